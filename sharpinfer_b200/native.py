"""ctypes binding of libsharpinfer_b200.so (the C ABI in include/sharpinfer_b200.h).

The library is loaded from the package directory; there is no fallback: if it
is missing or a call fails, an exception is raised.
"""
import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsharpinfer_b200.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "sharpinfer_b200.h")

SI_OK = 0
SI_F32, SI_F16, SI_Q8_0, SI_Q4_K, SI_Q6_K = 0, 1, 8, 12, 14
SI_Q4_0, SI_Q2_K, SI_Q3_K, SI_Q5_K = 2, 10, 11, 13
SYNTH_PLAIN, SYNTH_MODEL = 0, 1
BLOCK_ELEMS = {SI_Q4_K: 256, SI_Q6_K: 256, SI_Q8_0: 32, SI_Q4_0: 32, SI_Q2_K: 256, SI_Q3_K: 256, SI_Q5_K: 256}
BLOCK_BYTES = {SI_Q4_K: 144, SI_Q6_K: 210, SI_Q8_0: 34, SI_Q4_0: 18, SI_Q2_K: 84, SI_Q3_K: 110, SI_Q5_K: 176}

_c_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_f32 = ctypes.c_float


class ModelConfig(ctypes.Structure):
    """si_model_config (field names of the reference's ModelConfig)."""
    _fields_ = [("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("intermediate", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("vocab", ctypes.c_int), ("max_seq", ctypes.c_int), ("max_batch", ctypes.c_int),
                ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("weight_qtype", ctypes.c_int),
                ("lm_head_qtype", ctypes.c_int), ("emb_qtype", ctypes.c_int)]


T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_ATTN_NORM, T_FFN_NORM = range(9)
T_EMB, T_LM_HEAD, T_FINAL_NORM = 100, 101, 102


class SIError(RuntimeError):
    """A sharpinfer_b200 call returned a non-zero si_status."""

    def __init__(self, status, msg):
        super().__init__("si_status %d: %s" % (status, msg))
        self.status = status


# name -> (restype, argtypes)
_SIGS = {
    "si_version": (_i32, []),
    "si_last_error": (ctypes.c_char_p, []),
    "si_init": (_i32, [_i32, ctypes.POINTER(_c_p)]),
    "si_shutdown": (_i32, [_c_p]),
    "si_device_name": (_i32, [_c_p, ctypes.c_char_p, _i32]),
    "si_stream": (_i32, [_c_p, ctypes.POINTER(_c_p)]),
    "si_synchronize": (_i32, [_c_p]),
    "si_weight_upload": (_i32, [_c_p, _i32, _c_p, _i64, _i64, ctypes.POINTER(_c_p)]),
    "si_weight_synth": (_i32, [_c_p, _i32, _i64, _i64, _u64, _u64, _i32, _f32, ctypes.POINTER(_c_p)]),
    "si_weight_free": (_i32, [_c_p]),
    "si_weight_info": (_i32, [_c_p, ctypes.POINTER(_i32), ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                              ctypes.POINTER(_i64)]),
    "si_synth_blocks_host": (_i32, [_i32, _i64, _i64, _u64, _u64, _i32, _f32, _c_p]),
    "si_synth_f32_host": (_i32, [_i64, _u64, _u64, _f32, _f32, _c_p]),
    "si_synth_f16_host": (_i32, [_i64, _u64, _u64, _f32, _c_p]),
    "si_dequant": (_i32, [_c_p, _c_p, _c_p]),
    "si_qmatvec": (_i32, [_c_p, _c_p, _c_p, _c_p, _i32]),
    "si_act_prepare": (_i32, [_c_p, _c_p, _i64, _i32]),
    "si_qmatvec_prepared": (_i32, [_c_p, _c_p, _c_p, _i32, _i32]),
    "si_qmatvec_host": (_i32, [_c_p, _c_p, _c_p, _c_p, _i32]),
    "si_qmatvec_noalloc": (_i32, [_c_p, _c_p, _c_p, _i32, _c_p]),
    "si_qgemm": (_i32, [_c_p, _c_p, _c_p, _c_p, _i32]),
    "si_qgemm_cache_weight": (_i32, [_c_p, _c_p]),
    "si_attn_prefill": (_i32, [_c_p, _c_p, _c_p, _c_p, _c_p] + [_i32] * 6 + [ctypes.c_float, _i32, _i32]),
    "si_model_create_tp": (_i32, [_c_p, ctypes.POINTER(ModelConfig), _i32, _i32, ctypes.POINTER(_c_p)]),
    "si_model_tp_handle": (_i32, [_c_p, _c_p, _i32]),
    "si_model_tp_connect": (_i32, [_c_p, _c_p, _i32]),
    "si_model_tp_connect_local": (_i32, [_c_p, ctypes.POINTER(_c_p), _i32]),
    "si_tp_slice": (_i32, [ctypes.POINTER(ModelConfig), _i32, _i32, _i32] + [ctypes.POINTER(ctypes.c_int64)] * 5),
    "si_decode_step_kernels": (_i32, [_c_p, _i32, ctypes.POINTER(_i32)]),
    "cuda_init": (_c_p, [_i32]),
    "cuda_cleanup": (None, [_c_p]),
    "cuda_device_name": (None, [_c_p, _c_p, _i32]),
    "cuda_is_available": (_i32, []),
    "cuda_device_name_str": (ctypes.c_char_p, []),
    "cuda_mat_vec_mul": (None, [_c_p, _c_p, _c_p, _c_p, _i32, _i32]),
    "cuda_mat_mul": (None, [_c_p, _c_p, _c_p, _c_p, _i32, _i32, _i32]),
    "cuda_softmax": (None, [_c_p, _c_p, _i32]),
    "cuda_rms_norm": (None, [_c_p, _c_p, _c_p, _c_p, _i32, ctypes.c_float]),
    "cuda_silu": (None, [_c_p, _c_p, _i32]),
    "cuda_add_inplace": (None, [_c_p, _c_p, _c_p, _i32]),
    "flash_attention_forward": (None, [_c_p, _c_p, _c_p, _c_p] + [_i32] * 5 + [ctypes.c_float, _i32]),
    "si_model_create": (_i32, [_c_p, ctypes.POINTER(ModelConfig), ctypes.POINTER(_c_p)]),
    "si_model_free": (_i32, [_c_p]),
    "si_model_set_tensor": (_i32, [_c_p, _i32, _i32, _c_p]),
    "si_model_synth": (_i32, [_c_p, _u64]),
    "si_model_tensor_recipe": (_i32, [ctypes.POINTER(ModelConfig), _i32, _i32, ctypes.POINTER(_u64),
                                      ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_f32),
                                      ctypes.POINTER(_f32), ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "si_model_kv_synth": (_i32, [_c_p, _i32, _u64]),
    "si_model_kv_tag": (_u64, [_i32, _i32, _i32]),
    "si_model_kv_write": (_i32, [_c_p, _i32, _i32, _i32, _i32, _c_p, _c_p]),
    "si_decode_step": (_i32, [_c_p, _c_p, _i32, _i32, _c_p, _c_p]),
    "si_decode_generate": (_i32, [_c_p, _c_p, _i32, _i32, _i32, _c_p]),
    "si_model_attention": (_i32, [_c_p, _i32, _c_p, _c_p, _i32, _i32]),
    "si_model_prefill": (_i32, [_c_p, _i32, _c_p, _i32, _i32, _c_p, _c_p]),
    "si_model_get_config": (_i32, [_c_p, ctypes.POINTER(ModelConfig)]),
    "si_gguf_open": (_i32, [ctypes.c_char_p, ctypes.POINTER(_c_p)]),
    "si_gguf_close": (_i32, [_c_p]),
    "si_gguf_info": (_i32, [_c_p, ctypes.POINTER(_i32), ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                            ctypes.POINTER(_i64)]),
    "si_gguf_meta_int": (_i32, [_c_p, ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "si_gguf_meta_float": (_i32, [_c_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    "si_gguf_meta_string": (_i32, [_c_p, ctypes.c_char_p, ctypes.c_char_p, _i32]),
    "si_gguf_meta_array": (_i32, [_c_p, ctypes.c_char_p, ctypes.POINTER(_i32), ctypes.POINTER(_i64)]),
    "si_gguf_tensor_info": (_i32, [_c_p, _i64, ctypes.c_char_p, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i64),
                                   ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "si_gguf_find_tensor": (_i32, [_c_p, ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "si_gguf_tensor_data": (_i32, [_c_p, _i64, ctypes.POINTER(_c_p)]),
    "si_gguf_model_config": (_i32, [_c_p, _i32, _i32, ctypes.POINTER(ModelConfig)]),
    "si_model_load_gguf": (_i32, [_c_p, _c_p]),
    "si_model_kv_read": (_i32, [_c_p, _i32, _i32, _i32, _i32, _c_p, _c_p]),
    "si_model_kv_export": (_i32, [_c_p, _i32, _i32, _c_p, ctypes.c_size_t]),
    "si_model_kv_import": (_i32, [_c_p, _i32, _i32, _c_p, ctypes.c_size_t]),
}

_lib = None


def load():
    """Load the native library (once) and declare the signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            "libsharpinfer_b200.so not built (%s); run `python sharpinfer_b200/build.py`" % LIB_PATH)
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def declared_symbols(header=HEADER):
    """Names of the functions the public header declares with SI_EXPORT."""
    text = open(header).read()
    return re.findall(r"SI_EXPORT\s+[\w\s\*]+?\b(\w+)\s*\(", text)


def check(status):
    if status != SI_OK:
        raise SIError(status, load().si_last_error().decode(errors="replace"))
    return status


def call(name, *args):
    return check(getattr(load(), name)(*args))


def ptr(x):
    """Raw pointer of a torch tensor, numpy array, int address or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError("cannot take the address of %r" % type(x))
