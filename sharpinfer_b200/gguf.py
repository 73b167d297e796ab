"""GGUF files over the C ABI (si_gguf_*): the model loader behind
InferenceEngine.Load (src/SharpInfer.Core/Engine/InferenceEngine.cs:48-49).
The file is memory-mapped by the library; weights go to the device as their
raw GGUF blocks."""
import ctypes

from . import native as N


class GGUFFile:
    """An open GGUF v2/v3 file (si_gguf*)."""

    def __init__(self, path):
        h = ctypes.c_void_p()
        N.call("si_gguf_open", str(path).encode(), ctypes.byref(h))
        self.handle = h

    def close(self):
        if self.handle:
            N.call("si_gguf_close", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self):
        """(version, tensor count, key/value count, data-section offset)."""
        v, nt, nkv, off = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        N.call("si_gguf_info", self.handle, ctypes.byref(v), ctypes.byref(nt), ctypes.byref(nkv), ctypes.byref(off))
        return v.value, nt.value, nkv.value, off.value

    def meta_int(self, key):
        v = ctypes.c_int64()
        N.call("si_gguf_meta_int", self.handle, key.encode(), ctypes.byref(v))
        return v.value

    def meta_float(self, key):
        v = ctypes.c_double()
        N.call("si_gguf_meta_float", self.handle, key.encode(), ctypes.byref(v))
        return v.value

    def meta_string(self, key, maxlen=4096):
        buf = ctypes.create_string_buffer(maxlen)
        N.call("si_gguf_meta_string", self.handle, key.encode(), buf, maxlen)
        return buf.value.decode(errors="replace")

    def meta_array(self, key):
        """(item type, length) of an array value."""
        t, n = ctypes.c_int(), ctypes.c_int64()
        N.call("si_gguf_meta_array", self.handle, key.encode(), ctypes.byref(t), ctypes.byref(n))
        return t.value, n.value

    def tensors(self):
        """[(name, ggml type, rows, cols, bytes)] in file order."""
        out = []
        name = ctypes.create_string_buffer(512)
        qt, rows, cols, nb = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        for i in range(self.info()[1]):
            N.call("si_gguf_tensor_info", self.handle, i, name, 512, ctypes.byref(qt), ctypes.byref(rows),
                   ctypes.byref(cols), ctypes.byref(nb))
            out.append((name.value.decode(), qt.value, rows.value, cols.value, nb.value))
        return out

    def tensor_bytes(self, name):
        """The tensor's bytes in the mapped file (a copy)."""
        idx = ctypes.c_int64()
        N.call("si_gguf_find_tensor", self.handle, name.encode(), ctypes.byref(idx))
        p = ctypes.c_void_p()
        N.call("si_gguf_tensor_data", self.handle, idx.value, ctypes.byref(p))
        nb = [t for t in self.tensors() if t[0] == name][0][4]
        return ctypes.string_at(p.value, nb)

    def model_config(self, max_seq=0, max_batch=1):
        cfg = N.ModelConfig()
        N.call("si_gguf_model_config", self.handle, max_seq, max_batch, ctypes.byref(cfg))
        return cfg

    def load_into(self, model):
        """Upload every tensor into a DecodeModel built from model_config()."""
        N.call("si_model_load_gguf", model.handle, self.handle)
