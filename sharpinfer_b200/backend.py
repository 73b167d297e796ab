"""Host-side mirror of SharpInfer's compute-backend interface over the C ABI.

SharpInfer injects an IComputeBackend (src/SharpInfer.Core/Tensors/
TensorOps.cs:241-250) whose MatVecMul takes dequantised f32 spans.  The B200
path keeps the weights quantised and device-resident, so its entry points take
a QuantWeight handle instead of an f32 matrix.  Device tensors are torch CUDA
tensors (plumbing for memory and streams); all arithmetic runs in
libsharpinfer_b200.so.
"""
import ctypes
import weakref

import numpy as np

from . import native as N


def _torch():
    import torch
    return torch


class QuantWeight:
    """A device-resident GGUF-quantised [rows][cols] weight (si_weight*)."""

    def __init__(self, ctx, handle, qtype, rows, cols):
        self.ctx, self.handle, self.qtype, self.rows, self.cols = ctx, handle, qtype, rows, cols
        ctx._adopt(self)

    @property
    def device_bytes(self):
        b = ctypes.c_int64()
        N.call("si_weight_info", self.handle, None, None, None, ctypes.byref(b))
        return b.value

    @property
    def gguf_bytes(self):
        return self.rows * (self.cols // N.BLOCK_ELEMS[self.qtype]) * N.BLOCK_BYTES[self.qtype]

    def free(self):
        if self.handle:
            N.call("si_weight_free", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class B200Context:
    """One GPU and one CUDA stream (si_ctx*)."""

    def __init__(self, device=0):
        N.load()
        h = ctypes.c_void_p()
        N.call("si_init", int(device), ctypes.byref(h))
        self.handle = h
        self.device = device
        s = ctypes.c_void_p()
        N.call("si_stream", self.handle, ctypes.byref(s))
        self.stream_ptr = s.value
        self._torch_stream = None
        self._children = weakref.WeakSet()  # weights and models that live on this context

    def _adopt(self, obj):
        """Track an object whose native handle must be freed before the context."""
        self._children.add(obj)

    @property
    def name(self):
        buf = ctypes.create_string_buffer(256)
        N.call("si_device_name", self.handle, buf, 256)
        return buf.value.decode()

    @property
    def torch_stream(self):
        """The context's stream as a torch stream (for allocations and events)."""
        if self._torch_stream is None:
            torch = _torch()
            self._torch_stream = torch.cuda.ExternalStream(self.stream_ptr, device=self.device)
        return self._torch_stream

    def synchronize(self):
        N.call("si_synchronize", self.handle)

    def _enter(self):
        """Order the context stream after work queued on torch's current stream."""
        torch = _torch()
        cur = torch.cuda.current_stream(self.device)
        if cur.cuda_stream != self.stream_ptr:
            self.torch_stream.wait_stream(cur)
        return cur

    def _leave(self, cur):
        """Order torch's current stream after the work just queued on the context stream."""
        if cur.cuda_stream != self.stream_ptr:
            cur.wait_stream(self.torch_stream)

    def close(self):
        """Free the weights and models still open on this context, then the context."""
        if self.handle:
            for obj in list(self._children):
                try:
                    obj.free()
                except Exception:
                    pass
            N.call("si_shutdown", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights -----------------------------------------------------------------
    def upload(self, qtype, blocks, rows, cols):
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        want = rows * (cols // N.BLOCK_ELEMS[qtype]) * N.BLOCK_BYTES[qtype]
        if blocks.nbytes != want:
            raise ValueError("expected %d bytes of blocks, got %d" % (want, blocks.nbytes))
        h = ctypes.c_void_p()
        N.call("si_weight_upload", self.handle, qtype, N.ptr(blocks), rows, cols, ctypes.byref(h))
        return QuantWeight(self, h, qtype, rows, cols)

    def synth_weight(self, qtype, rows, cols, seed, tag, recipe=N.SYNTH_PLAIN, sigma=0.01):
        h = ctypes.c_void_p()
        N.call("si_weight_synth", self.handle, qtype, rows, cols, seed, tag, recipe, sigma,
               ctypes.byref(h))
        return QuantWeight(self, h, qtype, rows, cols)

    # ---- ops (device tensors, asynchronous on the context stream) ----------------
    def dequant(self, w, out=None):
        torch = _torch()
        cur = self._enter()
        with torch.cuda.stream(self.torch_stream):
            if out is None:
                out = torch.empty((w.rows, w.cols), dtype=torch.float32, device="cuda:%d" % self.device)
            N.call("si_dequant", self.handle, w.handle, N.ptr(out))
        self._leave(cur)
        return out

    def qmatvec(self, w, x, out=None):
        """y[b] = W x[b]; x is a [batch, cols] (or [cols]) f32 CUDA tensor."""
        torch = _torch()
        x2 = x.reshape(-1, w.cols)
        batch = x2.shape[0]
        cur = self._enter()
        with torch.cuda.stream(self.torch_stream):
            if out is None:
                out = torch.empty((batch, w.rows), dtype=torch.float32, device=x.device)
            N.call("si_qmatvec", self.handle, w.handle, N.ptr(x2), N.ptr(out), batch)
        self._leave(cur)
        return out

    def act_prepare(self, x):
        """Prepare x [batch, cols] once for several qmatvec_prepared calls."""
        torch = _torch()
        x2 = x.reshape(x.shape[0] if x.dim() > 1 else 1, -1)
        cur = self._enter()
        with torch.cuda.stream(self.torch_stream):
            N.call("si_act_prepare", self.handle, N.ptr(x2), x2.shape[1], x2.shape[0])
        self._leave(cur)
        return x2.shape[0]

    def qmatvec_prepared(self, w, batch, out=None, accumulate=False):
        torch = _torch()
        cur = self._enter()
        with torch.cuda.stream(self.torch_stream):
            if out is None:
                out = torch.empty((batch, w.rows), dtype=torch.float32, device="cuda:%d" % self.device)
            N.call("si_qmatvec_prepared", self.handle, w.handle, N.ptr(out), batch, int(accumulate))
        self._leave(cur)
        return out

    def qgemm(self, w, x, out=None):
        """y = x W^T for bf16 x [M, cols] (CUDA tensor) on the tensor cores; y f32 [M, rows]."""
        torch = _torch()
        assert x.dtype == torch.bfloat16 and x.shape[-1] == w.cols
        x2 = x.reshape(-1, w.cols).contiguous()
        M = x2.shape[0]
        cur = self._enter()
        with torch.cuda.stream(self.torch_stream):
            if out is None:
                out = torch.empty((M, w.rows), dtype=torch.float32, device=x.device)
            N.call("si_qgemm", self.handle, w.handle, N.ptr(x2), N.ptr(out), M)
        self._leave(cur)
        return out

    def attn_prefill(self, q, k, v, scale, causal=True, start_pos=None, out=None):
        """FlashAttention.Forward on the tensor cores: bf16 q [B, H, S, 128], k/v [B, Hkv, KV, 128]
        (CUDA tensors); returns f32 [B, H, S, 128].  start_pos defaults to KV - S."""
        torch = _torch()
        B, H, S, D = q.shape
        Hkv, KV = k.shape[1], k.shape[2]
        if start_pos is None:
            start_pos = KV - S
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        cur = self._enter()
        with torch.cuda.stream(self.torch_stream):
            if out is None:
                out = torch.empty((B, H, S, D), dtype=torch.float32, device=q.device)
            N.call("si_attn_prefill", self.handle, N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(out), B, H, Hkv, S, KV, D,
                   float(scale), int(bool(causal)), int(start_pos))
        self._leave(cur)
        return out

    def qgemm_cache_weight(self, w):
        """Keep a dequantised f16 copy of w for later qgemm calls."""
        N.call("si_qgemm_cache_weight", self.handle, w.handle)

    def qmatvec_host(self, w, x):
        """Same with host numpy arrays; synchronous (the cuda_mat_vec_mul convention)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, w.cols)
        y = np.empty((x.shape[0], w.rows), dtype=np.float32)
        N.call("si_qmatvec_host", self.handle, w.handle, N.ptr(x), N.ptr(y), x.shape[0])
        return y


# ---- seeded synthetic host data (same bytes as the device generator) -------------
def synth_blocks_host(qtype, rows, cols, seed, tag, recipe=N.SYNTH_PLAIN, sigma=0.01):
    nb = rows * (cols // N.BLOCK_ELEMS.get(qtype, 256))
    out = np.empty(max(nb * N.BLOCK_BYTES.get(qtype, 1), 1), dtype=np.uint8)
    N.call("si_synth_blocks_host", qtype, rows, cols, seed, tag, recipe, sigma, N.ptr(out))
    return out


def synth_f32_host(n, seed, tag, mean=0.0, sigma=1.0):
    out = np.empty(n, dtype=np.float32)
    N.call("si_synth_f32_host", n, seed, tag, mean, sigma, N.ptr(out))
    return out


def synth_f16_host(n, seed, tag, sigma=1.0):
    out = np.empty(n, dtype=np.uint16)
    N.call("si_synth_f16_host", n, seed, tag, sigma, N.ptr(out))
    return out
