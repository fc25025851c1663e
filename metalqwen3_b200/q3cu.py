"""ctypes binding of libq3cu.so (the C ABI in include/q3cu.h) over torch tensors.

torch is used only for device memory and streams; every op runs the library's
own sm_100a kernels.  There is no fallback: if the shared library is missing or
no sm_100 GPU is present, the calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libq3cu.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "q3cu.h")

F32, BF16 = 0, 1
GS = 64
DEV_BAD_INDEX, DEV_TIMEOUT = 0x1, 0x2
STATUS = {0: "OK", 1: "ERR_INVALID", 2: "ERR_ALIGN", 3: "ERR_GROUP", 4: "ERR_CUDA", 5: "ERR_INDEX",
          6: "ERR_TIMEOUT", 7: "ERR_NOT_INIT", 8: "ERR_OOM", 9: "ERR_DEVICE", 10: "ERR_FORMAT"}

_lib = None
_lock = threading.Lock()


class Q3Error(RuntimeError):
    def __init__(self, status: int, op: str, msg: str):
        super().__init__(f"{op}: {STATUS.get(status, status)}: {msg}")
        self.status = status


def header_functions(path: str = HEADER) -> list[str]:
    """Names of the entry points declared in include/q3cu.h."""
    text = open(path).read()
    return sorted(set(re.findall(r"\b(q3cu_[a-z0-9_]+)\s*\(", text)))


def load_library(path: str = LIB_PATH) -> C.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise ImportError(f"{path} is missing: run __graft_entry__.build() (make -C metalqwen3_b200/csrc)")
            lib = C.CDLL(path)
            vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float
            st = C.c_int
            sigs = {
                "q3cu_init": (st, [i32, C.POINTER(vp)]),
                "q3cu_destroy": (st, [vp]),
                "q3cu_is_initialized": (i32, [vp]),
                "q3cu_last_error_string": (C.c_char_p, []),
                "q3cu_status_string": (C.c_char_p, [st]),
                "q3cu_version": (i32, []),
                "q3cu_device_status": (st, [vp, vp, C.POINTER(C.c_uint32)]),
                "q3cu_selftest_wait_timeout": (st, [vp, vp]),
                "q3cu_check_header": (st, [vp, C.c_size_t, vp]),
                "q3cu_rmsnorm": (st, [vp, vp, i32, vp, i64, i32, f32, vp, vp]),
                "q3cu_rmsnorm_q8": (st, [vp, vp, i32, vp, i64, i32, f32, vp, vp, vp]),
                "q3cu_qk_norm_rope": (st, [vp, vp, vp, i32, vp, i64, i32, i32, i32, vp, vp, f32, f32, vp]),
                "q3cu_swiglu": (st, [vp, vp, vp, i32, i64, i32, vp]),
                "q3cu_swiglu_q8": (st, [vp, vp, vp, i32, i64, i32, vp, vp, vp]),
                "q3cu_softmax_rows": (st, [vp, vp, vp, vp, i64, vp]),
                "q3cu_quantize_q8": (st, [vp, vp, i32, i64, i32, vp, vp, vp]),
                "q3cu_dequantize_q8": (st, [vp, vp, vp, i64, vp, vp]),
                "q3cu_embed_gather": (st, [vp, vp, vp, i32, i32, vp, i64, vp, vp, vp, vp]),
                "q3cu_matmul_q8": (st, [vp, vp, vp, i32, vp, vp, i32, i32, vp, vp]),
                "q3cu_execute_quantized_matmul": (st, [vp, vp, vp, vp, vp, vp, i32, i32, i32]),
                "q3cu_attention": (st, [vp, vp, vp, vp, i32, i32, i32, i32, vp, i32, vp, vp, vp]),
                "q3cu_execute_attention": (st, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, C.c_uint64,
                                                i32]),
                "q3cu_model_load": (st, [vp, vp, C.c_size_t, i32, C.POINTER(vp)]),
                "q3cu_model_config": (st, [vp, vp]),
                "q3cu_model_forward": (st, [vp, i32, i32, vp, vp]),
                "q3cu_model_logits": (vp, [vp]),
                "q3cu_model_destroy": (st, [vp]),
                "q3cu_execute_rmsnorm": (st, [vp, vp, vp, vp, i32]),
                "q3cu_execute_softmax": (st, [vp, vp, i32]),
                "q3cu_execute_swiglu": (st, [vp, vp, vp, i32]),
                "q3cu_execute_rope": (st, [vp, vp, vp, i32, i32, i32, i32, vp, vp]),
                "q3cu_execute_quantize": (st, [vp, vp, vp, vp, i32]),
                "q3cu_execute_embedding": (st, [vp, vp, vp, vp, i32, i32]),
            }
            for name, (res, args) in sigs.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def _ptr(t):
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return C.c_void_p(t.data_ptr())
    return C.c_void_p(t.ctypes.data)      # numpy (host-pointer wrappers)


def _dtype(t):
    import torch
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


class Q3CU:
    """One library context on one device (not thread-safe)."""

    def __init__(self, device: int = 0):
        import torch
        self.torch = torch
        self.lib = load_library()
        self.device = device
        torch.cuda.set_device(device)
        h = C.c_void_p()
        self._check(self.lib.q3cu_init(device, C.byref(h)), "q3cu_init")
        self.ctx = h

    # -- plumbing ------------------------------------------------------------
    def _check(self, status, op):
        if status != 0:
            raise Q3Error(status, op, (self.lib.q3cu_last_error_string() or b"").decode())

    def _stream(self, stream=None):
        s = stream if stream is not None else self.torch.cuda.current_stream(self.device)
        return C.c_void_p(s.cuda_stream)

    def close(self):
        if getattr(self, "ctx", None):
            self.lib.q3cu_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def selftest_wait_timeout(self, stream=None) -> None:
        """Enqueue the failure-path self-test: a kernel whose bounded wait gives
        up (about 2 s) and sets the timeout bit; read it with device_status()."""
        self._check(self.lib.q3cu_selftest_wait_timeout(self.ctx, self._stream(stream)), "q3cu_selftest_wait_timeout")

    def device_status(self, stream=None) -> int:
        flags = C.c_uint32(0)
        st = self.lib.q3cu_device_status(self.ctx, self._stream(stream), C.byref(flags))
        if st not in (0, 5, 6):
            self._check(st, "q3cu_device_status")
        return flags.value

    # -- device-pointer ops ----------------------------------------------------
    def rmsnorm(self, x, w, eps=1e-6, out=None, stream=None):
        rows, dim = x.shape
        out = self.torch.empty_like(x) if out is None else out
        self._check(self.lib.q3cu_rmsnorm(self.ctx, _ptr(x), _dtype(x), _ptr(w), rows, dim, eps, _ptr(out),
                                          self._stream(stream)), "q3cu_rmsnorm")
        return out

    def rmsnorm_q8(self, x, w, eps=1e-6, q=None, s=None, stream=None):
        rows, dim = x.shape
        q = self.torch.empty((rows, dim), dtype=self.torch.int8, device=x.device) if q is None else q
        s = self.torch.empty((rows, dim // GS), dtype=self.torch.float32, device=x.device) if s is None else s
        self._check(self.lib.q3cu_rmsnorm_q8(self.ctx, _ptr(x), _dtype(x), _ptr(w), rows, dim, eps, _ptr(q),
                                             _ptr(s), self._stream(stream)), "q3cu_rmsnorm_q8")
        return q, s

    def qk_norm_rope(self, q, k, pos, q_norm, k_norm, theta=1e6, eps=1e-6, stream=None):
        """In place.  q: [rows, n_heads, hd], k: [rows, n_kv, hd]."""
        rows, nh, hd = q.shape
        nkv = k.shape[1]
        self._check(self.lib.q3cu_qk_norm_rope(self.ctx, _ptr(q), _ptr(k), _dtype(q), _ptr(pos), rows, nh, nkv, hd,
                                               _ptr(q_norm), _ptr(k_norm), theta, eps, self._stream(stream)),
                    "q3cu_qk_norm_rope")
        return q, k

    def swiglu(self, hb, hb2, stream=None):
        rows, hidden = hb.shape
        self._check(self.lib.q3cu_swiglu(self.ctx, _ptr(hb), _ptr(hb2), _dtype(hb), rows, hidden,
                                         self._stream(stream)), "q3cu_swiglu")
        return hb

    def swiglu_q8(self, hb, hb2, q=None, s=None, stream=None):
        rows, hidden = hb.shape
        q = self.torch.empty((rows, hidden), dtype=self.torch.int8, device=hb.device) if q is None else q
        s = self.torch.empty((rows, hidden // GS), dtype=self.torch.float32, device=hb.device) if s is None else s
        self._check(self.lib.q3cu_swiglu_q8(self.ctx, _ptr(hb), _ptr(hb2), _dtype(hb), rows, hidden, _ptr(q), _ptr(s),
                                            self._stream(stream)), "q3cu_swiglu_q8")
        return q, s

    def softmax_rows(self, x, off, lens, stream=None):
        self._check(self.lib.q3cu_softmax_rows(self.ctx, _ptr(x), _ptr(off), _ptr(lens), off.numel(),
                                               self._stream(stream)), "q3cu_softmax_rows")
        return x

    def quantize_q8(self, x, q=None, s=None, stream=None):
        rows, n = x.shape
        q = self.torch.empty((rows, n), dtype=self.torch.int8, device=x.device) if q is None else q
        s = self.torch.empty((rows, n // GS), dtype=self.torch.float32, device=x.device) if s is None else s
        self._check(self.lib.q3cu_quantize_q8(self.ctx, _ptr(x), _dtype(x), rows, n, _ptr(q), _ptr(s),
                                              self._stream(stream)), "q3cu_quantize_q8")
        return q, s

    def dequantize_q8(self, q, s, out=None, stream=None):
        n = q.numel()
        out = self.torch.empty(q.shape, dtype=self.torch.float32, device=q.device) if out is None else out
        self._check(self.lib.q3cu_dequantize_q8(self.ctx, _ptr(q), _ptr(s), n, _ptr(out), self._stream(stream)),
                    "q3cu_dequantize_q8")
        return out

    def embed_gather(self, tq, ts, ids, want_f32=True, want_q8=True, out=None, oq=None, os_=None, stream=None):
        vocab, dim = tq.shape
        n = ids.numel()
        T = self.torch
        if want_f32 and out is None:
            out = T.empty((n, dim), dtype=T.float32, device=tq.device)
        if want_q8 and oq is None:
            oq = T.empty((n, dim), dtype=T.int8, device=tq.device)
            os_ = T.empty((n, dim // GS), dtype=T.float32, device=tq.device)
        self._check(self.lib.q3cu_embed_gather(self.ctx, _ptr(tq), _ptr(ts), vocab, dim, _ptr(ids), n,
                                               _ptr(out if want_f32 else None), _ptr(oq if want_q8 else None),
                                               _ptr(os_ if want_q8 else None), self._stream(stream)),
                    "q3cu_embed_gather")
        return out, oq, os_

    def matmul_q8(self, xq, xs, wq, ws, out=None, stream=None):
        """out[b] = W @ x[b] for Q8_0 x (xq [B][n], xs [B][n/64]) and W (wq [d][n], ws [d][n/64])."""
        B, n = xq.shape
        d = wq.shape[0]
        if wq.shape[1] != n:
            raise ValueError(f"W is {tuple(wq.shape)}, x rows have {n} elements")
        out = self.torch.empty((B, d), dtype=self.torch.float32, device=xq.device) if out is None else out
        self._check(self.lib.q3cu_matmul_q8(self.ctx, _ptr(xq), _ptr(xs), B, _ptr(wq), _ptr(ws), n, d, _ptr(out),
                                            self._stream(stream)), "q3cu_matmul_q8")
        return out

    def attention(self, q, key_cache, value_cache, pos, kv_mul, att=None, probs=None, xb=None, stream=None):
        """One token's attention over cache rows 0..pos: q [n_heads][128];
        key_cache / value_cache [rows][kv_dim]; att: scratch for the scores;
        returns (xb [n_heads][128], probs [n_heads][att_stride] with the
        probabilities in columns 0..pos)."""
        T = self.torch
        n_heads = q.numel() // 128
        kv_dim = key_cache.shape[-1]
        att = T.zeros((n_heads, pos + 1), dtype=T.float32, device=q.device) if att is None else att
        probs = T.zeros_like(att) if probs is None else probs
        xb = T.empty((n_heads, 128), dtype=T.float32, device=q.device) if xb is None else xb
        self._check(self.lib.q3cu_attention(self.ctx, _ptr(q), _ptr(key_cache), _ptr(value_cache), pos, n_heads,
                                            kv_dim, kv_mul, _ptr(att), att.shape[-1], _ptr(probs), _ptr(xb),
                                            self._stream(stream)), "q3cu_attention")
        return xb, probs

    # -- host-pointer drop-in (numpy arrays, synchronous) -----------------------
    def execute_attention(self, xb, q, att, key_cache, value_cache, pos, head_dim, n_heads, n_kv_heads, seq_len,
                          kv_dim, loff, kv_mul):
        self._check(self.lib.q3cu_execute_attention(self.ctx, _ptr(xb), _ptr(q), _ptr(att), _ptr(key_cache),
                                                    _ptr(value_cache), pos, head_dim, n_heads, n_kv_heads, seq_len,
                                                    kv_dim, loff, kv_mul), "executeAttention")

    def execute_rmsnorm(self, out, inp, w):
        self._check(self.lib.q3cu_execute_rmsnorm(self.ctx, _ptr(out), _ptr(inp), _ptr(w), inp.size), "executeRMSNorm")

    def execute_softmax(self, x):
        self._check(self.lib.q3cu_execute_softmax(self.ctx, _ptr(x), x.size), "executeSoftmax")

    def execute_swiglu(self, hb, hb2):
        self._check(self.lib.q3cu_execute_swiglu(self.ctx, _ptr(hb), _ptr(hb2), hb.size), "executeSwiGLU")

    def execute_rope(self, q, k, head_dim, pos, n_heads, n_kv, qn, kn):
        self._check(self.lib.q3cu_execute_rope(self.ctx, _ptr(q), _ptr(k), head_dim, pos, n_heads, n_kv, _ptr(qn),
                                               _ptr(kn)), "executeRoPE")

    def execute_quantize(self, q, s, x):
        self._check(self.lib.q3cu_execute_quantize(self.ctx, _ptr(q), _ptr(s), _ptr(x), x.size), "executeQuantize")

    def execute_quantized_matmul(self, out, xq, xs, wq, ws, n, d, group_size=GS):
        self._check(self.lib.q3cu_execute_quantized_matmul(self.ctx, _ptr(out), _ptr(xq), _ptr(xs), _ptr(wq), _ptr(ws),
                                                           n, d, group_size), "executeQuantizedMatMul")

    def execute_embedding(self, out, tq, ts, token, dim):
        self._check(self.lib.q3cu_execute_embedding(self.ctx, _ptr(out), _ptr(tq), _ptr(ts), token, dim),
                    "executeEmbedding")


class Q3Model:
    """A checkpoint image (numpy uint8 array or bytes: the reference's file
    format) resident on the device of `q3` (a Q3CU context), with its KV cache;
    forward(token, pos) returns the logits as a numpy array."""

    def __init__(self, q3, image, ctx_length=0):
        import numpy as np
        self.q3, self.lib = q3, q3.lib
        self._img = np.ascontiguousarray(np.frombuffer(image, np.uint8) if isinstance(image, (bytes, bytearray))
                                         else image, np.uint8)
        self.m = C.c_void_p()
        q3._check(self.lib.q3cu_model_load(q3.ctx, self._img.ctypes.data, self._img.nbytes, ctx_length,
                                           C.byref(self.m)), "q3cu_model_load")
        cfg = (C.c_int32 * 12)()
        q3._check(self.lib.q3cu_model_config(self.m, cfg), "q3cu_model_config")
        keys = ("magic", "version", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
                "seq_len", "head_dim", "shared_classifier", "group_size")
        self.config = dict(zip(keys, list(cfg)))
        self._img = None                      # the weights live on the device now

    def forward(self, token, pos, stream=None, to_host=True, out=None):
        """Logits of `token` at `pos` as a new float32 array, or into `out` (a
        C-contiguous float32 array of vocab_size, e.g. over pinned memory), or
        left on the device (to_host=False; see logits_ptr)."""
        import numpy as np
        if to_host and out is None:
            out = np.empty(self.config["vocab_size"], np.float32)
        if to_host and (out.dtype != np.float32 or out.size != self.config["vocab_size"]
                        or not out.flags["C_CONTIGUOUS"]):
            raise ValueError("out must be a C-contiguous float32 array of vocab_size elements")
        self.q3._check(self.lib.q3cu_model_forward(self.m, int(token), int(pos),
                                                   out.ctypes.data if to_host else None, self.q3._stream(stream)),
                       "q3cu_model_forward")
        return out if to_host else None

    def logits_ptr(self):
        return self.lib.q3cu_model_logits(self.m)

    def close(self):
        if self.m:
            self.lib.q3cu_model_destroy(self.m)
            self.m = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
