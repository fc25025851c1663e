"""ctypes bindings for the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Two libraries are exposed:

* ``Oracle``     -- ``oracle/liboracle.so``, the plain-C restatement of the
  reference CPU engine (``oracle/q3_oracle.c``; each function cites
  ``src/cpu/qwen3_original.c`` line numbers).  Built on demand with ``make``.
* ``Reference``  -- ``oracle/_ref/libqwen3_ref.so``, the reference's own
  ``src/cpu/qwen3_original.c`` compiled unmodified (``make -C oracle ref``).
  Present only where the reference sources were available at build time.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only to check results against it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GS = 64
_build_lock = threading.Lock()


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def build_oracle(force: bool = False) -> str:
    path = os.path.join(HERE, "liboracle.so")
    with _build_lock:
        if force or not os.path.exists(path):
            subprocess.run(["make", "-s", "-C", HERE], check=True)
    return path


def reference_path() -> str:
    return os.path.join(HERE, "_ref", "libqwen3_ref.so")


def build_reference() -> str | None:
    """Compile the reference CPU engine if its sources are reachable."""
    root = os.environ.get("Q3_REFERENCE", os.path.join(HERE, "..", "..", "reference"))   # default: beside the repo
    src = os.path.join(root, "src", "cpu", "qwen3_original.c")
    if os.path.exists(src):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REFERENCE={os.path.abspath(root)}"], check=True)
    return reference_path() if os.path.exists(reference_path()) else None


class Oracle:
    """The restatement.  All array arguments are numpy arrays (C-contiguous)."""

    def __init__(self):
        self.lib = C.CDLL(build_oracle())
        L = self.lib
        vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "q3o_rmsnorm": (None, [vp, vp, vp, i32]),
            "q3o_softmax": (None, [vp, i32]),
            "q3o_quantize": (None, [vp, vp, vp, i32]),
            "q3o_dequantize": (None, [vp, vp, vp, i32]),
            "q3o_round_i8": (C.c_int8, [f32]),
            "q3o_qk_norm_rope_head_theta": (None, [vp, vp, i32, i32, f32]),
            "q3o_swiglu": (None, [vp, vp, i32]),
            "q3o_matmul": (None, [vp, vp, vp, vp, vp, i32, i32]),
            "q3o_attention": (None, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, C.c_uint64, i32]),
            "q3o_rows_rmsnorm": (None, [vp, i32, vp, i64, i32, vp, i32]),
            "q3o_rows_rmsnorm_q8": (None, [vp, i32, vp, i64, i32, vp, vp, i32]),
            "q3o_rows_quantize": (None, [vp, i32, i64, i32, vp, vp, i32]),
            "q3o_rows_swiglu": (None, [vp, vp, i32, i64, i32, i32]),
            "q3o_rows_swiglu_q8": (None, [vp, vp, i32, i64, i32, vp, vp, i32]),
            "q3o_rows_qk_norm_rope": (None, [vp, vp, i32, vp, i64, i32, i32, i32, vp, vp, f32, i32]),
            "q3o_rows_softmax": (None, [vp, vp, vp, i64, i32]),
            "q3o_rows_embed": (i64, [vp, vp, i32, i32, vp, i64, vp, vp, vp, i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args

    # ---- single-row primitives (reference semantics) -----------------------
    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        o = np.empty_like(x)
        self.lib.q3o_rmsnorm(_p(o), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size)
        return o

    def softmax(self, x):
        x = np.array(x, np.float32, copy=True)
        self.lib.q3o_softmax(_p(x), x.size)
        return x

    def quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        q = np.empty(x.size, np.int8)
        s = np.empty(x.size // GS, np.float32)
        self.lib.q3o_quantize(_p(q), _p(s), _p(x), x.size)
        return q, s

    def dequantize(self, q, s):
        q = np.ascontiguousarray(q, np.int8)
        x = np.empty(q.size, np.float32)
        self.lib.q3o_dequantize(_p(x), _p(q), _p(np.ascontiguousarray(s, np.float32)), q.size)
        return x

    def qk_norm_rope_head(self, v, w, pos, theta=1e6):
        v = np.array(v, np.float32, copy=True)
        self.lib.q3o_qk_norm_rope_head_theta(_p(v), _p(np.ascontiguousarray(w, np.float32)), v.size, pos, theta)
        return v

    def swiglu(self, hb, hb2):
        hb = np.array(hb, np.float32, copy=True)
        self.lib.q3o_swiglu(_p(hb), _p(np.ascontiguousarray(hb2, np.float32)), hb.size)
        return hb

    def matmul(self, xq, xs, wq, ws):
        """qwen3_original.c:310-331 for each row of x: xq [B][n], xs [B][n/64]; wq [d][n], ws [d][n/64] -> [B][d]."""
        xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
        xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
        wq = np.ascontiguousarray(wq, np.int8)
        ws = np.ascontiguousarray(ws, np.float32)
        B, n = xq.shape
        d = wq.shape[0]
        out = np.empty((B, d), np.float32)
        for b in range(B):
            self.lib.q3o_matmul(_p(out[b]), _p(xq[b]), _p(xs[b]), _p(wq), _p(ws), n, d)
        return out

    def attention(self, q, key_cache, value_cache, pos, n_heads, n_kv_heads, seq_len, loff=0, kv_mul=None):
        """qwen3_original.c:395-428 (q3o_attention): q [n_heads * 128]; the caches
        [.., kv_dim] flat; returns (xb [n_heads * hd], att [n_heads][seq_len])."""
        q = np.ascontiguousarray(q, np.float32).ravel()
        hd = q.size // n_heads
        kv_mul = kv_mul or n_heads // n_kv_heads
        kc = np.ascontiguousarray(key_cache, np.float32).ravel()
        vc = np.ascontiguousarray(value_cache, np.float32).ravel()
        xb = np.empty(n_heads * hd, np.float32)
        att = np.zeros((n_heads, seq_len), np.float32)
        self.lib.q3o_attention(_p(xb), _p(q), _p(att), _p(kc), _p(vc), int(pos), hd, n_heads, n_kv_heads,
                               seq_len, n_kv_heads * hd, C.c_uint64(loff), kv_mul)
        return xb, att

    # ---- row-batched forms ------------------------------------------------
    @staticmethod
    def _dt(a):
        if a.dtype == np.float32:
            return 0
        if a.dtype == np.uint16:   # bf16 bit patterns
            return 1
        raise TypeError(f"unsupported dtype {a.dtype}")

    def rows_rmsnorm(self, x, w, threads=1):
        rows, dim = x.shape
        out = np.empty_like(x)
        self.lib.q3o_rows_rmsnorm(_p(x), self._dt(x), _p(w), rows, dim, _p(out), threads)
        return out

    def rows_rmsnorm_q8(self, x, w, threads=1):
        rows, dim = x.shape
        q = np.empty((rows, dim), np.int8)
        s = np.empty((rows, dim // GS), np.float32)
        self.lib.q3o_rows_rmsnorm_q8(_p(x), self._dt(x), _p(w), rows, dim, _p(q), _p(s), threads)
        return q, s

    def rows_quantize(self, x, threads=1):
        rows, n = x.shape
        q = np.empty((rows, n), np.int8)
        s = np.empty((rows, n // GS), np.float32)
        self.lib.q3o_rows_quantize(_p(x), self._dt(x), rows, n, _p(q), _p(s), threads)
        return q, s

    def rows_swiglu(self, hb, hb2, threads=1):
        rows, n = hb.shape
        out = np.array(hb, copy=True)
        self.lib.q3o_rows_swiglu(_p(out), _p(hb2), self._dt(hb), rows, n, threads)
        return out

    def rows_swiglu_q8(self, hb, hb2, threads=1):
        rows, n = hb.shape
        q = np.empty((rows, n), np.int8)
        s = np.empty((rows, n // GS), np.float32)
        self.lib.q3o_rows_swiglu_q8(_p(hb), _p(hb2), self._dt(hb), rows, n, _p(q), _p(s), threads)
        return q, s

    def rows_qk_norm_rope(self, q, k, pos, q_norm, k_norm, theta=1e6, threads=1):
        """q: [rows, n_heads, hd], k: [rows, n_kv, hd]; returns new arrays."""
        rows, nh, hd = q.shape
        nkv = k.shape[1]
        qo, ko = np.array(q, copy=True), np.array(k, copy=True)
        pos = np.ascontiguousarray(pos, np.int32)
        self.lib.q3o_rows_qk_norm_rope(_p(qo), _p(ko), self._dt(q), _p(pos), rows, nh, nkv, hd,
                                       _p(np.ascontiguousarray(q_norm, np.float32)),
                                       _p(np.ascontiguousarray(k_norm, np.float32)), theta, threads)
        return qo, ko

    def rows_softmax(self, x, off, lens, threads=1):
        out = np.array(x, np.float32, copy=True)
        off = np.ascontiguousarray(off, np.int64)
        lens = np.ascontiguousarray(lens, np.int32)
        self.lib.q3o_rows_softmax(_p(out), _p(off), _p(lens), off.size, threads)
        return out

    def rows_embed(self, tq, ts, ids, want_f32=True, want_q8=True, threads=1):
        vocab, dim = tq.shape
        ids = np.ascontiguousarray(ids, np.int32)
        n = ids.size
        out = np.zeros((n, dim), np.float32) if want_f32 else None
        oq = np.zeros((n, dim), np.int8) if want_q8 else None
        os_ = np.zeros((n, dim // GS), np.float32) if want_q8 else None
        bad = self.lib.q3o_rows_embed(_p(tq), _p(ts), vocab, dim, _p(ids), n, _p(out), _p(oq), _p(os_), threads)
        return out, oq, os_, bad


class _QT(C.Structure):
    _fields_ = [("q", C.c_void_p), ("s", C.c_void_p)]


class _Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "magic_number", "version", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
        "vocab_size", "seq_len", "head_dim", "shared_classifier", "group_size")]


class _Transformer(C.Structure):
    """Layout of `Transformer` (src/cpu/qwen3_original.c:48-97)."""
    _fields_ = [("config", _Config)] + [(n, C.c_void_p) for n in (
        # TransformerWeights (:48-71)
        "q_tokens", "token_embedding_table", "rms_att_weight", "rms_ffn_weight", "wq", "wk", "wv", "wo",
        "q_norm_weights", "k_norm_weights", "w1", "w2", "w3", "rms_final_weight", "wcls",
        # RunState (:73-89)
        "x", "xb", "hb", "hb2")] + [("xq", _QT), ("hq", _QT)] + [(n, C.c_void_p) for n in (
        "q", "k", "v", "att", "logits", "key_cache", "value_cache", "data")] + [("file_size", C.c_ssize_t)]


class Reference:
    """The reference CPU engine compiled unmodified; exported symbols only."""

    def __init__(self, path: str | None = None):
        path = path or reference_path()
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        L = self.lib
        vp, i32 = C.c_void_p, C.c_int
        for name, res, args in (
            ("rmsnorm", None, [vp, vp, vp, i32]),
            ("softmax", None, [vp, i32]),
            ("quantize", None, [C.POINTER(_QT), vp, i32]),
            ("dequantize", None, [C.POINTER(_QT), vp, i32]),
            ("matmul", None, [vp, C.POINTER(_QT), C.POINTER(_QT), i32, i32]),
            ("qwen3_transformer_create", C.POINTER(_Transformer), [C.c_char_p, i32]),
            ("qwen3_transformer_free", None, [C.POINTER(_Transformer)]),
            ("qwen3_forward", C.POINTER(C.c_float), [C.POINTER(_Transformer), i32, i32]),
        ):
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        C.c_int.in_dll(L, "GS").value = GS   # the global at qwen3_original.c:20

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        o = np.empty_like(x)
        self.lib.rmsnorm(_p(o), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size)
        return o

    def softmax(self, x):
        x = np.array(x, np.float32, copy=True)
        self.lib.softmax(_p(x), x.size)
        return x

    def quantize(self, x):
        x = np.array(x, np.float32, copy=True)
        q = np.empty(x.size, np.int8)
        s = np.empty(x.size // GS, np.float32)
        qt = _QT(q.ctypes.data, s.ctypes.data)
        self.lib.quantize(C.byref(qt), _p(x), x.size)
        return q, s

    def dequantize(self, q, s):
        q = np.ascontiguousarray(q, np.int8)
        s = np.ascontiguousarray(s, np.float32)
        x = np.empty(q.size, np.float32)
        qt = _QT(q.ctypes.data, s.ctypes.data)
        self.lib.dequantize(C.byref(qt), _p(x), q.size)
        return x

    def matmul(self, xq, xs, wq, ws):
        """The reference's own `matmul` (OpenMP over output rows) for each row of x."""
        xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
        xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
        wq = np.ascontiguousarray(wq, np.int8)
        ws = np.ascontiguousarray(ws, np.float32)
        B, n = xq.shape
        d = wq.shape[0]
        out = np.empty((B, d), np.float32)
        wt = _QT(wq.ctypes.data, ws.ctypes.data)
        for b in range(B):
            xt = _QT(xq[b].ctypes.data, xs[b].ctypes.data)
            self.lib.matmul(_p(out[b]), C.byref(xt), C.byref(wt), n, d)
        return out

    # ---- whole decode step --------------------------------------------------
    def create(self, checkpoint_path: str, ctx_length: int = 0):
        t = self.lib.qwen3_transformer_create(checkpoint_path.encode(), ctx_length)
        if not t:
            raise RuntimeError("qwen3_transformer_create failed")
        return t

    def forward(self, t, token: int, pos: int) -> np.ndarray:
        ptr = self.lib.qwen3_forward(t, token, pos)
        return np.ctypeslib.as_array(ptr, shape=(t.contents.config.vocab_size,)).copy()

    @staticmethod
    def state(t, pos: int) -> dict:
        """Copies of the RunState buffers the reference leaves behind after forward()."""
        T = t.contents
        c = T.config
        hd, nh, nkv = c.head_dim, c.n_heads, c.n_kv_heads
        kvd, ahd = nkv * hd, nh * hd

        def arr(p, n, dt):
            return np.ctypeslib.as_array(C.cast(p, C.POINTER(dt)), shape=(n,)).copy()

        kc = arr(T.key_cache, c.n_layers * c.seq_len * kvd, C.c_float).reshape(c.n_layers, c.seq_len, kvd)
        vc = arr(T.value_cache, c.n_layers * c.seq_len * kvd, C.c_float).reshape(c.n_layers, c.seq_len, kvd)
        att = arr(T.att, nh * c.seq_len, C.c_float).reshape(nh, c.seq_len)[:, : pos + 1]
        return {
            "x": arr(T.x, c.dim, C.c_float),
            "q": arr(T.q, ahd, C.c_float),
            "hb": arr(T.hb, c.hidden_dim, C.c_float),
            "hb2": arr(T.hb2, c.hidden_dim, C.c_float),
            "xq_q": arr(T.xq.q, c.dim, C.c_int8),
            "xq_s": arr(T.xq.s, c.dim // GS, C.c_float),
            "hq_q": arr(T.hq.q, c.hidden_dim, C.c_int8),
            "hq_s": arr(T.hq.s, c.hidden_dim // GS, C.c_float),
            "att": att,
            "key_cache": kc[:, : pos + 1],
            "value_cache": vc[:, : pos + 1],
        }

    def free(self, t):
        self.lib.qwen3_transformer_free(t)


class ReferenceRows:
    """Row-batched, OpenMP driver of the compiled reference (oracle/ref_rows.c).

    Same method names and signatures as the f32 paths of ``Oracle`` so callers
    can time either; only f32 inputs.
    """

    def __init__(self, path: str | None = None):
        path = path or os.path.join(HERE, "_ref", "libref_rows.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        vp, i32, i64 = C.c_void_p, C.c_int, C.c_int64
        for name, args in (
            ("ref_rows_rmsnorm_q8", [vp, vp, i64, i32, vp, vp, i32]),
            ("ref_rows_quantize", [vp, i64, i32, vp, vp, i32]),
            ("ref_rows_qk_norm_rope", [vp, vp, vp, i64, i32, i32, i32, vp, vp, i32]),
            ("ref_rows_swiglu_q8", [vp, vp, i64, i32, vp, vp, i32]),
            ("ref_rows_softmax", [vp, vp, vp, i64, i32]),
            ("ref_rows_embed", [vp, vp, i32, i32, vp, i64, vp, vp, vp, i32]),
            ("ref_decode_ops", [vp, vp, i32, i32, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp,
                                i32, i32, vp, vp]),
        ):
            fn = getattr(self.lib, name)
            fn.restype = None
            fn.argtypes = args

    def rows_rmsnorm_q8(self, x, w, threads=1):
        rows, dim = x.shape
        q = np.empty((rows, dim), np.int8)
        s = np.empty((rows, dim // GS), np.float32)
        self.lib.ref_rows_rmsnorm_q8(_p(x), _p(w), rows, dim, _p(q), _p(s), threads)
        return q, s

    def rows_quantize(self, x, threads=1):
        rows, n = x.shape
        q = np.empty((rows, n), np.int8)
        s = np.empty((rows, n // GS), np.float32)
        self.lib.ref_rows_quantize(_p(np.ascontiguousarray(x, np.float32)), rows, n, _p(q), _p(s), threads)
        return q, s

    def rows_qk_norm_rope(self, q, k, pos, q_norm, k_norm, theta=1e6, threads=1):
        assert theta == 1e6, "the reference hard-codes theta = 1e6"
        rows, nh, hd = q.shape
        qo, ko = np.array(q, copy=True), np.array(k, copy=True)
        self.lib.ref_rows_qk_norm_rope(_p(qo), _p(ko), _p(np.ascontiguousarray(pos, np.int32)), rows, nh,
                                       k.shape[1], hd, _p(q_norm), _p(k_norm), threads)
        return qo, ko

    def rows_swiglu_q8(self, hb, hb2, threads=1):
        rows, n = hb.shape
        q = np.empty((rows, n), np.int8)
        s = np.empty((rows, n // GS), np.float32)
        self.lib.ref_rows_swiglu_q8(_p(hb), _p(hb2), rows, n, _p(q), _p(s), threads)
        return q, s

    def rows_softmax(self, x, off, lens, threads=1):
        out = np.array(x, np.float32, copy=True)
        off = np.ascontiguousarray(off, np.int64)
        lens = np.ascontiguousarray(lens, np.int32)
        self.lib.ref_rows_softmax(_p(out), _p(off), _p(lens), off.size, threads)
        return out

    def rows_embed(self, tq, ts, ids, want_q8=True, threads=1):
        vocab, dim = tq.shape
        ids = np.ascontiguousarray(ids, np.int32)
        n = ids.size
        out = np.zeros((n, dim), np.float32)
        oq = np.zeros((n, dim), np.int8) if want_q8 else None
        os_ = np.zeros((n, dim // GS), np.float32) if want_q8 else None
        self.lib.ref_rows_embed(_p(tq), _p(ts), vocab, dim, _p(ids), n, _p(out), _p(oq), _p(os_), threads)
        return out, oq, os_

    def decode_ops(self, tq, ts, token, x, w, q, k, pos, qn, kn, sc, ao, hb, hb2, layers):
        """One decode token through the path's ops (ref_decode_ops); q, k and sc
        in place."""
        dim = x.size
        n_heads, head_dim = q.shape[-2], q.shape[-1]
        n_kv = k.shape[-2]
        big = max(dim, hb.size, n_heads * head_dim)
        emb = np.empty(dim, np.float32)
        q8 = np.empty(big, np.int8)
        s8 = np.empty(big // GS, np.float32)
        self.lib.ref_decode_ops(_p(tq), _p(ts), dim, int(token), _p(emb), _p(x), _p(w), _p(q), _p(k), n_heads,
                                n_kv, head_dim, int(pos), _p(qn), _p(kn), _p(sc), _p(ao), _p(hb), _p(hb2), hb.size,
                                layers, _p(q8), _p(s8))
        return emb


class OracleModel:
    """The restated decode step (q3o_forward) over an in-memory checkpoint image."""

    class _M(C.Structure):
        _fields_ = [("c", _Config)] + [(n, C.c_void_p) for n in (
            "rms_att", "rms_ffn", "rms_final", "q_norm", "k_norm", "tok_q", "tok_s",
            "wq_q", "wk_q", "wv_q", "wo_q", "w1_q", "w2_q", "w3_q",
            "wq_s", "wk_s", "wv_s", "wo_s", "w1_s", "w2_s", "w3_s", "cls_q", "cls_s", "tok_f32")]

    class _S(C.Structure):
        _fields_ = [(n, C.c_void_p) for n in (
            "x", "xb", "hb", "hb2", "q", "att", "logits", "key_cache", "value_cache",
            "xq_q", "hq_q", "xq_s", "hq_s")]

    TAP_NAMES = [
        "embed", "att_rms_in", "att_rms_out", "att_xq_q", "att_xq_s", "q_pre", "k_pre", "q_post",
        "k_post", "scores", "probs", "att_out", "att_out_q", "att_out_s", "ffn_rms_in", "ffn_rms_out",
        "ffn_xq_q", "ffn_xq_s", "hb_pre", "hb2", "hb_post", "hq_q", "hq_s", "final_rms_in",
        "final_rms_out", "final_xq_q", "final_xq_s", "logits"]
    TAP_DTYPES = {n: (np.int8 if n.endswith("_q") else np.float32) for n in TAP_NAMES}
    TAP_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int64)

    def __init__(self, image: np.ndarray, ctx_length: int = 0, oracle: Oracle | None = None):
        self.o = oracle or Oracle()
        L = self.o.lib
        L.q3o_model_map.restype = C.c_int
        L.q3o_model_map.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int]
        L.q3o_state_alloc.restype = C.c_int
        L.q3o_state_alloc.argtypes = [C.c_void_p, C.c_void_p]
        L.q3o_forward.restype = C.POINTER(C.c_float)
        L.q3o_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, self.TAP_FN, C.c_void_p]
        L.q3o_model_free.argtypes = [C.c_void_p]
        L.q3o_state_free.argtypes = [C.c_void_p]
        self.image = np.ascontiguousarray(image, np.uint8)
        self.m = self._M()
        rc = L.q3o_model_map(C.byref(self.m), _p(self.image), self.image.size, ctx_length)
        if rc != 0:
            raise ValueError(f"q3o_model_map failed with {rc}")
        self.s = self._S()
        if L.q3o_state_alloc(C.byref(self.s), C.byref(self.m.c)) != 0:
            raise MemoryError("q3o_state_alloc")
        self.config = self.m.c

    def forward(self, token: int, pos: int, taps: dict | None = None) -> np.ndarray:
        cb = self.TAP_FN(0)
        if taps is not None:
            def _tap(_user, layer, tap, data, nbytes):
                name = self.TAP_NAMES[tap]
                dt = self.TAP_DTYPES[name]
                buf = C.string_at(data, nbytes)
                taps[(layer, name)] = np.frombuffer(buf, dtype=dt).copy()
            cb = self.TAP_FN(_tap)
        ptr = self.o.lib.q3o_forward(C.byref(self.m), C.byref(self.s), token, pos, cb, None)
        return np.ctypeslib.as_array(ptr, shape=(self.config.vocab_size,)).copy()

    def close(self):
        if getattr(self, "m", None) is not None:
            self.o.lib.q3o_state_free(C.byref(self.s))
            self.o.lib.q3o_model_free(C.byref(self.m))
            self.m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
