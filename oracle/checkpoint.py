"""Seeded synthetic qwen3.c v1 checkpoints -- TEST INFRASTRUCTURE ONLY.

No real Qwen3 weights are available offline, so the parity harnesses build
random-init checkpoints of a given shape in the reference's file format:

* header (scripts/export.py:108-131): uint32 magic 0x616A6331, int32 version 1,
  ten int32 fields (dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size,
  seq_len, head_dim, shared_classifier, group_size), zero-padded to 256 bytes;
* fp32 norm weights (export.py:135-146): rms_att[L][dim], rms_ffn[L][dim],
  rms_final[dim], q_norm[L][hd], k_norm[L][hd];
* Q8_0 tensors (export.py:150-160), each as int8 codes then fp32 scales, in the
  order tokens, wq*L, wk*L, wv*L, wo*L, w1*L, w2*L, w3*L (shared classifier);
  matrices are [out][in] row-major (qwen3_original.c:310-326).

Weights are N(0, 0.02) quantized with the exporter's rule (export.py:47-72:
scale = absmax/127, code = round-half-to-even(w/scale)); norm weights are
1 + N(0, 0.1).  The byte stream is a pure function of (shape, seed).
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np

GS = 64
MAGIC = 0x616A6331


def quantize_q80_export(w: np.ndarray):
    """export.py:47-72 in numpy (float32 throughout, round half to even)."""
    w = np.ascontiguousarray(w, np.float32).reshape(-1, GS)
    wmax = np.abs(w).max(axis=1)
    scale = (wmax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        quant = w / scale[:, None]
    q = np.nan_to_num(np.round(quant), nan=0.0).astype(np.int8)
    return q.reshape(-1), scale


def _chunks(dim, hidden, n_layers, n_heads, n_kv, vocab, seq_len, head_dim, seed):
    rng = np.random.default_rng(seed)
    yield struct.pack("I", MAGIC) + struct.pack("i", 1) + struct.pack(
        "iiiiiiiiii", dim, hidden, n_layers, n_heads, n_kv, vocab, seq_len, head_dim, 1, GS)
    yield b"\0" * (256 - 48)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32).tobytes()

    for _ in range(n_layers):
        yield norm(dim)
    for _ in range(n_layers):
        yield norm(dim)
    yield norm(dim)
    for _ in range(n_layers):
        yield norm(head_dim)
    for _ in range(n_layers):
        yield norm(head_dim)

    def q8(rows, cols):
        # generate in row blocks to bound memory for large shapes
        step = max(1, (1 << 24) // cols)
        qs, ss = [], []
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            w = 0.02 * rng.standard_normal((r1 - r0) * cols, dtype=np.float32)
            q, s = quantize_q80_export(w)
            qs.append(q.tobytes())
            ss.append(s.tobytes())
        return b"".join(qs) + b"".join(ss)

    ahd, kvd = n_heads * head_dim, n_kv * head_dim
    yield q8(vocab, dim)
    for shape in ([(ahd, dim)] * n_layers + [(kvd, dim)] * n_layers + [(kvd, dim)] * n_layers +
                  [(dim, ahd)] * n_layers + [(hidden, dim)] * n_layers + [(dim, hidden)] * n_layers +
                  [(hidden, dim)] * n_layers):
        yield q8(*shape)


def checkpoint_image(dim, hidden, n_layers, n_heads, n_kv, vocab, seq_len, head_dim, seed=0) -> np.ndarray:
    data = b"".join(_chunks(dim, hidden, n_layers, n_heads, n_kv, vocab, seq_len, head_dim, seed))
    return np.frombuffer(data, dtype=np.uint8).copy()


def write_checkpoint(path, dim, hidden, n_layers, n_heads, n_kv, vocab, seq_len, head_dim, seed=0) -> str:
    """Streams the checkpoint to `path`; returns the sha256 of the bytes written."""
    h = hashlib.sha256()
    with open(path, "wb") as f:
        for c in _chunks(dim, hidden, n_layers, n_heads, n_kv, vocab, seq_len, head_dim, seed):
            f.write(c)
            h.update(c)
    return h.hexdigest()
