"""Generates the golden fixtures in this folder from the reference itself.

The reference CPU engine (src/cpu/qwen3_original.c) is compiled unmodified by
`make -C oracle ref` into oracle/_ref/libqwen3_ref.so; this script calls its
exported functions (rmsnorm, softmax, quantize, dequantize, and the whole
decode step through qwen3_transformer_create / qwen3_forward) on seeded inputs
and stores inputs and outputs:

  primitives.npz    vectors of length 64..10240 (incl. the Q8_0 edge cases:
                    denormal groups, wrapped codes, inf/NaN, -0, exact .5
                    quotients) -> rmsnorm / softmax / quantize / dequantize
  matmul.npz        Q8_0 x Q8_0 matrix-vector products (`matmul`) on seeded
                    codes/scales, incl. extreme codes (-128, +-127), zero and
                    huge scales (inf outputs) and n = 64..1024
  forward_tiny.npz  a seeded 2-layer checkpoint (oracle/checkpoint.py, sha256
                    recorded) run for 8 positions: logits, and the RunState the
                    reference leaves behind (rotated q, SwiGLU output, softmax
                    probabilities, k cache of every layer)

Run from the repository root:  python tests/golden/make_golden.py
"""
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.checkpoint import write_checkpoint  # noqa: E402
from oracle.oracle import Reference, build_reference  # noqa: E402

TINY = dict(dim=128, hidden=384, n_layers=2, n_heads=4, n_kv=2, vocab=512, seq_len=64, head_dim=64)


def edge_vector():
    md = np.float32(1.4e-45)
    x = np.zeros(64 * 10, np.float32)
    x[64:128] = np.arange(64, dtype=np.float32) * md
    x[128:192] = 190 * md
    x[130] = -190 * md
    x[192:256] = 63 * md
    x[256] = np.inf
    x[320] = np.nan
    x[384] = -np.inf
    x[385] = 1.0
    x[448:512] = -0.0
    x[512:576] = np.linspace(-127.0, 127.0, 64, dtype=np.float32)
    x[576:640] = np.arange(64, dtype=np.float32) + 0.5
    return x


def main():
    if build_reference() is None:
        sys.exit("the reference sources are not available; cannot regenerate the fixtures")
    ref = Reference()
    rng = np.random.default_rng(20240601)
    out = {}
    vecs = []
    for n in (64, 128, 2560, 4096, 10240):
        vecs.append(rng.uniform(-1, 1, n).astype(np.float32))            # the reference's own test rule
        vecs.append((3 * rng.standard_normal(n)).astype(np.float32))
    vecs.append(edge_vector())
    for i, x in enumerate(vecs):
        w = (1 + 0.1 * rng.standard_normal(x.size)).astype(np.float32)
        out[f"x{i}"], out[f"w{i}"] = x, w
        with np.errstate(all="ignore"):
            out[f"rmsnorm{i}"] = ref.rmsnorm(x, w)
            out[f"softmax{i}"] = ref.softmax(x)
            q, s = ref.quantize(x)
            out[f"q{i}"], out[f"s{i}"] = q, s
            out[f"deq{i}"] = ref.dequantize(q, s)
    out["count"] = np.array(len(vecs))
    np.savez_compressed(os.path.join(HERE, "primitives.npz"), **out)

    mm = {}
    cases = [(64, 5), (128, 64), (1024, 96), (576, 33)]
    for i, (n, d) in enumerate(cases):
        xq = rng.integers(-127, 128, n, dtype=np.int8)
        xs = np.abs(0.05 * rng.standard_normal(n // 64)).astype(np.float32)
        wq = rng.integers(-127, 128, (d, n), dtype=np.int8)
        ws = np.abs(0.01 * rng.standard_normal((d, n // 64))).astype(np.float32)
        if i == 3:                                           # extremes
            xq[:64], wq[0, :64], wq[1, :64] = -128, -128, 127
            ws[2, :] = 0.0
            ws[3, 0], xs[0] = 3e38, 3e38                     # overflows to inf
        mm[f"xq{i}"], mm[f"xs{i}"], mm[f"wq{i}"], mm[f"ws{i}"] = xq, xs, wq, ws
        with np.errstate(all="ignore"):
            mm[f"out{i}"] = ref.matmul(xq, xs, wq, ws)[0]
    mm["count"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "matmul.npz"), **mm)

    fw = {}
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "tiny.bin")
        sha = write_checkpoint(path, seed=3, **TINY)
        t = ref.create(path, 0)
        toks = np.array([5, 77, 300, 1, 42, 511, 0, 256], np.int32)
        for pos, tok in enumerate(toks):
            fw[f"logits{pos}"] = ref.forward(t, int(tok), pos)
            st = ref.state(t, pos)
            fw[f"q{pos}"], fw[f"hb{pos}"] = st["q"], st["hb"]
            fw[f"att{pos}"] = st["att"].reshape(-1)
            for layer in range(TINY["n_layers"]):
                fw[f"k{pos}_{layer}"] = st["key_cache"][layer, pos]
        ref.free(t)
    fw["tokens"], fw["seed"], fw["sha256"] = toks, np.array(3), np.array(sha)
    for k, v in TINY.items():
        fw[f"shape_{k}"] = np.array(v)
    np.savez_compressed(os.path.join(HERE, "forward_tiny.npz"), **fw)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
