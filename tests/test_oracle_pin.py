"""Pins the CPU oracle (oracle/q3_oracle.c) to the reference.

* against the reference CPU engine itself, compiled unmodified from
  src/cpu/qwen3_original.c (oracle/_ref; skipped where it was not built):
  exported primitives bit for bit, and whole decode steps -- logits and the
  RunState buffers the reference leaves behind (k cache of every layer, last
  layer's rotated q, softmax probabilities, SwiGLU output, final Q8_0 codes);
* against the golden fixtures in tests/golden/, generated from that compiled
  reference by tests/golden/make_golden.py (these run everywhere).
"""
import os
import tempfile

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def u32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---------------------------------------------------------------- vs compiled reference
@pytest.mark.parametrize("n", [64, 128, 1024, 2560, 9728])
def test_primitives_vs_reference(oracle, reference, n):
    rng = np.random.default_rng(n)
    x = (3 * rng.standard_normal(n)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    assert np.array_equal(u32(oracle.rmsnorm(x, w)), u32(reference.rmsnorm(x, w)))
    assert np.array_equal(u32(oracle.softmax(x)), u32(reference.softmax(x)))
    qa, sa = oracle.quantize(x)
    qb, sb = reference.quantize(x)
    assert np.array_equal(qa, qb) and np.array_equal(u32(sa), u32(sb))
    assert np.array_equal(u32(oracle.dequantize(qa, sa)), u32(reference.dequantize(qa, sa)))


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


def test_quantize_edge_cases_vs_reference(oracle, reference):
    x = edge_vector()
    qa, sa = oracle.quantize(x)
    qb, sb = reference.quantize(x)
    assert np.array_equal(qa, qb) and np.array_equal(u32(sa), u32(sb))
    assert qb[128] == -66 and qb[130] == 66          # 190 wraps to -66 (low byte)
    assert (qb[192:256] == 0).all()                   # scale underflowed to 0 -> x/0 -> 0


def same_bits(a, b):
    """Bit-identical, except that any two NaNs compare equal (payloads differ between builds)."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return a.shape == b.shape and np.array_equal(na, nb) and np.array_equal(u32(a[~na]), u32(b[~nb]))


def matmul_case(rng, B, n, d, extremes=False):
    xq = rng.integers(-127, 128, (B, n), dtype=np.int8)
    xs = np.abs(0.05 * rng.standard_normal((B, n // 64))).astype(np.float32)
    wq = rng.integers(-127, 128, (d, n), dtype=np.int8)
    ws = np.abs(0.01 * rng.standard_normal((d, n // 64))).astype(np.float32)
    if extremes:
        xq[:, :64], wq[0, :64], wq[1, :64] = -128, -128, 127
        ws[2, :] = 0.0
        ws[3, 0], xs[:, 0] = 3e38, 3e38                 # inf
        ws[4, 1], xs[:, 1] = np.inf, 0.0                # inf * 0 = NaN
    return xq, xs, wq, ws


@pytest.mark.parametrize("B,n,d,ext", [(1, 64, 7, False), (2, 1024, 300, False), (1, 3072, 64, False),
                                       (3, 576, 40, True)])
def test_matmul_vs_reference(oracle, reference, B, n, d, ext):
    xq, xs, wq, ws = matmul_case(np.random.default_rng(n + d), B, n, d, ext)
    with np.errstate(all="ignore"):
        assert same_bits(oracle.matmul(xq, xs, wq, ws), reference.matmul(xq, xs, wq, ws))


def test_softmax_edges_vs_reference(oracle, reference):
    for x in (np.full(40, -3.0, np.float32), np.full(40, -200.0, np.float32), np.array([0.0], np.float32),
              np.array([np.nan, 1.0, 2.0], np.float32), np.array([88.0, 89.0, -1e30], np.float32)):
        a, b = oracle.softmax(x), reference.softmax(x)
        assert np.array_equal(u32(a), u32(b))


@pytest.mark.parametrize("shape", [
    dict(dim=128, hidden=384, n_layers=2, n_heads=4, n_kv=2, vocab=512, seq_len=64, head_dim=64),
    dict(dim=256, hidden=768, n_layers=3, n_heads=4, n_kv=2, vocab=300, seq_len=16, head_dim=128),
])
def test_forward_vs_reference(oracle, reference, shape):
    from oracle.checkpoint import checkpoint_image, write_checkpoint
    from oracle.oracle import OracleModel
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        write_checkpoint(path, seed=7, **shape)
        img = np.fromfile(path, np.uint8)
        assert np.array_equal(img, checkpoint_image(seed=7, **shape))
        t = reference.create(path, 0)
        om = OracleModel(img, oracle=oracle)
        L = shape["n_layers"]
        try:
            for pos, tok in enumerate([3, 77, 1, shape["vocab"] - 1, 42, 5, 9, 11]):
                la = reference.forward(t, tok, pos)
                taps = {}
                lb = om.forward(tok, pos, taps)
                st = reference.state(t, pos)
                assert np.array_equal(u32(la), u32(lb)), f"logits differ at pos {pos}"
                assert np.array_equal(u32(st["q"]), u32(taps[(L - 1, "q_post")]))
                assert np.array_equal(u32(st["hb"]), u32(taps[(L - 1, "hb_post")]))
                assert np.array_equal(u32(st["hb2"]), u32(taps[(L - 1, "hb2")]))
                assert np.array_equal(u32(st["att"].reshape(-1)), u32(taps[(L - 1, "probs")]))
                assert np.array_equal(st["hq_q"], taps[(L - 1, "hq_q")])
                assert np.array_equal(u32(st["hq_s"]), u32(taps[(L - 1, "hq_s")]))
                assert np.array_equal(st["xq_q"][: shape["dim"]], taps[(L, "final_xq_q")])
                assert np.array_equal(u32(st["x"]), u32(taps[(L, "final_rms_out")]))
                for layer in range(L):
                    assert np.array_equal(u32(st["key_cache"][layer, pos]), u32(taps[(layer, "k_post")]))
                # the attention loop alone (q3o_attention, executeAttention's arguments) on the
                # reference's own last-layer q and caches: its probabilities and head outputs
                xb, att = oracle.attention(st["q"], st["key_cache"][L - 1], st["value_cache"][L - 1], pos,
                                           shape["n_heads"], shape["n_kv"], shape["seq_len"])
                assert np.array_equal(u32(att[:, :pos + 1]), u32(st["att"]))
                assert np.array_equal(u32(xb), u32(taps[(L - 1, "att_out")]))
        finally:
            reference.free(t)
            om.close()


# ---------------------------------------------------------------- vs golden fixtures
def load_golden(name):
    p = os.path.join(GOLDEN, name)
    if not os.path.exists(p):
        pytest.fail(f"golden fixture {p} missing (run tests/golden/make_golden.py)")
    return np.load(p)


def test_golden_primitives(oracle):
    g = load_golden("primitives.npz")
    for i in range(int(g["count"])):
        x, w = g[f"x{i}"], g[f"w{i}"]
        assert np.array_equal(u32(oracle.rmsnorm(x, w)), u32(g[f"rmsnorm{i}"]))
        assert np.array_equal(u32(oracle.softmax(x)), u32(g[f"softmax{i}"]))
        q, s = oracle.quantize(x)
        assert np.array_equal(q, g[f"q{i}"]) and np.array_equal(u32(s), u32(g[f"s{i}"]))
        assert np.array_equal(u32(oracle.dequantize(q, s)), u32(g[f"deq{i}"]))


def test_golden_matmul(oracle):
    g = load_golden("matmul.npz")
    for i in range(int(g["count"])):
        with np.errstate(all="ignore"):
            o = oracle.matmul(g[f"xq{i}"], g[f"xs{i}"], g[f"wq{i}"], g[f"ws{i}"])[0]
        assert same_bits(o, g[f"out{i}"]), f"case {i}"


def test_golden_forward(oracle):
    from oracle.checkpoint import checkpoint_image
    from oracle.oracle import OracleModel
    g = load_golden("forward_tiny.npz")
    shape = {k: int(g[f"shape_{k}"]) for k in ("dim", "hidden", "n_layers", "n_heads", "n_kv", "vocab",
                                               "seq_len", "head_dim")}
    img = checkpoint_image(seed=int(g["seed"]), **shape)
    import hashlib
    assert hashlib.sha256(img.tobytes()).hexdigest() == str(g["sha256"])
    om = OracleModel(img, oracle=oracle)
    L = shape["n_layers"]
    toks = g["tokens"]
    for pos, tok in enumerate(toks):
        taps = {}
        logits = om.forward(int(tok), pos, taps)
        assert np.array_equal(u32(logits), u32(g[f"logits{pos}"]))
        assert np.array_equal(u32(taps[(L - 1, "q_post")]), u32(g[f"q{pos}"]))
        assert np.array_equal(u32(taps[(L - 1, "hb_post")]), u32(g[f"hb{pos}"]))
        assert np.array_equal(u32(taps[(L - 1, "probs")]), u32(g[f"att{pos}"]))
        for layer in range(L):
            assert np.array_equal(u32(taps[(layer, "k_post")]), u32(g[f"k{pos}_{layer}"]))
    om.close()
