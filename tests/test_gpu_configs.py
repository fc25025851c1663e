"""Parity at the exact shapes, seeds and sizes of the path's five workload
configurations (the kernel tests in test_gpu_parity.py cover edge cases at
small sizes; these pin the configurations themselves):

  1  Qwen3-0.6B decode step: 28 layers, seed-0 checkpoint (weights N(0, 0.02)
     through the exporter's Q8_0 rule, norm weights 1 + N(0, 0.1)), one
     uniform token (seed 0) at position 37 with a zero KV cache.  Every layer's
     op taps go through the kernels (test_gpu_decode_step.check_step), and the
     device decode step's logits are compared with the compiled reference's
     qwen3_forward (src/cpu/qwen3_original.c:333-468), bit for bit.
  3  Qwen3-8B batched decode: the ragged softmax over all 256 x 32 score rows of
     length pos + 1 (pos uniform in 0..32767, seed 0), at full size; bf16
     RMSNorm+Q8_0 (4096), QK-norm + RoPE (32 + 8 heads) and SwiGLU (12288).
  4  Q8_0 embedding gather at full scale: a 151936 x 4096 table, 1,048,576
     Zipf(1.1) ids, f32 rows and the re-quantized Q8_0 rows (17.2 GB + 4.6 GB of
     output, offsets past 2^31 elements), every row bit-exact against the
     oracle (qwen3_original.c:142-145 then :147-168).
  5  Qwen3-14B prefill layer, bf16 with 1% outlier channels: RMSNorm+Q8_0
     (5120), QK-norm + RoPE (40 + 8 heads, positions 0..4095), SwiGLU+Q8_0 and
     float SwiGLU (17408).

Tolerances: Q8_0 codes/scales, the embedding rows, RMSNorm and SwiGLU floats
bit-exact; RoPE and softmax 1e-5 relative / 1e-6 absolute in f32.  bf16 RoPE
outputs: 1e-2 relative, plus the f32 absolute floor of 1e-6 -- the arithmetic
is binary32 and only the inputs and outputs are bf16, so an output that
cancels to ~1e-6 carries the f32 path's absolute error, which no relative
bound covers.
"""
import os
import tempfile

import numpy as np
import pytest

from test_gpu_parity import ATOL, BF16_RTOL, RTOL, activations, assert_q8_equal, bf16_to_f32, bits, dev, host, \
    to_bf16

pytestmark = pytest.mark.gpu

GS = 64
BF16_ATOL = 1e-6


# --------------------------------------------------------------------------- config 1
QWEN3_06B = dict(dim=1024, hidden=3072, n_layers=28, n_heads=16, n_kv=8, vocab=151936, seq_len=64, head_dim=128)


def test_config1_decode_step_28_layers(q3, oracle):
    from metalqwen3_b200.q3cu import Q3Model
    from oracle.checkpoint import write_checkpoint
    from oracle.oracle import OracleModel
    from test_gpu_decode_step import check_step, norms_and_table
    from test_gpu_forward import expected_logits, same_bits

    shape = QWEN3_06B
    token = int(np.random.default_rng(0).integers(0, shape["vocab"]))
    pos = 37
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "qwen3_06b_seed0.bin")
        write_checkpoint(path, seed=0, **shape)
        img = np.fromfile(path, np.uint8)
        want = expected_logits(path, img, shape, [(token, pos)])[0]      # the compiled reference
    # every layer's ops through the kernels, against the oracle's taps
    taps = {}
    om = OracleModel(img, oracle=oracle)
    try:
        logits_o = om.forward(token, pos, taps)
    finally:
        om.close()
    assert same_bits(logits_o, want), "the oracle's forward differs from the reference's"
    check_step(q3, taps, shape, norms_and_table(img, **shape), token, pos)
    # the device decode step (zero KV cache, as the reference's calloc'd one)
    model = Q3Model(q3, img)
    try:
        got = model.forward(token, pos)
    finally:
        model.close()
    assert same_bits(got, want), f"logits differ (max |diff| {np.nanmax(np.abs(got - want))})"


# --------------------------------------------------------------------------- config 3
def test_config3_softmax_full_size(q3, oracle):
    """All 8192 score rows of the batched-decode step (139.9 M scores), rows of
    length pos + 1 back to back, f32 scores N(0, sigma = 2)."""
    import torch
    from test_gpu_parity import softmax_f64
    pos = np.random.default_rng(0).integers(0, 32768, size=256).astype(np.int32)
    lens = np.repeat(pos.astype(np.int64) + 1, 32)
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    x = (2.0 * np.random.default_rng(3).standard_normal(int(lens.sum()), dtype=np.float32)).astype(np.float32)
    t = dev(x)
    q3.softmax_rows(t, dev(off), dev(lens.astype(np.int32)))
    g = host(t)
    del t
    o = oracle.rows_softmax(x, off, lens.astype(np.int32), threads=os.cpu_count() or 1)
    r = softmax_f64(x, off, lens)
    tol = ATOL + RTOL * np.abs(r)
    assert not np.isnan(g).any()
    assert (np.abs(g - r) <= tol).all(), "outside tolerance of the binary64 softmax"
    assert (np.abs(g - o) <= np.abs(o - r) + tol).all(), "further from the oracle than allowed"
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dim,hidden,nh,posmax", [(4096, 12288, 32, 32768), (5120, 17408, 40, 4096)])
def test_bf16_layer_shapes(q3, oracle, dim, hidden, nh, posmax):
    """Configs 3 (dim 4096, hidden 12288, 32 + 8 heads) and 5 (dim 5120, hidden
    17408, 40 + 8 heads, 1% outlier channels) on bf16 rows.  RMSNorm, SwiGLU
    and their Q8_0 codes are bit-exact; RoPE is held to 1e-2 relative plus
    BF16_ATOL = 1e-6 absolute: the device's sincosf is within a few ulps of the
    host's cosf/sinf, and a rotated pair that cancels to near zero (|o| below
    1e-4 on these unit-variance rows) has no meaningful relative error, so the
    absolute term, 1e-6 of the data's scale, bounds those outputs instead."""
    rng = np.random.default_rng(dim)
    rows = 96
    outl = 0.01 if dim == 5120 else 0.0
    act = (lambda r, c: activations(rng, r, c)) if outl else (lambda r, c: rng.standard_normal((r, c), np.float32))
    # RMSNorm + Q8_0, and the float RMSNorm
    x = to_bf16(act(rows, dim), oracle)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    qg, sg = q3.rmsnorm_q8(dev(x), dev(w))
    qo, so = oracle.rows_rmsnorm_q8(x, w, threads=8)
    assert_q8_equal(qg, sg, qo, so)
    assert np.array_equal(host(q3.rmsnorm(dev(x), dev(w))), oracle.rows_rmsnorm(x, w, threads=8))
    # SwiGLU + Q8_0, and the float SwiGLU (bf16 out: the exact binary32 value rounded once)
    hb = to_bf16(act(rows, hidden), oracle)
    hb2 = to_bf16(act(rows, hidden), oracle)
    qg, sg = q3.swiglu_q8(dev(hb), dev(hb2))
    qo, so = oracle.rows_swiglu_q8(hb, hb2, threads=8)
    assert_q8_equal(qg, sg, qo, so)
    t = dev(hb)
    q3.swiglu(t, dev(hb2))
    assert np.array_equal(host(t), oracle.rows_swiglu(hb, hb2, threads=8)), "bf16 SwiGLU"
    # QK-norm + RoPE over the configuration's heads and positions
    qh = to_bf16(rng.standard_normal((rows, nh, 128), dtype=np.float32), oracle)
    kh = to_bf16(rng.standard_normal((rows, 8, 128), dtype=np.float32), oracle)
    pos = rng.integers(0, posmax, rows).astype(np.int32)
    pos[0], pos[-1] = 0, posmax - 1
    qn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    tq, tk = dev(qh), dev(kh)
    q3.qk_norm_rope(tq, tk, dev(pos), dev(qn), dev(kn))
    qo, ko = oracle.rows_qk_norm_rope(qh, kh, pos, qn, kn, threads=8)
    np.testing.assert_allclose(bf16_to_f32(host(tq)), bf16_to_f32(qo), rtol=BF16_RTOL, atol=BF16_ATOL)
    np.testing.assert_allclose(bf16_to_f32(host(tk)), bf16_to_f32(ko), rtol=BF16_RTOL, atol=BF16_ATOL)


# --------------------------------------------------------------------------- config 4
def test_config4_embed_full_scale(q3, oracle):
    """The whole embedding workload, with the table and ids the benchmark uses
    (its generator, seed 0): every output row equals the oracle's row for its
    id.  The oracle runs once per distinct id; rows are compared on the device,
    4 GiB of output at a time, through an index into those expected rows."""
    import torch
    from bench import Embed
    wl = Embed()
    d = wl.make(torch, torch.device("cuda", 0), seed=1234)
    tq, ts, ids = d["tq"], d["ts"], d["ids"]
    q3.embed_gather(tq, ts, ids, out=d["out"], oq=d["oq"], os_=d["os"])
    torch.cuda.synchronize()
    assert q3.device_status() == 0
    assert d["out"].numel() > 2 ** 31                        # element offsets past int32
    uniq, inv = np.unique(wl.ids, return_inverse=True)
    ro, rq, rs, bad = oracle.rows_embed(host(tq), host(ts), uniq.astype(np.int32), threads=os.cpu_count() or 1)
    assert bad == 0
    e_f, e_q, e_s = dev(ro.view(np.int32)), dev(rq), dev(rs.view(np.int32))
    del ro, rq, rs
    inv_d = torch.from_numpy(inv.astype(np.int64)).cuda()
    out_i, os_i = d["out"].view(torch.int32), d["os"].view(torch.int32)
    step = (4 << 30) // (wl.dim * 4)
    for a in range(0, wl.tokens, step):
        b = min(wl.tokens, a + step)
        sel = inv_d[a:b]
        assert torch.equal(out_i[a:b], e_f.index_select(0, sel)), f"f32 rows {a}..{b}"
        assert torch.equal(d["oq"][a:b], e_q.index_select(0, sel)), f"Q8_0 codes {a}..{b}"
        assert torch.equal(os_i[a:b], e_s.index_select(0, sel)), f"Q8_0 scales {a}..{b}"
    del d, e_f, e_q, e_s, out_i, os_i
    torch.cuda.empty_cache()
