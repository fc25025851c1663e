"""A whole decode step through the CUDA kernels, layer by layer, against the
oracle's taps (the parity half of the Qwen3-0.6B decode-step configuration).

The oracle runs qwen3.c's forward (src/cpu/qwen3_original.c:333-468; pinned
bit-exact to the compiled reference in test_oracle_pin.py) on a seeded
checkpoint and records every op's input and output per layer.  Each op's
tapped input is then fed to the matching kernel through the C ABI and the
result compared with the next tap:

  embedding row           tokens table -> `embed` tap            bit-exact
  attention RMSNorm+Q8_0  att_rms_in -> att_rms_out, att_xq_*    bit-exact
  QK-norm + RoPE          q_pre/k_pre -> q_post/k_post           1e-5 rel / 1e-6 abs
  softmax                 scores (n_heads rows of pos+1) -> probs 1e-5 rel / 1e-6 abs
  attention-out quantize  att_out -> att_out_q/_s                bit-exact
  FFN RMSNorm+Q8_0        ffn_rms_in -> ffn_rms_out, ffn_xq_*    bit-exact
  SwiGLU (+Q8_0)          hb_pre, hb2 -> hb_post, hq_*           bit-exact
  final RMSNorm+Q8_0      final_rms_in -> final_rms_out, *_xq_*  bit-exact

The Q8_0 matmuls between the ops are not on this path (the oracle's own).
"""
import numpy as np
import pytest

from test_gpu_parity import ATOL, RTOL, bits, dev, host

pytestmark = pytest.mark.gpu

GS = 64


def norms_and_table(img, dim, hidden, n_layers, n_heads, n_kv, vocab, seq_len, head_dim):
    """Norm weights and the Q8_0 token table from a checkpoint image (layout:
    oracle/checkpoint.py, the reference's export format)."""
    o = 256
    f32 = lambda n: img[o:o + 4 * n].view(np.float32)
    L, hd = n_layers, head_dim
    rms_att = f32(L * dim).reshape(L, dim); o += 4 * L * dim
    rms_ffn = f32(L * dim).reshape(L, dim); o += 4 * L * dim
    rms_final = f32(dim); o += 4 * dim
    q_norm = f32(L * hd).reshape(L, hd); o += 4 * L * hd
    k_norm = f32(L * hd).reshape(L, hd); o += 4 * L * hd
    tq = img[o:o + vocab * dim].view(np.int8).reshape(vocab, dim); o += vocab * dim
    ts = img[o:o + 4 * vocab * dim // GS].view(np.float32).reshape(vocab, dim // GS)
    return rms_att, rms_ffn, rms_final, q_norm, k_norm, tq, ts


def check_step(q3, taps, shape, w, token, pos):
    import torch
    rms_att, rms_ffn, rms_final, q_norm, k_norm, tq, ts = w
    L, nh, nkv, hd = shape["n_layers"], shape["n_heads"], shape["n_kv"], shape["head_dim"]
    t = lambda name, layer: taps[(layer, name)]

    # embedding row (dequantized on lookup)
    row = host(q3.embed_gather(dev(tq), dev(ts), dev(np.array([token], np.int32)), want_q8=False)[0])
    assert np.array_equal(bits(row[0]), bits(t("embed", -1))), "embedding row"

    def rms(x, wv, out_name, q_name, s_name, layer):
        x2 = dev(x.reshape(1, -1))
        g = host(q3.rmsnorm(x2, dev(wv)))[0]
        assert np.array_equal(bits(g), bits(t(out_name, layer))), f"{out_name} layer {layer}"
        qg, sg = q3.rmsnorm_q8(x2, dev(wv))
        assert np.array_equal(host(qg)[0], t(q_name, layer)), f"{q_name} layer {layer}"
        assert np.array_equal(bits(host(sg)[0]), bits(t(s_name, layer))), f"{s_name} layer {layer}"

    for l in range(L):
        rms(t("att_rms_in", l), rms_att[l], "att_rms_out", "att_xq_q", "att_xq_s", l)

        qd = dev(t("q_pre", l).reshape(1, nh, hd))
        kd = dev(t("k_pre", l).reshape(1, nkv, hd))
        q3.qk_norm_rope(qd, kd, dev(np.array([pos], np.int32)), dev(q_norm[l]), dev(k_norm[l]))
        np.testing.assert_allclose(host(qd).reshape(-1), t("q_post", l), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(host(kd).reshape(-1), t("k_post", l), rtol=RTOL, atol=ATOL)

        sc = t("scores", l).copy()
        n = pos + 1
        off = (np.arange(nh) * n).astype(np.int64)
        lens = np.full(nh, n, np.int32)
        sd = dev(sc)
        q3.softmax_rows(sd, dev(off), dev(lens))
        np.testing.assert_allclose(host(sd), t("probs", l), rtol=RTOL, atol=ATOL)

        qg, sg = q3.quantize_q8(dev(t("att_out", l).reshape(1, -1)))
        assert np.array_equal(host(qg)[0], t("att_out_q", l)), f"att_out_q layer {l}"
        assert np.array_equal(bits(host(sg)[0]), bits(t("att_out_s", l))), f"att_out_s layer {l}"

        rms(t("ffn_rms_in", l), rms_ffn[l], "ffn_rms_out", "ffn_xq_q", "ffn_xq_s", l)

        hb, hb2 = dev(t("hb_pre", l).reshape(1, -1)), dev(t("hb2", l).reshape(1, -1))
        qg, sg = q3.swiglu_q8(hb, hb2)
        assert np.array_equal(host(qg)[0], t("hq_q", l)), f"hq_q layer {l}"
        assert np.array_equal(bits(host(sg)[0]), bits(t("hq_s", l))), f"hq_s layer {l}"
        q3.swiglu(hb, hb2)
        assert np.array_equal(bits(host(hb)[0]), bits(t("hb_post", l))), f"hb_post layer {l}"

    rms(t("final_rms_in", L), rms_final, "final_rms_out", "final_xq_q", "final_xq_s", L)
    torch.cuda.synchronize()
    assert q3.device_status() == 0


SHAPES = {
    # head_dim 128 (the kernels' only head size); several positions so the
    # softmax rows grow and the KV cache fills
    "tiny": (dict(dim=256, hidden=768, n_layers=3, n_heads=4, n_kv=2, vocab=300, seq_len=16, head_dim=128),
             [(3, 0), (77, 1), (1, 2), (299, 3), (42, 4), (5, 5)]),
    # the Qwen3-0.6B layer shape (dim 1024, hidden 3072, 16 + 8 heads, vocab
    # 151936), 2 of its 28 layers, one token at position 37 with a zero KV cache
    "qwen3_0.6b_2layers": (dict(dim=1024, hidden=3072, n_layers=2, n_heads=16, n_kv=8, vocab=151936, seq_len=64,
                                head_dim=128), [(12345, 37)]),
}


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_decode_step_through_the_kernels(q3, oracle, name):
    from oracle.checkpoint import checkpoint_image
    from oracle.oracle import OracleModel
    shape, steps = SHAPES[name]
    img = checkpoint_image(seed=11, **shape)
    w = norms_and_table(img, **shape)
    om = OracleModel(img, oracle=oracle)
    try:
        for token, pos in steps:
            taps = {}
            om.forward(token, pos, taps)
            check_step(q3, taps, shape, w, token, pos)
    finally:
        om.close()
