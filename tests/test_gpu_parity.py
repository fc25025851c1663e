"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle.

Contract (from the reference, src/cpu/qwen3_original.c):
  * Q8_0 codes / scales and the embedding dequant: bit-exact;
  * RMSNorm (incl. the per-head QK-norm) and SwiGLU float outputs: bit-exact
    for f32 (sequential sum of squares, libm-identical expf);
  * RoPE and softmax: within RTOL = 1e-5, ATOL = 1e-6 (f32), 1e-2 relative for
    bf16 inputs; softmax is also held to "no further from the oracle than the
    oracle is from a binary64 softmax, plus the tolerance".
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6
BF16_RTOL = 1e-2


def dev(a):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    if a.dtype == np.uint16:
        t = t.view(torch.bfloat16)
    return t.cuda()


def host(t):
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint8)


def to_bf16(a, oracle):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_to_f32(u):
    return (u.astype(np.uint32) << 16).view(np.float32)


def activations(rng, rows, dim, outlier_frac=0.01, scale=20.0):
    """N(0,1) with a fixed 1% channel set scaled x20 (the prefill workloads' rule)."""
    x = rng.standard_normal((rows, dim), dtype=np.float32)
    k = max(1, int(round(dim * outlier_frac)))
    ch = np.random.default_rng(1234).choice(dim, size=k, replace=False)
    x[:, ch] *= np.float32(scale)
    return x


def assert_q8_equal(qg, sg, qo, so):
    qg, sg = host(qg), host(sg)
    assert qg.shape == qo.shape and sg.shape == so.shape
    nq = int((qg != qo).sum())
    ns = int((sg.view(np.uint32) != so.view(np.uint32)).sum())
    assert nq == 0 and ns == 0, f"{nq} code and {ns} scale mismatches"


# --------------------------------------------------------------------------- quantize
@pytest.mark.parametrize("rows,n", [(1, 64), (3, 128), (7, 2560), (33, 9728), (4096, 2560)])
def test_quantize_f32(q3, oracle, rows, n):
    rng = np.random.default_rng(rows * 7 + n)
    x = activations(rng, rows, n)
    qg, sg = q3.quantize_q8(dev(x))
    qo, so = oracle.rows_quantize(x, threads=8)
    assert_q8_equal(qg, sg, qo, so)


def test_quantize_edge_groups(q3, oracle):
    md = np.float32(1.4e-45)
    x = np.zeros((1, 64 * 12), np.float32)
    x[0, 64:128] = np.arange(64, dtype=np.float32) * md          # denormal group
    x[0, 128:192] = 190 * md; x[0, 130] = -190 * md                 # codes wrap past 127
    x[0, 192:256] = 63 * md                                        # scale underflows to 0
    x[0, 256] = np.inf; x[0, 320] = np.nan; x[0, 384] = -np.inf; x[0, 385] = 1.0
    x[0, 448:512] = -0.0
    x[0, 512:576] = np.linspace(-127.0, 127.0, 64, dtype=np.float32)   # exact .5 quotients
    x[0, 576:640] = (np.arange(64, dtype=np.float32) + 0.5)
    x[0, 640:704] = np.float32(3.4e38) * np.sign(np.arange(64) - 31.5).astype(np.float32)
    qg, sg = q3.quantize_q8(dev(x))
    qo, so = oracle.rows_quantize(x)
    assert_q8_equal(qg, sg, qo, so)


@pytest.mark.parametrize("rows,n", [(5, 256), (256, 4096)])
def test_quantize_bf16(q3, oracle, rows, n):
    rng = np.random.default_rng(5)
    xb = to_bf16(activations(rng, rows, n), oracle)
    qg, sg = q3.quantize_q8(dev(xb))
    qo, so = oracle.rows_quantize(xb)
    assert_q8_equal(qg, sg, qo, so)


def test_dequantize(q3, oracle):
    rng = np.random.default_rng(3)
    q = rng.integers(-127, 128, size=64 * 1000, dtype=np.int8)
    s = np.abs(0.01 * rng.standard_normal(1000)).astype(np.float32)
    g = host(q3.dequantize_q8(dev(q), dev(s)))
    assert np.array_equal(bits(g), bits(oracle.dequantize(q, s)))


# --------------------------------------------------------------------------- rmsnorm
@pytest.mark.parametrize("rows,dim", [(1, 64), (3, 128), (7, 1024), (300, 2560), (5, 4096), (9, 5120), (2, 1028)])
def test_rmsnorm_f32_bitexact(q3, oracle, rows, dim):
    rng = np.random.default_rng(rows + dim)
    x = activations(rng, rows, dim)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    g = host(q3.rmsnorm(dev(x), dev(w)))
    o = oracle.rows_rmsnorm(x, w, threads=8)
    assert np.array_equal(bits(g), bits(o)), f"max abs diff {np.abs(g - o).max()}"


def test_rmsnorm_in_place(q3, oracle):
    rng = np.random.default_rng(11)
    x = activations(rng, 17, 2560)
    w = (1 + 0.1 * rng.standard_normal(2560)).astype(np.float32)
    t = dev(x)
    q3.rmsnorm(t, dev(w), out=t)
    assert np.array_equal(bits(host(t)), bits(oracle.rows_rmsnorm(x, w)))


@pytest.mark.parametrize("rows,dim", [(1, 1024), (37, 2560), (4096, 2560)])
def test_rmsnorm_q8_f32(q3, oracle, rows, dim):
    rng = np.random.default_rng(rows)
    x = activations(rng, rows, dim)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    qg, sg = q3.rmsnorm_q8(dev(x), dev(w))
    qo, so = oracle.rows_rmsnorm_q8(x, w, threads=8)
    assert_q8_equal(qg, sg, qo, so)


@pytest.mark.parametrize("rows,dim,bf16", [
    (8192, 2560, False),      # persistent ring kernel: 2 blocks of 28 rows per SM (f32 below 65 rows per SM)
    (12000, 2560, False),     # TMA-fed, f32: 82 rows per SM, blocks of 41 rows, two chain warps
    (20011, 1024, False),     # TMA-fed: 2-3 blocks per SM (double-buffered row scales), a 1-row last block
    (1000, 2560, False),      # persistent ring kernel: 7 rows per SM
    (5000, 4096, True),       # TMA-fed, bf16, blocks of 34 rows
    (16384, 5120, True),      # TMA-fed, the Qwen3-14B prefill rows: 2 blocks of 56 per SM
])
def test_rmsnorm_many_rows(q3, oracle, rows, dim, bf16):
    """The prefill kernels (more rows than 4 per SM): codes, scales and floats
    bit for bit, also in place."""
    rng = np.random.default_rng(rows + dim)
    x = activations(rng, rows, dim)
    if bf16:
        x = to_bf16(x, oracle)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    qg, sg = q3.rmsnorm_q8(dev(x), dev(w))
    qo, so = oracle.rows_rmsnorm_q8(x, w, threads=8)
    assert_q8_equal(qg, sg, qo, so)
    o = oracle.rows_rmsnorm(x, w, threads=8)
    t = dev(x)
    assert np.array_equal(host(q3.rmsnorm(t, dev(w))), o)
    q3.rmsnorm(t, dev(w), out=t)                                     # in place
    assert np.array_equal(host(t), o)
    assert q3.device_status() == 0


@pytest.mark.parametrize("rows,dim", [(3, 512), (256, 4096), (2048, 5120)])
def test_rmsnorm_bf16(q3, oracle, rows, dim):
    rng = np.random.default_rng(dim)
    xb = to_bf16(activations(rng, rows, dim), oracle)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    qg, sg = q3.rmsnorm_q8(dev(xb), dev(w))
    qo, so = oracle.rows_rmsnorm_q8(xb, w, threads=8)
    assert_q8_equal(qg, sg, qo, so)
    g = host(q3.rmsnorm(dev(xb), dev(w)))
    o = oracle.rows_rmsnorm(xb, w, threads=8)
    np.testing.assert_allclose(bf16_to_f32(g), bf16_to_f32(o), rtol=BF16_RTOL)
    assert np.array_equal(g, o)      # the float result is exact, so is its bf16 rounding


@pytest.mark.parametrize("dim", [1024, 4096])
def test_rmsnorm_bf16_tiny_values(q3, oracle, dim):
    """bf16 rows of the few-row kernel fold each square with a fused
    multiply-add, which equals the reference's square-then-add only while the
    square is exact in binary32 (|v| >= 2^-63 or v == 0).  Rows holding
    smaller values must be folded the reference's way: all-tiny rows (where
    the two chains really differ), a few tiny values among normal ones, bf16
    subnormals, values on both sides of 2^-63, and exact zeros."""
    rng = np.random.default_rng(dim + 3)
    rows = []
    for scale in (2.0 ** -70, 2.0 ** -66, 2.0 ** -63):             # whole rows of tiny values
        rows.append(rng.standard_normal(dim).astype(np.float32) * np.float32(scale))
    r = rng.standard_normal(dim).astype(np.float32)                 # a few tiny values among normal ones
    r[rng.choice(dim, 5, replace=False)] *= np.float32(2.0 ** -80)
    rows.append(r)
    r = rng.standard_normal(dim).astype(np.float32) * np.float32(2.0 ** -64)
    r[: dim // 2] = rng.standard_normal(dim // 2).astype(np.float32)  # tiny tail after a normal head
    rows.append(r)
    r = rng.standard_normal(dim).astype(np.float32) * np.float32(2.0 ** -130)   # bf16 subnormals
    rows.append(r)
    r = np.where(rng.random(dim) < 0.5, np.float32(2.0 ** -63), np.float32(-(2.0 ** -63) * 0.99))
    rows.append(r.astype(np.float32))                              # both sides of 2^-63
    r = rng.standard_normal(dim).astype(np.float32)
    r[rng.random(dim) < 0.3] = 0.0                                  # exact zeros only: no fallback needed
    rows.append(r)
    xb = to_bf16(np.stack(rows), oracle)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    qg, sg = q3.rmsnorm_q8(dev(xb), dev(w))
    qo, so = oracle.rows_rmsnorm_q8(xb, w)
    assert_q8_equal(qg, sg, qo, so)
    g = host(q3.rmsnorm(dev(xb), dev(w)))
    o = oracle.rows_rmsnorm(xb, w)
    assert np.array_equal(g, o)
    assert q3.device_status() == 0


def test_rmsnorm_rejects_bad_shapes(q3):
    import torch
    from metalqwen3_b200.q3cu import Q3Error
    x = torch.zeros((2, 100), device="cuda")
    w = torch.ones(100, device="cuda")
    with pytest.raises(Q3Error) as e:
        q3.rmsnorm_q8(x, w)
    assert e.value.status == 3                       # ERR_GROUP
    x = torch.zeros((2, 130), device="cuda")
    with pytest.raises(Q3Error) as e:
        q3.rmsnorm(x, torch.ones(130, device="cuda"))
    assert e.value.status == 2                       # ERR_ALIGN (row bytes not a multiple of 16)


@pytest.mark.parametrize("rows", [4096, 12000])
def test_prefill_kernels_chained_on_one_stream(q3, oracle, rows):
    """The prefill kernels are programmatic dependent launches: each may start
    before the kernel ahead of it has finished, and must wait for it before
    touching memory.  Each op here reads what the launch just before it wrote,
    with no synchronisation in between (4096 rows: the RMSNorm ring kernel,
    12000: the TMA-fed one)."""
    import torch
    rng = np.random.default_rng(rows + 7)
    dim, hidden, nh, nkv = 2560, 9728, 32, 8
    x = activations(rng, rows, dim)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    w2 = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    qh = rng.standard_normal((rows, nh, 128), dtype=np.float32)
    kh = rng.standard_normal((rows, nkv, 128), dtype=np.float32)
    pos = (np.arange(rows) % 4096).astype(np.int32)
    qn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    hb = activations(rng, 4096, hidden)
    hb2 = rng.standard_normal((4096, hidden)).astype(np.float32)
    tx, tw, tw2, tq, tk, tp, tqn, tkn = (dev(a) for a in (x, w, w2, qh, kh, pos, qn, kn))
    thb, thb2 = dev(hb), dev(hb2)
    torch.cuda.synchronize()
    y = q3.rmsnorm(tx, tw)                        # RMSNorm -> y, then RMSNorm+Q8_0 of y
    qg, sg = q3.rmsnorm_q8(y, tw2)
    q3.qk_norm_rope(tq, tk, tp, tqn, tkn)         # twice in place
    q3.qk_norm_rope(tq, tk, tp, tqn, tkn)
    q3.swiglu(thb, thb2)                          # SwiGLU in place, then SwiGLU+Q8_0 of its output
    hq, hs = q3.swiglu_q8(thb, thb2)
    torch.cuda.synchronize()
    yo = oracle.rows_rmsnorm(x, w, threads=8)
    assert np.array_equal(bits(host(y)), bits(yo))
    qo, so = oracle.rows_rmsnorm_q8(yo, w2, threads=8)
    assert_q8_equal(qg, sg, qo, so)
    q1, k1 = oracle.rows_qk_norm_rope(qh, kh, pos, qn, kn, threads=8)
    q2, k2 = oracle.rows_qk_norm_rope(q1, k1, pos, qn, kn, threads=8)
    np.testing.assert_allclose(host(tq), q2, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(host(tk), k2, rtol=RTOL, atol=ATOL)
    ho = oracle.rows_swiglu(hb, hb2, threads=8)
    assert np.array_equal(bits(host(thb)), bits(ho))
    hqo, hso = oracle.rows_swiglu_q8(ho, hb2, threads=8)
    assert_q8_equal(hq, hs, hqo, hso)
    assert q3.device_status() == 0


# --------------------------------------------------------------------------- qk-norm + rope
@pytest.mark.parametrize("rows,nh,nkv,posmax", [(1, 16, 8, 37), (5, 32, 8, 4096), (4096, 32, 8, 4096), (64, 40, 8, 32768)])
def test_qk_norm_rope_f32(q3, oracle, rows, nh, nkv, posmax):
    rng = np.random.default_rng(rows + nh)
    qh = rng.standard_normal((rows, nh, 128), dtype=np.float32)
    kh = rng.standard_normal((rows, nkv, 128), dtype=np.float32)
    pos = (np.arange(rows) % posmax).astype(np.int32) if rows >= posmax else rng.integers(0, posmax, rows).astype(np.int32)
    if rows > 1:
        pos[0], pos[-1] = 0, posmax - 1
    qn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    tq, tk = dev(qh), dev(kh)
    q3.qk_norm_rope(tq, tk, dev(pos), dev(qn), dev(kn))
    qo, ko = oracle.rows_qk_norm_rope(qh, kh, pos, qn, kn, threads=8)
    np.testing.assert_allclose(host(tq), qo, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(host(tk), ko, rtol=RTOL, atol=ATOL)


def test_qk_norm_only_is_bitexact_at_pos0(q3, oracle):
    """At pos 0 the rotation is the identity (cos 0 = 1, sin 0 = 0), so the
    output is the QK-RMSNorm alone, which must match bit for bit."""
    rng = np.random.default_rng(2)
    qh = rng.standard_normal((9, 32, 128), dtype=np.float32)
    kh = rng.standard_normal((9, 8, 128), dtype=np.float32)
    pos = np.zeros(9, np.int32)
    qn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    tq, tk = dev(qh), dev(kh)
    q3.qk_norm_rope(tq, tk, dev(pos), dev(qn), dev(kn))
    qo, ko = oracle.rows_qk_norm_rope(qh, kh, pos, qn, kn)
    assert np.array_equal(bits(host(tq)), bits(qo)) and np.array_equal(bits(host(tk)), bits(ko))


@pytest.mark.parametrize("rows,nh", [(7, 32), (256, 32)])
def test_qk_norm_rope_bf16(q3, oracle, rows, nh):
    """bf16 head rows at positions up to 32767: 1e-2 relative, plus 1e-6
    absolute for outputs that cancel to near zero (the device sincosf is a few
    ulps from the host's cosf/sinf, which is no relative bound at |o| ~ 0)."""
    rng = np.random.default_rng(rows)
    qh = to_bf16(rng.standard_normal((rows, nh, 128), dtype=np.float32), oracle)
    kh = to_bf16(rng.standard_normal((rows, 8, 128), dtype=np.float32), oracle)
    pos = rng.integers(0, 32768, rows).astype(np.int32)
    qn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    tq, tk = dev(qh), dev(kh)
    q3.qk_norm_rope(tq, tk, dev(pos), dev(qn), dev(kn))
    qo, ko = oracle.rows_qk_norm_rope(qh, kh, pos, qn, kn)
    np.testing.assert_allclose(bf16_to_f32(host(tq)), bf16_to_f32(qo), rtol=BF16_RTOL, atol=1e-6)
    np.testing.assert_allclose(bf16_to_f32(host(tk)), bf16_to_f32(ko), rtol=BF16_RTOL, atol=1e-6)


# --------------------------------------------------------------------------- swiglu
@pytest.mark.parametrize("rows,hidden", [(1, 64), (3, 3072), (64, 9728), (4096, 9728)])
def test_swiglu_q8_f32(q3, oracle, rows, hidden):
    rng = np.random.default_rng(hidden + rows)
    hb = activations(rng, rows, hidden)
    hb2 = activations(rng, rows, hidden)
    qg, sg = q3.swiglu_q8(dev(hb), dev(hb2))
    qo, so = oracle.rows_swiglu_q8(hb, hb2, threads=8)
    assert_q8_equal(qg, sg, qo, so)


@pytest.mark.parametrize("rows,hidden", [(1, 4), (3, 3072), (64, 10240)])
def test_swiglu_f32_bitexact(q3, oracle, rows, hidden):
    rng = np.random.default_rng(hidden)
    hb = (4 * rng.standard_normal((rows, hidden))).astype(np.float32)
    hb2 = rng.standard_normal((rows, hidden)).astype(np.float32)
    t = dev(hb)
    q3.swiglu(t, dev(hb2))
    assert np.array_equal(bits(host(t)), bits(oracle.rows_swiglu(hb, hb2, threads=8)))


def test_swiglu_expf_sweep(q3, oracle):
    """hb swept over 2^24 binary32 values spanning the whole exponent range
    (incl. |hb| > 88, denormals, +-inf): SwiGLU outputs equal the oracle's bit
    for bit, i.e. the device expf returns the host libm's bits there."""
    u = (np.arange(1 << 24, dtype=np.uint64) * 256 + 17).astype(np.uint32)
    hb = u.view(np.float32).copy()
    hb[~np.isfinite(hb)] = 0.5
    hb[:4] = [np.inf, -np.inf, np.float32(88.72283), np.float32(-103.97)]
    hb = hb.reshape(-1, 4096)
    hb2 = np.ones_like(hb)
    t = dev(hb)
    q3.swiglu(t, dev(hb2))
    g, o = host(t), oracle.rows_swiglu(hb, hb2, threads=8)
    same = (bits(g) == bits(o)) | (np.isnan(g) & np.isnan(o))
    assert same.all(), f"{int((~same).sum())} mismatches"


@pytest.mark.parametrize("rows,hidden,bf16", [
    (2000, 1024, False),      # 2,048,000 elements: the last chunk of the streaming kernel is partial
    (512, 17408, True),       # the Qwen3-14B FFN rows, bf16
    (4096, 9728, True),
])
def test_swiglu_streaming(q3, oracle, rows, hidden, bf16):
    """The streaming (per-warp bulk-copy ring) kernel: Q8_0 codes/scales and the
    float output, in place, bit for bit."""
    rng = np.random.default_rng(rows + hidden)
    hb, hb2 = activations(rng, rows, hidden), activations(rng, rows, hidden)
    if bf16:
        hb, hb2 = to_bf16(hb, oracle), to_bf16(hb2, oracle)
    qg, sg = q3.swiglu_q8(dev(hb), dev(hb2))
    qo, so = oracle.rows_swiglu_q8(hb, hb2, threads=8)
    assert_q8_equal(qg, sg, qo, so)
    t = dev(hb)
    q3.swiglu(t, dev(hb2))
    g, o = host(t), oracle.rows_swiglu(hb, hb2, threads=8)
    assert np.array_equal(bits(g) if not bf16 else g, bits(o) if not bf16 else o)
    assert q3.device_status() == 0


def test_swiglu_bf16_every_input(q3, oracle):
    """Every one of the 65,536 bf16 bit patterns as hb (zeros, subnormals, the
    gate table's window and beyond, +-inf, NaN), 64 copies against random hb2,
    through the streaming kernel: the float output bit for bit (NaN where the
    reference gives NaN), and the Q8_0 codes of the finite part."""
    rng = np.random.default_rng(17)
    hb = np.tile(np.arange(65536, dtype=np.uint32).astype(np.uint16), 64).reshape(-1, 4096)
    hb2 = to_bf16(rng.standard_normal(hb.shape, dtype=np.float32), oracle)
    t = dev(hb)
    q3.swiglu(t, dev(hb2))
    g, o = bf16_to_f32(host(t)), bf16_to_f32(oracle.rows_swiglu(hb, hb2, threads=8))
    same = (g.view(np.uint32) == o.view(np.uint32)) | (np.isnan(g) & np.isnan(o))
    assert same.all(), f"{int((~same).sum())} mismatches"
    fin = np.isfinite(bf16_to_f32(hb)).all(axis=1)
    qg, sg = q3.swiglu_q8(dev(hb[fin]), dev(hb2[fin]))
    qo, so = oracle.rows_swiglu_q8(hb[fin], hb2[fin], threads=8)
    assert_q8_equal(qg, sg, qo, so)


@pytest.mark.parametrize("rows,hidden", [(3, 512), (256, 12288)])
def test_swiglu_q8_bf16(q3, oracle, rows, hidden):
    rng = np.random.default_rng(hidden)
    hb = to_bf16(activations(rng, rows, hidden), oracle)
    hb2 = to_bf16(activations(rng, rows, hidden), oracle)
    qg, sg = q3.swiglu_q8(dev(hb), dev(hb2))
    qo, so = oracle.rows_swiglu_q8(hb, hb2, threads=8)
    assert_q8_equal(qg, sg, qo, so)


# --------------------------------------------------------------------------- softmax
def softmax_f64(x, off, lens):
    out = np.empty(x.size, np.float64)
    for o_, n in zip(off, lens):
        r = x[o_:o_ + n].astype(np.float64)
        m = max(0.0, r.max()) if n else 0.0
        e = np.exp(r - m)
        out[o_:o_ + n] = e / e.sum()
    return out


def check_softmax(g, o, ref64, off, lens):
    nan_o = np.isnan(o)
    assert np.array_equal(np.isnan(g), nan_o)
    g, o, r = g[~nan_o], o[~nan_o], ref64[~nan_o]
    tol = ATOL + RTOL * np.abs(r)
    assert (np.abs(g - r) <= tol).all(), "GPU softmax outside tolerance of the binary64 softmax"
    assert (np.abs(g - o) <= np.abs(o - r) + tol).all(), "GPU softmax further from the oracle than allowed"


@pytest.mark.parametrize("lens", [
    [1, 2, 3, 38, 511, 512, 513, 1024, 1025, 2048, 2049, 4096, 4097, 16384, 32768],
    list(range(1, 300, 7)),
])
def test_softmax_ragged(q3, oracle, lens):
    rng = np.random.default_rng(len(lens))
    lens = np.array(lens, np.int32)
    gaps = rng.integers(0, 5, lens.size)                # unaligned row starts
    off = np.concatenate([[0], np.cumsum(lens + gaps)[:-1]]).astype(np.int64) + 1
    total = int(off[-1] + lens[-1] + 3)
    x = (2.0 * rng.standard_normal(total)).astype(np.float32)
    t = dev(x)
    q3.softmax_rows(t, dev(off), dev(lens))
    o = oracle.rows_softmax(x, off, lens)
    g = host(t)
    ref64 = softmax_f64(x, off, lens)
    inrow = np.zeros(total, bool)
    for a, n in zip(off, lens):
        inrow[a:a + n] = True
    check_softmax(g[inrow], o[inrow], ref64[inrow], off, lens)
    # elements between the rows are untouched
    assert np.array_equal(bits(g[~inrow]), bits(x[~inrow]))


@pytest.mark.parametrize("shift", [1, 2, 3])
def test_softmax_buffer_only_4_byte_aligned(q3, oracle, shift):
    """The API asks only 4-byte alignment of x: rows of a buffer that starts
    1-3 floats past a 16-byte boundary, short and long, ragged offsets."""
    rng = np.random.default_rng(shift)
    lens = np.array([5, 300, 4096, 4099, 9000, 1, 70], np.int32)
    off = np.concatenate([[0], np.cumsum(lens + rng.integers(0, 4, lens.size))[:-1]]).astype(np.int64)
    total = int(off[-1] + lens[-1])
    x = (2.0 * rng.standard_normal(total)).astype(np.float32)
    base = dev(np.concatenate([np.zeros(shift, np.float32), x]))
    view = base[shift:]
    assert view.data_ptr() % 16 == 4 * shift
    q3.softmax_rows(view, dev(off), dev(lens))
    o = oracle.rows_softmax(x, off, lens)
    g = host(view)
    inrow = np.zeros(total, bool)
    for a, n in zip(off, lens):
        inrow[a:a + n] = True
    check_softmax(g[inrow], o[inrow], softmax_f64(x, off, lens)[inrow], off, lens)
    assert np.array_equal(bits(g[~inrow]), bits(x[~inrow]))
    assert np.array_equal(bits(host(base[:shift])), bits(np.zeros(shift, np.float32)))


def test_softmax_max_starts_at_zero(q3, oracle):
    """All-negative rows: the reference's max is 0, not max(x); a row with
    every score below -104 underflows to 0/0 = NaN in the reference."""
    x = np.concatenate([np.full(100, -3.0, np.float32), np.full(50, -200.0, np.float32),
                        np.linspace(-90, -80, 20, dtype=np.float32)])
    lens = np.array([100, 50, 20], np.int32)
    off = np.array([0, 100, 150], np.int64)
    t = dev(x)
    q3.softmax_rows(t, dev(off), dev(lens))
    g, o = host(t), oracle.rows_softmax(x, off, lens)
    assert np.isnan(o[100:150]).all() and np.isnan(g[100:150]).all()
    np.testing.assert_allclose(g[:100], o[:100], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(g[150:], o[150:], rtol=RTOL, atol=ATOL)


def test_softmax_decode_batch(q3, oracle):
    """256 tokens x 32 heads, row length pos+1 with pos uniform in 0..32767,
    scores N(0, sigma=2): the batched-decode workload."""
    rng = np.random.default_rng(0)
    pos = rng.integers(0, 32768, 256)
    lens = np.repeat(pos + 1, 32).astype(np.int32)
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    x = (2.0 * rng.standard_normal(int(lens.sum()))).astype(np.float32)
    t = dev(x)
    q3.softmax_rows(t, dev(off), dev(lens))
    o = oracle.rows_softmax(x, off, lens, threads=8)
    sel = rng.choice(lens.size, 64, replace=False)     # binary64 reference on a row sample
    g = host(t)
    for r in sel:
        a, n = off[r], lens[r]
        check_softmax(g[a:a + n], o[a:a + n], softmax_f64(x[a:a + n], [0], [n]), [0], [n])
    np.testing.assert_allclose(g, o, rtol=1e-4, atol=ATOL)


def _ragged_case(rng, lens, scale=2.0):
    lens = np.asarray(lens, np.int32)
    gaps = rng.integers(0, 5, lens.size)
    off = np.concatenate([[0], np.cumsum(np.maximum(lens, 0) + gaps)[:-1]]).astype(np.int64) + 3
    total = int(off[-1] + max(int(lens[-1]), 0) + 2)
    x = (scale * rng.standard_normal(total)).astype(np.float32)
    return x, off, lens


def _check_ragged(g, x, o, off, lens):
    inrow = np.zeros(x.size, bool)
    for a, n in zip(off, lens):
        if n > 0:
            inrow[a:a + n] = True
    check_softmax(g[inrow], o[inrow], softmax_f64(x, off, np.maximum(lens, 0))[inrow], off, lens)
    assert np.array_equal(bits(g[~inrow]), bits(x[~inrow]))


@pytest.mark.parametrize("extra", [0, 400])
def test_softmax_row_classes(q3, oracle, extra):
    """Every path in one call.  With few rows (extra = 0) the one-CTA-per-row
    kernel: register rows (<= 16384 scores) and three-pass rows.  With 400
    extra short rows the ring kernel: rows of one warp (<= 4096), rows shared
    by the CTA and staged in shared memory, rows longer than the ring (global
    memory).  Empty and negative lengths; some rows hold scores far below
    their max (the exact-exp branch: subnormal and zero exponentials) and one
    holds a NaN."""
    rng = np.random.default_rng(7)
    lens = [0, 3, 4096, 4097, -5, 57340, 57344, 57345, 57347, 60000, 131072, 1, 9000, 20000]
    lens = lens + list(rng.integers(1, 9, extra))
    x, off, lens = _ragged_case(rng, lens)
    for r, n in ((3, 4097), (9, 60000), (12, 9000), (1, 3)):     # far-below-max scores
        idx = off[r] + rng.choice(n, min(n, 40), replace=False)
        x[idx] = rng.uniform(-110.0, -82.0, idx.size).astype(np.float32)
    x[off[13] + 777] = np.nan
    t = dev(x)
    q3.softmax_rows(t, dev(off), dev(lens))
    assert q3.device_status() == 0
    g, o = host(t), oracle.rows_softmax(x, off, np.maximum(lens, 0))
    assert np.isnan(g[off[13]:off[13] + 20000]).all()
    _check_ragged(g, x, o, off, lens)


def test_softmax_many_rows_repeat_and_two_streams(q3, oracle):
    """81920 rows (40 heads x 2048 tokens, lengths 1..512): the largest rows
    per unit.  The same call is made twice on one stream, then on two streams
    at once: the per-launch row counters must be back at zero each time."""
    import torch
    rng = np.random.default_rng(11)
    pos = np.arange(2048) % 512
    lens = np.repeat(pos + 1, 40).astype(np.int32)
    x, off, lens = _ragged_case(rng, lens)
    o = oracle.rows_softmax(x, off, lens, threads=8)
    doff, dlen = dev(off), dev(lens)
    for _ in range(2):
        t = dev(x)
        q3.softmax_rows(t, doff, dlen)
        g = host(t)
        for r in rng.choice(lens.size, 200, replace=False):            # binary64 bound on a row sample
            a, n = off[r], lens[r]
            check_softmax(g[a:a + n], o[a:a + n], softmax_f64(x[a:a + n], [0], [n]), [0], [n])
        np.testing.assert_allclose(g, o, rtol=1e-4, atol=ATOL)         # every row; gaps untouched
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    t1, t2 = dev(x), dev(x)
    torch.cuda.synchronize()
    q3.softmax_rows(t1, doff, dlen, stream=s1)
    q3.softmax_rows(t2, doff, dlen, stream=s2)
    torch.cuda.synchronize()
    assert q3.device_status() == 0
    g1, g2 = host(t1), host(t2)
    assert np.array_equal(bits(g1), bits(g2))
    np.testing.assert_allclose(g1, o, rtol=1e-4, atol=ATOL)


# --------------------------------------------------------------------------- embedding
@pytest.mark.parametrize("dim", [64, 1024, 4096, 4160])
def test_embed_gather(q3, oracle, dim):
    rng = np.random.default_rng(dim)
    vocab = 3000
    tq = rng.integers(-127, 128, size=(vocab, dim), dtype=np.int8)
    ts = np.abs(0.01 * rng.standard_normal((vocab, dim // 64))).astype(np.float32)
    ids = np.minimum(rng.zipf(1.1, 5000) - 1, vocab - 1).astype(np.int32)
    out, oq, os_ = q3.embed_gather(dev(tq), dev(ts), dev(ids))
    ro, rq, rs, bad = oracle.rows_embed(tq, ts, ids, threads=8)
    assert bad == 0
    assert np.array_equal(bits(host(out)), bits(ro))
    assert_q8_equal(oq, os_, rq, rs)
    f_only, _, _ = q3.embed_gather(dev(tq), dev(ts), dev(ids), want_q8=False)
    assert np.array_equal(bits(host(f_only)), bits(ro))
    _, q_only, s_only = q3.embed_gather(dev(tq), dev(ts), dev(ids), want_f32=False)
    assert_q8_equal(q_only, s_only, rq, rs)


def test_embed_bad_ids_flag_and_skip(q3, oracle):
    import torch
    rng = np.random.default_rng(9)
    tq = rng.integers(-127, 128, size=(100, 256), dtype=np.int8)
    ts = np.abs(0.01 * rng.standard_normal((100, 4))).astype(np.float32)
    ids = np.array([0, 5, -1, 99, 100, 7, 1 << 30], np.int32)
    assert q3.device_status() == 0
    out = torch.full((7, 256), 7.0, device="cuda")
    q3.embed_gather(dev(tq), dev(ts), dev(ids), want_q8=False, out=out)
    flags = q3.device_status()
    assert flags & 0x1
    assert q3.device_status() == 0                    # reading clears the word
    g = host(out)
    ro, _, _, bad = oracle.rows_embed(tq, ts, ids)
    assert bad == 3
    for i, t in enumerate(ids):
        if 0 <= t < 100:
            assert np.array_equal(bits(g[i]), bits(ro[i]))
        else:
            assert (g[i] == 7.0).all()


# --------------------------------------------------------------------------- drop-in (host pointers)
def test_execute_dropin(q3, oracle):
    rng = np.random.default_rng(42)
    # MetalContext::executeRMSNorm, incl. a size that is not a multiple of 4
    for size in (2560, 1023):
        x = rng.uniform(-1, 1, size).astype(np.float32)
        w = rng.uniform(-1, 1, size).astype(np.float32)
        out = np.empty_like(x)
        q3.execute_rmsnorm(out, x, w)
        assert np.array_equal(bits(out), bits(oracle.rmsnorm(x, w)))
    # executeSoftmax
    x = rng.uniform(-1, 1, 4096).astype(np.float32)
    y = x.copy()
    q3.execute_softmax(y)
    np.testing.assert_allclose(y, oracle.softmax(x), rtol=RTOL, atol=ATOL)
    assert abs(float(y.astype(np.float64).sum()) - 1.0) <= 1e-5
    # executeSwiGLU (size 10240 as in the reference's shader test, and a ragged one)
    for n in (10240, 1001):
        hb = rng.uniform(-1, 1, n).astype(np.float32)
        hb2 = rng.uniform(-1, 1, n).astype(np.float32)
        y = hb.copy()
        q3.execute_swiglu(y, hb2)
        assert np.array_equal(bits(y), bits(oracle.swiglu(hb, hb2)))
    # executeRoPE: 20 q heads / 4 kv heads at pos 42 (the reference's shader test shape)
    q = rng.uniform(-1, 1, 20 * 128).astype(np.float32)
    k = rng.uniform(-1, 1, 4 * 128).astype(np.float32)
    qn = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kn = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    qg, kg = q.copy(), k.copy()
    q3.execute_rope(qg, kg, 128, 42, 20, 4, qn, kn)
    qo = np.concatenate([oracle.qk_norm_rope_head(q[h * 128:(h + 1) * 128], qn, 42) for h in range(20)])
    ko = np.concatenate([oracle.qk_norm_rope_head(k[h * 128:(h + 1) * 128], kn, 42) for h in range(4)])
    np.testing.assert_allclose(qg, qo, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(kg, ko, rtol=RTOL, atol=ATOL)
    # executeQuantize, incl. a ragged tail the reference leaves untouched
    x = rng.standard_normal(1000).astype(np.float32)
    qq = np.full(1000, 99, np.int8)
    ss = np.zeros(1000 // 64, np.float32)
    q3.execute_quantize(qq, ss, x)
    qo, so = oracle.quantize(x[:960])
    assert np.array_equal(qq[:960], qo) and np.array_equal(bits(ss), bits(so)) and (qq[960:] == 99).all()
    # executeEmbedding from a Q8_0 table
    tq = rng.integers(-127, 128, size=(50, 1024), dtype=np.int8)
    ts = np.abs(0.01 * rng.standard_normal((50, 16))).astype(np.float32)
    out = np.empty(1024, np.float32)
    q3.execute_embedding(out, tq, ts, 17, 1024)
    assert np.array_equal(bits(out), bits(oracle.dequantize(tq[17], ts[17])))


@pytest.mark.parametrize("pos,n_heads,n_kv,seq_len,layer", [(0, 16, 8, 64, 0), (37, 16, 8, 64, 1), (700, 32, 8, 1024, 2),
                                                          (5000, 4, 4, 5001, 0),
                                                          (40959, 8, 4, 40960, 0)])   # 40,960 positions: chunked
def test_execute_attention(q3, oracle, pos, n_heads, n_kv, seq_len, layer):
    """MetalContext::executeAttention (the engine's metal_attention call,
    MetalQwen3.cpp:639): one token's heads over a layer's cache rows at loff,
    host pointers; head outputs and the probabilities left in att bit for bit
    against the reference's loop (qwen3_original.c:395-428).  Also the
    device-pointer q3cu_attention on the same rows."""
    import torch
    rng = np.random.default_rng(pos + n_heads)
    hd, kv_dim = 128, n_kv * 128
    kv_mul = n_heads // n_kv
    layers = layer + 1
    kc = rng.standard_normal(layers * seq_len * kv_dim).astype(np.float32)
    vc = rng.standard_normal(layers * seq_len * kv_dim).astype(np.float32)
    q = (0.3 * rng.standard_normal(n_heads * hd)).astype(np.float32)
    loff = layer * seq_len * kv_dim
    xb_o, att_o = oracle.attention(q, kc, vc, pos, n_heads, n_kv, seq_len, loff=loff)
    xb = np.full(n_heads * hd, np.nan, np.float32)
    att = np.full(n_heads * seq_len, -7.0, np.float32)
    q3.execute_attention(xb, q, att, kc, vc, pos, hd, n_heads, n_kv, seq_len, kv_dim, loff, kv_mul)
    assert np.array_equal(bits(xb), bits(xb_o))
    att = att.reshape(n_heads, seq_len)
    assert np.array_equal(bits(att[:, :pos + 1]), bits(att_o[:, :pos + 1]))
    assert (att[:, pos + 1:] == -7.0).all()                         # columns past pos untouched
    rows = slice(loff, loff + (pos + 1) * kv_dim)
    xg, ag = q3.attention(dev(q), dev(kc[rows].reshape(pos + 1, kv_dim)), dev(vc[rows].reshape(pos + 1, kv_dim)),
                          pos, kv_mul)
    torch.cuda.synchronize()
    assert np.array_equal(bits(host(xg).ravel()), bits(xb_o))
    assert np.array_equal(bits(host(ag)), bits(att_o[:, :pos + 1]))


def test_attention_rejects_bad_arguments(q3):
    import torch
    from metalqwen3_b200.q3cu import Q3Error
    q = torch.zeros(4 * 128, device="cuda")
    kc = torch.zeros(10, 256, device="cuda")
    with pytest.raises(Q3Error) as e:                                 # att narrower than pos + 1
        q3.attention(q, kc, kc, 9, 2, att=torch.zeros(4, 9, device="cuda"))
    assert e.value.status == 1
    with pytest.raises(Q3Error) as e:                                 # 4 heads / kv_mul 1 need 4 kv heads of 128
        q3.attention(q, kc, kc, 3, 1)
    assert e.value.status == 1
    a = torch.zeros(4, 10, device="cuda")
    with pytest.raises(Q3Error) as e:                                 # the probabilities may not overwrite the scores
        q3.attention(q, kc, kc, 3, 2, att=a, probs=a)
    assert e.value.status == 1
    with pytest.raises(Q3Error) as e:
        q3.execute_attention(np.zeros(512, np.float32), np.zeros(512, np.float32), np.zeros(40, np.float32),
                             np.zeros(2560, np.float32), np.zeros(2560, np.float32), 3, 64, 4, 2, 10, 256, 0, 2)
    assert e.value.status == 1                                         # head_dim 64


# --------------------------------------------------------------------------- Q8_0 matmul
def same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return a.shape == b.shape and np.array_equal(na, nb) and np.array_equal(bits(a[~na]), bits(b[~nb]))


def q8_operands(rng, B, n, d, extremes=False):
    """x codes / scales in the range quantize produces, W codes uniform in
    [-127, 127] with |N(0, 0.01)| group scales (the exporter's range)."""
    xq = rng.integers(-127, 128, (B, n), dtype=np.int8)
    xs = np.abs(0.05 * rng.standard_normal((B, n // 64))).astype(np.float32)
    wq = rng.integers(-127, 128, (d, n), dtype=np.int8)
    ws = np.abs(0.01 * rng.standard_normal((d, n // 64))).astype(np.float32)
    if extremes:
        xq[:, :64], wq[0, :64], wq[1, :64] = -128, -128, 127
        ws[2, :] = 0.0
        ws[3, 0], xs[:, 0] = 3e38, 3e38
        ws[4, 1], xs[:, 1] = np.inf, 0.0
    return xq, xs, wq, ws


# Qwen3-0.6B's matmul shapes (wq, wk/wv, wo, w1/w3, w2), an 8B-sized square one,
# odd row counts, 1..7 token rows (ragged blocks of 4), n from one group up.
@pytest.mark.parametrize("B,n,d", [(1, 1024, 2048), (1, 1024, 1024), (1, 2048, 1024), (1, 1024, 3072),
                                   (1, 3072, 1024), (2, 4096, 4096), (3, 2560, 9728), (4, 64, 5),
                                   (5, 1088, 333), (7, 9728, 77)])
def test_matmul_q8(q3, oracle, B, n, d):
    xq, xs, wq, ws = q8_operands(np.random.default_rng(B * 7 + n + d), B, n, d)
    g = host(q3.matmul_q8(dev(xq), dev(xs), dev(wq), dev(ws)))
    assert same_bits(g, oracle.matmul(xq, xs, wq, ws))


def test_matmul_q8_extremes_and_golden(q3, oracle):
    xq, xs, wq, ws = q8_operands(np.random.default_rng(5), 3, 576, 40, extremes=True)
    with np.errstate(all="ignore"):
        assert same_bits(host(q3.matmul_q8(dev(xq), dev(xs), dev(wq), dev(ws))), oracle.matmul(xq, xs, wq, ws))
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "matmul.npz"))
    for i in range(int(g["count"])):
        out = host(q3.matmul_q8(dev(g[f"xq{i}"][None]), dev(g[f"xs{i}"][None]), dev(g[f"wq{i}"]), dev(g[f"ws{i}"])))
        assert same_bits(out[0], g[f"out{i}"]), f"golden case {i}"


def test_matmul_q8_classifier(q3, oracle):
    """The 0.6B classifier: 151,936 x 1024 (155 MB of codes), one token."""
    xq, xs, wq, ws = q8_operands(np.random.default_rng(11), 1, 1024, 151936)
    g = host(q3.matmul_q8(dev(xq), dev(xs), dev(wq), dev(ws)))
    assert same_bits(g, oracle.matmul(xq, xs, wq, ws))


def test_execute_quantized_matmul(q3, oracle):
    """MetalContext::executeQuantizedMatMul drop-in (host pointers)."""
    xq, xs, wq, ws = q8_operands(np.random.default_rng(12), 1, 2048, 1024)
    out = np.empty(1024, np.float32)
    q3.execute_quantized_matmul(out, xq[0], xs[0], wq, ws, 2048, 1024)
    assert same_bits(out, oracle.matmul(xq, xs, wq, ws)[0])
    from metalqwen3_b200.q3cu import Q3Error
    with pytest.raises(Q3Error) as e:
        q3.execute_quantized_matmul(out, xq[0], xs[0], wq, ws, 2048, 1024, group_size=32)
    assert e.value.status == 3                       # ERR_GROUP


# --------------------------------------------------------------------------- tensor-core Q8_0 matmul
@pytest.mark.parametrize("B,n,d", [
    (128, 128, 128),          # one tile, one K-stage (two groups)
    (300, 2560, 1000),        # ragged token and output tiles, 40 groups (10 passes over the 4 accumulators)
    (1024, 1024, 3072),       # Qwen3-0.6B W1-shaped, several tiles per SM
    (256, 4224, 136),         # 66 groups: the last staged chunk holds 2 groups
    (200, 9728, 384),         # Qwen3-4B W2-shaped K (152 groups: ten staged chunks)
    (256, 256, 130),          # d % 4 != 0: outputs by plain stores instead of tensor stores
])
def test_matmul_q8_tensor_cores(q3, oracle, B, n, d):
    """Prefill-sized batches (>= 128 token rows) go through the tcgen05 kernel:
    every output bit-identical to the reference's matmul (qwen3_original.c:310-331)."""
    rng = np.random.default_rng(B + n + d)
    xq, xs, wq, wsc = q8_operands(rng, B, n, d)
    g = host(q3.matmul_q8(*(dev(a) for a in (xq, xs, wq, wsc))))
    o = oracle.matmul(xq, xs, wq, wsc)
    assert same_bits(g, o), f"{int((bits(g) != bits(o)).sum())} of {g.size} differ"
    assert q3.device_status() == 0


def test_matmul_q8_tensor_cores_extremes(q3, oracle):
    """The tensor-core path with -128 codes, zero, huge and infinite scales
    (inf * 0 = NaN in the reference's chain): the same bits or the same NaNs."""
    xq, xs, wq, ws = q8_operands(np.random.default_rng(5), 128, 640, 40, extremes=True)
    with np.errstate(all="ignore"):
        assert same_bits(host(q3.matmul_q8(dev(xq), dev(xs), dev(wq), dev(ws))), oracle.matmul(xq, xs, wq, ws))


def test_matmul_q8_tensor_cores_prefill_4b(q3, oracle):
    """The Qwen3-4B prefill W1 product (4096 tokens, 2560 -> 9728), with
    extreme codes (+-127 and -128) in some groups: 96 sampled token rows
    against the oracle, all 9728 outputs each, bit for bit."""
    rng = np.random.default_rng(7)
    B, n, d = 4096, 2560, 9728
    xq, xs, wq, wsc = q8_operands(rng, B, n, d)
    xq[5, :64] = 127; wq[:, :64] = 127; xq[6, 64:128] = -128; wq[:, 64:128] = -128
    g = host(q3.matmul_q8(*(dev(a) for a in (xq, xs, wq, wsc))))
    rows = np.unique(np.concatenate([[0, 5, 6, B - 1], rng.integers(0, B, 92)]))
    o = oracle.matmul(xq[rows], xs[rows], wq, wsc)
    assert same_bits(g[rows], o), f"{int((bits(g[rows]) != bits(o)).sum())} of {o.size} differ"
    assert q3.device_status() == 0
