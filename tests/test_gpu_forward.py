"""The whole decode step on the device (q3cu_model_load / q3cu_model_forward)
against the reference CPU engine itself (src/cpu/qwen3_original.c compiled
unmodified: qwen3_transformer_create + qwen3_forward on the same checkpoint
file): logits bit-identical at every position, the KV cache carried across
calls.  Checkpoints are seeded synthetic ones in the reference's export format
(oracle/checkpoint.py); where the compiled reference is absent the oracle's
restatement (pinned to it in test_oracle_pin.py) gives the expected logits.
"""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return a.shape == b.shape and np.array_equal(na, nb) and \
        np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


def expected_logits(path, img, shape, steps, ctx_length=0):
    """Logits of the reference (or, without it, the oracle) for each (token, pos)."""
    from oracle.oracle import Reference, build_reference, reference_path
    if not os.path.exists(reference_path()):
        build_reference()
    out = []
    if os.path.exists(reference_path()):
        ref = Reference()
        t = ref.create(path, ctx_length)
        try:
            for tok, pos in steps:
                out.append(ref.forward(t, tok, pos).copy())
        finally:
            ref.free(t)
        return out
    from oracle.oracle import OracleModel
    om = OracleModel(img, ctx_length=ctx_length)
    try:
        for tok, pos in steps:
            out.append(om.forward(tok, pos).copy())
    finally:
        om.close()
    return out


SHAPES = {
    "small": dict(dim=256, hidden=768, n_layers=3, n_heads=4, n_kv=2, vocab=300, seq_len=16, head_dim=128),
    # Qwen3-0.6B's layer shape and vocabulary, 2 layers
    "qwen3_06b_2l": dict(dim=1024, hidden=3072, n_layers=2, n_heads=16, n_kv=8, vocab=151936, seq_len=48,
                         head_dim=128),
}


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_forward_logits_bit_exact(q3, name):
    from metalqwen3_b200.q3cu import Q3Model
    from oracle.checkpoint import write_checkpoint
    shape = SHAPES[name]
    rng = np.random.default_rng(len(name))
    npos = 12 if name == "small" else 40
    steps = [(int(t), p) for p, t in enumerate(rng.integers(0, shape["vocab"], npos))]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        write_checkpoint(path, seed=5, **shape)
        img = np.fromfile(path, np.uint8)
        want = expected_logits(path, img, shape, steps)
    model = Q3Model(q3, img)
    try:
        for (tok, pos), w in zip(steps, want):
            got = model.forward(tok, pos)
            assert same_bits(got, w), f"{name}: logits differ at pos {pos} (max |diff| {np.nanmax(np.abs(got - w))})"
        # the same step again into a caller's buffer (the cache row at pos is rewritten with the same values)
        buf = np.full(shape["vocab"], np.nan, np.float32)
        assert model.forward(tok, pos, out=buf) is buf and same_bits(buf, want[-1])
        with pytest.raises(ValueError):
            model.forward(tok, pos, out=np.empty(shape["vocab"], np.float64))
    finally:
        model.close()


LONG = {
    # 32 query heads over 8 kv heads, every position of a 1800-position context:
    # the attention's score work items (32 heads x 15 chunks of 128 positions)
    # outnumber its grid of 3 CTAs per SM near the end, and the V ring of 4
    # chunks wraps several times
    "split_1800": (dict(dim=128, hidden=384, n_layers=2, n_heads=32, n_kv=8, vocab=200, seq_len=1800,
                        head_dim=128), range(1800)),
    # a context above 16,384 positions: the values launch keeps the
    # probabilities in shared memory while they fit its long-context
    # allocation (4,224 positions), over the first 300 positions here
    "long_16400": (dict(dim=256, hidden=768, n_layers=2, n_heads=4, n_kv=2, vocab=300, seq_len=16400,
                        head_dim=128), range(300)),
    # a 33,000-position context, 4,400 positions: past 4,224 the values
    # launch recomputes each chunk's probabilities instead of keeping them
    "long_33000_chunked": (dict(dim=256, hidden=768, n_layers=2, n_heads=4, n_kv=2, vocab=300, seq_len=33000,
                                head_dim=128), range(4400)),
}


@pytest.mark.parametrize("name", sorted(LONG))
def test_forward_long_context_bit_exact(q3, name):
    from metalqwen3_b200.q3cu import Q3Model
    from oracle.checkpoint import write_checkpoint
    shape, positions = LONG[name]
    rng = np.random.default_rng(11)
    steps = [(int(rng.integers(0, shape["vocab"])), p) for p in positions]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        write_checkpoint(path, seed=3, **shape)
        img = np.fromfile(path, np.uint8)
        want = expected_logits(path, img, shape, steps)
    model = Q3Model(q3, img)
    try:
        for (tok, pos), w in zip(steps, want):
            got = model.forward(tok, pos)
            assert same_bits(got, w), f"{name}: logits differ at pos {pos} (max |diff| {np.nanmax(np.abs(got - w))})"
    finally:
        model.close()


def test_forward_ctx_length_and_errors(q3):
    from metalqwen3_b200.q3cu import Q3Error, Q3Model
    from oracle.checkpoint import checkpoint_image, write_checkpoint
    shape = SHAPES["small"]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        write_checkpoint(path, seed=9, **shape)
        img = np.fromfile(path, np.uint8)
        steps = [(7, 0), (299, 1), (0, 2), (150, 3), (42, 4), (1, 5)]
        want = expected_logits(path, img, shape, steps, ctx_length=6)        # seq_len capped to 6
    m = Q3Model(q3, img, ctx_length=6)
    try:
        assert m.config["seq_len"] == 6
        for (tok, pos), w in zip(steps, want):
            assert same_bits(m.forward(tok, pos), w)
        with pytest.raises(Q3Error) as e:
            m.forward(1, 6)                                   # pos beyond the capped context
        assert e.value.status == 5                            # ERR_INDEX
        with pytest.raises(Q3Error) as e:
            m.forward(shape["vocab"], 0)                      # token beyond the vocabulary
        assert e.value.status == 5
    finally:
        m.close()
    bad = img.copy()
    bad[0] ^= 0xFF                                            # magic
    with pytest.raises(Q3Error) as e:
        Q3Model(q3, bad)
    assert e.value.status == 10                               # ERR_FORMAT
    with pytest.raises(Q3Error) as e:
        Q3Model(q3, img[: img.size - 1000])                   # truncated tensors
    assert e.value.status == 10
    assert np.array_equal(checkpoint_image(seed=9, **shape), img)


def test_cpp_engine_program(q3, tmp_path):
    """The C++ boundary end to end: CudaContext + CudaModel in a compiled program,
    run on a checkpoint file; its first logit has the reference's bits."""
    import subprocess
    from metalqwen3_b200.build import library_path
    from oracle.checkpoint import write_checkpoint
    from test_abi import CXX_PROGRAM, ROOT
    shape = SHAPES["small"]
    path = str(tmp_path / "m.bin")
    write_checkpoint(path, seed=4, **shape)
    want = expected_logits(path, np.fromfile(path, np.uint8), shape, [(1, 0)])[0]
    src = tmp_path / "engine.cpp"
    src.write_text(CXX_PROGRAM)
    libdir = os.path.dirname(library_path())
    exe = str(tmp_path / "engine")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), str(src), "-o", exe,
                    "-L", libdir, "-lq3cu", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([exe, path], check=True, capture_output=True, text=True, timeout=120).stdout.split()
    assert int(out[0]) == shape["vocab"]
    got = np.float32(float.fromhex(out[1]))
    assert got.view(np.uint32) == want[0].view(np.uint32)
