"""bench.py's host logic on CPU: the strong-scaling shards of the configurations
that split over GPUs, the parity check that compares a timed step's outputs with the
oracle (a mistake planted in the outputs must be counted), and the reference
arm's JSON line."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_strong_shards_cover_the_configuration(world):
    import bench
    for cls, total in ((bench.Decode8B, 256), (bench.Embed, 4096), (bench.Prefill14B, 131072)):
        kw = {"tokens": total}
        parts = [cls(shard=(r, world), **kw) for r in range(world)]
        assert sum(p.tokens for p in parts) == total
        full = cls(**kw)
        if cls is bench.Decode8B:
            assert np.array_equal(np.concatenate([p.pos for p in parts]), full.pos)
            work = [int(p.pos.astype(np.int64).sum() + p.pos.size) for p in parts]
            assert max(work) - min(work) <= 2 * 32768
        elif cls is bench.Embed:
            assert np.array_equal(np.concatenate([p.ids for p in parts]), full.ids)
        else:
            assert all(p.tokens % 4096 == 0 for p in parts)       # whole sequences
            # every rank reads the layer's norm weights once per launch besides its rows
            per_launch = full.dim * 4 + 2 * full.hd * 4
            assert sum(p.total_bytes() for p in parts) == full.total_bytes() + (world - 1) * per_launch


def _prefill_outputs(wl, d, oracle):
    """Fills the step's outputs as the kernels would (from the oracle itself)."""
    import torch
    x, w = d["x"].numpy(), d["w"].numpy()
    q, s = oracle.rows_rmsnorm_q8(x, w)
    d["xq"].copy_(torch.from_numpy(q)); d["xs"].copy_(torch.from_numpy(s))
    qo, ko = oracle.rows_qk_norm_rope(d["q"].numpy(), d["k"].numpy(), d["pos"].numpy(), d["qn"].numpy(),
                                      d["kn"].numpy())
    q, s = oracle.rows_swiglu_q8(d["hb"].numpy(), d["hb2"].numpy())
    d["hq"].copy_(torch.from_numpy(q)); d["hs"].copy_(torch.from_numpy(s))
    return qo, ko


def test_parity_check_counts_planted_mistakes(oracle):
    import torch
    import bench
    wl = bench.Prefill4B(tokens=40)
    d = wl.make(torch, torch.device("cpu"), seed=1)
    snap = wl.parity_snapshot(d)
    qo, ko = _prefill_outputs(wl, d, oracle)
    d["q"].copy_(torch.from_numpy(qo)); d["k"].copy_(torch.from_numpy(ko))
    r = wl.parity(oracle, snap, d)
    assert r["token_rows"] == 16 and r["rmsnorm_q8"] == 0 and r["qk_norm_rope"] == 0 and r["swiglu_q8"] == 0
    row = int(snap["rows"][3])
    d["xq"][row, 5] += 1                                  # one wrong code
    d["hs"][row, 0] = torch.nextafter(d["hs"][row, 0], torch.tensor(np.inf))   # one scale off by an ulp
    d["q"][row, 0, 0] += 1e-3                             # one RoPE value out of tolerance
    r = wl.parity(oracle, snap, d)
    assert (r["rmsnorm_q8"], r["swiglu_q8"], r["qk_norm_rope"]) == (1, 1, 1)


def test_end_to_end_parity_check_reads_the_host_buffers(oracle):
    """The end-to-end check as bench.py composes it: inputs from the host
    copies (q and k are rotated in place on the device, so the device tensors
    no longer hold them), outputs from the host copies of the results."""
    import torch
    import bench
    wl = bench.Prefill4B(tokens=40)
    assert wl.e2e_parity and bench.Matmul4B.e2e_parity and not bench.Decode8B.e2e_parity
    d = wl.make(torch, torch.device("cpu"), seed=2)
    hin = {k: d[k].clone() for k in wl.h2d_keys}
    qo, ko = _prefill_outputs(wl, d, oracle)
    d["q"].copy_(torch.from_numpy(qo)); d["k"].copy_(torch.from_numpy(ko))
    hout = {k: d[k].clone() for k in wl.d2h_keys}
    d["q"].add_(1.0)                                      # the device tensors moved on after the last step
    d["xq"].zero_()
    d_in = dict(d, **hin)
    r = wl.parity(oracle, wl.parity_snapshot(d_in), dict(d_in, **hout))
    assert (r["rmsnorm_q8"], r["qk_norm_rope"], r["swiglu_q8"]) == (0, 0, 0)
    row = int(wl.parity_snapshot(d_in)["rows"][2])
    hout["hq"][row, 7] += 1                               # one wrong code in the host output
    r = wl.parity(oracle, wl.parity_snapshot(d_in), dict(d_in, **hout))
    assert r["swiglu_q8"] == 1


def test_softmax_parity_check(oracle):
    import bench
    rng = np.random.default_rng(0)
    lens = [1, 38, 700, 4097]
    x = (2.0 * rng.standard_normal(sum(lens))).astype(np.float32)
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    g = oracle.rows_softmax(x, off, np.array(lens, np.int32))
    assert bench._softmax_mismatch(g, x, lens) == 0
    g[800] += 1e-4                                        # far outside 1e-5 rel + 1e-6 abs
    assert bench._softmax_mismatch(g, x, lens) == 1


def test_embed_parity_check(oracle):
    import torch
    import bench
    wl = bench.Embed(tokens=200, vocab=500, dim=128)
    d = wl.make(torch, torch.device("cpu"), seed=2)
    ro, rq, rs, bad = oracle.rows_embed(d["tq"].numpy(), d["ts"].numpy(), wl.ids)
    d["out"].copy_(torch.from_numpy(ro)); d["oq"].copy_(torch.from_numpy(rq)); d["os"].copy_(torch.from_numpy(rs))
    snap = wl.parity_snapshot(d)
    r = wl.parity(oracle, snap, d)
    assert r["f32_rows"] == 0 and r["q8_rows"] == 0 and r["bad_ids"] == 0
    d["out"][int(snap["rows"][1]), 7] += 1.0
    assert wl.parity(oracle, snap, d)["f32_rows"] == 1


def test_reference_arm_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["cores"] >= 1
