"""Benchmark of the fused Qwen3 layer kernels (HBM GB/s and tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads: prefill4b (default: the headline line), decode8b, embed, prefill14b,
decode06b (one Qwen3-0.6B decode token through 28 layers of the path's ops,
timed eagerly and as CUDA graphs: microseconds per op and per layer), matmul06b
(one Qwen3-0.6B decode token's Q8_0 matmuls, 113 launches replayed as a graph).

A step is one pass of the layer's memory-bound kernels over one batch of
token rows already resident in HBM.  Default workload `prefill4b`: the
Qwen3-4B-shaped prefill layer, 4096 fp32 tokens per GPU, dim 2560, 32 q / 8 kv
heads of 128, hidden 9728, positions 0..4095, theta 1e6:

    rmsnorm_q8    x[4096][2560] -> Q8_0 codes + scales            (fused)
    qk_norm_rope  q[4096][32][128], k[4096][8][128], in place
    swiglu_q8     hb, hb2 [4096][9728] -> Q8_0 codes + scales     (fused)

Inputs are seeded synthetic data with the workload's shapes and value rules
(activations N(0,1) with a fixed 1% of channels x20; norm weights 1+N(0,0.1)).
value = algorithmic bytes (every input read once + every output written once)
of all ranks / max-over-ranks device time.  Under torchrun each rank runs its own
batch on its own GPU (token rows are independent: weak scaling, no collective on
the data path).  Between timed steps L2 is flushed by writing a 256 MiB buffer
and then reading another 256 MiB buffer, outside the timed events (the read
makes the write's dirty lines drain there, not in the next step's first kernel).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GS = 64
E2E_CHUNKS = 8          # token-row chunks of the pipelined end-to-end step


# ---------------------------------------------------------------------------- parity helpers
# After timing, the parity check compares a sample of the last timed step's
# outputs with the oracle (oracle/, the CPU restatement of the reference pinned
# to it by the tests) applied to that step's inputs: mismatch counts go on the
# JSON line.  Inputs that the step updates in place are snapshotted (a few rows)
# between the last two timed steps, outside the timed events.  For prefill4b and
# matmul4b the same check also runs on the end-to-end path (`e2e.parity`): the
# pinned host outputs of its last step against the pinned host inputs.
RTOL, ATOL, BF16_RTOL = 1e-5, 1e-6, 1e-2


def _host(t):
    import numpy as np
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.detach().cpu().numpy()


def _sample_rows(n, k=16):
    import numpy as np
    return np.unique(np.linspace(0, max(n - 1, 0), min(n, k)).round().astype(np.int64)) if n else np.zeros(0, np.int64)


def _q8_mismatch(qg, sg, qo, so):
    import numpy as np
    return int((qg != qo).sum()) + int((np.ascontiguousarray(sg).view(np.uint32) !=
                                        np.ascontiguousarray(so).view(np.uint32)).sum())


def _f32(a):
    import numpy as np
    return (a.astype(np.uint32) << 16).view(np.float32) if a.dtype == np.uint16 else np.asarray(a, np.float32)


def _tol_mismatch(g, o, rtol, atol):
    """Elements of g outside atol + rtol*|o| of o (NaN must match NaN)."""
    import numpy as np
    g, o = _f32(g).ravel(), _f32(o).ravel()
    nan = np.isnan(o)
    bad = int((np.isnan(g) != nan).sum())
    return bad + int((np.abs(g[~nan] - o[~nan]) > atol + rtol * np.abs(o[~nan])).sum())


def _softmax_mismatch(g, x, lens):
    """Scores of the rows of g outside 1e-5 rel / 1e-6 abs of a binary64 softmax
    of the inputs x (the max starting at 0, as the reference's)."""
    import numpy as np
    bad, o = 0, 0
    for n in lens:
        r = x[o:o + n].astype(np.float64)
        e = np.exp(r - max(0.0, float(r.max())))
        bad += _tol_mismatch(g[o:o + n], (e / e.sum()).astype(np.float64), RTOL, ATOL)
        o += n
    return bad


# ---------------------------------------------------------------------------- workloads
class Workload:
    name = ""
    tokens = 0
    dtype = "f32"
    e2e_note = ""
    scaling = "weak"
    # True where the tensors copied in and out by the end-to-end step carry the
    # names the parity check reads, so the check also runs on the host
    # outputs of the last end-to-end step.
    e2e_parity = False

    def kernels(self):              # [(name, algorithmic bytes per launch)]
        raise NotImplementedError

    def total_bytes(self):
        return sum(b for _, b in self.kernels())


class Prefill4B(Workload):
    """Qwen3-4B-shaped prefill layer kernels, fp32, T tokens."""
    name = "prefill4b"
    e2e_parity = True

    def __init__(self, tokens=4096, dim=2560, nh=32, nkv=8, hd=128, hidden=9728):
        self.tokens, self.dim, self.nh, self.nkv, self.hd, self.hidden = tokens, dim, nh, nkv, hd, hidden

    def kernels(self):
        T, D, H = self.tokens, self.dim, self.hidden
        rms = T * D * 4 + T * D + T * (D // GS) * 4 + D * 4
        rope = 2 * T * (self.nh + self.nkv) * self.hd * 4 + T * 4 + 2 * self.hd * 4
        swi = 2 * T * H * 4 + T * H + T * (H // GS) * 4
        return [("rmsnorm_q8", rms), ("qk_norm_rope", rope), ("swiglu_q8", swi)]

    def config(self):
        return {"workload": "Qwen3-4B-shaped prefill layer kernels (rmsnorm_q8 + qk_norm_rope + swiglu_q8)",
                "tokens_per_gpu": self.tokens, "dim": self.dim, "n_heads": self.nh, "n_kv_heads": self.nkv,
                "head_dim": self.hd, "hidden": self.hidden, "positions": f"0..{self.tokens - 1}",
                "rope_theta": 1e6, "input_dtype": "f32"}

    # -- device data
    def make(self, torch, dev, seed):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        T, D, H = self.tokens, self.dim, self.hidden

        def act(rows, cols):
            a = torch.randn(rows, cols, device=dev, generator=g)
            k = max(1, round(cols * 0.01))
            ch = torch.randperm(cols, device=dev, generator=g)[:k]
            a[:, ch] *= 20.0
            return a

        d = {
            "x": act(T, D),
            "w": 1.0 + 0.1 * torch.randn(D, device=dev, generator=g),
            "q": torch.randn(T, self.nh, self.hd, device=dev, generator=g),
            "k": torch.randn(T, self.nkv, self.hd, device=dev, generator=g),
            "pos": torch.arange(T, device=dev, dtype=torch.int32),
            "qn": 1.0 + 0.1 * torch.randn(self.hd, device=dev, generator=g),
            "kn": 1.0 + 0.1 * torch.randn(self.hd, device=dev, generator=g),
            "hb": act(T, H),
            "hb2": act(T, H),
        }
        d["xq"] = torch.empty(T, D, dtype=torch.int8, device=dev)
        d["xs"] = torch.empty(T, D // GS, dtype=torch.float32, device=dev)
        d["hq"] = torch.empty(T, H, dtype=torch.int8, device=dev)
        d["hs"] = torch.empty(T, H // GS, dtype=torch.float32, device=dev)
        return d

    def launch(self, q3, d, stream, events=None):
        """Enqueues the step; events = list of (start, end) pairs per kernel."""
        ops = [
            lambda: q3.rmsnorm_q8(d["x"], d["w"], q=d["xq"], s=d["xs"], stream=stream),
            lambda: q3.qk_norm_rope(d["q"], d["k"], d["pos"], d["qn"], d["kn"], stream=stream),
            lambda: q3.swiglu_q8(d["hb"], d["hb2"], q=d["hq"], s=d["hs"], stream=stream),
        ]
        for i, op in enumerate(ops):
            if events is not None:
                events[i][0].record(stream)
            op()
            if events is not None:
                events[i][1].record(stream)
        return len(ops)

    # -- host (end-to-end) data: inputs copied in, outputs copied out each step
    h2d_keys = ("x", "q", "k", "pos", "hb", "hb2")
    d2h_keys = ("xq", "xs", "q", "k", "hq", "hs")

    def slice(self, d, a, b):
        """Views of token rows [a, b) of every per-token tensor (weights whole)."""
        return {k: (v if k in ("w", "qn", "kn") else v[a:b]) for k, v in d.items()}

    # -- CPU oracle on a token sample
    def cpu_step(self, oracle, np, sample, threads, rng):
        if not hasattr(self, "_cpu"):
            D, H = self.dim, self.hidden
            x = rng.standard_normal((sample, D), dtype=np.float32)
            w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
            q = rng.standard_normal((sample, self.nh, self.hd), dtype=np.float32)
            k = rng.standard_normal((sample, self.nkv, self.hd), dtype=np.float32)
            pos = np.arange(sample, dtype=np.int32)
            qn = (1 + 0.1 * rng.standard_normal(self.hd)).astype(np.float32)
            kn = (1 + 0.1 * rng.standard_normal(self.hd)).astype(np.float32)
            hb = rng.standard_normal((sample, H), dtype=np.float32)
            hb2 = rng.standard_normal((sample, H), dtype=np.float32)
            self._cpu = (x, w, q, k, pos, qn, kn, hb, hb2)
        x, w, q, k, pos, qn, kn, hb, hb2 = self._cpu
        oracle.rows_rmsnorm_q8(x, w, threads=threads)
        oracle.rows_qk_norm_rope(q, k, pos, qn, kn, threads=threads)
        oracle.rows_swiglu_q8(hb, hb2, threads=threads)

    def bytes_for_tokens(self, n):
        return self.total_bytes() * n / self.tokens

    def parity_snapshot(self, d):
        S = _sample_rows(self.tokens)
        return {"rows": S, "q": _host(d["q"][S]), "k": _host(d["k"][S])}

    def parity(self, oracle, snap, d, q3=None):
        S = snap["rows"]
        qn, kn, w = _host(d["qn"]), _host(d["kn"]), _host(d["w"])
        qo, so = oracle.rows_rmsnorm_q8(_host(d["x"][S]), w)
        qr, kr = oracle.rows_qk_norm_rope(snap["q"], snap["k"], _host(d["pos"][S]), qn, kn)
        ho, hs = oracle.rows_swiglu_q8(_host(d["hb"][S]), _host(d["hb2"][S]))
        rt, at = (BF16_RTOL, ATOL) if snap["q"].dtype.kind == "u" else (RTOL, ATOL)
        return {"token_rows": int(S.size),
                "rmsnorm_q8": _q8_mismatch(_host(d["xq"][S]), _host(d["xs"][S]), qo, so),
                "qk_norm_rope": _tol_mismatch(_host(d["q"][S]), qr, rt, at) + _tol_mismatch(_host(d["k"][S]), kr, rt, at),
                "swiglu_q8": _q8_mismatch(_host(d["hq"][S]), _host(d["hs"][S]), ho, hs)}


def _ragged(np, pos, nh):
    """Offsets and lengths of the attention score rows of tokens at `pos`:
    row t*nh + h has length pos[t] + 1 (causal)."""
    lens = np.repeat(pos.astype(np.int64) + 1, nh)
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    return off, lens.astype(np.int32)


class _BF16Layer(Workload):
    """Shared parts of the bf16 layer workloads: rmsnorm_q8 + qk_norm_rope +
    swiglu_q8 on bf16 token rows, then the attention softmax over every head's
    score row (length pos+1, f32 scores N(0, sigma=2), in place)."""
    dtype = "bf16 (softmax scores f32)"
    outliers = False

    def scores(self, pos):
        return int(pos.astype("int64").sum() + pos.size) * self.nh

    def kernel_bytes(self, pos):
        T, D, H = pos.size, self.dim, self.hidden
        rms = T * D * 2 + T * D + T * (D // GS) * 4 + D * 4
        rope = 2 * T * (self.nh + self.nkv) * self.hd * 2 + T * 4 + 2 * self.hd * 4
        swi = 2 * T * H * 2 + T * H + T * (H // GS) * 4
        smx = 8 * self.scores(pos) + 12 * T * self.nh
        return [("rmsnorm_q8", rms), ("qk_norm_rope", rope), ("swiglu_q8", swi), ("softmax_rows", smx)]

    def kernels(self):
        return self.kernel_bytes(self.pos)

    def _batch(self, torch, dev, g, pos):
        import numpy as np
        T, D, H = pos.size, self.dim, self.hidden
        off, lens = _ragged(np, pos, self.nh)

        def act(rows, cols):
            a = torch.randn(rows, cols, device=dev, generator=g)
            if self.outliers:
                ch = torch.randperm(cols, device=dev, generator=g)[:max(1, round(cols * 0.01))]
                a[:, ch] *= 20.0
            return a.to(torch.bfloat16)

        return {
            "x": act(T, D), "hb": act(T, H), "hb2": act(T, H),
            "q": torch.randn(T, self.nh, self.hd, device=dev, generator=g).to(torch.bfloat16),
            "k": torch.randn(T, self.nkv, self.hd, device=dev, generator=g).to(torch.bfloat16),
            "pos": torch.from_numpy(pos).to(dev),
            "att": torch.randn(int(lens.sum()), device=dev, generator=g).mul_(2.0),
            "off": torch.from_numpy(off).to(dev), "len": torch.from_numpy(lens).to(dev),
            "xq": torch.empty(T, D, dtype=torch.int8, device=dev),
            "xs": torch.empty(T, D // GS, dtype=torch.float32, device=dev),
            "hq": torch.empty(T, H, dtype=torch.int8, device=dev),
            "hs": torch.empty(T, H // GS, dtype=torch.float32, device=dev),
        }

    def make(self, torch, dev, seed):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        d = self._batch(torch, dev, g, self.pos)
        d["w"] = 1.0 + 0.1 * torch.randn(self.dim, device=dev, generator=g)
        d["qn"] = 1.0 + 0.1 * torch.randn(self.hd, device=dev, generator=g)
        d["kn"] = 1.0 + 0.1 * torch.randn(self.hd, device=dev, generator=g)
        if self.e2e_tokens < self.tokens:
            e = self._batch(torch, dev, g, self.pos[: self.e2e_tokens])
            for k, v in e.items():
                d[k + "_e2e"] = v
        else:
            for k in ("x", "hb", "hb2", "q", "k", "pos", "att", "off", "len", "xq", "xs", "hq", "hs"):
                d[k + "_e2e"] = d[k]
        return d

    def _ops(self, q3, d, stream, sfx=""):
        return [
            lambda: q3.rmsnorm_q8(d["x" + sfx], d["w"], q=d["xq" + sfx], s=d["xs" + sfx], stream=stream),
            lambda: q3.qk_norm_rope(d["q" + sfx], d["k" + sfx], d["pos" + sfx], d["qn"], d["kn"], stream=stream),
            lambda: q3.swiglu_q8(d["hb" + sfx], d["hb2" + sfx], q=d["hq" + sfx], s=d["hs" + sfx], stream=stream),
            lambda: q3.softmax_rows(d["att" + sfx], d["off" + sfx], d["len" + sfx], stream=stream),
        ]

    def launch(self, q3, d, stream, events=None):
        ops = self._ops(q3, d, stream)
        for i, op in enumerate(ops):
            if events is not None:
                events[i][0].record(stream)
            op()
            if events is not None:
                events[i][1].record(stream)
        return len(ops)

    def launch_e2e(self, q3, d, stream):
        for op in self._ops(q3, d, stream, "_e2e"):
            op()
        return 4

    h2d_keys = tuple(k + "_e2e" for k in ("x", "q", "k", "pos", "hb", "hb2", "att"))
    d2h_keys = tuple(k + "_e2e" for k in ("xq", "xs", "q", "k", "hq", "hs", "att"))

    def e2e_bytes(self):
        return sum(b for _, b in self.kernel_bytes(self.pos[: self.e2e_tokens]))

    def cpu_step(self, oracle, np, sample, threads, rng):
        # The reference computes in binary32: the CPU rows are f32 with the same shapes.
        if not hasattr(self, "_cpu"):
            D, H = self.dim, self.hidden
            f = lambda *shape: rng.standard_normal(shape, dtype=np.float32)
            pos = self.sample_pos(sample)
            off, lens = _ragged(np, pos, self.nh)
            self._cpu = (f(sample, D), (1 + 0.1 * f(D)).astype(np.float32), f(sample, self.nh, self.hd),
                         f(sample, self.nkv, self.hd), pos, (1 + 0.1 * f(self.hd)).astype(np.float32),
                         (1 + 0.1 * f(self.hd)).astype(np.float32), f(sample, H), f(sample, H),
                         (2.0 * f(int(lens.sum()))).astype(np.float32), off, lens)
        x, w, q, k, pos, qn, kn, hb, hb2, att, off, lens = self._cpu
        oracle.rows_rmsnorm_q8(x, w, threads=threads)
        oracle.rows_qk_norm_rope(q, k, pos, qn, kn, threads=threads)
        oracle.rows_swiglu_q8(hb, hb2, threads=threads)
        oracle.rows_softmax(att, off, lens, threads=threads)

    def bytes_for_tokens(self, n):
        return sum(b for _, b in self.kernel_bytes(self.sample_pos(n)))

    def parity_snapshot(self, d):
        import numpy as np
        snap = Prefill4B.parity_snapshot(self, d)
        off, lens = _ragged(np, self.pos, self.nh)
        R = _sample_rows(lens.size)
        R = np.unique(np.concatenate([R, [int(np.argmax(lens))]])) if lens.size else R
        att = d["att"]
        snap["sm_rows"], snap["sm_in"] = R, [_host(att[int(off[r]):int(off[r]) + int(lens[r])]) for r in R]
        return snap

    def parity(self, oracle, snap, d, q3=None):
        import numpy as np
        out = Prefill4B.parity(self, oracle, snap, d, q3)
        off, lens = _ragged(np, self.pos, self.nh)
        R, att = snap["sm_rows"], d["att"]
        g = np.concatenate([_host(att[int(off[r]):int(off[r]) + int(lens[r])]) for r in R]) if R.size else \
            np.zeros(0, np.float32)
        x = np.concatenate(snap["sm_in"]) if R.size else g
        out["softmax_rows"] = _softmax_mismatch(g, x, [int(lens[r]) for r in R])
        out["softmax_row_count"] = int(R.size)
        return out


class Decode8B(_BF16Layer):
    """Qwen3-8B-shaped batched decode: T bf16 tokens at positions uniform in
    0..32767 (seed 0).  Under torchrun the tokens are split over the ranks in
    contiguous runs of near-equal softmax work (sum of pos + 1; strong
    scaling)."""
    name = "decode8b"

    scaling = "strong"

    def __init__(self, tokens=256, dim=4096, nh=32, nkv=8, hd=128, hidden=12288, maxpos=32767, seed=0, shard=None):
        import numpy as np
        from metalqwen3_b200.shard import split_by_work
        self.dim, self.nh, self.nkv, self.hd, self.hidden = dim, nh, nkv, hd, hidden
        pos = np.random.default_rng(seed).integers(0, maxpos + 1, size=tokens).astype(np.int32)
        self.total_tokens = tokens
        if shard is not None:          # this rank's tokens: contiguous, cut at equal softmax work (sum of pos + 1)
            a, b = split_by_work(pos.astype(np.int64) + 1, shard[1])[shard[0]]
            pos = pos[a:b]
        self.pos, self.tokens = pos, int(pos.size)
        self.e2e_tokens = self.tokens

    def sample_pos(self, n):
        return self.pos[:n]

    def config(self):
        return {"workload": "Qwen3-8B-shaped batched decode (rmsnorm_q8 + qk_norm_rope + swiglu_q8 on bf16 rows; "
                            "softmax over each head's score row of length pos+1)",
                "tokens_per_gpu": self.tokens, "dim": self.dim, "n_heads": self.nh, "n_kv_heads": self.nkv,
                "head_dim": self.hd, "hidden": self.hidden, "positions": "uniform 0..32767 (seed 0)",
                "softmax_rows": self.tokens * self.nh, "softmax_scores": self.scores(self.pos),
                "scores": "f32 N(0, sigma=2)", "rope_theta": 1e6, "input_dtype": "bf16"}


class Prefill14B(_BF16Layer):
    """Qwen3-14B-shaped long-context prefill, one layer: T bf16 tokens in all
    (131,072 = 32 sequences of 4096, positions 0..4095 each), 1% outlier
    channels x20, causal softmax of every head's row.  Under torchrun the
    sequences are split over the ranks (strong scaling); --weak runs T on every
    GPU."""
    name = "prefill14b"
    outliers = True

    scaling = "strong"

    def __init__(self, tokens=131072, dim=5120, nh=40, nkv=8, hd=128, hidden=17408, seqlen=4096, e2e_tokens=512,
                 shard=None):
        import numpy as np
        from metalqwen3_b200.shard import split_even
        self.dim, self.nh, self.nkv, self.hd, self.hidden, self.seqlen = dim, nh, nkv, hd, hidden, seqlen
        self.total_tokens = tokens
        if shard is not None:          # this rank's whole sequences (token rows are independent)
            a, b = split_even((tokens + seqlen - 1) // seqlen, shard[1])[shard[0]]
            tokens = max(0, min(tokens, b * seqlen) - a * seqlen)
        self.tokens = tokens
        self.pos = (np.arange(tokens) % seqlen).astype(np.int32)
        self.e2e_tokens = min(e2e_tokens, tokens)
        self.e2e_note = (f"end to end on the first {self.e2e_tokens} tokens of a sequence per step (a full step "
                         f"would move {self.scores(self.pos) * 4 / 1e9:.1f} GB of scores each way)")

    def sample_pos(self, n):
        import numpy as np
        return ((np.arange(n) * self.seqlen) // max(n, 1)).astype(np.int32)    # spread over 0..seqlen-1

    def config(self):
        return {"workload": "Qwen3-14B-shaped long-context prefill, one layer (rmsnorm_q8 + qk_norm_rope + "
                            "swiglu_q8 on bf16 rows; causal softmax of every head's row)",
                "tokens_per_gpu": self.tokens, "sequences_per_gpu": self.tokens // self.seqlen,
                "positions": f"0..{self.seqlen - 1} per sequence", "dim": self.dim, "n_heads": self.nh,
                "n_kv_heads": self.nkv, "head_dim": self.hd, "hidden": self.hidden,
                "softmax_scores": self.scores(self.pos), "scores": "f32 N(0, sigma=2)", "rope_theta": 1e6,
                "input_dtype": "bf16 (1% outlier channels x20)"}


class Embed(Workload):
    """Q8_0 embedding dequant/gather: a vocab x dim Q8_0 table on the device, N
    Zipf(1.1)-distributed token ids; each lookup writes the f32 row and its
    re-quantized Q8_0 codes + scales.  Under torchrun the table is replicated on
    every GPU (made outside the timed region) and the ids are split over the
    ranks (strong scaling)."""
    name = "embed"
    dtype = "int8 codes + f32 scales -> f32 rows + Q8_0"

    scaling = "strong"

    def __init__(self, tokens=1048576, vocab=151936, dim=4096, seed=0, e2e_lookups=65536, shard=None):
        import numpy as np
        from metalqwen3_b200.shard import split_even
        self.vocab, self.dim = vocab, dim
        rng = np.random.default_rng(seed)
        ranks = np.empty(0, np.int64)
        while ranks.size < tokens:                     # Zipf(1.1), truncated to the vocab by rejection
            r = rng.zipf(1.1, size=tokens)
            ranks = np.concatenate([ranks, r[r <= vocab]])
        perm = rng.permutation(vocab)                  # rank -> token id: a seeded permutation
        ids = perm[ranks[:tokens] - 1].astype(np.int32)
        self.total_tokens = tokens
        if shard is not None:                          # this rank's lookups (the table is replicated)
            a, b = split_even(tokens, shard[1])[shard[0]]
            ids = ids[a:b]
        self.ids, self.tokens = ids, int(ids.size)
        tokens = self.tokens
        self.e2e_lookups = min(e2e_lookups, tokens)
        self.e2e_note = (f"end to end on a sub-batch of {self.e2e_lookups} lookups per step (one full step "
                         f"moves {tokens * dim * 5 / 1e9:.1f} GB of rows to the host)")

    def kernels(self):
        D = self.dim
        per = 4 + D + D // 16 + 4 * D + D + D // 16
        return [("embed_gather", per * self.tokens)]

    def config(self):
        return {"workload": "Q8_0 embedding dequant/gather with fused re-quantize",
                "lookups_per_gpu": self.tokens, "vocab": self.vocab, "dim": self.dim,
                "ids": "Zipf(s=1.1) ranks truncated to the vocab, mapped through a seeded permutation (seed 0)",
                "table": "codes uniform in [-127,127], scales |N(0,0.01)|", "outputs": "f32 rows + Q8_0 codes/scales"}

    def make(self, torch, dev, seed):
        g = torch.Generator(device=dev)
        g.manual_seed(1234)                            # the same (replicated) table on every rank
        V, D, N = self.vocab, self.dim, self.tokens
        d = {
            "tq": torch.randint(-127, 128, (V, D), device=dev, dtype=torch.int8, generator=g),
            "ts": (0.01 * torch.randn(V, D // GS, device=dev, generator=g)).abs(),
            "ids": torch.from_numpy(self.ids).to(dev),
            "out": torch.empty(N, D, dtype=torch.float32, device=dev),
            "oq": torch.empty(N, D, dtype=torch.int8, device=dev),
            "os": torch.empty(N, D // GS, dtype=torch.float32, device=dev),
        }
        n = self.e2e_lookups
        d["ids_e2e"] = d["ids"][:n].clone()
        d["out_e2e"], d["oq_e2e"], d["os_e2e"] = d["out"][:n], d["oq"][:n], d["os"][:n]
        return d

    def launch(self, q3, d, stream, events=None):
        if events is not None:
            events[0][0].record(stream)
        q3.embed_gather(d["tq"], d["ts"], d["ids"], out=d["out"], oq=d["oq"], os_=d["os"], stream=stream)
        if events is not None:
            events[0][1].record(stream)
        return 1

    def launch_e2e(self, q3, d, stream):
        q3.embed_gather(d["tq"], d["ts"], d["ids_e2e"], out=d["out_e2e"], oq=d["oq_e2e"], os_=d["os_e2e"],
                        stream=stream)
        return 1

    h2d_keys = ("ids_e2e",)
    d2h_keys = ("out_e2e", "oq_e2e", "os_e2e")

    def e2e_bytes(self):
        return self.kernels()[0][1] * self.e2e_lookups / self.tokens

    def cpu_step(self, oracle, np, sample, threads, rng):
        if not hasattr(self, "_cpu"):
            tq = rng.integers(-127, 128, size=(self.vocab, self.dim), dtype=np.int8)
            ts = np.abs(0.01 * rng.standard_normal((self.vocab, self.dim // GS))).astype(np.float32)
            self._cpu = (tq, ts, self.ids[: max(sample, 1)])
        tq, ts, ids = self._cpu
        oracle.rows_embed(tq, ts, ids[:sample], want_q8=True, threads=threads)

    def bytes_for_tokens(self, n):
        return self.total_bytes() * n / self.tokens

    def parity_snapshot(self, d):
        return {"rows": _sample_rows(self.tokens, 64)}

    def parity(self, oracle, snap, d, q3=None):
        import numpy as np
        import torch
        S = snap["rows"]
        ids = torch.from_numpy(self.ids[S].astype(np.int64)).to(d["tq"].device)
        ro, rq, rs, bad = oracle.rows_embed(_host(d["tq"][ids]), _host(d["ts"][ids]), np.arange(S.size, dtype=np.int32))
        return {"lookups": int(S.size), "bad_ids": int(bad),
                "f32_rows": int((_host(d["out"][S]).view(np.uint32) != ro.view(np.uint32)).sum()),
                "q8_rows": _q8_mismatch(_host(d["oq"][S]), _host(d["os"][S]), rq, rs)}


class Decode06B(Workload):
    """Qwen3-0.6B decode step through the path's ops: T token rows (1: one
    decode token) at position 37, the embedding row, then 28 layers of
    attention RMSNorm+Q8_0 (1024), QK-norm+RoPE (16 + 8 heads of 128), the 16
    score rows of 38 (zero KV cache), the attention-output quantize (2048),
    FFN RMSNorm+Q8_0 and SwiGLU+Q8_0 (3072), and the final RMSNorm+Q8_0 -- in
    layer order, each op on its own layer's inputs.  Latency-bound: read as
    microseconds per op and per layer (the `graph` key: the same op sequence
    captured in a CUDA graph and replayed, per op type and for the whole step),
    not as a roofline fraction."""
    name = "decode06b"
    dtype = "f32"

    def __init__(self, tokens=1, dim=1024, nh=16, nkv=8, hd=128, hidden=3072, layers=28, pos=37, vocab=151936):
        self.tokens, self.dim, self.nh, self.nkv, self.hd = tokens, dim, nh, nkv, hd
        self.hidden, self.layers, self.pos, self.vocab = hidden, layers, pos, vocab

    def op_bytes(self):
        T, D, H, A, n = self.tokens, self.dim, self.hidden, self.nh * self.hd, self.pos + 1
        return {
            "embed_gather": T * (4 + D + D // 16 + 4 * D),
            "rmsnorm_q8": T * (4 * D + D + D // 16 * 4) + 4 * D,
            "qk_norm_rope": 2 * T * (self.nh + self.nkv) * self.hd * 4 + T * 4 + 2 * self.hd * 4,
            "softmax_rows": 8 * T * self.nh * n + 12 * T * self.nh,
            "quantize_q8": T * (4 * A + A + A // 16 * 4),
            "swiglu_q8": T * (2 * 4 * H + H + H // 16 * 4),
        }

    def op_counts(self):
        L = self.layers
        return {"embed_gather": 1, "rmsnorm_q8": 2 * L + 1, "qk_norm_rope": L, "softmax_rows": L,
                "quantize_q8": L, "swiglu_q8": L}

    def kernels(self):
        b, c = self.op_bytes(), self.op_counts()
        return [("decode_step_ops", sum(b[k] * c[k] for k in b))]

    def config(self):
        return {"workload": "Qwen3-0.6B decode step through the path's ops (28 layers; the Q8_0 matmuls are not "
                            "on the path)", "tokens_per_gpu": self.tokens, "dim": self.dim, "n_heads": self.nh,
                "n_kv_heads": self.nkv, "head_dim": self.hd, "hidden": self.hidden, "layers": self.layers,
                "position": self.pos, "vocab": self.vocab, "input_dtype": "f32"}

    def make(self, torch, dev, seed):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        L, T, D, H, A = self.layers, self.tokens, self.dim, self.hidden, self.nh * self.hd
        n = self.pos + 1
        r = lambda *shape: torch.randn(*shape, device=dev, generator=g)
        rows = T * self.nh
        d = {
            "xa": r(L, T, D), "xf": r(L, T, D), "xfin": r(T, D),
            "wa": 1 + 0.1 * r(L, D), "wf": 1 + 0.1 * r(L, D), "wfin": 1 + 0.1 * r(D),
            "q": r(L, T, self.nh, self.hd), "k": r(L, T, self.nkv, self.hd),
            "qn": 1 + 0.1 * r(L, self.hd), "kn": 1 + 0.1 * r(L, self.hd),
            "pos": torch.full((T,), self.pos, dtype=torch.int32, device=dev),
            "sc": 2.0 * r(L, rows * n), "off": torch.arange(rows, device=dev, dtype=torch.int64) * n,
            "len": torch.full((rows,), n, dtype=torch.int32, device=dev),
            "ao": r(L, T, A), "hb": r(L, T, H), "hb2": r(L, T, H),
            "tq": torch.randint(-127, 128, (self.vocab, D), dtype=torch.int8, device=dev, generator=g),
            "ts": (0.01 * r(self.vocab, D // GS)).abs(),
            "ids": torch.randint(0, self.vocab, (T,), dtype=torch.int32, device=dev, generator=g),
            "emb": torch.empty(T, D, device=dev),
            "xq": torch.empty(T, D, dtype=torch.int8, device=dev), "xs": torch.empty(T, D // GS, device=dev),
            "aq": torch.empty(T, A, dtype=torch.int8, device=dev), "as": torch.empty(T, A // GS, device=dev),
            "hq": torch.empty(T, H, dtype=torch.int8, device=dev), "hs": torch.empty(T, H // GS, device=dev),
        }
        return d

    def _ops(self, q3, d, stream):
        """(op type, launch) in layer order; per-layer views are taken here once."""
        ops = [("embed_gather", lambda: q3.embed_gather(d["tq"], d["ts"], d["ids"], want_q8=False, out=d["emb"],
                                                         stream=stream))]
        for l in range(self.layers):
            xa, xf, wa, wf = d["xa"][l], d["xf"][l], d["wa"][l], d["wf"][l]
            q, k, qn, kn, sc = d["q"][l], d["k"][l], d["qn"][l], d["kn"][l], d["sc"][l]
            ao, hb, hb2 = d["ao"][l], d["hb"][l], d["hb2"][l]
            ops += [
                ("rmsnorm_q8", lambda xa=xa, wa=wa: q3.rmsnorm_q8(xa, wa, q=d["xq"], s=d["xs"], stream=stream)),
                ("qk_norm_rope", lambda q=q, k=k, qn=qn, kn=kn: q3.qk_norm_rope(q, k, d["pos"], qn, kn,
                                                                                stream=stream)),
                ("softmax_rows", lambda sc=sc: q3.softmax_rows(sc, d["off"], d["len"], stream=stream)),
                ("quantize_q8", lambda ao=ao: q3.quantize_q8(ao, q=d["aq"], s=d["as"], stream=stream)),
                ("rmsnorm_q8", lambda xf=xf, wf=wf: q3.rmsnorm_q8(xf, wf, q=d["xq"], s=d["xs"], stream=stream)),
                ("swiglu_q8", lambda hb=hb, hb2=hb2: q3.swiglu_q8(hb, hb2, q=d["hq"], s=d["hs"], stream=stream)),
            ]
        ops.append(("rmsnorm_q8", lambda: q3.rmsnorm_q8(d["xfin"], d["wfin"], q=d["xq"], s=d["xs"], stream=stream)))
        return ops

    def launch(self, q3, d, stream, events=None):
        if not hasattr(self, "_opl") or self._opl[0] is not d or self._opl[1] is not stream:
            self._opl = (d, stream, self._ops(q3, d, stream))
        ops = self._opl[2]
        if events is not None:
            events[0][0].record(stream)
        for _, op in ops:
            op()
        if events is not None:
            events[0][1].record(stream)
        return len(ops)

    def graph_report(self, torch, q3, d, stream, reps=20):
        """The step's ops captured in CUDA graphs and replayed: the whole step
        in layer order, and each op type's launches alone; device microseconds."""
        ops = self._ops(q3, d, stream)
        groups = {"step": ops}
        for name in self.op_counts():
            groups[name] = [o for o in ops if o[0] == name]
        out = {}
        for name, lst in groups.items():
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for _, op in lst:
                    op()
            for _ in range(3):
                gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(reps):
                    gr.replay()
                e1.record(stream)
            stream.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            out[name] = {"us_per_replay": round(us, 2), "launches": len(lst), "us_per_op": round(us / len(lst), 2)}
            del gr
        out["us_per_layer"] = round((out["step"]["us_per_replay"] - out["embed_gather"]["us_per_replay"]) /
                                    self.layers, 2)
        return out

    h2d_keys = ("xa", "xf", "xfin", "q", "k", "sc", "ao", "hb", "hb2", "ids")
    d2h_keys = ("emb", "xq", "xs", "aq", "as", "hq", "hs")

    def cpu_step(self, oracle, np, sample, threads, rng):
        """One decode token of the reference's CPU code, on one core (the
        reference runs these ops serially per token)."""
        if not hasattr(self, "_cpu"):
            D, H, A, n = self.dim, self.hidden, self.nh * self.hd, self.pos + 1
            f = lambda *shape: rng.standard_normal(shape, dtype=np.float32)
            self._cpu = dict(x=f(1, D), w=(1 + 0.1 * f(D)).astype(np.float32), q=f(1, self.nh, self.hd),
                             k=f(1, self.nkv, self.hd), pos=np.array([self.pos], np.int32),
                             qn=(1 + 0.1 * f(self.hd)).astype(np.float32), kn=(1 + 0.1 * f(self.hd)).astype(np.float32),
                             sc=(2.0 * f(self.nh * n)).astype(np.float32),
                             off=(np.arange(self.nh) * n).astype(np.int64), lens=np.full(self.nh, n, np.int32),
                             ao=f(1, A), hb=f(1, H), hb2=f(1, H),
                             tq=rng.integers(-127, 128, size=(1024, D), dtype=np.int8),
                             ts=np.abs(0.01 * f(1024, D // GS)).astype(np.float32),
                             ids=np.array([7], np.int32))
        c = self._cpu
        if hasattr(oracle, "decode_ops"):           # the reference's code, the whole sequence in C
            oracle.decode_ops(c["tq"], c["ts"], int(c["ids"][0]), c["x"], c["w"], c["q"], c["k"], self.pos, c["qn"],
                              c["kn"], c["sc"], c["ao"], c["hb"], c["hb2"], self.layers)
            return
        oracle.rows_embed(c["tq"], c["ts"], c["ids"], want_q8=False, threads=1)
        for _ in range(self.layers):
            oracle.rows_rmsnorm_q8(c["x"], c["w"], threads=1)
            oracle.rows_qk_norm_rope(c["q"], c["k"], c["pos"], c["qn"], c["kn"], threads=1)
            oracle.rows_softmax(c["sc"], c["off"], c["lens"], threads=1)
            oracle.rows_quantize(c["ao"], threads=1)
            oracle.rows_rmsnorm_q8(c["x"], c["w"], threads=1)
            oracle.rows_swiglu_q8(c["hb"], c["hb2"], threads=1)
        oracle.rows_rmsnorm_q8(c["x"], c["w"], threads=1)

    cpu_tokens = 1                      # cpu_step runs one decode token whatever the sample
    cpu_threads = 1                     # ... on one core

    def bytes_for_tokens(self, n):
        return self.total_bytes()

    def parity_snapshot(self, d):
        return {}

    def parity(self, oracle, snap, d, q3=None):
        """The outputs the step leaves behind: the embedding row, the final
        RMSNorm+Q8_0 and the last layer's quantize and SwiGLU+Q8_0."""
        import numpy as np
        import torch
        L = self.layers
        ids = d["ids"].to(torch.int64)
        ro, _, _, _ = oracle.rows_embed(_host(d["tq"][ids]), _host(d["ts"][ids]),
                                        np.arange(self.tokens, dtype=np.int32), want_q8=False)
        xq, xs = oracle.rows_rmsnorm_q8(_host(d["xfin"]), _host(d["wfin"]))
        aq, as_ = oracle.rows_quantize(_host(d["ao"][L - 1]))
        hq, hs = oracle.rows_swiglu_q8(_host(d["hb"][L - 1]), _host(d["hb2"][L - 1]))
        return {"embed_gather": int((_host(d["emb"]).view(np.uint32) != ro.view(np.uint32)).sum()),
                "rmsnorm_q8": _q8_mismatch(_host(d["xq"]), _host(d["xs"]), xq, xs),
                "quantize_q8": _q8_mismatch(_host(d["aq"]), _host(d["as"]), aq, as_),
                "swiglu_q8": _q8_mismatch(_host(d["hq"]), _host(d["hs"]), hq, hs)}


class Matmul06B(Workload):
    """Qwen3-0.6B decode-token Q8_0 matmuls (qwen3_original.c:357-359, :432,
    :444-445, :454, :466), T token rows (1: one decode token): per layer the
    Q/K/V projections as one concatenated [2048+1024+1024][1024] matrix (they
    share their input), wo [1024][2048], W1|W3 as one [6144][1024], w2
    [1024][3072]; then the classifier [151936][1024] (the shared token table).
    28 layers + 1 = 113 launches per step, replayed as one CUDA graph.
    Weights: codes uniform in [-127, 127], scales |N(0, 0.01)| (the exporter's
    ranges); each matmul reads its own seeded activation codes.  HBM-bound in
    principle (633 MB of weights per token), latency-bound per launch at this
    model size."""
    name = "matmul06b"
    dtype = "int8 codes (dp4a, exact int32) -> f32"

    def __init__(self, tokens=1, dim=1024, nh=16, nkv=8, hd=128, hidden=3072, layers=28, vocab=151936):
        self.tokens, self.dim, self.layers, self.vocab = tokens, dim, layers, vocab
        A, K = nh * hd, nkv * hd
        self.shapes = [("qkv", dim, A + 2 * K), ("wo", A, dim), ("w13", dim, 2 * hidden), ("w2", hidden, dim)]

    def _mats(self):
        return [(f"{nm}{l}", n, d) for l in range(self.layers) for nm, n, d in self.shapes] + \
               [("cls", self.dim, self.vocab)]

    def kernels(self):
        B = self.tokens
        b = sum(d * n + d * n // 16 + B * (n + n // 16) + 4 * B * d for _, n, d in self._mats())
        return [("matmul_q8", b)]

    def config(self):
        return {"workload": "Qwen3-0.6B decode-token Q8_0 matmuls (28 layers: QKV, wo, W1|W3, w2; classifier)",
                "tokens_per_gpu": self.tokens, "dim": self.dim, "layers": self.layers, "vocab": self.vocab,
                "launches_per_step": len(self._mats()), "weights": "codes uniform [-127,127], scales |N(0,0.01)|",
                "launch": "one CUDA graph replay per step"}

    def make(self, torch, dev, seed):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        B = self.tokens
        d = {}
        for nm, n, m in self._mats():
            d["wq_" + nm] = torch.randint(-127, 128, (m, n), dtype=torch.int8, device=dev, generator=g)
            d["ws_" + nm] = (0.01 * torch.randn(m, n // GS, device=dev, generator=g)).abs()
            d["xq_" + nm] = torch.randint(-127, 128, (B, n), dtype=torch.int8, device=dev, generator=g)
            d["xs_" + nm] = (0.05 * torch.randn(B, n // GS, device=dev, generator=g)).abs()
            d["o_" + nm] = torch.empty(B, m, device=dev)
        self.h2d_keys = tuple(k for k in d if k.startswith(("xq_", "xs_")))
        self.d2h_keys = tuple(k for k in d if k.startswith("o_"))
        return d

    def _replay(self, q3, d, stream):
        import torch
        key = (id(d), id(stream))
        if getattr(self, "_gkey", None) != key:
            mats = self._mats()
            for nm, _, _ in mats:          # once eagerly (lazy init outside the capture)
                q3.matmul_q8(d["xq_" + nm], d["xs_" + nm], d["wq_" + nm], d["ws_" + nm], out=d["o_" + nm], stream=stream)
            stream.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for nm, _, _ in mats:
                    q3.matmul_q8(d["xq_" + nm], d["xs_" + nm], d["wq_" + nm], d["ws_" + nm], out=d["o_" + nm],
                                 stream=stream)
            self._graph, self._gkey = gr, key
        self._graph.replay()
        return len(self._mats())

    def launch(self, q3, d, stream, events=None):
        if events is not None:
            n = self._replay(q3, d, stream)            # the graph exists before the first timed step
            events[0][0].record(stream)
            self._graph.replay()
            events[0][1].record(stream)
            return n
        return self._replay(q3, d, stream)

    def launch_e2e(self, q3, d, stream):
        return self._replay(q3, d, stream)

    def cpu_step(self, oracle, np, sample, threads, rng):
        """One decode token's matmuls by the reference's own `matmul` (OpenMP over
        output rows, its own pragma), on all host cores."""
        if not hasattr(self, "_cpu"):
            from oracle.oracle import Oracle, Reference
            try:
                self._mm = Reference().matmul
            except Exception:
                self._mm = Oracle().matmul
            mats = {}
            for nm, n, m in self.shapes + [("cls", self.dim, self.vocab)]:
                mats[nm] = (rng.integers(-127, 128, (1, n), dtype=np.int8),
                            np.abs(0.05 * rng.standard_normal((1, n // GS))).astype(np.float32),
                            rng.integers(-127, 128, (m, n), dtype=np.int8),
                            np.abs(0.01 * rng.standard_normal((m, n // GS))).astype(np.float32))
            self._cpu = mats
        for _ in range(self.layers):
            for nm, _, _ in self.shapes:
                self._mm(*self._cpu[nm])
        self._mm(*self._cpu["cls"])

    cpu_tokens = 1
    cpu_note = ("the reference's own matmul (src/cpu/qwen3_original.c:310-331, compiled unmodified, its "
                "#pragma omp parallel for over output rows), one decode token per pass")

    def bytes_for_tokens(self, n):
        return self.total_bytes() / self.tokens

    def parity_snapshot(self, d):
        return {}

    def parity(self, oracle, snap, d, q3=None):
        """256 classifier rows and the whole last-layer w2 product, bit for bit."""
        import numpy as np
        out = {}
        for nm, rows in (("cls", _sample_rows(self.vocab, 256)), (f"w2{self.layers - 1}", None)):
            wq, ws = d["wq_" + nm], d["ws_" + nm]
            if rows is not None:
                wq, ws = wq[rows], ws[rows]
            o = oracle.matmul(_host(d["xq_" + nm]), _host(d["xs_" + nm]), _host(wq), _host(ws))
            g = _host(d["o_" + nm])
            g = g[:, rows] if rows is not None else g
            out[nm] = int((np.ascontiguousarray(g).view(np.uint32) != o.view(np.uint32)).sum())
        return out


class Matmul4B(Workload):
    """The prefill form of the Q8_0 matmul (qwen3_original.c:310-331 applied to
    every token row) on the tensor cores: the Qwen3-4B FFN up-projection of a
    4096-token batch, x codes/scales [4096][2560] (the rmsnorm_q8 output) times
    W1 [9728][2560] into f32 [4096][9728].  tcgen05 int8 MMA, the float chain
    per group in the reference's order (bit-exact).  Compute-bound: the
    roofline is int8 tensor throughput (2 ops per multiply-add)."""
    name = "matmul4b"
    dtype = "int8 codes (tcgen05 int8 MMA, exact int32) -> f32"
    bound = "tensor"
    e2e_parity = True

    def __init__(self, tokens=4096, n=2560, d=9728):
        self.tokens, self.n, self.d = tokens, n, d

    def kernels(self):
        T, n, d = self.tokens, self.n, self.d
        return [("matmul_q8_tc", T * n + T * (n // GS) * 4 + d * n + d * (n // GS) * 4 + 4 * T * d)]

    def flops(self):
        return 2 * self.tokens * self.n * self.d

    def config(self):
        return {"workload": "Qwen3-4B prefill FFN up-projection, Q8_0 x Q8_0 on the tcgen05 tensor cores",
                "tokens_per_gpu": self.tokens, "n": self.n, "d": self.d,
                "weights": "codes uniform [-127,127], scales |N(0,0.01)|; x scales |N(0,0.05)|"}

    def make(self, torch, dev, seed):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        T, n, d = self.tokens, self.n, self.d
        return {"xq": torch.randint(-127, 128, (T, n), dtype=torch.int8, device=dev, generator=g),
                "xs": (0.05 * torch.randn(T, n // GS, device=dev, generator=g)).abs(),
                "wq": torch.randint(-127, 128, (d, n), dtype=torch.int8, device=dev, generator=g),
                "ws": (0.01 * torch.randn(d, n // GS, device=dev, generator=g)).abs(),
                "out": torch.empty(T, d, device=dev)}

    def launch(self, q3, d, stream, events=None):
        if events is not None:
            events[0][0].record(stream)
        q3.matmul_q8(d["xq"], d["xs"], d["wq"], d["ws"], out=d["out"], stream=stream)
        if events is not None:
            events[0][1].record(stream)
        return 1

    h2d_keys = ("xq", "xs")
    d2h_keys = ("out",)

    def cpu_step(self, oracle, np, sample, threads, rng):
        """The reference's own matmul (OpenMP over output rows) on a few token rows."""
        if not hasattr(self, "_cpu"):
            from oracle.oracle import Oracle, Reference
            try:
                self._mm = Reference().matmul
            except Exception:
                self._mm = Oracle().matmul
            n, d = self.n, self.d
            self._cpu = (rng.integers(-127, 128, (4, n), dtype=np.int8),
                         np.abs(0.05 * rng.standard_normal((4, n // GS))).astype(np.float32),
                         rng.integers(-127, 128, (d, n), dtype=np.int8),
                         np.abs(0.01 * rng.standard_normal((d, n // GS))).astype(np.float32))
        self._mm(*self._cpu)

    cpu_tokens = 4
    cpu_note = ("the reference's own matmul (src/cpu/qwen3_original.c:310-331, compiled unmodified, OpenMP over "
                "output rows), 4 token rows per pass")

    def bytes_for_tokens(self, n):
        return self.total_bytes() * n / self.tokens

    def parity_snapshot(self, d):
        return {"rows": _sample_rows(self.tokens, 16)}

    def parity(self, oracle, snap, d, q3=None):
        import numpy as np
        S = snap["rows"]
        o = oracle.matmul(_host(d["xq"][S]), _host(d["xs"][S]), _host(d["wq"]), _host(d["ws"]))
        return {"token_rows": int(S.size), "outputs": int((_host(d["out"][S]).view(np.uint32) != o.view(np.uint32)).sum())}


class Forward06B(Workload):
    """One Qwen3-0.6B decode token through the whole model on the device
    (q3cu_model_load + q3cu_model_forward: qwen3_original.c:333-468), at
    position `pos` (attention over pos + 1 KV rows): the embedding row, 28
    layers of RMSNorm+Q8_0, Q/K/V matmuls, QK-norm+RoPE, attention, quantize,
    wo + residual, RMSNorm+Q8_0, W1|W3, SwiGLU+Q8_0, w2 + residual, then the
    final RMSNorm+Q8_0 and the classifier -- 171 launches (Q|K|V one matmul;
    the layer's two RMSNorm+Q8_0 and its SwiGLU+Q8_0 computed by the matmuls
    that consume them; attention as a scores launch that also does QK-norm+RoPE
    and a softmax/values launch that quantizes its output), every launch after
    the first a programmatic dependent, replayed as one
    CUDA graph per timed step.  The checkpoint is a seeded synthetic image in the
    reference's file format (codes uniform in [-127, 127], scales
    |N(0, 0.01)|, norm weights 1 + N(0, 0.1)); the reference arm runs its own
    qwen3_forward on the same file."""
    name = "forward06b"
    dtype = "f32 activations, Q8_0 weights (int8 dp4a, exact int32)"

    def __init__(self, tokens=1, pos=511, layers=28, dim=1024, hidden=3072, nh=16, nkv=8, hd=128, vocab=151936):
        self.tokens, self.pos, self.layers, self.dim, self.hidden = 1, pos, layers, dim, hidden
        self.nh, self.nkv, self.hd, self.vocab = nh, nkv, hd, vocab

    def _bytes(self):
        D, H, L, V = self.dim, self.hidden, self.layers, self.vocab
        A, K = self.nh * self.hd, self.nkv * self.hd
        codes = V * D + L * (A * D + 2 * K * D + D * A + 3 * H * D)
        norms = 4 * (2 * L * D + D + 2 * L * self.hd)
        kv = 2 * L * (self.pos + 1) * K * 4 + 2 * L * K * 4      # cache rows read, this position's rows written
        return codes + codes // 16 + norms + kv + 4 * V

    def kernels(self):
        return [("decode_step", self._bytes())]

    def config(self):
        return {"workload": "Qwen3-0.6B decode token through the whole model on the device (28 layers, classifier)",
                "tokens_per_gpu": 1, "position": self.pos, "dim": self.dim, "hidden": self.hidden,
                "layers": self.layers, "n_heads": self.nh, "n_kv_heads": self.nkv, "head_dim": self.hd,
                "vocab": self.vocab, "launches_per_step": 6 * self.layers + 3,
                "weights": "seeded synthetic checkpoint, codes uniform [-127,127], scales |N(0,0.01)|",
                "launch": "one CUDA graph replay per step; e2e: the q3cu_model_forward call with logits to the host"}

    def image(self, seed=0):
        """The checkpoint bytes (the reference's format), as a numpy uint8 array."""
        import struct
        import numpy as np
        rng = np.random.default_rng(seed)
        D, H, L, V, hd = self.dim, self.hidden, self.layers, self.vocab, self.hd
        A, K = self.nh * hd, self.nkv * hd
        parts = [struct.pack("I", 0x616A6331) + struct.pack("i", 1) +
                 struct.pack("10i", D, H, L, self.nh, self.nkv, V, self.pos + 1, hd, 1, GS), bytes(256 - 48)]
        norm = lambda n: (1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32).tobytes()
        parts += [norm(L * D), norm(L * D), norm(D), norm(L * hd), norm(L * hd)]

        def q8(rows, cols):
            n = rows * cols
            return (rng.integers(-127, 128, n, dtype=np.int8).tobytes() +
                    np.abs(0.01 * rng.standard_normal(n // GS, dtype=np.float32)).astype(np.float32).tobytes())
        parts.append(q8(V, D))
        for shape in [(A, D)] * L + [(K, D)] * L + [(K, D)] * L + [(D, A)] * L + [(H, D)] * L + [(D, H)] * L + \
                [(H, D)] * L:
            parts.append(q8(*shape))
        return np.frombuffer(b"".join(parts), np.uint8)

    def make(self, torch, dev, seed):
        return {"img": self.image(seed)}

    def _model(self, q3, d):
        if "model" not in d:
            from metalqwen3_b200.q3cu import Q3Model
            d["model"] = Q3Model(q3, d.pop("img"))
        return d["model"]

    def _replay(self, q3, d, stream):
        import torch
        m = self._model(q3, d)
        if getattr(self, "_gkey", None) != (id(d), id(stream)):
            m.forward(7, self.pos, stream=stream, to_host=False)         # eager once, outside the capture
            stream.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                m.forward(7, self.pos, stream=stream, to_host=False)
            self._graph, self._gkey = gr, (id(d), id(stream))
        return self._graph

    def launch(self, q3, d, stream, events=None):
        gr = self._replay(q3, d, stream)
        if events is not None:
            events[0][0].record(stream)
        gr.replay()
        if events is not None:
            events[0][1].record(stream)
        return 6 * self.layers + 4                 # + the kernel that stores the step parameters

    def launch_e2e(self, q3, d, stream):
        if "logits_host" not in d:                 # the caller's pinned logits buffer, reused every step
            import torch
            d["logits_host"] = torch.empty(self.vocab, dtype=torch.float32, pin_memory=True).numpy()
        self._model(q3, d).forward(7, self.pos, stream=stream, out=d["logits_host"])
        return 6 * self.layers + 3

    h2d_keys = ()
    d2h_keys = ()
    lib_h2d_bytes = 528                     # the step parameters: position, token, 64 cos + 64 sin

    @property
    def lib_d2h_bytes(self):
        return 4 * self.vocab                    # the logits

    e2e_note = ("the token id and position go in by value (the library copies them and RoPE's table to the "
                "device and replays its own graph of the step); the logits come back to the host inside the call "
                "(607,744 bytes, into the caller's pinned buffer)")

    def cpu_step(self, oracle, np, sample, threads, rng):
        """One decode token by the reference's own qwen3_forward on the same checkpoint file."""
        if not hasattr(self, "_ref"):
            import tempfile
            from oracle.oracle import Reference
            self._dir = tempfile.TemporaryDirectory()
            path = os.path.join(self._dir.name, "m.bin")
            self.image(1234).tofile(path)
            self._ref = Reference()
            self._t = self._ref.create(path, self.pos + 1)
        self._ref.forward(self._t, 7, self.pos)

    cpu_tokens = 1
    cpu_note = ("the reference's own qwen3_transformer_create + qwen3_forward (src/cpu/qwen3_original.c compiled "
                "unmodified, OpenMP in its matmul and attention), one decode token per pass")

    def bytes_for_tokens(self, n):
        return self.total_bytes()

    def parity_snapshot(self, d):
        return {}

    def parity(self, oracle, snap, d, q3=None):
        """The logits of the timed step (run once more after timing: the same
        graph on the same inputs) against the reference's own
        qwen3_forward (the oracle's restatement where it is not built) on the
        same checkpoint, token and position, with the same zero KV cache below
        pos: every one of the vocab logits bit for bit."""
        import numpy as np
        g = np.empty(self.vocab, np.float32)
        self._model(q3, d).forward(7, self.pos, out=g)          # the timed step once more, logits to the host
        try:
            self.cpu_step(None, np, 1, 1, None)          # builds the reference model on the same image
            want = self._ref.forward(self._t, 7, self.pos)
        except (FileNotFoundError, OSError):
            from oracle.oracle import OracleModel
            om = OracleModel(self.image(1234), ctx_length=self.pos + 1, oracle=oracle)
            want = om.forward(7, self.pos)
            om.close()
        nan = np.isnan(want)
        return {"logits": int((np.isnan(g) != nan).sum() +
                              (g[~nan].view(np.uint32) != want[~nan].view(np.uint32)).sum()),
                "vocab": int(want.size)}


WORKLOADS = {"prefill4b": Prefill4B, "decode8b": Decode8B, "embed": Embed, "prefill14b": Prefill14B,
             "decode06b": Decode06B, "matmul06b": Matmul06B, "matmul4b": Matmul4B, "forward06b": Forward06B}


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every 10 ms."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index):
        self.index, self.samples, self.reasons, self.max_mhz = index, [], set(), None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML unavailable: report nothing rather than guess
            self.err = str(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h) if hasattr(
                    nv, "nvmlDeviceGetCurrentClocksEventReasons") else nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()
        if not self.ok or not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml 10 ms"}


# ---------------------------------------------------------------------------- helpers
def measured_hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense int8 tensor throughput for the roofline: twice the measured dense
    bf16 burst figure (MEASURED_PEAKS.json bf16_tflops; B200's dense int8 rate
    is twice its bf16 rate), else twice the fallback 1.59 PFLOP/s."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            v = float(json.load(f)["bf16_tflops"])
        return 2 * v, "2 x measured dense bf16 burst (MEASURED_PEAKS.json bf16_tflops): int8 rate"
    except Exception:
        return 2 * 1590.0, "2 x fallback 1590 TFLOP/s bf16: int8 rate"


def profiled_traffic(workload, kernel, alg_bytes=None):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, or None.

    A capture taken on a smaller case of the same kernel is scaled to this
    launch by the ratio of algorithmic bytes (the kernel's traffic grows in
    proportion: every input read once, every output written once)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            e = json.load(f)[workload][kernel]
    except Exception:
        return None
    b = e["dram_bytes_per_launch"]
    if alg_bytes is not None and e.get("algorithmic_bytes") and alg_bytes != e["algorithmic_bytes"]:
        b = round(b * alg_bytes / e["algorithmic_bytes"])
    return b


def cpu_baseline(workload, seconds=10.0):
    import numpy as np
    impl, kind = cpu_impl()
    threads = getattr(workload, "cpu_threads", os.cpu_count() or 1)
    sample = 128
    rng = np.random.default_rng(0)
    workload.cpu_step(impl, np, sample, threads, rng)          # warm up (allocations, page faults)
    t0 = time.perf_counter()
    n = 0
    while True:
        workload.cpu_step(impl, np, sample, threads, rng)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = workload.bytes_for_tokens(sample) * n / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{n} passes over {getattr(workload, 'cpu_tokens', sample)} tokens of the same step "
                      f"({el:.1f} s), OpenMP over rows; " + getattr(workload, "cpu_note", CPU_NOTE[kind]),
            "tokens_per_s": round(getattr(workload, "cpu_tokens", sample) * n / el, 1)}


# ---------------------------------------------------------------------------- reference arm
def cpu_impl():
    """The reference compiled from its sources (oracle/_ref) if present, else the port."""
    try:
        from oracle.oracle import ReferenceRows
        return ReferenceRows(), "reference"
    except Exception:
        from oracle.oracle import Oracle
        return Oracle(), "port"


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    impl, kind = cpu_impl()
    threads = getattr(wl, "cpu_threads", os.cpu_count() or 1)
    sample = 32
    rng = np.random.default_rng(0)
    for _ in range(args.warmup):
        wl.cpu_step(impl, np, sample, threads, rng)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wl.cpu_step(impl, np, sample, threads, rng)
    el = time.perf_counter() - t0
    val = wl.bytes_for_tokens(sample) * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": wl.scaling if not args.weak else "weak", "vs_baseline": None,
        "dtype": wl.dtype, "data": "synthetic",
        "config": dict(wl.config(), sample_tokens_per_step=sample),
        "tokens_per_s": round(getattr(wl, "cpu_tokens", sample) * args.steps / el, 2),
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{getattr(wl, 'cpu_tokens', sample)} tokens per step of the same workload, "
                                   f"{threads} host threads "
                                   f"(OpenMP over rows); " + getattr(wl, "cpu_note", CPU_NOTE[kind])},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# The CPU implementation's row functions, by the kernel they stand for.
CPU_KERNEL = {"rows_rmsnorm_q8": "rmsnorm_q8", "rows_qk_norm_rope": "qk_norm_rope", "rows_swiglu_q8": "swiglu_q8",
              "rows_softmax": "softmax_rows", "rows_embed": "embed_gather", "rows_quantize": "quantize_q8"}


class _TimedImpl:
    """Wraps the CPU implementation and adds up the wall time of each row function."""

    def __init__(self, impl):
        self._impl, self.seconds = impl, {}

    def __getattr__(self, name):
        f = getattr(self._impl, name)
        if name not in CPU_KERNEL:
            return f

        def timed(*a, **kw):
            t0 = time.perf_counter()
            r = f(*a, **kw)
            k = CPU_KERNEL[name]
            self.seconds[k] = self.seconds.get(k, 0.0) + time.perf_counter() - t0
            return r
        return timed


def cpu_kernels(args, wl):
    """Per-kernel GB/s of the reference's CPU code on this host, on one core and
    on all cores (OpenMP over rows), on a token sample of the workload; one JSON
    line."""
    import numpy as np
    impl, kind = cpu_impl()
    cores = os.cpu_count() or 1
    sample = 128
    if hasattr(wl, "op_bytes"):
        kb = {k: b * wl.op_counts()[k] for k, b in wl.op_bytes().items()}
    elif hasattr(wl, "kernel_bytes"):
        kb = dict(wl.kernel_bytes(wl.sample_pos(sample)))
    else:
        kb = {n: b * sample / wl.tokens for n, b in wl.kernels()}
    out, passes = {}, {}
    for threads in (1, cores):
        timed = _TimedImpl(impl)
        rng = np.random.default_rng(0)
        wl.cpu_step(impl, np, sample, threads, rng)              # builds the sample; warm-up
        t0, n = time.perf_counter(), 0
        while True:
            wl.cpu_step(timed, np, sample, threads, rng)
            n += 1
            if time.perf_counter() - t0 >= args.cpu_seconds:
                break
        passes[str(threads)] = n
        for k, sec in timed.seconds.items():
            out.setdefault(k, {})[str(threads)] = round(kb[k] * n / sec / 1e9, 3)
    print(json.dumps({"cpu_kernels": out, "unit": "GB/s (algorithmic bytes of the workload's kernels)",
                      "workload": wl.name, "threads": [1, cores], "kind": kind,
                      "sample": f"{sample} tokens per pass; passes per thread count {passes}", "note": CPU_NOTE[kind]}),
          flush=True)
    return 0


CPU_NOTE = {
    "reference": "src/cpu/qwen3_original.c compiled unmodified (rmsnorm, softmax, quantize, dequantize); its "
                 "inline RoPE and SwiGLU loops restated in oracle/ref_rows.c",
    "port": "oracle/q3_oracle.c, the restatement of src/cpu/qwen3_original.c",
}


METRIC = "fused layer-kernel HBM GB/s & tokens/s at 1/2/4/8 B200; % of HBM roofline"


# ---------------------------------------------------------------------------- our arm
def h2d_probe(args):
    """Host<->device copy bandwidth of every rank at once (pinned host memory,
    1 GiB per copy, CUDA events on the copying stream, max over ranks): the
    ceiling of the end-to-end numbers at N GPUs.  One JSON line."""
    import torch
    import torch.distributed as dist
    world, rank, local, dev = _dist_init(torch, dist)
    nbytes = 1 << 30
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    g = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s = torch.cuda.Stream(device=dev)
    out = {}
    for name, (dst, src) in (("h2d", (g, h)), ("d2h", (h, g))):
        for _ in range(2):
            with torch.cuda.stream(s):
                dst.copy_(src, non_blocking=True)
        s.synchronize()
        _barrier(dist, world, local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            for _ in range(args.steps):
                dst.copy_(src, non_blocking=True)
            e1.record(s)
        s.synchronize()
        ms = e0.elapsed_time(e1)
        per = torch.tensor([nbytes * args.steps / (ms / 1e3) / 1e9], device=dev, dtype=torch.float64)
        mx = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            allv = [torch.zeros_like(per) for _ in range(world)]
            dist.all_gather(allv, per)
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        else:
            allv = [per]
        out[name] = {"per_rank_gbs": [round(float(v.item()), 2) for v in allv],
                     "aggregate_gbs": round(world * nbytes * args.steps / (float(mx.item()) / 1e3) / 1e9, 2)}
    if rank == 0:
        aff = sorted(os.sched_getaffinity(0))
        print(json.dumps({"probe": "pinned host <-> device copies, all ranks at once", "n_gpus": world,
                          "bytes_per_copy": nbytes, "copies": args.steps, **out,
                          "rank0_cpu_affinity": f"{aff[0]}-{aff[-1]} ({len(aff)} cpus)" if aff else None}),
              flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def _dist_init(torch, dist):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        # once per process: every workload of a multi-workload launch shares the group
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return world, rank, local, dev


def _barrier(dist, world, local):
    if world > 1:
        dist.barrier(device_ids=[local])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="prefill4b")
    ap.add_argument("--tokens", type=int, default=0,
                    help="token rows (lookups): per GPU for weak workloads, the total for strong ones")
    ap.add_argument("--weak", action="store_true",
                    help="run a strong-scaling workload with its whole size on every GPU (replicas)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-kernels", action="store_true",
                    help="time each kernel of the workload on the reference's CPU code (1 core and all cores) and exit")
    ap.add_argument("--h2d-probe", action="store_true",
                    help="measure pinned host<->device copy bandwidth on every rank at once and exit")
    ap.set_defaults(workload_list=None)
    argv = sys.argv[1:]
    wi = argv.index("--workload") if "--workload" in argv else -1
    names = argv[wi + 1].split(",") if wi >= 0 else ["prefill4b"]
    if wi >= 0:
        argv = argv[:wi + 1] + [names[0]] + argv[wi + 2:]
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)
    if args.h2d_probe:
        return h2d_probe(args)
    rc = 0
    for name in names:                   # several workloads in one launch: one JSON line each
        if name not in WORKLOADS:
            raise SystemExit(f"unknown workload {name}")
        args.workload = name
        rc = rc or run_one(args)
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
    return rc


def run_one(args):
    cls = WORKLOADS[args.workload]
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    rank_env = int(os.environ.get("RANK", "0"))
    strong = cls.scaling == "strong" and not args.weak
    kw = {"tokens": args.tokens} if args.tokens else {}
    if strong:
        kw["shard"] = (rank_env, world_env)
    wl = cls(**kw)

    if args.impl == "reference":
        return run_reference(args, wl)
    if args.cpu_kernels:
        return cpu_kernels(args, wl)

    import torch
    import torch.distributed as dist

    world, rank, local, dev = _dist_init(torch, dist)

    from metalqwen3_b200.q3cu import Q3CU
    q3 = Q3CU(local)
    stream = torch.cuda.Stream(device=dev)
    d = wl.make(torch, dev, seed=1234 + rank)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.zeros(32 << 20, dtype=torch.int64, device=dev)
    nk = len(wl.kernels())

    def cold_l2():
        # Write 256 MiB, then read another 256 MiB: the step's inputs leave L2
        # and the lines the write left dirty are written back here, not inside
        # the next step's first kernel.
        flush.fill_(1)
        flush_r.amax()

    def barrier():
        _barrier(dist, world, local)

    # warm-up; the host time to enqueue one step sizes the start gate below
    enq = []
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            t0 = time.perf_counter()
            wl.launch(q3, d, stream)
            enq.append(time.perf_counter() - t0)
            cold_l2()
    stream.synchronize()
    if q3.device_status(stream) != 0:
        raise RuntimeError("device status set during warm-up")
    # Every timed step starts from a common point on all ranks: a host barrier,
    # then a fixed-length device sleep (torch's bounded spin kernel) on the
    # stream while the host enqueues the step behind it.  The step's start event
    # follows the sleep, so neither the barrier's skew between hosts nor the
    # host's launch latency falls inside the step; its end event follows the
    # step's last kernel.  Step time = max over ranks of end - start, per step.
    gate_s = max(100e-6, 3.0 * statistics.median(enq[1:] or enq))
    gate_cycles = int(gate_s * 2.0e9)

    # The timed region alternates two kinds of step: K plain steps (events only
    # at the step's start and end: `value`) and, before each, a profiled step
    # with an event pair around every kernel (the per-kernel durations behind
    # `kernels` and `roofline`).  Events between kernels cost a few microseconds
    # of front-end time per boundary, which would otherwise be charged to the
    # step.
    clocks = ClockSampler(local)
    clocks.start()
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(nk)] for _ in range(args.steps)]
    sev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    snap = None
    barrier()
    torch.cuda.synchronize(dev)
    launches = 0
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            launches += wl.launch(q3, d, stream, events=ev[i])      # profiled step
            cold_l2()
            if i == args.steps - 1 and hasattr(wl, "parity_snapshot"):
                stream.synchronize()
                snap = wl.parity_snapshot(d)        # inputs of the last step that it updates in place
                cold_l2()
            barrier()
            torch.cuda._sleep(gate_cycles)
            sev[i][0].record(stream)
            launches += wl.launch(q3, d, stream)                     # plain step
            sev[i][1].record(stream)
            cold_l2()                           # outside the events: L2 cold for the next step
    stream.synchronize()
    torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop()
    if q3.device_status(stream) != 0:
        raise RuntimeError("device status set during the timed region")
    parity = None
    if rank == 0 and hasattr(wl, "parity"):
        # the parity check: a sample of the last timed step against the oracle
        from oracle.oracle import Oracle
        parity = {"checked": "last timed step (sampled rows) vs the oracle on the same inputs; counts of "
                             "mismatching values (bit-exact ops) or of values outside the tolerance (RoPE, softmax)",
                  **wl.parity(Oracle(), snap or {}, d, q3)}

    per_kernel = [[ev[i][k][0].elapsed_time(ev[i][k][1]) for i in range(args.steps)] for k in range(nk)]
    step_ms = torch.tensor([sev[i][0].elapsed_time(sev[i][1]) for i in range(args.steps)], dtype=torch.float64,
                           device=dev)
    kern_ms = torch.tensor([sum(per_kernel[k][i] for k in range(nk)) for i in range(args.steps)],
                           dtype=torch.float64, device=dev)
    step_bytes = torch.tensor([float(wl.total_bytes()), float(wl.tokens)], dtype=torch.float64, device=dev)
    own_ms = float(step_ms.sum().item())
    if world > 1:
        dist.all_reduce(step_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(kern_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(step_bytes, op=dist.ReduceOp.SUM)
        rank_ms = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(rank_ms, torch.tensor([own_ms], dtype=torch.float64, device=dev))
        rank_ms = [float(t.item()) / args.steps for t in rank_ms]
    else:
        rank_ms = [own_ms / args.steps]
    total_ms = float(step_ms.sum().item())
    kernel_ms = float(kern_ms.sum().item())
    all_bytes, all_tokens = float(step_bytes[0].item()), float(step_bytes[1].item())

    # ---- CUDA graphs of the step's ops (latency-bound workloads) -----------
    graph = wl.graph_report(torch, q3, d, stream) if hasattr(wl, "graph_report") else None

    # ---- end to end: host buffers, copies inside the timed region ----------
    hin = {k: d[k].detach().to("cpu").pin_memory() for k in wl.h2d_keys}
    hout = {k: torch.empty(d[k].shape, dtype=d[k].dtype).pin_memory() for k in wl.d2h_keys}
    h2d = sum(t.numel() * t.element_size() for t in hin.values()) + getattr(wl, "lib_h2d_bytes", 0)
    d2h = sum(t.numel() * t.element_size() for t in hout.values()) + getattr(wl, "lib_d2h_bytes", 0)

    # Row-sliceable workloads pipeline each step over E2E_CHUNKS token-row chunks:
    # copy-in on two streams (alternate chunks), kernels on another, copy-out on
    # a fourth, so PCIe moves inputs and outputs at the same time (it is full
    # duplex).  A chunk's copy-in for the next step waits for its copy-out (q and
    # k are updated in place).  Other workloads copy in, run and copy out on one
    # stream.
    chunks = [(i * wl.tokens // E2E_CHUNKS, (i + 1) * wl.tokens // E2E_CHUNKS)
              for i in range(E2E_CHUNKS)] if hasattr(wl, "slice") else None
    s_ins = [torch.cuda.Stream(device=dev) for _ in range(2)]     # chunks alternate between two copy-in streams
    s_out = torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(E2E_CHUNKS)]
    ev_done = [torch.cuda.Event() for _ in range(E2E_CHUNKS)]
    ev_out = [torch.cuda.Event() for _ in range(E2E_CHUNKS)]

    def e2e_step():
        if chunks is None:
            with torch.cuda.stream(stream):
                for k, t in hin.items():
                    d[k].copy_(t, non_blocking=True)
                (wl.launch_e2e if hasattr(wl, "launch_e2e") else wl.launch)(q3, d, stream)
                for k, t in hout.items():
                    t.copy_(d[k], non_blocking=True)
            return
        for c, (a, b) in enumerate(chunks):
            s_in = s_ins[c % 2]
            s_in.wait_event(ev_out[c])
            with torch.cuda.stream(s_in):
                for k, t in hin.items():
                    d[k][a:b].copy_(t[a:b], non_blocking=True)
                ev_in[c].record(s_in)
            stream.wait_event(ev_in[c])
            with torch.cuda.stream(stream):
                wl.launch(q3, wl.slice(d, a, b), stream)
                ev_done[c].record(stream)
            s_out.wait_event(ev_done[c])
            with torch.cuda.stream(s_out):
                for k, t in hout.items():
                    t[a:b].copy_(d[k][a:b], non_blocking=True)
                ev_out[c].record(s_out)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    first, last = (stream, stream) if chunks is None else (s_ins[0], s_out)
    e0.record(first)
    if chunks is not None:
        s_ins[1].wait_event(e0)                 # nothing of the timed region starts before e0
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(last)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    e2e_b = torch.tensor([float(wl.e2e_bytes() if hasattr(wl, "e2e_bytes") else wl.total_bytes())],
                         dtype=torch.float64, device=dev)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(e2e_b, op=dist.ReduceOp.SUM)
        e2e_ms = float(t.item())
        barrier()
    e2e_all_bytes = float(e2e_b.item())
    # The parity check on the end-to-end path: the pinned host outputs of the last
    # end-to-end step against the oracle applied to the pinned host inputs.
    e2e_check = None
    if rank == 0 and parity is not None and wl.e2e_parity:
        from oracle.oracle import Oracle
        d_in = dict(d, **hin)
        e2e_check = wl.parity(Oracle(), wl.parity_snapshot(d_in), dict(d_in, **hout), q3)

    # ---- report ---------------------------------------------------------------
    if rank == 0:
        ms_per_step = total_ms / args.steps
        gbs = all_bytes * args.steps / (total_ms / 1e3) / 1e9
        kern = {}
        for k, (name, b) in enumerate(wl.kernels()):
            avg = statistics.mean(per_kernel[k])
            kern[name] = {"bytes": b, "avg_us": round(avg * 1e3, 3), "gbs": round(b / (avg / 1e3) / 1e9, 1)}
        peak, peak_kind = measured_hbm_peak()
        dom_name, dom_bytes = max(wl.kernels(), key=lambda kb: kb[1])
        dom_avg_s = statistics.mean(per_kernel[[n for n, _ in wl.kernels()].index(dom_name)]) / 1e3
        achieved = dom_bytes / dom_avg_s / 1e9
        tensor = getattr(wl, "bound", "hbm") == "tensor"
        if tensor:
            tpeak, tkind = measured_tensor_peak()
        scaling = "strong" if strong else "weak"
        par = (f"token rows split over {world} GPUs (strong: the configuration's total is fixed)" if strong else
               f"token rows x{world} (weak: the same batch on every GPU)")
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
            "config": dict(wl.config(), parallelism=par,
                           total_tokens=int(all_tokens),
                           l2="flushed between timed steps (256 MiB write + 256 MiB read of another buffer, outside the events); "
                              f"step working set {wl.total_bytes() / 1e6:.0f} MB per GPU vs 126 MB L2"),
            "timing": ("per step: host barrier, a fixed device sleep while the step is enqueued, then CUDA events "
                       "around the step on the launching stream; step time = max over ranks; value = all ranks' "
                       "algorithmic bytes / sum of step times; each timed step is preceded by a profiled step "
                       "(an event pair around each kernel: `kernels`, `roofline`)"),
            "kernel_sum_ms_per_step": round(kernel_ms / args.steps, 5),
            "rank_ms_per_step": [round(x, 5) for x in rank_ms],
            "tokens_per_s": round(all_tokens * args.steps / (total_ms / 1e3), 1),
            "hbm_frac": round(gbs / world / peak, 4),
            "kernels": kern,
            "roofline": ({"bound": "tensor", "kernel": dom_name,
                          "achieved": round(wl.flops() / dom_avg_s / 1e12, 1), "peak": tpeak, "peak_source": tkind,
                          "unit": "TFLOP/s", "frac": round(wl.flops() / dom_avg_s / 1e12 / tpeak, 4),
                          "traffic": profiled_traffic(wl.name, dom_name, dom_bytes),
                          "hbm_gbs": round(achieved, 1), "algorithmic_flops_per_launch": wl.flops(),
                          "algorithmic_bytes_per_launch": dom_bytes} if tensor else
                         {"bound": "hbm", "kernel": dom_name, "achieved": round(achieved, 1), "peak": peak,
                          "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                          else "fallback 6650 GB/s", "unit": "GB/s", "frac": round(achieved / peak, 4),
                          "traffic": profiled_traffic(wl.name, dom_name, dom_bytes),
                          "algorithmic_bytes_per_launch": dom_bytes}),
            "e2e": {"value": round(e2e_all_bytes * args.e2e_steps / (e2e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms / args.e2e_steps, 3),
                    "path": ("pinned host inputs -> cudaMemcpyAsync H2D -> q3cu C ABI kernels -> D2H, per step"
                             + (f", pipelined over {E2E_CHUNKS} token-row chunks on four streams (two copy-in, "
                                "kernels, copy-out)" if chunks else "") + (f"; {wl.e2e_note}" if wl.e2e_note else "")),
                    **({"parity": e2e_check} if e2e_check is not None else {})},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if graph is not None:
            line["graph"] = graph
        if parity is not None:
            line["parity"] = parity
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
        print(json.dumps(line), flush=True)

    q3.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
