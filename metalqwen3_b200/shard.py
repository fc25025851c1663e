"""Token-row sharding across the GPUs of one box.

Every kernel of this path is independent per token row (per lookup for the
embedding gather, per (token, head) row for softmax), so N GPUs split the rows
and exchange nothing on the data path.  These helpers compute each rank's
contiguous share:

* ``split_even(n, world)``   -- rows of equal cost (RMSNorm, RoPE, SwiGLU,
  quantize, embedding lookups): shares differ by at most one row;
* ``split_by_work(lens, world)`` -- ragged softmax rows, whose cost is their
  length: cut the prefix sum of the lengths at equal-work points so every rank
  gets ~sum(lens)/world elements.

All functions are pure host code (numpy); the returned ranges are half-open
[start, end) row indices.
"""
from __future__ import annotations

import numpy as np


def split_even(n: int, world: int) -> list[tuple[int, int]]:
    if world <= 0:
        raise ValueError("world must be positive")
    base, extra = divmod(n, world)
    out, s = [], 0
    for r in range(world):
        e = s + base + (1 if r < extra else 0)
        out.append((s, e))
        s = e
    return out


def split_by_work(lens, world: int) -> list[tuple[int, int]]:
    """Contiguous row ranges with near-equal total length."""
    if world <= 0:
        raise ValueError("world must be positive")
    lens = np.asarray(lens, dtype=np.int64)
    n = lens.size
    if n == 0:
        return [(0, 0)] * world
    csum = np.cumsum(lens)
    total = int(csum[-1])
    cuts = [0]
    for r in range(1, world):
        target = total * r / world
        # first row whose inclusive prefix reaches the target ends rank r-1's share
        i = int(np.searchsorted(csum, target, side="left")) + 1
        i = max(cuts[-1], min(i, n))
        cuts.append(i)
    cuts.append(n)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def shard_offsets(off, lens, rng: tuple[int, int]):
    """Row metadata of one rank's share, rebased to a compact local buffer.

    Returns (local_off, local_len, global_start, global_end): the rank copies
    x[global_start:global_end] into its own buffer and runs softmax_rows with
    local_off / local_len.
    """
    off = np.asarray(off, dtype=np.int64)
    lens = np.asarray(lens, dtype=np.int32)
    a, b = rng
    if a == b:
        return off[:0].copy(), lens[:0].copy(), 0, 0
    g0 = int(off[a:b].min())
    g1 = int((off[a:b] + lens[a:b]).max())
    return (off[a:b] - g0).astype(np.int64), lens[a:b].copy(), g0, g1
