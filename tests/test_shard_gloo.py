"""Multi-rank host logic on CPU (gloo, world size 2).

* the row split covers every row exactly once and balances work;
* two ranks each run their share of a ragged softmax and of an RMSNorm->Q8_0
  batch through the oracle, all-gather the results, and the assembled output
  equals the single-process result bit for bit (no data-path collective is
  needed: the gather here only checks the assembly);
* a rank that fails reports it on the host (through the store) before the next
  step, and the other rank stops instead of waiting in a collective.
"""
import os
import socket

import numpy as np
import pytest

from metalqwen3_b200.shard import shard_offsets, split_by_work, split_even


def test_split_even():
    for n in (0, 1, 7, 4096):
        for w in (1, 2, 3, 8):
            parts = split_even(n, w)
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
            sizes = [e - s for s, e in parts]
            assert max(sizes) - min(sizes) <= 1


def test_split_by_work_balances_ragged_rows():
    rng = np.random.default_rng(0)
    pos = rng.integers(0, 32768, 256)
    lens = np.repeat(pos + 1, 32)
    for w in (1, 2, 4, 8):
        parts = split_by_work(lens, w)
        assert parts[0][0] == 0 and parts[-1][1] == lens.size
        work = [int(lens[s:e].sum()) for s, e in parts]
        assert max(work) - min(work) <= 2 * lens.max()
    assert split_by_work([], 3) == [(0, 0)] * 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        o = Oracle()
        rng = np.random.default_rng(5)
        # ragged softmax share
        lens = rng.integers(1, 3000, 37).astype(np.int32)
        off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        x = (2 * rng.standard_normal(int(lens.sum()))).astype(np.float32)
        a, b = split_by_work(lens, world)[rank]
        loff, llen, g0, g1 = shard_offsets(off, lens, (a, b))
        part = o.rows_softmax(x[g0:g1], loff, llen) if b > a else np.zeros(0, np.float32)
        parts = [None] * world
        dist.all_gather_object(parts, (g0, part))
        # RMSNorm -> Q8_0 share
        xs = rng.standard_normal((23, 256)).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
        s, e = split_even(23, world)[rank]
        qq, ss = o.rows_rmsnorm_q8(np.ascontiguousarray(xs[s:e]), w)
        qparts = [None] * world
        dist.all_gather_object(qparts, (s, qq, ss))
        # failure detection on the host: rank 1 reports an error for step 1
        store = dist.distributed_c10d._get_default_store()
        stopped_at = None
        for step in range(3):
            if rank == 1 and step == 1:
                store.set(f"fail/{step}/{rank}", "device status 0x1")
            store.set(f"done/{step}/{rank}", "1")
            store.wait([f"done/{step}/{r}" for r in range(world)], datetime.timedelta(seconds=10))
            failed = [r for r in range(world) if store.check([f"fail/{step}/{r}"])]
            if failed:
                stopped_at = (step, failed)
                break
            dist.barrier()
        if rank == 0:
            full = o.rows_softmax(x, off, lens)
            got = np.array(x, copy=True)
            for g0_, p in parts:
                got[g0_:g0_ + p.size] = p
            qfull, sfull = o.rows_rmsnorm_q8(xs, w)
            qg = np.concatenate([p[1] for p in sorted(qparts, key=lambda t: t[0])])
            sg = np.concatenate([p[2] for p in sorted(qparts, key=lambda t: t[0])])
            q.put((np.array_equal(got.view(np.uint32), full.view(np.uint32)),
                   np.array_equal(qg, qfull) and np.array_equal(sg.view(np.uint32), sfull.view(np.uint32)),
                   stopped_at))
        dist.destroy_process_group()
    except Exception as ex:  # report instead of hanging the parent
        q.put(("error", rank, repr(ex)))


def test_two_rank_gloo_sharding():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    res = q.get(timeout=5)
    assert res[0] != "error", res
    softmax_ok, q8_ok, stopped_at = res
    assert softmax_ok and q8_ok
    assert stopped_at == (1, [1])
