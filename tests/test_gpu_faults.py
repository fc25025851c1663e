"""Failure detection on the GPU without a fault: a device-side bounded wait
that runs out reports Q3CU_DEV_TIMEOUT through the status word, the host reads
it, and the context keeps working.  (The host-side rank failure is tested on
CPU gloo ranks in test_shard_gloo.py.)"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DEV_TIMEOUT = 0x2


def test_bounded_wait_timeout_is_reported(q3, oracle):
    import torch
    from metalqwen3_b200.q3cu import Q3Error
    assert q3.device_status() == 0
    t0 = time.time()
    q3.selftest_wait_timeout()
    flags = q3.device_status()               # synchronises: the wait gave up at its limit (~2 s)
    elapsed = time.time() - t0
    assert flags & DEV_TIMEOUT, f"status 0x{flags:x}"
    assert 0.5 < elapsed < 30, elapsed
    assert q3.device_status() == 0           # read once, then cleared
    # the C ABI reports the same as a status code
    q3.selftest_wait_timeout()
    st = q3.lib.q3cu_device_status(q3.ctx, None, None)
    assert st == 6                            # Q3CU_ERR_TIMEOUT
    # the context is still usable: a normal op, bit-exact
    rng = np.random.default_rng(1)
    x = rng.standard_normal((4, 2560), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(2560)).astype(np.float32)
    g = q3.rmsnorm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()).cpu().numpy()
    assert np.array_equal(g.view(np.uint32), oracle.rows_rmsnorm(x, w).view(np.uint32))
    assert q3.device_status() == 0
