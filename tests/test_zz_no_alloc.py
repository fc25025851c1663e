"""q3cu_execute_rmsnorm_static: the allocation-free executeRMSNorm.

Called through the C ABI and compared with q3cu_execute_rmsnorm (the context
entry point) on the same inputs, two calls in a row per size.  Both run the same
RMSNorm kernel, so the tolerance is zero: the outputs must be bit-identical.
The file name sorts last, so in a full run it executes after every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX = 16384          # Q3CU_STATIC_RMSNORM_MAX


@pytest.fixture(scope="module")
def static_rmsnorm(q3):
    fn = q3.lib.q3cu_execute_rmsnorm_static
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
    return fn


def _call(fn, out, x, w, size):
    return fn(out.ctypes.data, x.ctypes.data, w.ctypes.data, size, None)


@pytest.mark.parametrize("size", [2560, 1027, 5, MAX])
def test_static_matches_context_entry_point_twice(q3, static_rmsnorm, size):
    rng = np.random.default_rng(size)
    for call in range(2):
        x = (rng.standard_normal(size) * (1 + call)).astype(np.float32)
        w = (0.5 + rng.random(size)).astype(np.float32)
        want = np.empty(size, np.float32)
        got = np.full(size, np.nan, np.float32)
        q3.execute_rmsnorm(want, x, w)
        assert _call(static_rmsnorm, got, x, w, size) == 0, q3.lib.q3cu_last_error_string()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_static_rejects_sizes_beyond_the_limit(q3, static_rmsnorm):
    x = np.ones(MAX + 1, np.float32)
    out = np.full(MAX + 1, 7.0, np.float32)
    assert _call(static_rmsnorm, out, x, x, MAX + 1) == 1          # Q3CU_ERR_INVALID
    assert b"exceeds the limit" in q3.lib.q3cu_last_error_string()
    assert np.all(out == 7.0)
    assert _call(static_rmsnorm, out, x, x, 0) == 1
