"""Checks of the fast arithmetic used by the Q8_0 epilogues, SwiGLU and RMSNorm.

* Q8_0 scale RN(wmax/127) by a Markstein correction step == IEEE division
  for every binary32 wmax in [2^-100, 2^100]  (CPU, exhaustive, fmaf);
* the bf16 RMSNorm chain's fused square: every bf16 value whose square is
  not exact in binary32 is caught by the kernel's guard (CPU, exhaustive);
* on the GPU (tests/native/check_device_math.cu, built with nvcc):
  the Markstein reciprocal == __frcp_rn for every binary32 d >= 1 (two
  steps) and every d in [1, 2^120) (one step); softmax's binary32 exp within
  1e-6 relative of exp on every binary32 d in [-80, 0], and its packed pair
  form bit-identical to it on the same range; and the
  multiply-by-reciprocal code path == the IEEE-division path on 2^20 random
  scales x values placed on and around every rounding tie.
"""
import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "metalqwen3_b200", "csrc")

DIV127 = r"""
#include <stdio.h>
#include <stdint.h>
#include <string.h>
#include <math.h>
int main(void) {
    const float c = 0x1.020408p-7f;
    long long bad = 0;
    #pragma omp parallel for reduction(+:bad) schedule(dynamic, 1 << 16)
    for (long long i = 0x0d800000LL; i <= 0x71800000LL; i++) {          /* 2^-100 .. 2^100 */
        uint32_t u = (uint32_t)i; float m; memcpy(&m, &u, 4);
        float s0 = m * c;
        float s = fmaf(fmaf(-s0, 127.0f, m), c, s0);
        float ref = m / 127.0f;
        uint32_t a, b; memcpy(&a, &s, 4); memcpy(&b, &ref, 4);
        if (a != b) bad++;
    }
    printf("%lld\n", bad);
    return 0;
}
"""


def test_scale_div127_exhaustive():
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "a.c"), os.path.join(d, "a")
        open(src, "w").write(DIV127)
        subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", src, "-o", exe, "-lm"], check=True)
        bad = int(subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()[0])
    assert bad == 0


def test_bf16_fused_square_guard_exhaustive():
    """The few-row RMSNorm kernel folds a bf16 row's squares as fma(v, v, acc),
    which rounds acc + v*v once where the reference rounds v*v and then the sum:
    the same bits whenever v*v is exact in binary32.  Over all 65,536 bf16
    values: every value whose square is not exact is caught by the kernel's
    guard (0 < |bits| < 0x2000, i.e. 0 < |v| < 2^-63), and the guard catches
    nothing else but values below 2^-63."""
    import numpy as np
    b = np.arange(1 << 16, dtype=np.uint32)
    v = (b << 16).view(np.float32)
    fin = np.isfinite(v)
    with np.errstate(over="ignore"):
        sq32 = (v[fin] * v[fin]).astype(np.float32)                   # RN(v*v) in binary32
        sq64 = v[fin].astype(np.float64) ** 2                        # exact (16-bit significand)
        exact = np.ones(b.size, bool)
        exact[fin] = (sq32.astype(np.float64) == sq64) | np.isinf(sq32)   # overflow: inf either way
    guard = ((b & 0x7FFF) - 1) < 0x1FFF                               # the kernel's predicate, per half word
    assert not np.any(~exact & ~guard), "a square that is not exact escapes the guard"
    assert np.all(np.abs(v[guard]) < 2.0 ** -63) and np.all(v[guard] != 0)
    assert np.any(~exact)                                             # the guard is needed


@pytest.mark.gpu
def test_fast_device_math_on_gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "check")
        subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "--fmad=false",
                        "-I", CSRC, "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "native", "check_device_math.cu"), "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=300).stdout.split()
    bad_rcp, bad_scale, bad_code, bad_rcp1, exp80_e12, bad_pair = map(int, out[:6])
    assert bad_pair == 0, f"{bad_pair} d in [-80, 0] where the packed exp differs from the scalar one"
    assert exp80_e12 < 1_000_000, f"softmax exp: relative error {exp80_e12 * 1e-12:.3g} on [-80, 0] (bound 1e-6)"
    assert bad_rcp == 0, f"{bad_rcp} binary32 d >= 1 where the Markstein reciprocal != __frcp_rn"
    assert bad_rcp1 == 0, f"{bad_rcp1} binary32 d in [1, 2^120) where the one-step reciprocal != __frcp_rn"
    assert bad_scale == 0, f"{bad_scale} scales differ from the IEEE quotient"
    assert bad_code == 0, f"{bad_code} codes differ between the fast and the exact path"
