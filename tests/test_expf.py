"""The device expf (metalqwen3_b200/csrc/q3_expf.h) against the host libm.

The header is plain C under a host compiler, so the same source that runs on
the GPU is compiled here (-ffp-contract=off, explicit fma()) and compared with
the C library's expf on every one of the 2^32 binary32 inputs.  The GPU build
of the same source is checked against the host on a 2^24-point sweep in
tests/test_gpu_parity.py::test_swiglu_expf_sweep.
"""
import os
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "metalqwen3_b200", "csrc")

HARNESS = r"""
#include <stdio.h>
#include <stdint.h>
#include <string.h>
#include <math.h>
#include "q3_expf.h"
static const uint64_t TAB[32] = Q3_EXP2_TAB32_INIT;
int main(void) {
    uint32_t HI[32], LO[32];
    for (int i = 0; i < 32; i++) { HI[i] = (uint32_t)(TAB[i] >> 32); LO[i] = (uint32_t)TAB[i]; }
    long long bad = 0, checked = 0, bad_fast = 0;
    #pragma omp parallel for reduction(+:bad,checked) schedule(dynamic, 1 << 16)
    for (long long i = 0; i < (1LL << 32); i++) {
        uint32_t u = (uint32_t)i; float x; memcpy(&x, &u, 4);
        float a = expf(x), b = q3_expf_tab(x, TAB), c = q3_expf_fast(x, HI, LO);
        uint32_t ua, ub, uc; memcpy(&ua, &a, 4); memcpy(&ub, &b, 4); memcpy(&uc, &c, 4);
        checked++;
        if (ua != ub && !(isnan(a) && isnan(b))) bad++;
        if (ua != uc && !(isnan(a) && isnan(c))) bad_fast++;
    }
    printf("%lld %lld %lld\n", checked, bad, bad_fast);
    return 0;
}
"""


def test_table_matches_generator():
    import importlib.util
    spec = importlib.util.spec_from_file_location("gen", os.path.join(CSRC, "gen_exp_table.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    text = open(os.path.join(CSRC, "q3_expf.h")).read()
    body = text.split("#define Q3_EXP2_TAB32_INIT {")[1].split("}")[0]
    vals = [int(t.strip().rstrip("ULL"), 16) for t in body.replace("\\", "").split(",") if t.strip()]
    assert vals == gen.table()


def test_expf_all_binary32_inputs():
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "h.c")
        exe = os.path.join(d, "h")
        open(src, "w").write(HARNESS)
        subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-I", CSRC, src, "-o", exe, "-lm"], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()
    checked, bad, bad_fast = int(out[0]), int(out[1]), int(out[2])
    assert checked == 1 << 32
    assert bad == 0, f"{bad} binary32 inputs where q3_expf_tab differs from the host expf"
    assert bad_fast == 0, f"{bad_fast} binary32 inputs where q3_expf_fast differs from the host expf"
