"""The C ABI library: loads, exports every entry point that include/q3cu.h
declares, and validates arguments on the host (no kernel is launched here)."""
import ctypes as C
import os
import struct

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from metalqwen3_b200.build import build_library, library_path
    if not os.path.exists(library_path()):
        build_library()
    from metalqwen3_b200.q3cu import load_library
    return load_library()


def test_exports_every_declared_symbol(lib):
    from metalqwen3_b200.q3cu import header_functions
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared in include/q3cu.h but not exported: {missing}"


def test_cudacontext_symbols_exported():
    import subprocess
    from metalqwen3_b200.build import library_path
    syms = subprocess.run(["nm", "-D", "-C", library_path()], capture_output=True, text=True).stdout
    for m in ("CudaContext::executeRMSNorm", "CudaContext::executeSoftmax", "CudaContext::executeSwiGLU",
              "CudaContext::executeRoPE", "CudaContext::executeQuantize", "CudaContext::executeEmbedding",
              "CudaContext::initialize", "CudaContext::cleanup", "CudaContext::executeQuantizedMatMul",
              "CudaModel::CudaModel", "CudaModel::forward"):
        assert m in syms, m


CXX_PROGRAM = r'''
#include "CudaContext.h"
#include <cstdio>
#include <fstream>
#include <iterator>
#include <vector>
// The engine-side use of the C++ boundary: context, MetalContext-style calls, a model and its decode step.
int main(int argc, char **argv) {
    CudaContext ctx(0);
    if (!ctx.initialize()) { std::printf("%s\n", ctx.lastError().c_str()); return 2; }
    float x[64], w[64], o[64];
    for (int i = 0; i < 64; ++i) { x[i] = 0.1f * i; w[i] = 1.0f; }
    ctx.executeRMSNorm(o, x, w, 64);
    if (argc > 1) {
        std::ifstream f(argv[1], std::ios::binary);
        std::vector<char> img((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
        CudaModel m(ctx, img.data(), img.size());
        const float *logits = m.forward(1, 0);
        std::printf("%d %a\n", m.config().vocab_size, logits[0]);
    }
    return 0;
}
'''


def test_cpp_boundary_compiles_and_links(tmp_path):
    """An engine-side C++ program using CudaContext and CudaModel builds against the
    headers and links against libq3cu.so (running it needs a GPU)."""
    import subprocess
    from metalqwen3_b200.build import library_path
    src = tmp_path / "engine.cpp"
    src.write_text(CXX_PROGRAM)
    libdir = os.path.dirname(library_path())
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), str(src), "-o",
                    str(tmp_path / "engine"), "-L", libdir, "-lq3cu", f"-Wl,-rpath,{libdir}"], check=True)
    assert (tmp_path / "engine").exists()


ENGINE_CALL_SITES = r'''
#include "CudaContext.h"
#include <memory>
#include <stdexcept>
// The calls the reference engine makes on its backend object, with its member
// and argument names (src/metal/MetalQwen3.cpp: the error handler :56-57 and
// metal_rmsnorm / metal_softmax / metal_swiglu / metal_rope / metal_attention
// :479-639), compiled against CudaContext in place of MetalContext.
struct Engine {
    std::unique_ptr<CudaContext> metalContext;
    void on_error() {
        if (metalContext->isBatching()) {
            metalContext->endBatch();
        }
    }
    void rmsnorm(float *o, float *x, float *weight, int size) { metalContext->executeRMSNorm(o, x, weight, size); }
    void softmax(float *x, int size) { metalContext->executeSoftmax(x, size); }
    void swiglu(float *hb, float *hb2, int hidden_dim) { metalContext->executeSwiGLU(hb, hb2, hidden_dim); }
    void rope(float *q, float *k, int head_dim, int pos, int n_heads, int n_kv_heads, float *q_norm, float *k_norm) {
        metalContext->executeRoPE(q, k, head_dim, pos, n_heads, n_kv_heads, q_norm, k_norm);
    }
    void attention(float *xb, float *q, float *att, float *key_cache, float *value_cache, int pos, int head_dim,
                   int n_heads, int n_kv_heads, int seq_len, int kv_dim, uint64_t loff, int kv_mul) {
        metalContext->executeAttention(xb, q, att, key_cache, value_cache, pos, head_dim, n_heads, n_kv_heads,
                                       seq_len, kv_dim, loff, kv_mul);
    }
    void matmul(float *xout, int8_t *xq, float *xs, int8_t *wq, float *ws, int n, int d) {
        metalContext->executeQuantizedMatMul(xout, xq, xs, wq, ws, n, d, 64);
    }
};
int main() {
    Engine e;
    e.metalContext = std::make_unique<CudaContext>(0);
    e.metalContext->beginBatch();
    e.on_error();
    return e.metalContext->isInitialized() ? 1 : 0;
}
'''


def test_engine_call_sites_compile(tmp_path):
    """Every backend call of the reference engine compiles against CudaContext
    unchanged apart from the type name (the drop-in claim: only the member's
    type and the header change on the engine side)."""
    import subprocess
    from metalqwen3_b200.build import library_path
    src = tmp_path / "engine_calls.cpp"
    src.write_text(ENGINE_CALL_SITES)
    libdir = os.path.dirname(library_path())
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                    "-o", str(tmp_path / "engine_calls"), "-L", libdir, "-lq3cu", f"-Wl,-rpath,{libdir}"], check=True)
    syms = subprocess.run(["nm", "-D", "-C", library_path()], capture_output=True, text=True).stdout
    assert "CudaContext::executeAttention" in syms


def test_status_strings(lib):
    for s in range(11):
        assert lib.q3cu_status_string(s)
    assert lib.q3cu_version() >= 100


def test_null_context_is_rejected(lib):
    # every op checks the context before touching CUDA
    assert lib.q3cu_rmsnorm(None, None, 0, None, 1, 64, 1e-6, None, None) == 7
    assert lib.q3cu_rmsnorm_q8(None, None, 0, None, 1, 64, 1e-6, None, None, None) == 7
    assert lib.q3cu_swiglu_q8(None, None, None, 0, 1, 64, None, None, None) == 7
    assert lib.q3cu_softmax_rows(None, None, None, None, 1, None) == 7
    assert lib.q3cu_quantize_q8(None, None, 0, 1, 64, None, None, None) == 7
    assert lib.q3cu_embed_gather(None, None, None, 1, 64, None, 1, None, None, None, None) == 7
    assert lib.q3cu_execute_rmsnorm(None, None, None, None, 4) == 7
    assert lib.q3cu_destroy(None) == 7
    assert lib.q3cu_is_initialized(None) == 0
    assert b"context" in lib.q3cu_last_error_string()


def header(**kw):
    f = dict(magic=0x616A6331, version=1, dim=1024, hidden=3072, n_layers=28, n_heads=16, n_kv=8, vocab=151936,
             seq_len=64, head_dim=128, shared=1, gs=64)
    f.update(kw)
    return struct.pack("Iiiiiiiiiiii", f["magic"], f["version"], f["dim"], f["hidden"], f["n_layers"], f["n_heads"],
                       f["n_kv"], f["vocab"], f["seq_len"], f["head_dim"], f["shared"], f["gs"]) + b"\0" * 208


def test_check_header(lib):
    cfg = (C.c_int32 * 12)()
    h = header()
    assert lib.q3cu_check_header(h, len(h), cfg) == 0
    assert cfg[2] == 1024 and cfg[7] == 151936
    for bad in (header(magic=0x12345678), header(version=2), header(gs=32), header(n_kv=3)):
        assert lib.q3cu_check_header(bad, len(bad), None) == 10
    assert lib.q3cu_check_header(h, 20, None) == 10
    assert lib.q3cu_check_header(None, 0, None) == 1


def test_init_without_gpu_reports_device_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    assert lib.q3cu_init(0, C.byref(h)) == 9
    assert not h.value
