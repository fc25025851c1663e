// q3cu_api.cu -- the C ABI declared in include/q3cu.h.
//
// Host-side only: argument checks, the per-context device status word, the
// host frequency table for RoPE, kernel launches, and the synchronous
// host-pointer wrappers that keep MetalContext's execute* signatures
// (src/metal/MetalContext.h:78-87).  Where the reference exits or throws
// (src/metal/MetalContext.cpp:577-586, :738-754) this returns a status code.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "q3cu_internal.h"

// Softmax launches take their row counters from a ring of pairs (see
// launch_softmax below).
constexpr int SCHED_PAIRS = 64;

struct q3cu_ctx {
    int device = -1;
    int sms = 0;
    uint32_t *d_status = nullptr;           // device status word (Q3CU_DEV_* bits)
    uint32_t *d_sched = nullptr;            // SCHED_PAIRS softmax counter pairs, zero between launches
    cudaEvent_t sched_ev[SCHED_PAIRS] = {}; // the latest launch on each pair
    uint32_t sched_next = 0;
    std::mutex sched_mu;
    cudaStream_t stream = nullptr;          // the host-pointer wrappers' stream
    void *d_scratch = nullptr;              // staging for the host-pointer wrappers
    size_t scratch_bytes = 0;
    std::map<std::pair<int, uint32_t>, q3::InvFreq> inv_freq;   // (head_dim, bits of theta)
    bool alive = false;
};

namespace {

thread_local char g_err[512] = "";

q3cu_status fail(q3cu_status s, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return s;
}

q3cu_status cuda_fail(cudaError_t e, const char *what) {
    return fail(e == cudaErrorMemoryAllocation ? Q3CU_ERR_OOM : Q3CU_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CHECK_CTX(ctx)                                                                       \
    do {                                                                                     \
        if (!(ctx) || !(ctx)->alive) return fail(Q3CU_ERR_NOT_INIT, "context is NULL or destroyed"); \
    } while (0)

q3cu_status use_device(q3cu_ctx *ctx) {
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != ctx->device) {
        e = cudaSetDevice(ctx->device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    }
    return Q3CU_OK;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t esize(q3cu_dtype dt) { return dt == Q3CU_F32 ? 4 : 2; }

q3cu_status check_dtype(q3cu_dtype dt) {
    if (dt != Q3CU_F32 && dt != Q3CU_BF16) return fail(Q3CU_ERR_INVALID, "unknown dtype %d", int(dt));
    return Q3CU_OK;
}

q3cu_status launched(cudaError_t e, const char *what) {
    if (e != cudaSuccess) return cuda_fail(e, what);
    return Q3CU_OK;
}

// freq_j = powf(theta, -(float)j / (head_dim/2)): the expression of
// src/cpu/qwen3_original.c:367/:384 (theta = 1e6 there), evaluated with the host
// C library so that the angle pos*freq_j matches the reference bit for bit.
const q3::InvFreq &inv_freq_for(q3cu_ctx *ctx, int head_dim, float theta) {
    uint32_t tb;
    std::memcpy(&tb, &theta, 4);
    auto key = std::make_pair(head_dim, tb);
    auto it = ctx->inv_freq.find(key);
    if (it != ctx->inv_freq.end()) return it->second;
    q3::InvFreq f{};
    const int half = head_dim / 2;
    for (int j = 0; j < half && j < 64; ++j) f.v[j] = powf(theta, -(float)j / half);
    return ctx->inv_freq.emplace(key, f).first->second;
}

// The softmax kernel balances rows across SMs with a pair of device counters
// that must be zero at launch; the kernel's last CTA zeroes them again.  Each
// launch takes the next pair of a ring of SCHED_PAIRS, and the stream first
// waits for the previous launch on that pair (its event), so launches on
// different streams never share a pair while running.  Inside a stream capture
// the wait and record are left out (the event was recorded outside the
// capture); the captured launch keeps its pair.
q3cu_status launch_softmax(q3cu_ctx *ctx, float *x, const int64_t *off, const int32_t *len, int64_t rows,
                           cudaStream_t stream) {
    if (rows == 0) return Q3CU_OK;
    std::lock_guard<std::mutex> lock(ctx->sched_mu);
    const uint32_t i = ctx->sched_next++ % SCHED_PAIRS;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(stream, &cs);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
    const bool eager = cs == cudaStreamCaptureStatusNone;
    if (eager && (e = cudaStreamWaitEvent(stream, ctx->sched_ev[i], 0)) != cudaSuccess)
        return cuda_fail(e, "cudaStreamWaitEvent");
    e = q3::launch_softmax_rows(x, off, len, rows, ctx->d_sched + size_t(i) * q3::SMX_SCHED_WORDS, ctx->d_status,
                                stream, ctx->sms);
    if (e != cudaSuccess) return cuda_fail(e, "softmax launch");
    if (eager && (e = cudaEventRecord(ctx->sched_ev[i], stream)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    return Q3CU_OK;
}

q3cu_status grow_scratch(q3cu_ctx *ctx, size_t bytes) {
    if (bytes <= ctx->scratch_bytes) return Q3CU_OK;
    if (ctx->d_scratch) cudaFree(ctx->d_scratch);
    ctx->d_scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    cudaError_t e = cudaMalloc(&ctx->d_scratch, want);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (host-pointer staging)");
    ctx->scratch_bytes = want;
    return Q3CU_OK;
}

size_t up16(size_t b) { return (b + 15) & ~size_t(15); }
size_t up32(size_t b) { return (b + 31) & ~size_t(31); }

}  // namespace

namespace q3 {
cudaError_t ensure_smem_attr(const void *kernel, size_t bytes, int slot) {
    static std::atomic<uint32_t> done[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || slot < 0 || slot >= 32) return cudaErrorInvalidValue;
    const uint32_t bit = 1u << slot;
    if (done[dev].load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    if (e == cudaSuccess) done[dev].fetch_or(bit, std::memory_order_release);
    return e;
}

q3cu_status set_error(q3cu_status s, const char *msg) { return fail(s, "%s", msg); }
bool ctx_alive(const q3cu_ctx *ctx) { return ctx && ctx->alive; }
q3cu_status ctx_use_device(q3cu_ctx *ctx) { return use_device(ctx); }
int ctx_sms(const q3cu_ctx *ctx) { return ctx->sms; }
uint32_t *ctx_status_word(const q3cu_ctx *ctx) { return ctx->d_status; }
}  // namespace q3

extern "C" {

int q3cu_version(void) { return 100; }

const char *q3cu_last_error_string(void) { return g_err; }

const char *q3cu_status_string(q3cu_status s) {
    switch (s) {
        case Q3CU_OK: return "ok";
        case Q3CU_ERR_INVALID: return "invalid argument";
        case Q3CU_ERR_ALIGN: return "misaligned pointer or row";
        case Q3CU_ERR_GROUP: return "length not a multiple of the Q8_0 group size (64)";
        case Q3CU_ERR_CUDA: return "CUDA runtime error";
        case Q3CU_ERR_INDEX: return "token id out of range";
        case Q3CU_ERR_TIMEOUT: return "device wait timed out";
        case Q3CU_ERR_NOT_INIT: return "context not initialised";
        case Q3CU_ERR_OOM: return "out of memory";
        case Q3CU_ERR_DEVICE: return "unsupported or missing device";
        case Q3CU_ERR_FORMAT: return "bad checkpoint header";
    }
    return "unknown status";
}

q3cu_status q3cu_init(int device, q3cu_ctx **out) {
    if (!out) return fail(Q3CU_ERR_INVALID, "q3cu_init: out is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return fail(Q3CU_ERR_DEVICE, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    if (device < 0 || device >= n) return fail(Q3CU_ERR_DEVICE, "device %d not present (%d devices)", device, n);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(Q3CU_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", device,
                    prop.major, prop.minor);
    auto *ctx = new (std::nothrow) q3cu_ctx();
    if (!ctx) return fail(Q3CU_ERR_OOM, "host allocation of the context failed");
    ctx->device = device;
    ctx->sms = prop.multiProcessorCount;
    int prev = 0;
    cudaGetDevice(&prev);
    e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_status, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    const size_t sched_bytes = size_t(SCHED_PAIRS) * q3::SMX_SCHED_WORDS * sizeof(uint32_t);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_sched, sched_bytes);
    if (e == cudaSuccess) e = cudaMemset(ctx->d_sched, 0, sched_bytes);
    for (int i = 0; i < SCHED_PAIRS && e == cudaSuccess; ++i)
        e = cudaEventCreateWithFlags(&ctx->sched_ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) {
        for (int i = 0; i < SCHED_PAIRS; ++i)
            if (ctx->sched_ev[i]) cudaEventDestroy(ctx->sched_ev[i]);
        if (ctx->d_sched) cudaFree(ctx->d_sched);
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        if (ctx->d_status) cudaFree(ctx->d_status);
        cudaSetDevice(prev);
        delete ctx;
        return cuda_fail(e, "q3cu_init");
    }
    cudaSetDevice(prev);
    ctx->alive = true;
    *out = ctx;
    return Q3CU_OK;
}

q3cu_status q3cu_destroy(q3cu_ctx *ctx) {
    CHECK_CTX(ctx);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->d_scratch) cudaFree(ctx->d_scratch);
    for (int i = 0; i < SCHED_PAIRS; ++i) {
        if (ctx->sched_ev[i]) cudaEventSynchronize(ctx->sched_ev[i]);
        if (ctx->sched_ev[i]) cudaEventDestroy(ctx->sched_ev[i]);
    }
    if (ctx->d_sched) cudaFree(ctx->d_sched);
    if (ctx->d_status) cudaFree(ctx->d_status);
    cudaSetDevice(prev);
    ctx->alive = false;
    delete ctx;
    return Q3CU_OK;
}

int q3cu_is_initialized(const q3cu_ctx *ctx) { return ctx && ctx->alive ? 1 : 0; }

q3cu_status q3cu_selftest_wait_timeout(q3cu_ctx *ctx, q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (q3cu_status st = use_device(ctx)) return st;
    return launched(q3::launch_selftest_wait(ctx->d_status, static_cast<cudaStream_t>(stream)),
                    "wait-timeout self-test launch");
}

q3cu_status q3cu_device_status(q3cu_ctx *ctx, q3cu_stream stream, uint32_t *flags) {
    CHECK_CTX(ctx);
    q3cu_status st = use_device(ctx);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    uint32_t h = 0;
    e = cudaMemcpy(&h, ctx->d_status, sizeof(h), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && h) e = cudaMemset(ctx->d_status, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
    if (flags) *flags = h;
    if (h & Q3CU_DEV_TIMEOUT) return fail(Q3CU_ERR_TIMEOUT, "a device-side wait gave up (status 0x%x)", h);
    if (h & Q3CU_DEV_BAD_INDEX) return fail(Q3CU_ERR_INDEX, "a token id was out of range (status 0x%x)", h);
    return Q3CU_OK;
}

q3cu_status q3cu_check_header(const void *header, size_t bytes, q3cu_config *out) {
    if (!header) return fail(Q3CU_ERR_INVALID, "header is NULL");
    if (bytes < sizeof(q3cu_config)) return fail(Q3CU_ERR_FORMAT, "header shorter than %zu bytes", sizeof(q3cu_config));
    q3cu_config c;
    std::memcpy(&c, header, sizeof(c));
    if (uint32_t(c.magic_number) != 0x616a6331u) return fail(Q3CU_ERR_FORMAT, "bad magic 0x%08x", uint32_t(c.magic_number));
    if (c.version != 1) return fail(Q3CU_ERR_FORMAT, "checkpoint version %d, need 1", c.version);
    if (c.group_size != Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_FORMAT, "group size %d, need 64", c.group_size);
    if (c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
        c.vocab_size <= 0 || c.seq_len <= 0 || c.head_dim <= 0 || c.n_heads % c.n_kv_heads != 0)
        return fail(Q3CU_ERR_FORMAT, "non-positive or inconsistent shape fields");
    if (out) *out = c;
    return Q3CU_OK;
}

// ---------------------------------------------------------------------------
// device-pointer ops
// ---------------------------------------------------------------------------

static q3cu_status rms_common(q3cu_ctx *ctx, const void *x, q3cu_dtype dt, const float *w, int64_t rows, int dim,
                              bool q8, const void *out, const int8_t *q, const float *s) {
    CHECK_CTX(ctx);
    if (q3cu_status st = check_dtype(dt)) return st;
    if (rows < 0 || dim <= 0) return fail(Q3CU_ERR_INVALID, "rows=%lld dim=%d", (long long)rows, dim);
    if (rows > 0 && (!x || !w)) return fail(Q3CU_ERR_INVALID, "x or w is NULL");
    if (q8 && rows > 0 && (!q || !s)) return fail(Q3CU_ERR_INVALID, "q or s is NULL");
    if (!q8 && rows > 0 && !out) return fail(Q3CU_ERR_INVALID, "out is NULL");
    if (q8 && dim % Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_GROUP, "dim %d is not a multiple of 64", dim);
    if ((size_t(dim) * esize(dt)) % 16) return fail(Q3CU_ERR_ALIGN, "dim * sizeof(dtype) must be a multiple of 16");
    if (!aligned(x, 16) || !aligned(w, 16) || (!q8 && !aligned(out, 16)))
        return fail(Q3CU_ERR_ALIGN, "x, w and out must be 16-byte aligned");
    if (q8 && (!aligned(q, dt == Q3CU_F32 ? 4 : 8) || !aligned(s, 4)))
        return fail(Q3CU_ERR_ALIGN, "q must be %d-byte aligned, s 4-byte aligned", dt == Q3CU_F32 ? 4 : 8);
    return use_device(ctx);
}

q3cu_status q3cu_rmsnorm(q3cu_ctx *ctx, const void *x, q3cu_dtype dtype, const float *w, int64_t rows, int dim,
                         float eps, void *out, q3cu_stream stream) {
    if (q3cu_status st = rms_common(ctx, x, dtype, w, rows, dim, false, out, nullptr, nullptr)) return st;
    return launched(q3::launch_rmsnorm(x, dtype, w, rows, dim, eps, out, nullptr, nullptr, ctx->d_status,
                                       static_cast<cudaStream_t>(stream), ctx->sms),
                    "rmsnorm launch");
}

q3cu_status q3cu_rmsnorm_q8(q3cu_ctx *ctx, const void *x, q3cu_dtype dtype, const float *w, int64_t rows, int dim,
                            float eps, int8_t *q, float *s, q3cu_stream stream) {
    if (q3cu_status st = rms_common(ctx, x, dtype, w, rows, dim, true, nullptr, q, s)) return st;
    return launched(q3::launch_rmsnorm(x, dtype, w, rows, dim, eps, nullptr, q, s, ctx->d_status,
                                       static_cast<cudaStream_t>(stream), ctx->sms),
                    "rmsnorm_q8 launch");
}

q3cu_status q3cu_qk_norm_rope(q3cu_ctx *ctx, void *q, void *k, q3cu_dtype dtype, const int32_t *pos, int64_t rows,
                              int n_heads, int n_kv, int head_dim, const float *q_norm, const float *k_norm,
                              float theta, float eps, q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (q3cu_status st = check_dtype(dtype)) return st;
    if (head_dim != 128) return fail(Q3CU_ERR_INVALID, "head_dim %d: only 128 is supported", head_dim);
    if (rows < 0 || n_heads < 0 || n_kv < 0) return fail(Q3CU_ERR_INVALID, "negative size");
    if (rows > 0 && ((n_heads > 0 && (!q || !q_norm)) || (n_kv > 0 && (!k || !k_norm)) || !pos))
        return fail(Q3CU_ERR_INVALID, "NULL pointer");
    if ((q && !aligned(q, 16)) || (k && !aligned(k, 16)) || (q_norm && !aligned(q_norm, 8)) ||
        (k_norm && !aligned(k_norm, 8)) || !aligned(pos, 4))
        return fail(Q3CU_ERR_ALIGN, "q and k must be 16-byte aligned, norm weights 8-byte aligned");
    if (!(theta > 0.0f)) return fail(Q3CU_ERR_INVALID, "theta must be positive");
    if (q3cu_status st = use_device(ctx)) return st;
    const q3::InvFreq &f = inv_freq_for(ctx, head_dim, theta);
    return launched(q3::launch_qk_norm_rope(q, k, dtype, pos, rows, n_heads, n_kv, q_norm, k_norm, f, eps,
                                            ctx->d_status, static_cast<cudaStream_t>(stream), ctx->sms),
                    "qk_norm_rope launch");
}

static q3cu_status swiglu_common(q3cu_ctx *ctx, const void *hb, const void *hb2, q3cu_dtype dt, int64_t rows,
                                 int hidden, bool q8, const int8_t *q, const float *s) {
    CHECK_CTX(ctx);
    if (q3cu_status st = check_dtype(dt)) return st;
    if (rows < 0 || hidden <= 0) return fail(Q3CU_ERR_INVALID, "rows=%lld hidden=%d", (long long)rows, hidden);
    if (rows > 0 && (!hb || !hb2)) return fail(Q3CU_ERR_INVALID, "hb or hb2 is NULL");
    if (q8 && rows > 0 && (!q || !s)) return fail(Q3CU_ERR_INVALID, "q or s is NULL");
    if (q8 && hidden % Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_GROUP, "hidden %d is not a multiple of 64", hidden);
    if ((size_t(hidden) * esize(dt)) % 16) return fail(Q3CU_ERR_ALIGN, "hidden * sizeof(dtype) must be a multiple of 16");
    if (!aligned(hb, 16) || !aligned(hb2, 16)) return fail(Q3CU_ERR_ALIGN, "hb and hb2 must be 16-byte aligned");
    if (q8 && (!aligned(q, dt == Q3CU_F32 ? 4 : 8) || !aligned(s, 4)))
        return fail(Q3CU_ERR_ALIGN, "q or s misaligned");
    return use_device(ctx);
}

q3cu_status q3cu_swiglu(q3cu_ctx *ctx, void *hb, const void *hb2, q3cu_dtype dtype, int64_t rows, int hidden,
                        q3cu_stream stream) {
    if (q3cu_status st = swiglu_common(ctx, hb, hb2, dtype, rows, hidden, false, nullptr, nullptr)) return st;
    return launched(q3::launch_swiglu(hb, hb2, dtype, rows * int64_t(hidden), hb, nullptr, nullptr, ctx->d_status,
                                      static_cast<cudaStream_t>(stream), ctx->sms),
                    "swiglu launch");
}

q3cu_status q3cu_swiglu_q8(q3cu_ctx *ctx, const void *hb, const void *hb2, q3cu_dtype dtype, int64_t rows, int hidden,
                           int8_t *q, float *s, q3cu_stream stream) {
    if (q3cu_status st = swiglu_common(ctx, hb, hb2, dtype, rows, hidden, true, q, s)) return st;
    return launched(q3::launch_swiglu(hb, hb2, dtype, rows * int64_t(hidden), nullptr, q, s, ctx->d_status,
                                      static_cast<cudaStream_t>(stream), ctx->sms),
                    "swiglu_q8 launch");
}

q3cu_status q3cu_softmax_rows(q3cu_ctx *ctx, float *x, const int64_t *row_off, const int32_t *row_len, int64_t rows,
                              q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (rows < 0) return fail(Q3CU_ERR_INVALID, "rows < 0");
    if (rows > 0 && (!x || !row_off || !row_len)) return fail(Q3CU_ERR_INVALID, "NULL pointer");
    if (!aligned(x, 4) || !aligned(row_off, 8) || !aligned(row_len, 4)) return fail(Q3CU_ERR_ALIGN, "misaligned array");
    if (q3cu_status st = use_device(ctx)) return st;
    return launch_softmax(ctx, x, row_off, row_len, rows, static_cast<cudaStream_t>(stream));
}

q3cu_status q3cu_quantize_q8(q3cu_ctx *ctx, const void *x, q3cu_dtype dtype, int64_t rows, int n, int8_t *q, float *s,
                             q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (q3cu_status st = check_dtype(dtype)) return st;
    if (rows < 0 || n <= 0) return fail(Q3CU_ERR_INVALID, "rows=%lld n=%d", (long long)rows, n);
    if (n % Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_GROUP, "n %d is not a multiple of 64", n);
    if (rows > 0 && (!x || !q || !s)) return fail(Q3CU_ERR_INVALID, "NULL pointer");
    if (!aligned(x, 16) || !aligned(q, dtype == Q3CU_F32 ? 4 : 8) || !aligned(s, 4))
        return fail(Q3CU_ERR_ALIGN, "x must be 16-byte aligned");
    if (q3cu_status st = use_device(ctx)) return st;
    return launched(q3::launch_quantize_q8(x, dtype, rows * int64_t(n), q, s, static_cast<cudaStream_t>(stream),
                                           ctx->sms),
                    "quantize launch");
}

q3cu_status q3cu_dequantize_q8(q3cu_ctx *ctx, const int8_t *q, const float *s, int64_t n, float *x, q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (n < 0) return fail(Q3CU_ERR_INVALID, "n < 0");
    if (n % Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_GROUP, "n is not a multiple of 64");
    if (n > 0 && (!q || !s || !x)) return fail(Q3CU_ERR_INVALID, "NULL pointer");
    if (!aligned(q, 16) || !aligned(x, 16) || !aligned(s, 4)) return fail(Q3CU_ERR_ALIGN, "q and x must be 16-byte aligned");
    if (q3cu_status st = use_device(ctx)) return st;
    return launched(q3::launch_dequantize_q8(q, s, n, x, static_cast<cudaStream_t>(stream), ctx->sms),
                    "dequantize launch");
}

q3cu_status q3cu_embed_gather(q3cu_ctx *ctx, const int8_t *tq, const float *ts, int vocab, int dim, const int32_t *ids,
                              int64_t n, float *out_f32, int8_t *out_q, float *out_s, q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (vocab <= 0 || dim <= 0 || n < 0) return fail(Q3CU_ERR_INVALID, "vocab=%d dim=%d n=%lld", vocab, dim, (long long)n);
    if (dim % Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_GROUP, "dim %d is not a multiple of 64", dim);
    if ((out_q == nullptr) != (out_s == nullptr)) return fail(Q3CU_ERR_INVALID, "out_q and out_s must both be set or both NULL");
    if (!out_f32 && !out_q) return fail(Q3CU_ERR_INVALID, "no output requested");
    if (n > 0 && (!tq || !ts || !ids)) return fail(Q3CU_ERR_INVALID, "NULL pointer");
    if (!aligned(tq, 16) || !aligned(ts, 4) || !aligned(ids, 4) || (out_f32 && !aligned(out_f32, 16)) ||
        (out_q && !aligned(out_q, 16)) || (out_s && !aligned(out_s, 4)))
        return fail(Q3CU_ERR_ALIGN, "table codes and outputs must be 16-byte aligned");
    if (q3cu_status st = use_device(ctx)) return st;
    return launched(q3::launch_embed_gather(tq, ts, vocab, dim, ids, n, out_f32, out_q, out_s, ctx->d_status,
                                            static_cast<cudaStream_t>(stream), ctx->sms),
                    "embed_gather launch");
}

q3cu_status q3cu_matmul_q8(q3cu_ctx *ctx, const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws,
                           int n, int d, float *out, q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (B < 0 || n <= 0 || d < 0) return fail(Q3CU_ERR_INVALID, "B=%d n=%d d=%d", B, n, d);
    if (n % Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_GROUP, "n %d is not a multiple of 64", n);
    if (B > 0 && d > 0 && (!xq || !xs || !wq || !ws || !out)) return fail(Q3CU_ERR_INVALID, "NULL pointer");
    if (!aligned(xq, 32) || !aligned(wq, 32) || !aligned(xs, 4) || !aligned(ws, 4) || !aligned(out, 4))
        return fail(Q3CU_ERR_ALIGN, "xq and wq must be 32-byte aligned, xs, ws and out 4-byte aligned");
    if (q3cu_status st = use_device(ctx)) return st;
    if (q3::matmul_q8_tc_supported(B, n, d))               // prefill batches: the tensor-core kernel
        return launched(q3::launch_matmul_q8_tc(xq, xs, B, wq, ws, n, d, out, ctx->d_status,
                                                static_cast<cudaStream_t>(stream), ctx->sms),
                        "matmul_q8 (tensor cores) launch");
    return launched(q3::launch_matmul_q8(xq, xs, B, wq, ws, n, d, out, static_cast<cudaStream_t>(stream), ctx->sms),
                    "matmul_q8 launch");
}

static q3cu_status check_attention(const float *q, const float *kc, const float *vc, int pos, int n_heads,
                                   int kv_dim, int kv_mul, const float *att, int att_stride, const float *xb) {
    if (!q || !kc || !vc || !att || !xb || pos < 0 || n_heads <= 0 || kv_mul <= 0 || att_stride <= pos)
        return fail(Q3CU_ERR_INVALID, "attention: bad argument (pos=%d n_heads=%d kv_mul=%d att_stride=%d)", pos,
                    n_heads, kv_mul, att_stride);
    if (int64_t(kv_dim) < int64_t((n_heads - 1) / kv_mul + 1) * 128)
        return fail(Q3CU_ERR_INVALID, "attention: kv_dim %d holds fewer than the %d kv heads of 128 used", kv_dim,
                    (n_heads - 1) / kv_mul + 1);
    if (kv_dim % 4 || !aligned(kc, 16) || !aligned(vc, 16) || !aligned(q, 4) || !aligned(att, 4) || !aligned(xb, 4))
        return fail(Q3CU_ERR_ALIGN, "attention: caches 16-byte aligned with kv_dim %% 4 == 0");
    return Q3CU_OK;
}

q3cu_status q3cu_attention(q3cu_ctx *ctx, const float *q, const float *key_cache, const float *value_cache, int pos,
                           int n_heads, int kv_dim, int kv_mul, float *att, int att_stride, float *probs, float *xb,
                           q3cu_stream stream) {
    CHECK_CTX(ctx);
    if (q3cu_status st = check_attention(q, key_cache, value_cache, pos, n_heads, kv_dim, kv_mul, att, att_stride, xb))
        return st;
    if (probs == att || (probs && !aligned(probs, 4)))
        return fail(Q3CU_ERR_INVALID, "attention: probs must be NULL or a 4-byte aligned buffer other than att");
    if (q3cu_status st = use_device(ctx)) return st;
    return launched(q3::launch_attention_rows(q, key_cache, value_cache, att, probs, xb, pos, n_heads, kv_dim, kv_mul,
                                              att_stride, static_cast<cudaStream_t>(stream), ctx->sms),
                    "attention launch");
}

// ---------------------------------------------------------------------------
// host-pointer drop-in wrappers (synchronous)
// ---------------------------------------------------------------------------
#define TRY_CUDA(expr, what)                                   \
    do {                                                       \
        cudaError_t e_ = (expr);                               \
        if (e_ != cudaSuccess) return cuda_fail(e_, what);     \
    } while (0)

static q3cu_status finish(q3cu_ctx *ctx) {
    TRY_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return q3cu_device_status(ctx, ctx->stream, nullptr);
}

q3cu_status q3cu_execute_rmsnorm(q3cu_ctx *ctx, float *output, const float *input, const float *weight, int size) {
    CHECK_CTX(ctx);
    if (!output || !input || !weight || size <= 0) return fail(Q3CU_ERR_INVALID, "executeRMSNorm: bad argument");
    if (q3cu_status st = use_device(ctx)) return st;
    // Pad the row to a multiple of 4 floats with zeros: the kernel sums x*x over
    // the padded row (adding +0 leaves the sum unchanged) and divides by `size`.
    const int padded = (size + 3) & ~3;
    const size_t rb = up16(size_t(padded) * 4);
    if (q3cu_status st = grow_scratch(ctx, 3 * rb)) return st;
    auto *d = static_cast<uint8_t *>(ctx->d_scratch);
    float *dx = reinterpret_cast<float *>(d), *dw = reinterpret_cast<float *>(d + rb),
          *dout = reinterpret_cast<float *>(d + 2 * rb);
    if (padded != size) TRY_CUDA(cudaMemsetAsync(d, 0, 2 * rb, ctx->stream), "memset");
    TRY_CUDA(cudaMemcpyAsync(dx, input, size_t(size) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dw, weight, size_t(size) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(q3::launch_rmsnorm_padded(dx, dw, size, padded, dout, ctx->d_status, ctx->stream, ctx->sms), "rmsnorm");
    TRY_CUDA(cudaMemcpyAsync(output, dout, size_t(size) * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

q3cu_status q3cu_execute_softmax(q3cu_ctx *ctx, float *x, int size) {
    CHECK_CTX(ctx);
    if (!x || size < 0) return fail(Q3CU_ERR_INVALID, "executeSoftmax: bad argument");
    if (size == 0) return Q3CU_OK;
    if (q3cu_status st = use_device(ctx)) return st;
    const size_t xb = up16(size_t(size) * 4);
    if (q3cu_status st = grow_scratch(ctx, xb + 16)) return st;
    auto *d = static_cast<uint8_t *>(ctx->d_scratch);
    float *dx = reinterpret_cast<float *>(d);
    int64_t *doff = reinterpret_cast<int64_t *>(d + xb);
    int32_t *dlen = reinterpret_cast<int32_t *>(d + xb + 8);
    const int64_t off = 0;
    const int32_t len = size;
    TRY_CUDA(cudaMemcpyAsync(dx, x, size_t(size) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(doff, &off, 8, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dlen, &len, 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    if (q3cu_status st = launch_softmax(ctx, dx, doff, dlen, 1, ctx->stream)) return st;
    TRY_CUDA(cudaMemcpyAsync(x, dx, size_t(size) * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

q3cu_status q3cu_execute_swiglu(q3cu_ctx *ctx, float *hb, const float *hb2, int hidden_dim) {
    CHECK_CTX(ctx);
    if (!hb || !hb2 || hidden_dim <= 0) return fail(Q3CU_ERR_INVALID, "executeSwiGLU: bad argument");
    if (q3cu_status st = use_device(ctx)) return st;
    const int padded = (hidden_dim + 3) & ~3;           // zero tail: silu(0)*0 = 0, discarded
    const size_t rb = up16(size_t(padded) * 4);
    if (q3cu_status st = grow_scratch(ctx, 2 * rb)) return st;
    auto *d = static_cast<uint8_t *>(ctx->d_scratch);
    float *da = reinterpret_cast<float *>(d), *db = reinterpret_cast<float *>(d + rb);
    if (padded != hidden_dim) TRY_CUDA(cudaMemsetAsync(d, 0, 2 * rb, ctx->stream), "memset");
    TRY_CUDA(cudaMemcpyAsync(da, hb, size_t(hidden_dim) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(db, hb2, size_t(hidden_dim) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(q3::launch_swiglu(da, db, Q3CU_F32, padded, da, nullptr, nullptr, ctx->d_status, ctx->stream, ctx->sms),
             "swiglu");
    TRY_CUDA(cudaMemcpyAsync(hb, da, size_t(hidden_dim) * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

q3cu_status q3cu_execute_rope(q3cu_ctx *ctx, float *q, float *k, int head_dim, int pos, int n_heads, int n_kv_heads,
                              const float *q_norm_weights, const float *k_norm_weights) {
    CHECK_CTX(ctx);
    if (!q || !k || !q_norm_weights || !k_norm_weights || n_heads < 0 || n_kv_heads < 0)
        return fail(Q3CU_ERR_INVALID, "executeRoPE: bad argument");
    if (head_dim != 128) return fail(Q3CU_ERR_INVALID, "executeRoPE: head_dim %d, only 128 is supported", head_dim);
    if (q3cu_status st = use_device(ctx)) return st;
    const size_t qb = up16(size_t(n_heads) * head_dim * 4), kb = up16(size_t(n_kv_heads) * head_dim * 4);
    const size_t wb = up16(size_t(head_dim) * 4);
    if (q3cu_status st = grow_scratch(ctx, qb + kb + 2 * wb + 16)) return st;
    auto *d = static_cast<uint8_t *>(ctx->d_scratch);
    float *dq = reinterpret_cast<float *>(d), *dk = reinterpret_cast<float *>(d + qb);
    float *dqn = reinterpret_cast<float *>(d + qb + kb), *dkn = reinterpret_cast<float *>(d + qb + kb + wb);
    int32_t *dpos = reinterpret_cast<int32_t *>(d + qb + kb + 2 * wb);
    TRY_CUDA(cudaMemcpyAsync(dq, q, size_t(n_heads) * head_dim * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dk, k, size_t(n_kv_heads) * head_dim * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dqn, q_norm_weights, size_t(head_dim) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dkn, k_norm_weights, size_t(head_dim) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dpos, &pos, 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaStreamSynchronize(ctx->stream), "sync");      // &pos is a stack address
    const q3::InvFreq &f = inv_freq_for(ctx, head_dim, 1e6f);  // the reference's theta
    TRY_CUDA(q3::launch_qk_norm_rope(dq, dk, Q3CU_F32, dpos, 1, n_heads, n_kv_heads, dqn, dkn, f, 1e-6f,
                                     ctx->d_status, ctx->stream, ctx->sms), "qk_norm_rope");
    TRY_CUDA(cudaMemcpyAsync(q, dq, size_t(n_heads) * head_dim * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    TRY_CUDA(cudaMemcpyAsync(k, dk, size_t(n_kv_heads) * head_dim * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

q3cu_status q3cu_execute_attention(q3cu_ctx *ctx, float *xb, const float *q, float *att, float *key_cache,
                                   float *value_cache, int pos, int head_dim, int n_heads, int n_kv_heads,
                                   int seq_len, int kv_dim, uint64_t loff, int kv_mul) {
    CHECK_CTX(ctx);
    if (head_dim != 128) return fail(Q3CU_ERR_INVALID, "executeAttention: head_dim %d, only 128 is supported", head_dim);
    if (n_kv_heads <= 0 || seq_len <= pos || kv_mul <= 0 || (n_heads - 1) / kv_mul >= n_kv_heads)
        return fail(Q3CU_ERR_INVALID, "executeAttention: bad argument (pos=%d seq_len=%d n_heads=%d n_kv=%d kv_mul=%d)",
                    pos, seq_len, n_heads, n_kv_heads, kv_mul);
    // The layer's rows 0..pos are staged on the device as they lie in the host
    // cache (row stride kv_dim, padded to a multiple of 4 floats for 16-byte
    // rows); the probabilities come back into att's columns 0..pos.
    const int npos = pos + 1, kvp = (kv_dim + 3) & ~3;
    const size_t qb = up16(size_t(n_heads) * 128 * 4), cb = up16(size_t(npos) * kvp * 4),
                 ab = up16(size_t(n_heads) * npos * 4);          // scores, then the probabilities
    if (!xb || !q || !att || !key_cache || !value_cache || n_heads <= 0 || int64_t(kv_dim) < int64_t(n_kv_heads) * 128)
        return fail(Q3CU_ERR_INVALID, "executeAttention: bad argument (n_heads=%d kv_dim=%d n_kv=%d)", n_heads, kv_dim,
                    n_kv_heads);
    if (q3cu_status st = use_device(ctx)) return st;
    if (q3cu_status st = grow_scratch(ctx, qb + 2 * cb + 2 * ab + qb)) return st;
    auto *d = static_cast<uint8_t *>(ctx->d_scratch);
    float *dq = reinterpret_cast<float *>(d), *dk = reinterpret_cast<float *>(d + qb),
          *dv = reinterpret_cast<float *>(d + qb + cb), *da = reinterpret_cast<float *>(d + qb + 2 * cb),
          *dp = reinterpret_cast<float *>(d + qb + 2 * cb + ab), *dx = reinterpret_cast<float *>(d + qb + 2 * cb + 2 * ab);
    TRY_CUDA(cudaMemcpyAsync(dq, q, size_t(n_heads) * 128 * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpy2DAsync(dk, size_t(kvp) * 4, key_cache + loff, size_t(kv_dim) * 4, size_t(kv_dim) * 4, npos,
                               cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpy2DAsync(dv, size_t(kvp) * 4, value_cache + loff, size_t(kv_dim) * 4, size_t(kv_dim) * 4, npos,
                               cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(q3::launch_attention_rows(dq, dk, dv, da, dp, dx, pos, n_heads, kvp, kv_mul, npos, ctx->stream,
                                       ctx->sms),
             "attention");
    TRY_CUDA(cudaMemcpyAsync(xb, dx, size_t(n_heads) * 128 * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    TRY_CUDA(cudaMemcpy2DAsync(att, size_t(seq_len) * 4, dp, size_t(npos) * 4, size_t(npos) * 4, n_heads,
                               cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

q3cu_status q3cu_execute_quantize(q3cu_ctx *ctx, int8_t *q, float *s, const float *x, int n) {
    CHECK_CTX(ctx);
    if (!q || !s || !x || n < 0) return fail(Q3CU_ERR_INVALID, "executeQuantize: bad argument");
    // The reference quantizes n/64 whole groups and leaves a ragged tail
    // untouched (src/cpu/qwen3_original.c:148).
    const int groups = n / Q3CU_GROUP_SIZE;
    if (groups == 0) return Q3CU_OK;
    if (q3cu_status st = use_device(ctx)) return st;
    const int m = groups * Q3CU_GROUP_SIZE;
    const size_t xb = up16(size_t(m) * 4), qb = up16(size_t(m));
    if (q3cu_status st = grow_scratch(ctx, xb + qb + size_t(groups) * 4)) return st;
    auto *d = static_cast<uint8_t *>(ctx->d_scratch);
    float *dx = reinterpret_cast<float *>(d);
    int8_t *dq = reinterpret_cast<int8_t *>(d + xb);
    float *ds = reinterpret_cast<float *>(d + xb + qb);
    TRY_CUDA(cudaMemcpyAsync(dx, x, size_t(m) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(q3::launch_quantize_q8(dx, Q3CU_F32, m, dq, ds, ctx->stream, ctx->sms), "quantize");
    TRY_CUDA(cudaMemcpyAsync(q, dq, size_t(m), cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    TRY_CUDA(cudaMemcpyAsync(s, ds, size_t(groups) * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

q3cu_status q3cu_execute_quantized_matmul(q3cu_ctx *ctx, float *output, const int8_t *x_q, const float *x_s,
                                          const int8_t *w_q, const float *w_s, int n, int d, int group_size) {
    CHECK_CTX(ctx);
    if (!output || !x_q || !x_s || !w_q || !w_s || n <= 0 || d < 0)
        return fail(Q3CU_ERR_INVALID, "executeQuantizedMatMul: bad argument");
    if (group_size != Q3CU_GROUP_SIZE || n % Q3CU_GROUP_SIZE)
        return fail(Q3CU_ERR_GROUP, "group_size %d / n %d: only 64-element groups are supported", group_size, n);
    if (d == 0) return Q3CU_OK;
    if (q3cu_status st = use_device(ctx)) return st;
    const int g = n / Q3CU_GROUP_SIZE;
    const size_t xqb = up32(size_t(n)), xsb = up32(size_t(g) * 4), wqb = up32(size_t(d) * n),
                 wsb = up32(size_t(d) * g * 4);
    if (q3cu_status st = grow_scratch(ctx, xqb + xsb + wqb + wsb + size_t(d) * 4)) return st;
    auto *p = static_cast<uint8_t *>(ctx->d_scratch);
    int8_t *dxq = reinterpret_cast<int8_t *>(p);
    float *dxs = reinterpret_cast<float *>(p + xqb);
    int8_t *dwq = reinterpret_cast<int8_t *>(p + xqb + xsb);
    float *dws = reinterpret_cast<float *>(p + xqb + xsb + wqb);
    float *dout = reinterpret_cast<float *>(p + xqb + xsb + wqb + wsb);
    TRY_CUDA(cudaMemcpyAsync(dxq, x_q, size_t(n), cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dxs, x_s, size_t(g) * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dwq, w_q, size_t(d) * n, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dws, w_s, size_t(d) * g * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(q3::launch_matmul_q8(dxq, dxs, 1, dwq, dws, n, d, dout, ctx->stream, ctx->sms), "matmul");
    TRY_CUDA(cudaMemcpyAsync(output, dout, size_t(d) * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

q3cu_status q3cu_execute_embedding(q3cu_ctx *ctx, float *out, const int8_t *q, const float *s, int token, int dim) {
    CHECK_CTX(ctx);
    if (!out || !q || !s || dim <= 0 || token < 0) return fail(Q3CU_ERR_INVALID, "executeEmbedding: bad argument");
    if (dim % Q3CU_GROUP_SIZE) return fail(Q3CU_ERR_GROUP, "dim %d is not a multiple of 64", dim);
    if (q3cu_status st = use_device(ctx)) return st;
    const size_t qb = up16(size_t(dim)), sb = up16(size_t(dim / Q3CU_GROUP_SIZE) * 4);
    if (q3cu_status st = grow_scratch(ctx, qb + sb + size_t(dim) * 4)) return st;
    auto *d = static_cast<uint8_t *>(ctx->d_scratch);
    int8_t *dq = reinterpret_cast<int8_t *>(d);
    float *ds = reinterpret_cast<float *>(d + qb), *dx = reinterpret_cast<float *>(d + qb + sb);
    TRY_CUDA(cudaMemcpyAsync(dq, q + int64_t(token) * dim, size_t(dim), cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(cudaMemcpyAsync(ds, s + int64_t(token) * (dim / Q3CU_GROUP_SIZE), size_t(dim / Q3CU_GROUP_SIZE) * 4,
                             cudaMemcpyHostToDevice, ctx->stream), "H2D");
    TRY_CUDA(q3::launch_dequantize_q8(dq, ds, dim, dx, ctx->stream, ctx->sms), "dequantize");
    TRY_CUDA(cudaMemcpyAsync(out, dx, size_t(dim) * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    return finish(ctx);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// executeRMSNorm without device allocation (q3cu_execute_rmsnorm_static)
// ---------------------------------------------------------------------------
// q3cu_execute_rmsnorm stages its row in a per-context buffer that grows with
// cudaMalloc, and creating the context allocates too.  Some callers cannot
// allocate at the moment they normalise a row: an engine that reserved all of
// the device's memory for weights and KV cache up front (a new allocation
// fails, or fragments its pool); a decode loop with a latency budget, where
// cudaMalloc / cudaFree may synchronise the device and stall other streams; a
// host application that forbids allocations once it is running.  This path
// stages through a fixed array in the library's own device image instead, and
// reuses the RMSNorm launcher unchanged.
//
// Layout of the array (one instance per device, zero when the module loads):
//   [0, 4)                 status word (Q3CU_DEV_* bits).  Must be 0 when the
//                          kernel starts: every call clears it first.
//   [256, 256 + R)         x, then zeros up to a multiple of 4 elements
//   [256 + R, 256 + 2R)    w, same zero tail
//   [256 + 2R, 256 + 3R)   output
// with R = 4 * Q3CU_STATIC_RMSNORM_MAX bytes.  The zero tails (elements
// size..padded-1 of x and w) must be zero when the kernel runs, since the
// kernel sums over the padded row: every call writes them.
namespace {

constexpr size_t kStaticRow = size_t(4) * Q3CU_STATIC_RMSNORM_MAX;
static_assert(Q3CU_STATIC_SCRATCH_BYTES == 256 + 3 * kStaticRow, "scratch layout");

struct StaticScratch {
    std::atomic<uint8_t *> base{nullptr};
    int sms = 0;
};
StaticScratch g_static[64];
std::mutex g_static_mu;

}  // namespace

static __device__ __align__(256) uint8_t g_static_scratch[Q3CU_STATIC_SCRATCH_BYTES];

namespace {

// The array's address on `dev` (the current device), looked up on the first
// call for that device.
q3cu_status static_scratch(int dev, uint8_t **base, int *sms) {
    if (dev < 0 || dev >= 64) return fail(Q3CU_ERR_DEVICE, "device %d out of range", dev);
    StaticScratch &s = g_static[dev];
    uint8_t *b = s.base.load(std::memory_order_acquire);
    if (!b) {
        std::lock_guard<std::mutex> lock(g_static_mu);
        b = s.base.load(std::memory_order_acquire);
        if (!b) {
            int major = 0, minor = 0, n = 0;
            cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
            if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
            if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
            if (major != 10 || minor != 0)
                return fail(Q3CU_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major,
                            minor);
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_static_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (static scratch)");
            s.sms = n;
            b = static_cast<uint8_t *>(p);
            s.base.store(b, std::memory_order_release);
        }
    }
    *base = b;
    *sms = s.sms;
    return Q3CU_OK;
}

}  // namespace

extern "C" q3cu_status q3cu_execute_rmsnorm_static(float *output, const float *input, const float *weight, int size,
                                                   q3cu_stream stream) {
    if (!output || !input || !weight || size <= 0)
        return fail(Q3CU_ERR_INVALID, "executeRMSNorm (static scratch): bad argument");
    if (size > Q3CU_STATIC_RMSNORM_MAX)
        return fail(Q3CU_ERR_INVALID, "executeRMSNorm (static scratch): size %d exceeds the limit of %d elements", size,
                    Q3CU_STATIC_RMSNORM_MAX);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    uint8_t *base = nullptr;
    int sms = 0;
    if (q3cu_status st = static_scratch(dev, &base, &sms)) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int padded = (size + 3) & ~3;
    uint32_t *d_status = reinterpret_cast<uint32_t *>(base);
    float *dx = reinterpret_cast<float *>(base + 256), *dw = reinterpret_cast<float *>(base + 256 + kStaticRow),
          *dout = reinterpret_cast<float *>(base + 256 + 2 * kStaticRow);
    TRY_CUDA(cudaMemsetAsync(d_status, 0, 4, s), "memset (status)");
    if (padded != size) {
        TRY_CUDA(cudaMemsetAsync(dx + size, 0, size_t(padded - size) * 4, s), "memset (tail)");
        TRY_CUDA(cudaMemsetAsync(dw + size, 0, size_t(padded - size) * 4, s), "memset (tail)");
    }
    TRY_CUDA(cudaMemcpyAsync(dx, input, size_t(size) * 4, cudaMemcpyHostToDevice, s), "H2D");
    TRY_CUDA(cudaMemcpyAsync(dw, weight, size_t(size) * 4, cudaMemcpyHostToDevice, s), "H2D");
    TRY_CUDA(q3::launch_rmsnorm_padded(dx, dw, size, padded, dout, d_status, s, sms), "rmsnorm");
    TRY_CUDA(cudaMemcpyAsync(output, dout, size_t(size) * 4, cudaMemcpyDeviceToHost, s), "D2H");
    uint32_t flags = 0;
    TRY_CUDA(cudaMemcpyAsync(&flags, d_status, 4, cudaMemcpyDeviceToHost, s), "D2H (status)");
    TRY_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (flags & Q3CU_DEV_TIMEOUT) return fail(Q3CU_ERR_TIMEOUT, "executeRMSNorm (static scratch): a device wait gave up");
    return Q3CU_OK;
}
