// q3cu_model.cu -- a Qwen3 checkpoint resident on the device, and the
// reference's decode step (forward) run on it with the library's kernels.
//
// Reference: src/cpu/qwen3_original.c
//   read_checkpoint / memory_map_weights (:185-248): 256-byte header, fp32
//   norms (rms_att[L][dim], rms_ffn[L][dim], rms_final[dim], q_norm[L][hd],
//   k_norm[L][hd]), then Q8_0 tensors, each as int8 codes then f32 scales:
//   token table, wq[L], wk[L], wv[L], wo[L], w1[L], w2[L], w3[L] (and the
//   classifier unless shared_classifier).  ctx_length caps seq_len (:240-241).
//   forward (:333-468): the op sequence reproduced in q3cu_model_forward.
//
// Every step keeps the reference's roundings, so the logits are its bits:
// the embedding row is dequantized on lookup (the reference dequantizes the
// whole table at load, :203-205; same product per element); the layer's
// RMSNorm+Q8_0 and SwiGLU+Q8_0 are computed, with the operations of the
// library's bit-exact kernels, by every CTA of the matmul that consumes them
// (launch_matmul_q8_pro); the final RMSNorm+Q8_0 is its own kernel, because
// the classifier's grid is more than one wave; QK-norm+RoPE takes
// its cos/sin from the host's libm for the step's position (as the reference
// computes them) instead of the device's sincosf; the
// matmuls keep the group order (k_matmul.cu) and fuse the residual add
// (x += W x, one rounding as in :434/:457); attention keeps its three orders
// and quantizes its own output (k_attn.cu).  Weights that share an input are
// stored as one matrix -- Q|K|V as [A+2K][dim] into one [q | k | v] buffer,
// W1|W3 as [2H][dim] -- so a layer is 6 launches (QK-norm+RoPE and the
// cache-row writes inside the attention's first launch).  Every launch after
// the embedding row is a programmatic dependent of the kernel before it (its
// weight loads or its prologue start while that kernel finishes; each waits
// for it before touching what it wrote, and no kernel here writes what its
// predecessor reads).  Weights, KV cache and run state
// live in one device allocation made at load; forward allocates nothing.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "q3cu_internal.h"

struct q3cu_model {
    q3cu_ctx *ctx = nullptr;
    q3cu_config cfg{};
    int kv_dim = 0, ahd = 0, kv_mul = 0, sms = 0;
    void *arena = nullptr;
    float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    int8_t *tok_q = nullptr, *cls_q = nullptr;
    float *tok_s = nullptr, *cls_s = nullptr;
    std::vector<int8_t *> wqkv, wo, w13, w2;
    std::vector<float *> sqkv, so, s13, s2;
    float *kc = nullptr, *vc = nullptr, *x = nullptr, *qkv = nullptr, *att = nullptr, *hb = nullptr,
          *logits = nullptr, *xs = nullptr;
    int8_t *xq = nullptr;
    q3::StepParams *step = nullptr;           // this step's position, token and RoPE table
    cudaStream_t own = nullptr;               // the model's stream: its graph runs there
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    cudaGraphExec_t graph = nullptr;          // one decode step, captured at the first call
    // pinned host staging: the step parameters copied in, the status word read back
    q3::StepParams *h_step = nullptr;
    uint32_t *h_status = nullptr;
    cudaEvent_t ev_step = nullptr;            // the copy of h_step has been made
};

namespace {

q3cu_status err(q3cu_status s, const char *fmt, ...) {
    char buf[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return q3::set_error(s, buf);
}

q3cu_status cuda_err(cudaError_t e, const char *what) {
    return err(e == cudaErrorMemoryAllocation ? Q3CU_ERR_OOM : Q3CU_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define MTRY(expr, what)                                     \
    do {                                                     \
        cudaError_t e_ = (expr);                             \
        if (e_ != cudaSuccess) return cuda_err(e_, what);    \
    } while (0)
#define MCHK(expr)                                           \
    do {                                                     \
        q3cu_status s_ = (expr);                             \
        if (s_ != Q3CU_OK) return s_;                        \
    } while (0)

size_t up256(size_t b) { return (b + 255) & ~size_t(255); }

// Bump allocator over the arena: first pass sizes it, second hands out pointers.
struct Layout {
    uint8_t *base = nullptr;
    size_t off = 0;
    template <typename T> T *take(size_t count) {
        T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
        off += up256(count * sizeof(T));
        return p;
    }
};

// Reads the checkpoint image in file order.
struct Reader {
    const uint8_t *p, *end;
    bool ok = true;
    const uint8_t *take(size_t n) {
        if (size_t(end - p) < n) {
            ok = false;
            return nullptr;
        }
        const uint8_t *r = p;
        p += n;
        return r;
    }
};

}  // namespace

static void place(q3cu_model *m, Layout &L) {
    const q3cu_config &c = m->cfg;
    const size_t D = c.dim, H = c.hidden_dim, V = c.vocab_size, S = c.seq_len, hd = c.head_dim;
    const int nl = c.n_layers;
    m->rms_att = L.take<float>(size_t(nl) * D);
    m->rms_ffn = L.take<float>(size_t(nl) * D);
    m->rms_final = L.take<float>(D);
    m->q_norm = L.take<float>(size_t(nl) * hd);
    m->k_norm = L.take<float>(size_t(nl) * hd);
    m->tok_q = L.take<int8_t>(V * D);
    m->tok_s = L.take<float>(V * D / 64);
    for (auto *v : {&m->wqkv, &m->wo, &m->w13, &m->w2}) v->assign(nl, nullptr);
    for (auto *v : {&m->sqkv, &m->so, &m->s13, &m->s2}) v->assign(nl, nullptr);
    const size_t A = m->ahd, K = m->kv_dim;
    for (int l = 0; l < nl; ++l) {
        m->wqkv[l] = L.take<int8_t>((A + 2 * K) * D); m->sqkv[l] = L.take<float>((A + 2 * K) * D / 64);
        m->wo[l] = L.take<int8_t>(D * A);      m->so[l] = L.take<float>(D * A / 64);
        m->w13[l] = L.take<int8_t>(2 * H * D); m->s13[l] = L.take<float>(2 * H * D / 64);
        m->w2[l] = L.take<int8_t>(D * H);      m->s2[l] = L.take<float>(D * H / 64);
    }
    if (c.shared_classifier) {
        m->cls_q = m->tok_q;
        m->cls_s = m->tok_s;
    } else {
        m->cls_q = L.take<int8_t>(V * D);
        m->cls_s = L.take<float>(V * D / 64);
    }
    m->kc = L.take<float>(size_t(nl) * S * K);
    m->vc = L.take<float>(size_t(nl) * S * K);
    m->x = L.take<float>(D);
    m->qkv = L.take<float>(A + 2 * K);
    m->att = L.take<float>(size_t(c.n_heads) * S);
    m->hb = L.take<float>(2 * H);
    m->logits = L.take<float>(V);
    const size_t qmax = D > A ? (D > H ? D : H) : (A > H ? A : H);
    m->xq = L.take<int8_t>(qmax);
    m->xs = L.take<float>(qmax / 64);
    m->step = L.take<q3::StepParams>(1);
}

extern "C" {

q3cu_status q3cu_model_load(q3cu_ctx *ctx, const void *checkpoint, size_t bytes, int ctx_length, q3cu_model **out) {
    if (!out) return err(Q3CU_ERR_INVALID, "out is NULL");
    *out = nullptr;
    if (!q3::ctx_alive(ctx)) return err(Q3CU_ERR_NOT_INIT, "context is NULL or destroyed");
    if (!checkpoint) return err(Q3CU_ERR_INVALID, "checkpoint is NULL");
    q3cu_config c;
    MCHK(q3cu_check_header(checkpoint, bytes, &c));
    if (bytes < 256) return err(Q3CU_ERR_FORMAT, "image shorter than its 256-byte header");
    if (ctx_length < 0) return err(Q3CU_ERR_INVALID, "ctx_length %d", ctx_length);
    if (ctx_length != 0 && ctx_length <= c.seq_len) c.seq_len = ctx_length;     // :240-241
    if (c.head_dim != 128) return err(Q3CU_ERR_INVALID, "head_dim %d: the kernels take 128", c.head_dim);
    const int A = c.n_heads * c.head_dim;
    if (c.dim % 64 || c.hidden_dim % 64 || A % 64)
        return err(Q3CU_ERR_FORMAT, "dim, hidden_dim and n_heads*head_dim must be multiples of 64");

    q3cu_model *m = new q3cu_model();
    m->ctx = ctx;
    m->cfg = c;
    m->ahd = A;
    m->kv_dim = c.n_kv_heads * c.head_dim;
    m->kv_mul = c.n_heads / c.n_kv_heads;
    m->sms = q3::ctx_sms(ctx);
    auto fail_free = [&](q3cu_status s) {
        if (m->arena) cudaFree(m->arena);
        delete m;
        return s;
    };
    if (q3cu_status s = q3::ctx_use_device(ctx)) return fail_free(s);
    Layout sizing;
    place(m, sizing);
    cudaError_t e = cudaMalloc(&m->arena, sizing.off);
    if (e != cudaSuccess) return fail_free(cuda_err(e, "cudaMalloc (model)"));
    Layout L{static_cast<uint8_t *>(m->arena), 0};
    place(m, L);

    // copy the image in file order
    const size_t D = c.dim, H = c.hidden_dim, V = c.vocab_size, hd = c.head_dim, K = m->kv_dim;
    const int nl = c.n_layers;
    Reader r{static_cast<const uint8_t *>(checkpoint) + 256, static_cast<const uint8_t *>(checkpoint) + bytes};
    auto up = [&](void *dst, size_t n) -> cudaError_t {
        const uint8_t *src = r.take(n);
        if (!src) return cudaSuccess;                       // r.ok reports the short image
        return cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice);
    };
    auto up_q8 = [&](int8_t *q, float *s, size_t n) -> cudaError_t {   // codes then scales
        cudaError_t e1 = up(q, n);
        if (e1 != cudaSuccess) return e1;
        return up(s, n / 64 * 4);
    };
    cudaError_t ce = cudaSuccess;
    auto step = [&](cudaError_t e2) { if (ce == cudaSuccess) ce = e2; };
    step(up(m->rms_att, size_t(nl) * D * 4));
    step(up(m->rms_ffn, size_t(nl) * D * 4));
    step(up(m->rms_final, D * 4));
    step(up(m->q_norm, size_t(nl) * hd * 4));
    step(up(m->k_norm, size_t(nl) * hd * 4));
    step(up_q8(m->tok_q, m->tok_s, V * D));
    for (int l = 0; l < nl; ++l) step(up_q8(m->wqkv[l], m->sqkv[l], size_t(A) * D));                 // wq: rows 0..A-1
    for (int l = 0; l < nl; ++l)                                                                        // wk: A..A+K-1
        step(up_q8(m->wqkv[l] + size_t(A) * D, m->sqkv[l] + size_t(A) * D / 64, K * D));
    for (int l = 0; l < nl; ++l)                                                                        // wv: A+K..
        step(up_q8(m->wqkv[l] + (size_t(A) + K) * D, m->sqkv[l] + (size_t(A) + K) * D / 64, K * D));
    for (int l = 0; l < nl; ++l) step(up_q8(m->wo[l], m->so[l], D * size_t(A)));
    for (int l = 0; l < nl; ++l) step(up_q8(m->w13[l], m->s13[l], H * D));                       // w1: rows 0..H-1
    for (int l = 0; l < nl; ++l) step(up_q8(m->w2[l], m->s2[l], D * H));
    for (int l = 0; l < nl; ++l) step(up_q8(m->w13[l] + H * D, m->s13[l] + H * D / 64, H * D));  // w3: rows H..2H-1
    if (!c.shared_classifier) step(up_q8(m->cls_q, m->cls_s, V * D));
    if (ce != cudaSuccess) return fail_free(cuda_err(ce, "cudaMemcpy (weights)"));
    if (!r.ok) return fail_free(err(Q3CU_ERR_FORMAT, "image of %zu bytes is shorter than its header's tensors", bytes));
    // the KV cache starts at zero, as the reference's calloc'd RunState (:113-114)
    e = cudaMemset(m->kc, 0, size_t(nl) * c.seq_len * K * 4);
    if (e == cudaSuccess) e = cudaMemset(m->vc, 0, size_t(nl) * c.seq_len * K * 4);
    if (e != cudaSuccess) return fail_free(cuda_err(e, "cudaMemset (KV cache)"));
    e = cudaStreamCreateWithFlags(&m->own, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->ev_step, cudaEventDisableTiming);
    void *hb = nullptr;
    if (e == cudaSuccess) e = cudaHostAlloc(&hb, sizeof(q3::StepParams) + 16, cudaHostAllocDefault);
    if (e != cudaSuccess) {
        if (m->ev_in) cudaEventDestroy(m->ev_in);
        if (m->ev_out) cudaEventDestroy(m->ev_out);
        if (m->ev_step) cudaEventDestroy(m->ev_step);
        if (m->own) cudaStreamDestroy(m->own);
        return fail_free(cuda_err(e, "stream / events / pinned staging"));
    }
    m->h_step = static_cast<q3::StepParams *>(hb);
    m->h_status = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(hb) + sizeof(q3::StepParams));
    *out = m;
    return Q3CU_OK;
}

q3cu_status q3cu_model_config(const q3cu_model *m, q3cu_config *out) {
    if (!m || !out) return err(Q3CU_ERR_INVALID, "NULL argument");
    *out = m->cfg;
    return Q3CU_OK;
}

const float *q3cu_model_logits(const q3cu_model *m) { return m ? m->logits : nullptr; }

}  // extern "C"

// Every launch of one decode step, in order, on stream s (the step's position
// and token are read from m->step on the device).
static q3cu_status enqueue_step(q3cu_model *m, cudaStream_t s) {
    q3cu_ctx *ctx = m->ctx;
    const q3cu_config &c = m->cfg;
    const int D = c.dim, H = c.hidden_dim, A = m->ahd, K = m->kv_dim, hd = c.head_dim, S = c.seq_len;
    const float eps = 1e-6f;                                   // rmsnorm's constant (:283)
    const q3cu_stream st = s;
    // token embedding (:342): the row of the dequantized table
    MCHK(q3cu_embed_gather(ctx, m->tok_q, m->tok_s, c.vocab_size, D, &m->step->token, 1, m->x, nullptr, nullptr, st));
    for (int l = 0; l < c.n_layers; ++l) {
        const int64_t loff = int64_t(l) * S * K;
        // attention rmsnorm + quantize, Q|K|V (:353-359): one launch, every CTA
        // normalizes and quantizes x into its shared memory
        MTRY(q3::launch_matmul_q8_pro(q3::PRO_RMS, q3::MmPro{m->x, nullptr, m->rms_att + int64_t(l) * D, eps}, D,
                                      m->wqkv[l], m->sqkv[l], A + 2 * K,
                                      q3::MmOut{m->qkv, m->qkv, m->qkv, A + 2 * K, A + 2 * K}, s, m->sms, nullptr),
             "rmsnorm + wq|wk|wv");
        // Q/K RMSNorm + RoPE, the key and the value into their cache rows,
        // attention and the quantize of its output (:349-350, :361-428, :431)
        MTRY(q3::launch_attention_step(m->qkv, m->kc + loff, m->vc + loff, m->att, m->xq, m->xs, m->step, c.n_heads,
                                       c.n_kv_heads, m->q_norm + int64_t(l) * hd, m->k_norm + int64_t(l) * hd, eps,
                                       S, s, m->sms),
             "attention");
        // output projection + residual (:432-435)
        MTRY(q3::launch_matmul_q8_seg(m->xq, m->xs, 1, m->wo[l], m->so[l], A, D, q3::MmOut{m->x, m->x, m->x, D, D}, s,
                                      m->sms, m->x, true),
             "wo");
        // FFN (:438-458)
        MTRY(q3::launch_matmul_q8_pro(q3::PRO_RMS, q3::MmPro{m->x, nullptr, m->rms_ffn + int64_t(l) * D, eps}, D,
                                      m->w13[l], m->s13[l], 2 * H, q3::MmOut{m->hb, m->hb, m->hb, 2 * H, 2 * H}, s,
                                      m->sms, nullptr),
             "rmsnorm + w1|w3");
        MTRY(q3::launch_matmul_q8_pro(q3::PRO_SWIGLU, q3::MmPro{m->hb, m->hb + H, nullptr, 0.0f}, H, m->w2[l],
                                      m->s2[l], D, q3::MmOut{m->x, m->x, m->x, D, D}, s, m->sms, m->x),
             "swiglu + w2");
    }
    // final rmsnorm + classifier (:462-466)
    MCHK(q3cu_rmsnorm_q8(ctx, m->x, Q3CU_F32, m->rms_final, 1, D, eps, m->xq, m->xs, st));
    MTRY(q3::launch_matmul_q8_seg(m->xq, m->xs, 1, m->cls_q, m->cls_s, D, c.vocab_size,
                                  q3::MmOut{m->logits, m->logits, m->logits, c.vocab_size, c.vocab_size}, s, m->sms,
                                  nullptr, true),
         "classifier");
    return Q3CU_OK;
}

// The step captured once as a CUDA graph on the model's own stream.
static q3cu_status capture_step(q3cu_model *m) {
    MTRY(cudaStreamBeginCapture(m->own, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture");
    const q3cu_status st = enqueue_step(m, m->own);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(m->own, &g);
    if (st != Q3CU_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (e != cudaSuccess) return cuda_err(e, "cudaStreamEndCapture");
    const cudaError_t e2 = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    if (e2 != cudaSuccess) {
        m->graph = nullptr;
        return cuda_err(e2, "cudaGraphInstantiate");
    }
    return Q3CU_OK;
}

extern "C" {

q3cu_status q3cu_model_forward(q3cu_model *m, int token, int pos, float *logits_host, q3cu_stream stream) {
    if (!m) return err(Q3CU_ERR_INVALID, "model is NULL");
    q3cu_ctx *ctx = m->ctx;
    if (!q3::ctx_alive(ctx)) return err(Q3CU_ERR_NOT_INIT, "the model's context is destroyed");
    const q3cu_config &c = m->cfg;
    if (token < 0 || token >= c.vocab_size) return err(Q3CU_ERR_INDEX, "token %d outside [0, %d)", token, c.vocab_size);
    if (pos < 0 || pos >= c.seq_len) return err(Q3CU_ERR_INDEX, "pos %d outside [0, %d)", pos, c.seq_len);
    MCHK(q3::ctx_use_device(ctx));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The step's parameters: RoPE's cos/sin for this position with the C
    // library's calls, as the reference makes them (:367-368):
    // freq = powf(1e6, -(float)j / (hd/2)), cosf / sinf of the binary32 product pos * freq.
    q3::StepParams sp{};
    sp.pos = pos;
    sp.token = token;
    const int hd = c.head_dim;
    for (int j = 0; j < hd / 2; ++j) {
        const float freq = powf(1e6f, -float(j) / float(hd / 2));
        const float ang = float(pos) * freq;
        sp.c[j] = cosf(ang);
        sp.s[j] = sinf(ang);
    }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    MTRY(cudaStreamIsCapturing(s, &cap), "cudaStreamIsCapturing");
    if (cap != cudaStreamCaptureStatusNone) {
        // inside the caller's capture: the launches join it, the parameters as a kernel
        MTRY(q3::launch_set_step(m->step, sp, s), "step parameters");
        MCHK(enqueue_step(m, s));
    } else {
        // the model's own graph, replayed on its stream between two events on the caller's
        MTRY(cudaEventSynchronize(m->ev_step), "cudaEventSynchronize");   // the last step's copy has read h_step
        *m->h_step = sp;
        MTRY(cudaEventRecord(m->ev_in, s), "cudaEventRecord");
        MTRY(cudaStreamWaitEvent(m->own, m->ev_in, 0), "cudaStreamWaitEvent");
        MTRY(cudaMemcpyAsync(m->step, m->h_step, sizeof(sp), cudaMemcpyHostToDevice, m->own), "step parameters");
        MTRY(cudaEventRecord(m->ev_step, m->own), "cudaEventRecord");
        if (!m->graph) MCHK(capture_step(m));
        MTRY(cudaGraphLaunch(m->graph, m->own), "cudaGraphLaunch");
        MTRY(cudaEventRecord(m->ev_out, m->own), "cudaEventRecord");
        MTRY(cudaStreamWaitEvent(s, m->ev_out, 0), "cudaStreamWaitEvent");
    }
    if (logits_host) {
        // the logits and the status word back in one round trip; a set word is
        // reported (and cleared) by q3cu_device_status
        MTRY(cudaMemcpyAsync(logits_host, m->logits, size_t(c.vocab_size) * 4, cudaMemcpyDeviceToHost, s), "logits D2H");
        MTRY(cudaMemcpyAsync(m->h_status, q3::ctx_status_word(ctx), sizeof(uint32_t), cudaMemcpyDeviceToHost, s),
             "status D2H");
        MTRY(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        if (*m->h_status) MCHK(q3cu_device_status(ctx, stream, nullptr));
    }
    return Q3CU_OK;
}

q3cu_status q3cu_model_destroy(q3cu_model *m) {
    if (!m) return Q3CU_OK;
    if (q3::ctx_alive(m->ctx)) q3::ctx_use_device(m->ctx);
    if (m->own) cudaStreamSynchronize(m->own);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->ev_in) cudaEventDestroy(m->ev_in);
    if (m->ev_out) cudaEventDestroy(m->ev_out);
    if (m->ev_step) cudaEventDestroy(m->ev_step);
    if (m->own) cudaStreamDestroy(m->own);
    if (m->h_step) cudaFreeHost(m->h_step);
    cudaError_t e = m->arena ? cudaFree(m->arena) : cudaSuccess;
    delete m;
    return e == cudaSuccess ? Q3CU_OK : cuda_err(e, "cudaFree (model)");
}

}  // extern "C"
