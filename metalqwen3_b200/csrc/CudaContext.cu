// CudaContext.cu -- the C++ MetalContext drop-in (include/CudaContext.h), a thin
// layer over the C ABI.
#include "CudaContext.h"

#include <stdexcept>

CudaContext::CudaContext(int device) : device_(device) {}

CudaContext::~CudaContext() { cleanup(); }

bool CudaContext::initialize() {
    if (ctx_) return true;
    q3cu_status s = q3cu_init(device_, &ctx_);
    if (s != Q3CU_OK) {
        last_error_ = q3cu_last_error_string();
        ctx_ = nullptr;
        return false;
    }
    return true;
}

void CudaContext::cleanup() {
    if (ctx_) q3cu_destroy(ctx_);
    ctx_ = nullptr;
}

void CudaContext::check(q3cu_status s, const char *op) {
    if (s == Q3CU_OK) return;
    last_error_ = std::string(op) + ": " + q3cu_status_string(s) + " (" + q3cu_last_error_string() + ")";
    throw std::runtime_error(last_error_);
}

void CudaContext::executeRMSNorm(float *output, const float *input, const float *weight, int size) {
    check(q3cu_execute_rmsnorm(ctx_, output, input, weight, size), "executeRMSNorm");
}
void CudaContext::executeSoftmax(float *x, int size) { check(q3cu_execute_softmax(ctx_, x, size), "executeSoftmax"); }
void CudaContext::executeSwiGLU(float *hb, const float *hb2, int hidden_dim) {
    check(q3cu_execute_swiglu(ctx_, hb, hb2, hidden_dim), "executeSwiGLU");
}
void CudaContext::executeRoPE(float *q, float *k, int head_dim, int pos, int n_heads, int n_kv_heads,
                              const float *q_norm_weights, const float *k_norm_weights) {
    check(q3cu_execute_rope(ctx_, q, k, head_dim, pos, n_heads, n_kv_heads, q_norm_weights, k_norm_weights),
          "executeRoPE");
}
void CudaContext::executeAttention(float *xb, const float *q, float *att, float *key_cache, float *value_cache,
                                   int pos, int head_dim, int n_heads, int n_kv_heads, int seq_len, int kv_dim,
                                   uint64_t loff, int kv_mul) {
    check(q3cu_execute_attention(ctx_, xb, q, att, key_cache, value_cache, pos, head_dim, n_heads, n_kv_heads, seq_len,
                                 kv_dim, loff, kv_mul),
          "executeAttention");
}
void CudaContext::executeQuantize(int8_t *q, float *s, const float *x, int n) {
    check(q3cu_execute_quantize(ctx_, q, s, x, n), "executeQuantize");
}
void CudaContext::executeEmbedding(float *out, const int8_t *q, const float *s, int token, int dim) {
    check(q3cu_execute_embedding(ctx_, out, q, s, token, dim), "executeEmbedding");
}

void CudaContext::executeQuantizedMatMul(float *output, const int8_t *x_q, const float *x_s, const int8_t *w_q,
                                         const float *w_s, int n, int d, int group_size) {
    check(q3cu_execute_quantized_matmul(ctx_, output, x_q, x_s, w_q, w_s, n, d, group_size), "executeQuantizedMatMul");
}
void CudaContext::matmulQ8(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n, int d,
                           float *out, q3cu_stream stream) {
    check(q3cu_matmul_q8(ctx_, xq, xs, B, wq, ws, n, d, out, stream), "matmulQ8");
}
void CudaContext::rmsnormQ8(const void *x, q3cu_dtype dt, const float *w, int64_t rows, int dim, int8_t *q, float *s,
                            q3cu_stream stream, float eps) {
    check(q3cu_rmsnorm_q8(ctx_, x, dt, w, rows, dim, eps, q, s, stream), "rmsnormQ8");
}
void CudaContext::rmsnorm(const void *x, q3cu_dtype dt, const float *w, int64_t rows, int dim, void *out,
                          q3cu_stream stream, float eps) {
    check(q3cu_rmsnorm(ctx_, x, dt, w, rows, dim, eps, out, stream), "rmsnorm");
}
void CudaContext::qkNormRope(void *q, void *k, q3cu_dtype dt, const int32_t *pos, int64_t rows, int n_heads, int n_kv,
                             int head_dim, const float *q_norm, const float *k_norm, q3cu_stream stream, float theta,
                             float eps) {
    check(q3cu_qk_norm_rope(ctx_, q, k, dt, pos, rows, n_heads, n_kv, head_dim, q_norm, k_norm, theta, eps, stream),
          "qkNormRope");
}
void CudaContext::swigluQ8(const void *hb, const void *hb2, q3cu_dtype dt, int64_t rows, int hidden, int8_t *q,
                           float *s, q3cu_stream stream) {
    check(q3cu_swiglu_q8(ctx_, hb, hb2, dt, rows, hidden, q, s, stream), "swigluQ8");
}
void CudaContext::softmaxRows(float *x, const int64_t *row_off, const int32_t *row_len, int64_t rows,
                              q3cu_stream stream) {
    check(q3cu_softmax_rows(ctx_, x, row_off, row_len, rows, stream), "softmaxRows");
}
void CudaContext::quantizeQ8(const void *x, q3cu_dtype dt, int64_t rows, int n, int8_t *q, float *s,
                             q3cu_stream stream) {
    check(q3cu_quantize_q8(ctx_, x, dt, rows, n, q, s, stream), "quantizeQ8");
}
void CudaContext::embedGather(const int8_t *tq, const float *ts, int vocab, int dim, const int32_t *ids, int64_t n,
                              float *out_f32, int8_t *out_q, float *out_s, q3cu_stream stream) {
    check(q3cu_embed_gather(ctx_, tq, ts, vocab, dim, ids, n, out_f32, out_q, out_s, stream), "embedGather");
}
void CudaContext::attention(const float *q, const float *key_cache, const float *value_cache, int pos, int n_heads,
                            int kv_dim, int kv_mul, float *att, int att_stride, float *probs, float *xb,
                            q3cu_stream stream) {
    check(q3cu_attention(ctx_, q, key_cache, value_cache, pos, n_heads, kv_dim, kv_mul, att, att_stride, probs, xb,
                         stream),
          "attention");
}
void CudaContext::checkDeviceStatus(q3cu_stream stream) {
    check(q3cu_device_status(ctx_, stream, nullptr), "checkDeviceStatus");
}

static void model_check(q3cu_status s, const char *op) {
    if (s == Q3CU_OK) return;
    throw std::runtime_error(std::string(op) + ": " + q3cu_status_string(s) + " (" + q3cu_last_error_string() + ")");
}

CudaModel::CudaModel(CudaContext &ctx, const void *checkpoint, size_t bytes, int ctx_length) {
    model_check(q3cu_model_load(ctx.raw(), checkpoint, bytes, ctx_length, &m_), "q3cu_model_load");
    model_check(q3cu_model_config(m_, &cfg_), "q3cu_model_config");
    logits_.resize(size_t(cfg_.vocab_size));
}

CudaModel::~CudaModel() {
    if (m_) q3cu_model_destroy(m_);
}

const float *CudaModel::forward(int token, int pos) {
    model_check(q3cu_model_forward(m_, token, pos, logits_.data(), nullptr), "q3cu_model_forward");
    return logits_.data();
}

const float *CudaModel::deviceLogits() const { return q3cu_model_logits(m_); }
