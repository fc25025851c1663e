/*
 * CudaContext.h -- C++ drop-in for MetalContext (src/metal/MetalContext.h:35-123)
 * over the q3cu C ABI (q3cu.h).
 *
 * The engine's wrappers MetalQwen3::metal_rmsnorm / metal_softmax /
 * metal_swiglu / metal_rope / metal_attention (src/metal/MetalQwen3.cpp:479-639)
 * and its error handler (isBatching / endBatch, :56-57) call these methods with
 * the same host-pointer signatures; only the type name changes.
 * Like MetalContext, each execute* call is synchronous (copy in, run, copy
 * out).  Failures throw std::runtime_error, the exception type MetalContext
 * throws on buffer and command-buffer errors (src/metal/MetalContext.cpp:438-442,
 * :738-754), instead of calling exit(1).
 *
 * The batched device-pointer methods are the throughput path: they take
 * device pointers and a stream, enqueue one launch over all rows and return.
 */
#ifndef Q3CU_CUDA_CONTEXT_H
#define Q3CU_CUDA_CONTEXT_H

#include <cstdint>
#include <string>
#include <vector>

#include "q3cu.h"

class CudaContext {
public:
    explicit CudaContext(int device = 0);
    ~CudaContext();
    CudaContext(const CudaContext &) = delete;
    CudaContext &operator=(const CudaContext &) = delete;

    // MetalContext::initialize / cleanup / isInitialized (MetalContext.h:40-43)
    bool initialize();
    void cleanup();
    bool isInitialized() const { return ctx_ != nullptr; }
    const std::string &lastError() const { return last_error_; }

    // MetalContext::beginBatch / endBatch / isBatching (MetalContext.h:58-60).
    // Every call here is already synchronous and complete on return, so there
    // is never an open batch: the first two do nothing, isBatching() is false.
    void beginBatch() {}
    void endBatch() {}
    bool isBatching() const { return false; }

    // MetalContext::execute* (MetalContext.h:79-87), host pointers, synchronous
    void executeRMSNorm(float *output, const float *input, const float *weight, int size);
    void executeSoftmax(float *x, int size);
    void executeSwiGLU(float *hb, const float *hb2, int hidden_dim);
    void executeRoPE(float *q, float *k, int head_dim, int pos, int n_heads, int n_kv_heads,
                     const float *q_norm_weights, const float *k_norm_weights);
    // MetalContext::executeAttention (MetalContext.h:86-87): one token's heads
    // over the cache rows 0..pos at key_cache + loff / value_cache + loff.
    void executeAttention(float *xb, const float *q, float *att, float *key_cache, float *value_cache, int pos,
                          int head_dim, int n_heads, int n_kv_heads, int seq_len, int kv_dim, uint64_t loff,
                          int kv_mul);
    // the engine's CPU quantize (MetalQwen3.cpp:308-329) and embedding copy (:228)
    void executeQuantize(int8_t *q, float *s, const float *x, int n);
    void executeEmbedding(float *out, const int8_t *q, const float *s, int token, int dim);
    // MetalContext::executeQuantizedMatMul (src/metal/MetalContext.h:81-82).
    void executeQuantizedMatMul(float *output, const int8_t *x_q, const float *x_s, const int8_t *w_q,
                                const float *w_s, int n, int d, int group_size);

    // batched device-pointer path (asynchronous on `stream`)
    void rmsnormQ8(const void *x, q3cu_dtype dt, const float *w, int64_t rows, int dim, int8_t *q, float *s,
                   q3cu_stream stream, float eps = 1e-6f);
    void matmulQ8(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n, int d,
                  float *out, q3cu_stream stream);
    void rmsnorm(const void *x, q3cu_dtype dt, const float *w, int64_t rows, int dim, void *out,
                 q3cu_stream stream, float eps = 1e-6f);
    void qkNormRope(void *q, void *k, q3cu_dtype dt, const int32_t *pos, int64_t rows, int n_heads, int n_kv,
                    int head_dim, const float *q_norm, const float *k_norm, q3cu_stream stream,
                    float theta = 1e6f, float eps = 1e-6f);
    void swigluQ8(const void *hb, const void *hb2, q3cu_dtype dt, int64_t rows, int hidden, int8_t *q, float *s,
                  q3cu_stream stream);
    void softmaxRows(float *x, const int64_t *row_off, const int32_t *row_len, int64_t rows, q3cu_stream stream);
    void quantizeQ8(const void *x, q3cu_dtype dt, int64_t rows, int n, int8_t *q, float *s, q3cu_stream stream);
    void embedGather(const int8_t *tq, const float *ts, int vocab, int dim, const int32_t *ids, int64_t n,
                     float *out_f32, int8_t *out_q, float *out_s, q3cu_stream stream);
    void attention(const float *q, const float *key_cache, const float *value_cache, int pos, int n_heads,
                   int kv_dim, int kv_mul, float *att, int att_stride, float *probs, float *xb, q3cu_stream stream);
    // synchronises `stream` and throws if a kernel flagged a device-side error
    void checkDeviceStatus(q3cu_stream stream);

    q3cu_ctx *raw() const { return ctx_; }

private:
    void check(q3cu_status s, const char *op);
    int device_;
    q3cu_ctx *ctx_ = nullptr;
    std::string last_error_;
};

// The reference's Transformer on the device: a checkpoint image loaded once
// (build_transformer / read_checkpoint, src/cpu/qwen3_original.c:185-258) and
// its decode step (forward, :333-468), through q3cu_model_*.  forward()
// returns the logits like the reference's forward does (a buffer the object
// owns, valid until the next call), with the reference's bits.  Throws
// std::runtime_error on failure.
class CudaModel {
public:
    CudaModel(CudaContext &ctx, const void *checkpoint, size_t bytes, int ctx_length = 0);
    ~CudaModel();
    CudaModel(const CudaModel &) = delete;
    CudaModel &operator=(const CudaModel &) = delete;

    const q3cu_config &config() const { return cfg_; }
    const float *forward(int token, int pos);          // host logits [vocab], synchronous
    const float *deviceLogits() const;                 // the same logits on the device

private:
    q3cu_model *m_ = nullptr;
    q3cu_config cfg_{};
    std::vector<float> logits_;
};

#endif
