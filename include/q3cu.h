/*
 * q3cu.h -- C ABI of the B200 (sm_100a) fused Qwen3 layer kernels.
 *
 * This library replaces the operator backend that the qwen3.c-derived engine
 * calls once per op per layer: `MetalContext::execute*` in
 * src/metal/MetalContext.h:78-87 (Metal shaders under shaders/) and the CPU
 * helpers the engine runs between those calls (`quantize`, the embedding
 * gather).  Results follow the reference CPU engine src/cpu/qwen3_original.c:
 *
 *   - Q8_0 codes and scales, and the embedding dequant, are bit-exact;
 *   - RMSNorm (also the per-head QK-norm) and SwiGLU float outputs are
 *     bit-exact for f32 inputs (sequential sum of squares; an expf that
 *     reproduces the host libm's);
 *   - RoPE and softmax outputs are within 1e-5 relative / 1e-6 absolute (f32)
 *     and 1e-2 relative (bf16 inputs).
 *
 * Conventions
 *   - Device-pointer entry points (`q3cu_<op>`) take caller-owned device
 *     memory, run asynchronously on `stream` (NULL = the legacy default
 *     stream) and allocate nothing.  Row-major, contiguous rows.
 *   - Every entry point returns a q3cu_status; none exits or throws.  The
 *     message of the last failure on the calling thread is available from
 *     q3cu_last_error_string().
 *   - Errors found on the device (an out-of-range token id, a wait that gave
 *     up) set bits in a per-context status word and skip the affected row;
 *     q3cu_device_status() synchronises the stream and returns and clears
 *     them.
 *   - Q8_0 tensors are two arrays, as QuantizedTensor in
 *     src/cpu/qwen3_original.c:43-46: int8 codes [rows][n] and float scales
 *     [rows][n/64].  The group size is fixed at 64; n must be a multiple of 64.
 *   - The host-pointer entry points (`q3cu_execute_*`) keep the reference's
 *     signatures and are synchronous: copy in, run, copy out (the drop-in for
 *     MetalQwen3::metal_* -> MetalContext::execute*).
 *   - One context per device per host thread; a context is not thread-safe.
 */
#ifndef Q3CU_H
#define Q3CU_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    Q3CU_OK = 0,
    Q3CU_ERR_INVALID = 1,    /* bad argument: NULL pointer, negative or zero size ...   */
    Q3CU_ERR_ALIGN = 2,      /* a pointer or row is not aligned as required             */
    Q3CU_ERR_GROUP = 3,      /* a Q8_0 length is not a multiple of the group size (64)  */
    Q3CU_ERR_CUDA = 4,       /* a CUDA runtime call failed                              */
    Q3CU_ERR_INDEX = 5,      /* device status: a token id was out of range              */
    Q3CU_ERR_TIMEOUT = 6,    /* device status: a bounded wait gave up                   */
    Q3CU_ERR_NOT_INIT = 7,   /* NULL or destroyed context                               */
    Q3CU_ERR_OOM = 8,        /* device or host allocation failed                        */
    Q3CU_ERR_DEVICE = 9,     /* no such device, or not an sm_100 device                 */
    Q3CU_ERR_FORMAT = 10     /* checkpoint header: bad magic, version or group size     */
} q3cu_status;

typedef enum { Q3CU_F32 = 0, Q3CU_BF16 = 1 } q3cu_dtype;

/* Bits of the device status word (q3cu_device_status). */
#define Q3CU_DEV_BAD_INDEX 0x1u
#define Q3CU_DEV_TIMEOUT   0x2u

#define Q3CU_GROUP_SIZE 64

typedef struct q3cu_ctx q3cu_ctx;
typedef void *q3cu_stream;               /* a cudaStream_t */

/* Mirrors the header fields of a v1 checkpoint (`Config`,
 * src/cpu/qwen3_original.c:28-41). */
typedef struct {
    int32_t magic_number, version, dim, hidden_dim, n_layers, n_heads, n_kv_heads,
            vocab_size, seq_len, head_dim, shared_classifier, group_size;
} q3cu_config;

/* ---- lifecycle (MetalContext::initialize/cleanup/isInitialized,
 *      src/metal/MetalContext.h:40-43) ------------------------------------- */
q3cu_status q3cu_init(int device, q3cu_ctx **out);
q3cu_status q3cu_destroy(q3cu_ctx *ctx);
int         q3cu_is_initialized(const q3cu_ctx *ctx);
const char *q3cu_last_error_string(void);
const char *q3cu_status_string(q3cu_status s);
int         q3cu_version(void);
/* Synchronises `stream`, returns the device status bits in *flags and clears
 * them.  Returns Q3CU_ERR_INDEX / Q3CU_ERR_TIMEOUT when the matching bit is set. */
q3cu_status q3cu_device_status(q3cu_ctx *ctx, q3cu_stream stream, uint32_t *flags);
/* Failure-path self-test (no counterpart in the reference): enqueues one CTA
 * whose threads wait on a shared-memory barrier that nothing completes, with
 * the same bounded wait the kernels use (about 2 s).  The wait gives up, sets
 * Q3CU_DEV_TIMEOUT in the status word and the kernel returns; nothing faults
 * and the context stays usable.  For testing a caller's handling of a
 * device-side timeout (read it with q3cu_device_status). */
q3cu_status q3cu_selftest_wait_timeout(q3cu_ctx *ctx, q3cu_stream stream);

/* Validates a checkpoint header (src/cpu/qwen3_original.c:236-244 exits on a bad
 * magic or version; this returns Q3CU_ERR_FORMAT instead). */
q3cu_status q3cu_check_header(const void *header, size_t bytes, q3cu_config *out);

/* ---- device-pointer ops ------------------------------------------------- */

/* RMSNorm of each row (src/cpu/qwen3_original.c:278-289;
 * shaders/rmsnorm.metal:23-66): out = w * (ss * x), ss = 1/sqrtf(sum(x^2)/dim + eps).
 * x, out: [rows][dim] of `dtype` (out may equal x); w: [dim] f32.
 * dim * sizeof(dtype) must be a multiple of 16 and x, out 16-byte aligned. */
q3cu_status q3cu_rmsnorm(q3cu_ctx *ctx, const void *x, q3cu_dtype dtype, const float *w,
                         int64_t rows, int dim, float eps, void *out, q3cu_stream stream);

/* RMSNorm fused with the Q8_0 quantize that follows it in the forward pass
 * (qwen3_original.c:353 then :356, :439 then :443, :462 then :465): the float
 * row never leaves the chip.  q: [rows][dim] int8, s: [rows][dim/64] f32. */
q3cu_status q3cu_rmsnorm_q8(q3cu_ctx *ctx, const void *x, q3cu_dtype dtype, const float *w,
                            int64_t rows, int dim, float eps, int8_t *q, float *s,
                            q3cu_stream stream);

/* Per-head QK-RMSNorm + rotate-half RoPE, in place (qwen3_original.c:361-393;
 * MetalContext::executeRoPE, src/metal/MetalContext.cpp:826-913;
 * shaders/rope.metal:6-77).  q: [rows][n_heads][head_dim],
 * k: [rows][n_kv][head_dim] of `dtype`; pos: [rows] int32 (device);
 * q_norm, k_norm: [head_dim] f32 (device).  freq_j = powf(theta, -j/(hd/2)) is
 * evaluated on the host with the C library's powf, as the reference does.
 * head_dim must be 128. */
q3cu_status q3cu_qk_norm_rope(q3cu_ctx *ctx, void *q, void *k, q3cu_dtype dtype,
                              const int32_t *pos, int64_t rows, int n_heads, int n_kv,
                              int head_dim, const float *q_norm, const float *k_norm,
                              float theta, float eps, q3cu_stream stream);

/* SwiGLU in place: hb = hb * (hb2 * (1/(1+expf(-hb)))) (qwen3_original.c:449-450;
 * MetalContext::executeSwiGLU, src/metal/MetalContext.cpp:772-824).
 * hb, hb2: [rows][hidden] of `dtype`; hidden * sizeof(dtype) % 16 == 0. */
q3cu_status q3cu_swiglu(q3cu_ctx *ctx, void *hb, const void *hb2, q3cu_dtype dtype,
                        int64_t rows, int hidden, q3cu_stream stream);

/* SwiGLU fused with the following Q8_0 quantize (qwen3_original.c:449-453). */
q3cu_status q3cu_swiglu_q8(q3cu_ctx *ctx, const void *hb, const void *hb2, q3cu_dtype dtype,
                           int64_t rows, int hidden, int8_t *q, float *s, q3cu_stream stream);

/* In-place softmax of ragged f32 rows (qwen3_original.c:291-308, called per
 * head at :416; MetalContext::executeSoftmax, src/metal/MetalContext.cpp:633-677).
 * Row r is x[row_off[r] .. row_off[r] + row_len[r]) (device arrays).
 * The running max starts at 0, as in the reference. */
q3cu_status q3cu_softmax_rows(q3cu_ctx *ctx, float *x, const int64_t *row_off,
                              const int32_t *row_len, int64_t rows, q3cu_stream stream);

/* Q8_0 quantize of each row (qwen3_original.c:147-168; engine copy
 * src/metal/MetalQwen3.cpp:308-329; shaders/quantize.metal:18-47). */
q3cu_status q3cu_quantize_q8(q3cu_ctx *ctx, const void *x, q3cu_dtype dtype, int64_t rows,
                             int n, int8_t *q, float *s, q3cu_stream stream);

/* Q8_0 dequantize (qwen3_original.c:142-145): x = q * s[i/64].  n = element count. */
q3cu_status q3cu_dequantize_q8(q3cu_ctx *ctx, const int8_t *q, const float *s, int64_t n,
                               float *x, q3cu_stream stream);

/* Embedding lookup from a Q8_0 table (qwen3_original.c:142-145 applied at load,
 * :203-205, then the row memcpy at :342; engine src/metal/MetalQwen3.cpp:228,362-365):
 * row i of the output is table row ids[i] dequantized, optionally re-quantized
 * to Q8_0 (:147-168).  tq: [vocab][dim] int8, ts: [vocab][dim/64] f32.
 * out_f32 [n][dim] may be NULL; out_q [n][dim] and out_s [n][dim/64] may both be
 * NULL.  An out-of-range id sets Q3CU_DEV_BAD_INDEX and leaves its row untouched. */
q3cu_status q3cu_embed_gather(q3cu_ctx *ctx, const int8_t *tq, const float *ts, int vocab,
                              int dim, const int32_t *ids, int64_t n, float *out_f32,
                              int8_t *out_q, float *out_s, q3cu_stream stream);

/* Q8_0 x Q8_0 matrix products for B token rows (qwen3_original.c:310-331
 * `matmul`, applied to each row; engine src/metal/MetalQwen3.cpp:530-533,
 * shaders/quantized_matmul.metal): out[b][i] = sum over the 64-groups j of row
 * i, in order, of RN(RN((float) dot(xq[b] group j, wq[i] group j) * ws[i][j])
 * * xs[b][j]) -- the reference's bits.  xq [B][n], xs [B][n/64]; wq [d][n],
 * ws [d][n/64] (row-major [out][in]); out [B][d].  n % 64 == 0; xq and wq
 * 32-byte aligned.  W is streamed once per block of up to 4 token rows. */
q3cu_status q3cu_matmul_q8(q3cu_ctx *ctx, const int8_t *xq, const float *xs, int B,
                           const int8_t *wq, const float *ws, int n, int d, float *out,
                           q3cu_stream stream);

/* Multi-head attention of one token over positions 0..pos
 * (qwen3_original.c:395-428; MetalContext::executeAttention,
 * src/metal/MetalContext.h:86-87, shaders/attention.metal): per query head h,
 * scores q_h . k_t / sqrtf(128) in index order, the reference's softmax (max
 * from 0), then xb_h = sum over t in order of att[t] * v_t; kv head h / kv_mul.
 * Device pointers: q [n_heads][128] (after QK-norm + RoPE); key_cache,
 * value_cache [pos + 1 or more][kv_dim] (this layer's rows); att
 * [n_heads][att_stride] is scratch for the scores (att_stride > pos); probs
 * (NULL, or a different buffer of the same shape) receives the probabilities,
 * the reference's att after its softmax; xb [n_heads][128].  head_dim is 128;
 * kv_dim % 4 == 0.  Any number of positions.  Same bits as the reference. */
q3cu_status q3cu_attention(q3cu_ctx *ctx, const float *q, const float *key_cache, const float *value_cache,
                           int pos, int n_heads, int kv_dim, int kv_mul, float *att, int att_stride, float *probs,
                           float *xb, q3cu_stream stream);

/* ---- a checkpoint on the device and its decode step --------------------- */
typedef struct q3cu_model q3cu_model;

/* Loads a checkpoint image -- the file's bytes: 256-byte header, fp32 norms,
 * Q8_0 tensors (qwen3_original.c:185-248 read_checkpoint/memory_map_weights,
 * written by scripts/export.py:108-170) -- into device memory on ctx's device,
 * with a zeroed KV cache of seq_len positions (ctx_length > 0 caps seq_len as
 * :240-241 does).  The token table stays Q8_0: rows are dequantized on lookup
 * instead of keeping the reference's fp32 copy (:203-205).  head_dim must be
 * 128.  One device allocation, made here; a short image is Q3CU_ERR_FORMAT. */
q3cu_status q3cu_model_load(q3cu_ctx *ctx, const void *checkpoint, size_t bytes, int ctx_length,
                            q3cu_model **out);
q3cu_status q3cu_model_config(const q3cu_model *m, q3cu_config *out);
/* One decode step, `forward(token, pos)` (qwen3_original.c:333-468; the
 * library entry qwen3_forward, :1062): the token at `pos` attends to the KV
 * rows 0..pos written by earlier calls.  The logits [vocab] stay on the device
 * (q3cu_model_logits); with logits_host set they are also copied there and the
 * call synchronises `stream`.  Same bits as the reference.  Allocates nothing;
 * an out-of-range token or pos is Q3CU_ERR_INDEX. */
q3cu_status q3cu_model_forward(q3cu_model *m, int token, int pos, float *logits_host,
                               q3cu_stream stream);
const float *q3cu_model_logits(const q3cu_model *m);
q3cu_status q3cu_model_destroy(q3cu_model *m);

/* ---- host-pointer drop-in (synchronous), MetalContext signatures -------- */

/* MetalContext::executeRMSNorm (src/metal/MetalContext.h:79). */
q3cu_status q3cu_execute_rmsnorm(q3cu_ctx *ctx, float *output, const float *input,
                                 const float *weight, int size);
/* MetalContext::executeSoftmax (src/metal/MetalContext.h:80). */
q3cu_status q3cu_execute_softmax(q3cu_ctx *ctx, float *x, int size);
/* MetalContext::executeSwiGLU (src/metal/MetalContext.h:83). */
q3cu_status q3cu_execute_swiglu(q3cu_ctx *ctx, float *hb, const float *hb2, int hidden_dim);
/* MetalContext::executeRoPE (src/metal/MetalContext.h:84-85): QK-norm + RoPE
 * of one token's n_heads query heads and n_kv_heads key heads at `pos`. */
q3cu_status q3cu_execute_rope(q3cu_ctx *ctx, float *q, float *k, int head_dim, int pos,
                              int n_heads, int n_kv_heads, const float *q_norm_weights,
                              const float *k_norm_weights);
/* MetalContext::executeAttention (src/metal/MetalContext.h:86-87; called from
 * MetalQwen3::metal_attention, src/metal/MetalQwen3.cpp:639): one token's
 * attention over the layer's cache rows 0..pos at key_cache + loff and
 * value_cache + loff (row stride kv_dim), host pointers.  Writes xb
 * [n_heads][head_dim] and, as the reference's CPU loop does, the probabilities
 * into att [n_heads][seq_len] (columns 0..pos).  head_dim must be 128. */
q3cu_status q3cu_execute_attention(q3cu_ctx *ctx, float *xb, const float *q, float *att, float *key_cache,
                                   float *value_cache, int pos, int head_dim, int n_heads, int n_kv_heads,
                                   int seq_len, int kv_dim, uint64_t loff, int kv_mul);
/* The engine's CPU quantize (src/metal/MetalQwen3.cpp:308-329). */
q3cu_status q3cu_execute_quantize(q3cu_ctx *ctx, int8_t *q, float *s, const float *x, int n);
/* MetalContext::executeQuantizedMatMul (src/metal/MetalContext.h:81-82): one
 * token, W (d,n) @ x (n,) -> output (d,), all host pointers (copied in per
 * call, as the Metal path does).  group_size must be 64. */
q3cu_status q3cu_execute_quantized_matmul(q3cu_ctx *ctx, float *output, const int8_t *x_q,
                                          const float *x_s, const int8_t *w_q, const float *w_s,
                                          int n, int d, int group_size);
/* The engine's embedding row copy (src/metal/MetalQwen3.cpp:228) from a Q8_0
 * table row instead of a dequantized fp32 table. */
q3cu_status q3cu_execute_embedding(q3cu_ctx *ctx, float *out, const int8_t *q, const float *s,
                                   int token, int dim);

/* ---- allocation-free executeRMSNorm ----------------------------------------
 * No counterpart in the reference.  Same result as q3cu_execute_rmsnorm, for
 * callers that must not allocate device memory when they normalise a row: it
 * takes no context and stages x, w and the output in a fixed array inside the
 * library's device image (Q3CU_STATIC_SCRATCH_BYTES per device) instead of a
 * cudaMalloc'd buffer.  Synchronous on `stream` (NULL: the legacy default
 * stream) of the current device.
 *   - size must be 1..Q3CU_STATIC_RMSNORM_MAX; larger sizes return
 *     Q3CU_ERR_INVALID and touch nothing.
 *   - The first call on a device looks up the array's address (and loads the
 *     library's device code if that has not happened yet); make one call per
 *     device before any stream capture.
 *   - There is one array per device: calls that overlap on the same device
 *     (several host threads or streams) race and must be serialised by the
 *     caller. */
#define Q3CU_STATIC_RMSNORM_MAX 16384
#define Q3CU_STATIC_SCRATCH_BYTES (256 + 3 * 4 * Q3CU_STATIC_RMSNORM_MAX)
q3cu_status q3cu_execute_rmsnorm_static(float *output, const float *input, const float *weight,
                                        int size, q3cu_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* Q3CU_H */
