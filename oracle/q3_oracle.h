/*
 * q3_oracle.h -- CPU oracle for the fused Qwen3 layer kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the arithmetic in
 * the reference CPU engine `src/cpu/qwen3_original.c` (qwen3.c, int8 Q8_0 forward
 * pass).  It exists so that tests, the smoke check and the CPU baseline leg of
 * the benchmark can check the CUDA library against the reference's semantics.
 * No product code path may link, load or call it.
 *
 * Every function follows one reference function or inline loop, cited as
 * file:line below.  Operation order, rounding points and libm calls are kept
 * identical so that results are bit-identical to the reference when this file
 * is compiled with `-O2 -ffp-contract=off` (no -ffast-math): float arithmetic is
 * IEEE binary32 with one rounding per operator, sums are sequential in index
 * order, and transcendental functions are the host libm's (`expf`, `powf`,
 * `sinf`, `cosf`, `sqrtf`, `round`), exactly as in the reference.
 *
 * Pinning: `tests/test_oracle_pin.py` checks these functions against the
 * reference itself compiled from its own sources (oracle/Makefile, target
 * `ref`) and against the golden fixtures in tests/golden/ that were generated
 * from that compiled reference.
 */
#ifndef Q3_ORACLE_H
#define Q3_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Q8_0 group size.  The reference keeps it in the global `int GS`
 * (src/cpu/qwen3_original.c:20), set from the checkpoint header at :244; every
 * checkpoint the exporter writes uses 64 (scripts/export.py:76). */
#define Q3O_GS 64

/* ---- primitives ------------------------------------------------------- */

/* qwen3_original.c:278-289 `rmsnorm`.  o may alias x. */
void q3o_rmsnorm(float *o, const float *x, const float *w, int size);

/* qwen3_original.c:291-308 `softmax`, in place.  The running max starts at 0. */
void q3o_softmax(float *x, int size);

/* qwen3_original.c:147-168 `quantize`: n/64 groups, scale = absmax/127,
 * code = (int8_t)round(x/scale).  n must be a multiple of 64 (the reference
 * silently ignores a ragged tail: the loop runs n/GS groups). */
void q3o_quantize(int8_t *q, float *s, const float *x, int n);

/* qwen3_original.c:142-145 `dequantize`: x[i] = q[i] * s[i/64]. */
void q3o_dequantize(float *x, const int8_t *q, const float *s, int n);

/* The float-to-int8 conversion of quantize, `(int8_t) round(quant_value)`
 * (qwen3_original.c:164).  Out-of-range results are undefined in C; the x86-64
 * build truncates with cvttsd2si, whose invalid result (NaN, +-inf, |v| >= 2^31)
 * is INT_MIN, and keeps the low byte.  This restates that observed behaviour
 * (pinned against the compiled reference in tests/test_oracle_pin.py). */
int8_t q3o_round_i8(float v);

/* qwen3_original.c:361-376 (query heads) and :378-393 (key heads): per-head
 * RMSNorm with the layer's q_norm/k_norm weights (:365, :382), then the
 * rotate-half RoPE with freq = powf(1e6, -(float)j/(hd/2)) (:367, :384). */
void q3o_qk_norm_rope_head(float *v, const float *norm_w, int head_dim, int pos);

/* Same with theta as a parameter (the reference hard-codes 1e6). */
void q3o_qk_norm_rope_head_theta(float *v, const float *norm_w, int head_dim, int pos, float theta);

/* qwen3_original.c:449-450: hb[i] *= hb2[i] * (1/(1+expf(-hb[i]))), in place. */
void q3o_swiglu(float *hb, const float *hb2, int n);

/* qwen3_original.c:310-331 `matmul`: W (d,n) Q8_0 @ x (n,) Q8_0 -> xout (d,). */
void q3o_matmul(float *xout, const int8_t *xq, const float *xs,
                const int8_t *wq, const float *ws, int n, int d);

/* qwen3_original.c:395-428: scores q.k / sqrtf(head_dim) over positions
 * 0..pos, softmax, weighted sum of the values, for every query head (kv head
 * h / kv_mul); arguments as MetalContext::executeAttention
 * (src/metal/MetalContext.h:86-87).  att: [n_heads][seq_len] scratch (rows hold
 * the probabilities afterwards); xb: [n_heads][head_dim]. */
void q3o_attention(float *xb, const float *q, float *att, const float *key_cache, const float *value_cache,
                   int pos, int head_dim, int n_heads, int n_kv_heads, int seq_len, int kv_dim, uint64_t loff,
                   int kv_mul);

/* ---- bf16 helpers (inputs of the bf16 configurations) ------------------- */

/* bf16 -> f32 is exact (a 16-bit shift).  f32 -> bf16 rounds to nearest even,
 * NaN kept quiet. */
float q3o_bf16_to_f32(uint16_t b);
uint16_t q3o_f32_to_bf16(float f);

/* ---- row-batched forms (one reference call per row) --------------------- */
/* dtype: 0 = f32, 1 = bf16.  Float outputs of bf16 inputs are rounded to bf16.
 * `threads` <= 1 runs single-threaded, else an OpenMP parallel-for over rows
 * (each row is independent, so results do not depend on the thread count). */

void q3o_rows_rmsnorm(const void *x, int dtype, const float *w, int64_t rows, int dim,
                      void *out, int threads);
void q3o_rows_rmsnorm_q8(const void *x, int dtype, const float *w, int64_t rows, int dim,
                         int8_t *q, float *s, int threads);
void q3o_rows_quantize(const void *x, int dtype, int64_t rows, int n,
                       int8_t *q, float *s, int threads);
void q3o_rows_swiglu(void *hb, const void *hb2, int dtype, int64_t rows, int n, int threads);
void q3o_rows_swiglu_q8(const void *hb, const void *hb2, int dtype, int64_t rows, int n,
                        int8_t *q, float *s, int threads);
/* q: [rows][n_heads][head_dim], k: [rows][n_kv][head_dim], in place; pos[rows]. */
void q3o_rows_qk_norm_rope(void *q, void *k, int dtype, const int32_t *pos, int64_t rows,
                           int n_heads, int n_kv, int head_dim,
                           const float *q_norm, const float *k_norm, float theta, int threads);
/* Ragged rows: row r is x[off[r] .. off[r]+len[r]). */
void q3o_rows_softmax(float *x, const int64_t *off, const int32_t *len, int64_t rows, int threads);
/* Embedding lookup: dequantize table row ids[i] (qwen3_original.c:142-145
 * applied to the table at :203-205, gathered by the memcpy at :342), then
 * optionally re-quantize it (:147-168).  Out-of-range ids leave the row
 * untouched and are counted in the return value. */
int64_t q3o_rows_embed(const int8_t *tq, const float *ts, int vocab, int dim,
                       const int32_t *ids, int64_t n, float *out, int8_t *oq, float *os,
                       int threads);

/* ---- restated decode step (qwen3_original.c:333-468) -------------------- */

typedef struct {
    int magic_number, version, dim, hidden_dim, n_layers, n_heads, n_kv_heads,
        vocab_size, seq_len, head_dim, shared_classifier, group_size;
} q3o_config;   /* qwen3_original.c:28-41 */

typedef struct {
    q3o_config c;
    const float *rms_att, *rms_ffn, *rms_final, *q_norm, *k_norm;
    const int8_t *tok_q;  const float *tok_s;
    const int8_t **wq_q, **wk_q, **wv_q, **wo_q, **w1_q, **w2_q, **w3_q;
    const float  **wq_s, **wk_s, **wv_s, **wo_s, **w1_s, **w2_s, **w3_s;
    const int8_t *cls_q; const float *cls_s;
    float *tok_f32;      /* whole table dequantized at load, as the reference does */
} q3o_model;

typedef struct {
    float *x, *xb, *hb, *hb2, *q, *att, *logits, *key_cache, *value_cache;
    int8_t *xq_q, *hq_q; float *xq_s, *hq_s;
} q3o_state;

/* Tap ids passed to the tap callback, one per op input/output of a layer. */
enum {
    Q3O_TAP_EMBED = 0,        /* x after the embedding gather (layer -1)            */
    Q3O_TAP_ATT_RMS_IN,       /* x fed to the attention rmsnorm                     */
    Q3O_TAP_ATT_RMS_OUT,      /* xb                                                 */
    Q3O_TAP_ATT_XQ_Q,         /* int8 codes of quantize(xb, dim)                    */
    Q3O_TAP_ATT_XQ_S,         /* scales                                             */
    Q3O_TAP_Q_PRE,            /* q before QK-norm + RoPE (n_heads*hd)               */
    Q3O_TAP_K_PRE,            /* k before (n_kv*hd)                                 */
    Q3O_TAP_Q_POST,           /* q after                                            */
    Q3O_TAP_K_POST,           /* k after                                            */
    Q3O_TAP_SCORES,           /* attention scores before softmax, [n_heads][pos+1]  */
    Q3O_TAP_PROBS,            /* after softmax                                      */
    Q3O_TAP_ATT_OUT,          /* xb attention output (all_heads_dim)                */
    Q3O_TAP_ATT_OUT_Q,        /* codes of quantize(xb, all_heads_dim)               */
    Q3O_TAP_ATT_OUT_S,
    Q3O_TAP_FFN_RMS_IN,
    Q3O_TAP_FFN_RMS_OUT,
    Q3O_TAP_FFN_XQ_Q,
    Q3O_TAP_FFN_XQ_S,
    Q3O_TAP_HB_PRE,           /* w1 output (hidden)                                 */
    Q3O_TAP_HB2,              /* w3 output                                          */
    Q3O_TAP_HB_POST,          /* after SwiGLU                                       */
    Q3O_TAP_HQ_Q,             /* codes of quantize(hb, hidden)                      */
    Q3O_TAP_HQ_S,
    Q3O_TAP_FINAL_RMS_IN,     /* layer = n_layers                                   */
    Q3O_TAP_FINAL_RMS_OUT,
    Q3O_TAP_FINAL_XQ_Q,
    Q3O_TAP_FINAL_XQ_S,
    Q3O_TAP_LOGITS,
    Q3O_TAP_COUNT
};

typedef void (*q3o_tap_fn)(void *user, int layer, int tap, const void *data, int64_t bytes);

/* Map a v1 checkpoint image (qwen3_original.c:185-217, header checks :236-244).
 * Returns 0 on success, 1 bad magic, 2 bad version, 3 group size != 64,
 * 4 image too small, 5 allocation failure. */
int q3o_model_map(q3o_model *m, const void *image, int64_t bytes, int ctx_length);
void q3o_model_free(q3o_model *m);
int q3o_state_alloc(q3o_state *s, const q3o_config *c);
void q3o_state_free(q3o_state *s);
/* One decode step; returns logits.  `tap` may be NULL. */
float *q3o_forward(q3o_model *m, q3o_state *s, int token, int pos, q3o_tap_fn tap, void *user);

#ifdef __cplusplus
}
#endif
#endif
