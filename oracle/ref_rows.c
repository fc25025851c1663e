/*
 * ref_rows.c -- row-batched, multi-threaded driver of the reference CPU engine.
 *
 * TEST AND CPU-BASELINE INFRASTRUCTURE ONLY: used by the CPU-baseline and reference
 * legs of bench.py to time the reference's own code on the host cores.
 *
 * Linked against oracle/_ref/libqwen3_ref.so, i.e. src/cpu/qwen3_original.c
 * compiled unmodified.  Each row calls the reference's exported functions
 * (`rmsnorm` :278-289, `quantize` :147-168, `dequantize` :142-145, `softmax`
 * :291-308) exactly as its forward() does.  The QK-norm rotation (:366-375)
 * and the SwiGLU gate (:449-450) are inline loops in forward() with no symbol
 * of their own, so those few lines are restated here (as in q3_oracle.c, which
 * tests/test_oracle_pin.py pins bit-exactly against the reference's forward()).
 * Rows are spread over `threads` OpenMP threads; rows are independent.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct { int8_t *q; float *s; } QuantizedTensor;   /* qwen3_original.c:43-46 */
extern int GS;                                             /* :20 */
void rmsnorm(float *o, float *x, float *weight, int size);
void softmax(float *x, int size);
void quantize(QuantizedTensor *qx, float *x, int n);
void dequantize(QuantizedTensor *qx, float *x, int n);

#define NT(t) ((t) > 1 ? (t) : 1)

void ref_rows_rmsnorm_q8(const float *x, const float *w, int64_t rows, int dim, int8_t *q, float *s, int threads) {
    GS = 64;
    #pragma omp parallel num_threads(NT(threads))
    {
        float *o = malloc((size_t)dim * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            rmsnorm(o, (float *)(x + r * dim), (float *)w, dim);
            QuantizedTensor qt = {q + r * dim, s + r * (dim / 64)};
            quantize(&qt, o, dim);
        }
        free(o);
    }
}

void ref_rows_quantize(const float *x, int64_t rows, int n, int8_t *q, float *s, int threads) {
    GS = 64;
    #pragma omp parallel for schedule(static) num_threads(NT(threads))
    for (int64_t r = 0; r < rows; r++) {
        QuantizedTensor qt = {q + r * n, s + r * (n / 64)};
        quantize(&qt, (float *)(x + r * n), n);
    }
}

void ref_rows_qk_norm_rope(float *q, float *k, const int32_t *pos, int64_t rows, int n_heads, int n_kv,
                           int head_dim, const float *q_norm, const float *k_norm, int threads) {
    GS = 64;
    #pragma omp parallel for num_threads(NT(threads)) schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int t = 0; t < 2; t++) {
            int nh = t == 0 ? n_heads : n_kv;
            float *base = t == 0 ? q + r * n_heads * head_dim : k + r * n_kv * head_dim;
            const float *nw = t == 0 ? q_norm : k_norm;
            for (int h = 0; h < nh; h++) {
                float *v = base + h * head_dim;
                rmsnorm(v, v, (float *)nw, head_dim);
                for (int j = 0; j < head_dim / 2; j++) {
                    float freq = powf(1e6, -(float)j / (head_dim / 2));
                    float c = cosf(pos[r] * freq), sn = sinf(pos[r] * freq);
                    float a = v[j], b = v[j + head_dim / 2];
                    v[j] = a * c - b * sn;
                    v[j + head_dim / 2] = a * sn + b * c;
                }
            }
        }
    }
}

void ref_rows_swiglu_q8(const float *hb, const float *hb2, int64_t rows, int n, int8_t *q, float *s, int threads) {
    GS = 64;
    #pragma omp parallel num_threads(NT(threads))
    {
        float *a = malloc((size_t)n * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            const float *h = hb + r * n, *g = hb2 + r * n;
            for (int i = 0; i < n; i++)
                a[i] = h[i] * (g[i] * (1.0f / (1.0f + expf(-h[i]))));
            QuantizedTensor qt = {q + r * n, s + r * (n / 64)};
            quantize(&qt, a, n);
        }
        free(a);
    }
}

void ref_rows_softmax(float *x, const int64_t *off, const int32_t *len, int64_t rows, int threads) {
    GS = 64;
    #pragma omp parallel for num_threads(NT(threads)) schedule(dynamic, 16)
    for (int64_t r = 0; r < rows; r++)
        softmax(x + off[r], len[r]);
}

void ref_rows_embed(const int8_t *tq, const float *ts, int vocab, int dim, const int32_t *ids, int64_t n,
                    float *out, int8_t *oq, float *os, int threads) {
    GS = 64;
    #pragma omp parallel for num_threads(NT(threads)) schedule(static)
    for (int64_t i = 0; i < n; i++) {
        int t = ids[i];
        if (t < 0 || t >= vocab) continue;
        QuantizedTensor src = {(int8_t *)tq + (int64_t)t * dim, (float *)ts + (int64_t)t * (dim / 64)};
        float *row = out + i * dim;
        dequantize(&src, row, dim);
        if (oq) {
            QuantizedTensor dst = {oq + i * dim, os + i * (dim / 64)};
            quantize(&dst, row, dim);
        }
    }
}

/* One decode token through the path's ops, in the order of forward()
 * (qwen3_original.c:333-468 without its matmuls and attention dot products):
 * the embedding row, then per layer RMSNorm + quantize (:353-356), the QK-norm
 * + RoPE loop (:361-393), softmax of the n_heads score rows of pos+1 (:416),
 * quantize of the attention output (:431), RMSNorm + quantize (:439-443),
 * SwiGLU + quantize (:449-453); then the final RMSNorm + quantize (:462-465).
 * Every layer reuses the same inputs (the matmuls that would produce fresh ones
 * are not on the path); q, k and the scores are updated in place. */
void ref_decode_ops(const int8_t *tq, const float *ts, int dim, int token, float *emb, const float *x,
                    const float *w, float *q, float *k, int n_heads, int n_kv, int head_dim, int pos,
                    const float *qn, const float *kn, float *sc, const float *ao, const float *hb,
                    const float *hb2, int hidden, int layers, int8_t *q8, float *s8) {
    GS = 64;
    const int ahd = n_heads * head_dim, n = pos + 1;
    const int big = dim > hidden ? dim : hidden;
    float *o = malloc((size_t)(big > ahd ? big : ahd) * 4);
    QuantizedTensor row = {(int8_t *)tq + (int64_t)token * dim, (float *)ts + (int64_t)token * (dim / 64)};
    dequantize(&row, emb, dim);
    QuantizedTensor out = {q8, s8};
    for (int l = 0; l < layers; l++) {
        rmsnorm(o, (float *)x, (float *)w, dim);
        quantize(&out, o, dim);
        ref_rows_qk_norm_rope(q, k, &pos, 1, n_heads, n_kv, head_dim, qn, kn, 1);
        for (int h = 0; h < n_heads; h++) softmax(sc + (int64_t)h * n, n);
        quantize(&out, (float *)ao, ahd);
        rmsnorm(o, (float *)x, (float *)w, dim);
        quantize(&out, o, dim);
        for (int i = 0; i < hidden; i++) o[i] = hb[i] * (hb2[i] * (1.0f / (1.0f + expf(-hb[i]))));
        quantize(&out, o, hidden);
    }
    rmsnorm(o, (float *)x, (float *)w, dim);
    quantize(&out, o, dim);
    free(o);
}
