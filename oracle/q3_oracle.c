/*
 * q3_oracle.c -- CPU oracle for the fused Qwen3 layer kernels.
 *
 * TEST INFRASTRUCTURE ONLY: the reference results the CUDA library is tested against, and the timed CPU
 * baseline.  Never linked into, loaded by or called from the product.
 *
 * Plain-C restatement of src/cpu/qwen3_original.c (the reference's CPU engine).
 * Build with `-O2 -ffp-contract=off` and without -ffast-math so that every
 * float operator rounds once, in the reference's order (see oracle/Makefile).
 */
#include "q3_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define GS Q3O_GS

/* ------------------------------------------------------------------------ */
/* primitives                                                                */
/* ------------------------------------------------------------------------ */

/* qwen3_original.c:278-289. */
void q3o_rmsnorm(float *o, const float *x, const float *w, int size) {
    float ss = 0;                                   /* sequential, index order */
    for (int j = 0; j < size; j++)
        ss += x[j] * x[j];
    ss = 1.0f / sqrtf((ss / size) + 1e-6f);
    for (int j = 0; j < size; j++)
        o[j] = w[j] * (ss * x[j]);
}

/* qwen3_original.c:291-308.  Note the max starts at 0, not -inf. */
void q3o_softmax(float *x, int size) {
    float max_val = 0;
    for (int i = 0; i < size; i++)
        if (x[i] > max_val)
            max_val = x[i];
    float sum = 0;
    for (int i = 0; i < size; i++) {
        x[i] = expf(x[i] - max_val);
        sum += x[i];
    }
    for (int i = 0; i < size; i++)
        x[i] /= sum;
}

/* qwen3_original.c:164: `(int8_t) round(quant_value)`. */
int8_t q3o_round_i8(float v) {
    double r = round((double)v);
    if (!(r > -2147483649.0 && r < 2147483648.0))   /* NaN, inf, out of int32 */
        return 0;                                   /* low byte of INT_MIN    */
    return (int8_t)(uint8_t)((uint32_t)(int32_t)r & 0xffu);
}

/* qwen3_original.c:147-168. */
void q3o_quantize(int8_t *q, float *s, const float *x, int n) {
    for (int g = 0; g < n / GS; g++) {
        float wmax = 0;
        for (int i = 0; i < GS; i++) {
            float val = fabsf(x[g * GS + i]);       /* fabs of a float is exact */
            if (val > wmax)
                wmax = val;
        }
        float scale = wmax / 127.0f;
        s[g] = scale;
        for (int i = 0; i < GS; i++) {
            float qv = x[g * GS + i] / scale;
            q[g * GS + i] = q3o_round_i8(qv);
        }
    }
}

/* qwen3_original.c:142-145. */
void q3o_dequantize(float *x, const int8_t *q, const float *s, int n) {
    for (int i = 0; i < n; i++)
        x[i] = q[i] * s[i / GS];
}

/* qwen3_original.c:361-376 / :378-393 for one head. */
void q3o_qk_norm_rope_head_theta(float *v, const float *norm_w, int head_dim, int pos, float theta) {
    q3o_rmsnorm(v, v, norm_w, head_dim);
    int half = head_dim / 2;
    for (int j = 0; j < half; j++) {
        float freq = powf(theta, -(float)j / half);
        float c = cosf(pos * freq), s = sinf(pos * freq);
        float x = v[j];
        float y = v[j + half];
        v[j] = x * c - y * s;
        v[j + half] = x * s + y * c;
    }
}

void q3o_qk_norm_rope_head(float *v, const float *norm_w, int head_dim, int pos) {
    q3o_qk_norm_rope_head_theta(v, norm_w, head_dim, pos, 1e6f);
}

/* qwen3_original.c:449-450. */
void q3o_swiglu(float *hb, const float *hb2, int n) {
    for (int i = 0; i < n; i++)
        hb[i] = hb[i] * (hb2[i] * (1.0f / (1.0f + expf(-hb[i]))));
}

/* qwen3_original.c:310-331. */
void q3o_matmul(float *xout, const int8_t *xq, const float *xs,
                const int8_t *wq, const float *ws, int n, int d) {
    #pragma omp parallel for
    for (int i = 0; i < d; i++) {
        float val = 0;
        int in = i * n;
        for (int j = 0; j <= n - GS; j += GS) {
            int32_t ival = 0;
            for (int k = 0; k < GS; k++)
                ival += xq[j + k] * wq[in + j + k];
            val += ((float)ival) * ws[(in + j) / GS] * xs[j / GS];
        }
        xout[i] = val;
    }
}

/* qwen3_original.c:395-428, the multi-head attention loop of one decode step,
 * with MetalContext::executeAttention's arguments (src/metal/MetalContext.h:86-87):
 * per query head h, kv head h / kv_mul, over positions 0..pos of the layer's
 * cache rows at key_cache + loff / value_cache + loff. */
void q3o_attention(float *xb, const float *q, float *att, const float *key_cache, const float *value_cache,
                   int pos, int head_dim, int n_heads, int n_kv_heads, int seq_len, int kv_dim, uint64_t loff,
                   int kv_mul) {
    (void)n_kv_heads;
    for (int h = 0; h < n_heads; h++) {
        const float *qh = q + h * head_dim;
        float *a = att + (int64_t)h * seq_len;
        for (int t = 0; t <= pos; t++) {
            const float *k = key_cache + loff + (int64_t)t * kv_dim + (h / kv_mul) * head_dim;
            float score = 0;
            for (int i = 0; i < head_dim; i++)
                score += qh[i] * k[i];
            a[t] = score / sqrtf(head_dim);
        }
        q3o_softmax(a, pos + 1);
        float *xh = xb + h * head_dim;
        memset(xh, 0, (size_t)head_dim * sizeof(float));
        for (int t = 0; t <= pos; t++) {
            const float *v = value_cache + loff + (int64_t)t * kv_dim + (h / kv_mul) * head_dim;
            float w = a[t];
            for (int i = 0; i < head_dim; i++)
                xh[i] += w * v[i];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* bf16                                                                      */
/* ------------------------------------------------------------------------ */

float q3o_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t q3o_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u)
        return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static void load_row(float *dst, const void *src, int dtype, int64_t off, int n) {
    if (dtype == 0) {
        memcpy(dst, (const float *)src + off, (size_t)n * 4);
    } else {
        const uint16_t *b = (const uint16_t *)src + off;
        for (int i = 0; i < n; i++) dst[i] = q3o_bf16_to_f32(b[i]);
    }
}

static void store_row(void *dst, int dtype, int64_t off, const float *src, int n) {
    if (dtype == 0) {
        memcpy((float *)dst + off, src, (size_t)n * 4);
    } else {
        uint16_t *b = (uint16_t *)dst + off;
        for (int i = 0; i < n; i++) b[i] = q3o_f32_to_bf16(src[i]);
    }
}

/* ------------------------------------------------------------------------ */
/* row-batched forms                                                         */
/* ------------------------------------------------------------------------ */

#define NT(t) ((t) > 1 ? (t) : 1)

void q3o_rows_rmsnorm(const void *x, int dtype, const float *w, int64_t rows, int dim,
                      void *out, int threads) {
    #pragma omp parallel num_threads(NT(threads)) if (threads > 1)
    {
        float *a = malloc((size_t)dim * 4), *o = malloc((size_t)dim * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            load_row(a, x, dtype, r * dim, dim);
            q3o_rmsnorm(o, a, w, dim);
            store_row(out, dtype, r * dim, o, dim);
        }
        free(a); free(o);
    }
}

void q3o_rows_rmsnorm_q8(const void *x, int dtype, const float *w, int64_t rows, int dim,
                         int8_t *q, float *s, int threads) {
    #pragma omp parallel num_threads(NT(threads)) if (threads > 1)
    {
        float *a = malloc((size_t)dim * 4), *o = malloc((size_t)dim * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            load_row(a, x, dtype, r * dim, dim);
            q3o_rmsnorm(o, a, w, dim);
            q3o_quantize(q + r * dim, s + r * (dim / GS), o, dim);
        }
        free(a); free(o);
    }
}

void q3o_rows_quantize(const void *x, int dtype, int64_t rows, int n,
                       int8_t *q, float *s, int threads) {
    #pragma omp parallel num_threads(NT(threads)) if (threads > 1)
    {
        float *a = malloc((size_t)n * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            load_row(a, x, dtype, r * n, n);
            q3o_quantize(q + r * n, s + r * (n / GS), a, n);
        }
        free(a);
    }
}

void q3o_rows_swiglu(void *hb, const void *hb2, int dtype, int64_t rows, int n, int threads) {
    #pragma omp parallel num_threads(NT(threads)) if (threads > 1)
    {
        float *a = malloc((size_t)n * 4), *b = malloc((size_t)n * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            load_row(a, hb, dtype, r * n, n);
            load_row(b, hb2, dtype, r * n, n);
            q3o_swiglu(a, b, n);
            store_row(hb, dtype, r * n, a, n);
        }
        free(a); free(b);
    }
}

void q3o_rows_swiglu_q8(const void *hb, const void *hb2, int dtype, int64_t rows, int n,
                        int8_t *q, float *s, int threads) {
    #pragma omp parallel num_threads(NT(threads)) if (threads > 1)
    {
        float *a = malloc((size_t)n * 4), *b = malloc((size_t)n * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            load_row(a, hb, dtype, r * n, n);
            load_row(b, hb2, dtype, r * n, n);
            q3o_swiglu(a, b, n);
            q3o_quantize(q + r * n, s + r * (n / GS), a, n);
        }
        free(a); free(b);
    }
}

void q3o_rows_qk_norm_rope(void *q, void *k, int dtype, const int32_t *pos, int64_t rows,
                           int n_heads, int n_kv, int head_dim,
                           const float *q_norm, const float *k_norm, float theta, int threads) {
    #pragma omp parallel num_threads(NT(threads)) if (threads > 1)
    {
        float *a = malloc((size_t)head_dim * 4);
        #pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            for (int h = 0; h < n_heads; h++) {
                int64_t off = (r * n_heads + h) * head_dim;
                load_row(a, q, dtype, off, head_dim);
                q3o_qk_norm_rope_head_theta(a, q_norm, head_dim, pos[r], theta);
                store_row(q, dtype, off, a, head_dim);
            }
            for (int h = 0; h < n_kv; h++) {
                int64_t off = (r * n_kv + h) * head_dim;
                load_row(a, k, dtype, off, head_dim);
                q3o_qk_norm_rope_head_theta(a, k_norm, head_dim, pos[r], theta);
                store_row(k, dtype, off, a, head_dim);
            }
        }
        free(a);
    }
}

void q3o_rows_softmax(float *x, const int64_t *off, const int32_t *len, int64_t rows, int threads) {
    #pragma omp parallel for num_threads(NT(threads)) if (threads > 1) schedule(dynamic, 16)
    for (int64_t r = 0; r < rows; r++)
        q3o_softmax(x + off[r], len[r]);
}

int64_t q3o_rows_embed(const int8_t *tq, const float *ts, int vocab, int dim,
                       const int32_t *ids, int64_t n, float *out, int8_t *oq, float *os,
                       int threads) {
    int64_t bad = 0;
    #pragma omp parallel num_threads(NT(threads)) if (threads > 1) reduction(+:bad)
    {
        float *row = malloc((size_t)dim * 4);
        #pragma omp for schedule(static)
        for (int64_t i = 0; i < n; i++) {
            int t = ids[i];
            if (t < 0 || t >= vocab) { bad++; continue; }
            q3o_dequantize(row, tq + (int64_t)t * dim, ts + (int64_t)t * (dim / GS), dim);
            if (out) memcpy(out + i * dim, row, (size_t)dim * 4);
            if (oq) q3o_quantize(oq + i * dim, os + i * (dim / GS), row, dim);
        }
        free(row);
    }
    return bad;
}

/* ------------------------------------------------------------------------ */
/* restated decode step                                                      */
/* ------------------------------------------------------------------------ */

/* qwen3_original.c:171-183: each tensor is int8 codes followed by f32 scales. */
static const uint8_t *map_q8(const uint8_t *p, int n, int64_t each,
                             const int8_t **qs, const float **ss) {
    for (int i = 0; i < n; i++) {
        qs[i] = (const int8_t *)p;
        p += each;
        ss[i] = (const float *)p;
        p += (each / GS) * 4;
    }
    return p;
}

int q3o_model_map(q3o_model *m, const void *image, int64_t bytes, int ctx_length) {
    memset(m, 0, sizeof(*m));
    if (bytes < 256) return 4;
    memcpy(&m->c, image, sizeof(q3o_config));
    q3o_config *c = &m->c;
    if (c->magic_number != 0x616a6331) return 1;           /* :238 */
    if (c->version != 1) return 2;                          /* :239 */
    if (c->group_size != GS) return 3;                      /* GS fixed at 64 */
    if (ctx_length != 0 && ctx_length <= c->seq_len)        /* :241-242 */
        c->seq_len = ctx_length;
    int64_t L = c->n_layers, dim = c->dim, hd = c->head_dim, hid = c->hidden_dim;
    int64_t ahd = (int64_t)c->n_heads * hd, kvd = (int64_t)c->n_kv_heads * hd;
    int64_t q8 = 0;
    #define Q8B(n) ((n) + ((n) / GS) * 4)
    q8 += Q8B((int64_t)c->vocab_size * dim);
    q8 += L * (Q8B(dim * ahd) + 2 * Q8B(dim * kvd) + Q8B(ahd * dim) + 3 * Q8B(dim * hid));
    if (!c->shared_classifier) q8 += Q8B(dim * (int64_t)c->vocab_size);
    int64_t need = 256 + 4 * (2 * L * dim + dim + 2 * L * hd) + q8;
    if (bytes < need) return 4;

    const float *f = (const float *)((const uint8_t *)image + 256);   /* :185-198 */
    m->rms_att = f;   f += L * dim;
    m->rms_ffn = f;   f += L * dim;
    m->rms_final = f; f += dim;
    m->q_norm = f;    f += L * hd;
    m->k_norm = f;    f += L * hd;
    const uint8_t *p = (const uint8_t *)f;
    const int8_t *tq; const float *tsc;
    p = map_q8(p, 1, (int64_t)c->vocab_size * dim, &tq, &tsc);       /* :201 */
    m->tok_q = tq; m->tok_s = tsc;
    #define ALLOC_LAYERS(a) do { m->a##_q = malloc(L * sizeof(void *)); m->a##_s = malloc(L * sizeof(void *)); \
        if (!m->a##_q || !m->a##_s) return 5; } while (0)
    ALLOC_LAYERS(wq); ALLOC_LAYERS(wk); ALLOC_LAYERS(wv); ALLOC_LAYERS(wo);
    ALLOC_LAYERS(w1); ALLOC_LAYERS(w2); ALLOC_LAYERS(w3);
    p = map_q8(p, L, dim * ahd, m->wq_q, m->wq_s);                    /* :207-214 */
    p = map_q8(p, L, dim * kvd, m->wk_q, m->wk_s);
    p = map_q8(p, L, dim * kvd, m->wv_q, m->wv_s);
    p = map_q8(p, L, ahd * dim, m->wo_q, m->wo_s);
    p = map_q8(p, L, dim * hid, m->w1_q, m->w1_s);
    p = map_q8(p, L, hid * dim, m->w2_q, m->w2_s);
    p = map_q8(p, L, dim * hid, m->w3_q, m->w3_s);
    if (c->shared_classifier) { m->cls_q = m->tok_q; m->cls_s = m->tok_s; }   /* :216 */
    else { const int8_t *cq; const float *cs; map_q8(p, 1, dim * (int64_t)c->vocab_size, &cq, &cs);
           m->cls_q = cq; m->cls_s = cs; }
    /* :203-205: the whole embedding table is dequantized at load. */
    m->tok_f32 = malloc((size_t)c->vocab_size * dim * 4);
    if (!m->tok_f32) return 5;
    for (int64_t v = 0; v < c->vocab_size; v++)
        q3o_dequantize(m->tok_f32 + v * dim, m->tok_q + v * dim, m->tok_s + v * (dim / GS), (int)dim);
    return 0;
}

void q3o_model_free(q3o_model *m) {
    free(m->wq_q); free(m->wq_s); free(m->wk_q); free(m->wk_s); free(m->wv_q); free(m->wv_s);
    free(m->wo_q); free(m->wo_s); free(m->w1_q); free(m->w1_s); free(m->w2_q); free(m->w2_s);
    free(m->w3_q); free(m->w3_s); free(m->tok_f32);
    memset(m, 0, sizeof(*m));
}

/* qwen3_original.c:98-121 (calloc'd buffers, zero KV cache). */
int q3o_state_alloc(q3o_state *s, const q3o_config *c) {
    int64_t ahd = (int64_t)c->n_heads * c->head_dim, kvd = (int64_t)c->n_kv_heads * c->head_dim;
    memset(s, 0, sizeof(*s));
    s->x = calloc(c->dim, 4);
    s->xb = calloc(ahd, 4);
    s->hb = calloc(c->hidden_dim, 4);
    s->hb2 = calloc(c->hidden_dim, 4);
    s->xq_q = calloc(ahd, 1); s->xq_s = calloc(ahd / GS, 4);
    s->hq_q = calloc(c->hidden_dim, 1); s->hq_s = calloc(c->hidden_dim / GS, 4);
    s->q = calloc(ahd, 4);
    s->att = calloc((int64_t)c->n_heads * c->seq_len, 4);
    s->logits = calloc(c->vocab_size, 4);
    s->key_cache = calloc((int64_t)c->n_layers * c->seq_len * kvd, 4);
    s->value_cache = calloc((int64_t)c->n_layers * c->seq_len * kvd, 4);
    if (!s->x || !s->xb || !s->hb || !s->hb2 || !s->q || !s->att || !s->logits ||
        !s->key_cache || !s->value_cache || !s->xq_q || !s->xq_s || !s->hq_q || !s->hq_s)
        return 5;
    return 0;
}

void q3o_state_free(q3o_state *s) {
    free(s->x); free(s->xb); free(s->hb); free(s->hb2); free(s->xq_q); free(s->xq_s);
    free(s->hq_q); free(s->hq_s); free(s->q); free(s->att); free(s->logits);
    free(s->key_cache); free(s->value_cache);
    memset(s, 0, sizeof(*s));
}

#define TAP(layer, id, ptr, nbytes) do { if (tap) tap(user, (layer), (id), (ptr), (int64_t)(nbytes)); } while (0)

/* qwen3_original.c:333-468. */
float *q3o_forward(q3o_model *m, q3o_state *s, int token, int pos, q3o_tap_fn tap, void *user) {
    const q3o_config *p = &m->c;
    int dim = p->dim, hd = p->head_dim, hid = p->hidden_dim;
    int kv_dim = p->n_kv_heads * hd;
    int kv_mul = p->n_heads / p->n_kv_heads;
    int ahd = p->n_heads * hd;

    memcpy(s->x, m->tok_f32 + (int64_t)token * dim, (size_t)dim * 4);      /* :342 */
    TAP(-1, Q3O_TAP_EMBED, s->x, dim * 4);

    for (int l = 0; l < p->n_layers; l++) {
        uint64_t loff = l * (uint64_t)p->seq_len * kv_dim;                  /* :348 */
        float *k = s->key_cache + loff + (int64_t)pos * kv_dim;
        float *v = s->value_cache + loff + (int64_t)pos * kv_dim;

        TAP(l, Q3O_TAP_ATT_RMS_IN, s->x, dim * 4);
        q3o_rmsnorm(s->xb, s->x, m->rms_att + (int64_t)l * dim, dim);      /* :353 */
        TAP(l, Q3O_TAP_ATT_RMS_OUT, s->xb, dim * 4);
        q3o_quantize(s->xq_q, s->xq_s, s->xb, dim);                         /* :356 */
        TAP(l, Q3O_TAP_ATT_XQ_Q, s->xq_q, dim);
        TAP(l, Q3O_TAP_ATT_XQ_S, s->xq_s, (dim / GS) * 4);
        q3o_matmul(s->q, s->xq_q, s->xq_s, m->wq_q[l], m->wq_s[l], dim, ahd);    /* :357-359 */
        q3o_matmul(k, s->xq_q, s->xq_s, m->wk_q[l], m->wk_s[l], dim, kv_dim);
        q3o_matmul(v, s->xq_q, s->xq_s, m->wv_q[l], m->wv_s[l], dim, kv_dim);
        TAP(l, Q3O_TAP_Q_PRE, s->q, ahd * 4);
        TAP(l, Q3O_TAP_K_PRE, k, kv_dim * 4);

        for (int h = 0; h < p->n_heads; h++)                                /* :361-376 */
            q3o_qk_norm_rope_head(s->q + h * hd, m->q_norm + (int64_t)l * hd, hd, pos);
        for (int h = 0; h < p->n_kv_heads; h++)                             /* :378-393 */
            q3o_qk_norm_rope_head(k + h * hd, m->k_norm + (int64_t)l * hd, hd, pos);
        TAP(l, Q3O_TAP_Q_POST, s->q, ahd * 4);
        TAP(l, Q3O_TAP_K_POST, k, kv_dim * 4);

        /* :395-428 (the reference parallelises over heads; heads are independent). */
        float *scores = tap ? malloc((size_t)p->n_heads * (pos + 1) * 4) : NULL;
        for (int h = 0; h < p->n_heads; h++) {
            float *qh = s->q + h * hd;
            float *att = s->att + (int64_t)h * p->seq_len;
            for (int t = 0; t <= pos; t++) {
                float *kt = s->key_cache + loff + (int64_t)t * kv_dim + (h / kv_mul) * hd;
                float score = 0;
                for (int i = 0; i < hd; i++)
                    score += qh[i] * kt[i];
                att[t] = score / sqrtf(hd);                                 /* :412 */
            }
            if (scores) memcpy(scores + (int64_t)h * (pos + 1), att, (size_t)(pos + 1) * 4);
            q3o_softmax(att, pos + 1);                                      /* :416 */
            float *xbh = s->xb + h * hd;
            memset(xbh, 0, (size_t)hd * 4);
            for (int t = 0; t <= pos; t++) {
                float *vt = s->value_cache + loff + (int64_t)t * kv_dim + (h / kv_mul) * hd;
                float a = att[t];
                for (int i = 0; i < hd; i++)
                    xbh[i] += a * vt[i];
            }
        }
        if (scores) {
            TAP(l, Q3O_TAP_SCORES, scores, (int64_t)p->n_heads * (pos + 1) * 4);
            for (int h = 0; h < p->n_heads; h++)
                memcpy(scores + (int64_t)h * (pos + 1), s->att + (int64_t)h * p->seq_len, (size_t)(pos + 1) * 4);
            TAP(l, Q3O_TAP_PROBS, scores, (int64_t)p->n_heads * (pos + 1) * 4);
            free(scores);
        }
        TAP(l, Q3O_TAP_ATT_OUT, s->xb, ahd * 4);

        q3o_quantize(s->xq_q, s->xq_s, s->xb, ahd);                         /* :431 */
        TAP(l, Q3O_TAP_ATT_OUT_Q, s->xq_q, ahd);
        TAP(l, Q3O_TAP_ATT_OUT_S, s->xq_s, (ahd / GS) * 4);
        q3o_matmul(s->xb, s->xq_q, s->xq_s, m->wo_q[l], m->wo_s[l], ahd, dim);   /* :432 */
        for (int i = 0; i < dim; i++)                                       /* :435-436 */
            s->x[i] += s->xb[i];

        TAP(l, Q3O_TAP_FFN_RMS_IN, s->x, dim * 4);
        q3o_rmsnorm(s->xb, s->x, m->rms_ffn + (int64_t)l * dim, dim);      /* :439 */
        TAP(l, Q3O_TAP_FFN_RMS_OUT, s->xb, dim * 4);
        q3o_quantize(s->xq_q, s->xq_s, s->xb, dim);                         /* :443 */
        TAP(l, Q3O_TAP_FFN_XQ_Q, s->xq_q, dim);
        TAP(l, Q3O_TAP_FFN_XQ_S, s->xq_s, (dim / GS) * 4);
        q3o_matmul(s->hb, s->xq_q, s->xq_s, m->w1_q[l], m->w1_s[l], dim, hid);   /* :444-445 */
        q3o_matmul(s->hb2, s->xq_q, s->xq_s, m->w3_q[l], m->w3_s[l], dim, hid);
        TAP(l, Q3O_TAP_HB_PRE, s->hb, hid * 4);
        TAP(l, Q3O_TAP_HB2, s->hb2, hid * 4);
        q3o_swiglu(s->hb, s->hb2, hid);                                     /* :449-450 */
        TAP(l, Q3O_TAP_HB_POST, s->hb, hid * 4);
        q3o_quantize(s->hq_q, s->hq_s, s->hb, hid);                         /* :453 */
        TAP(l, Q3O_TAP_HQ_Q, s->hq_q, hid);
        TAP(l, Q3O_TAP_HQ_S, s->hq_s, (hid / GS) * 4);
        q3o_matmul(s->xb, s->hq_q, s->hq_s, m->w2_q[l], m->w2_s[l], hid, dim);   /* :454 */
        for (int i = 0; i < dim; i++)                                       /* :457-458 */
            s->x[i] += s->xb[i];
    }

    int L = p->n_layers;
    TAP(L, Q3O_TAP_FINAL_RMS_IN, s->x, dim * 4);
    q3o_rmsnorm(s->x, s->x, m->rms_final, dim);                             /* :462 */
    TAP(L, Q3O_TAP_FINAL_RMS_OUT, s->x, dim * 4);
    q3o_quantize(s->xq_q, s->xq_s, s->x, dim);                              /* :465 */
    TAP(L, Q3O_TAP_FINAL_XQ_Q, s->xq_q, dim);
    TAP(L, Q3O_TAP_FINAL_XQ_S, s->xq_s, (dim / GS) * 4);
    q3o_matmul(s->logits, s->xq_q, s->xq_s, m->cls_q, m->cls_s, dim, p->vocab_size);   /* :466 */
    TAP(L, Q3O_TAP_LOGITS, s->logits, (int64_t)p->vocab_size * 4);
    return s->logits;
}
