// k_attn.cu -- decode attention for one token, bit-exact with the reference.
//
// Reference: src/cpu/qwen3_original.c:395-428 (per query head h, kv head
// h / kv_mul, positions t = 0..pos):
//     score = 0; for i < head_dim: score += q[i] * k_t[i]      (index order)
//     att[t] = score / sqrtf(head_dim)
//     softmax(att, pos + 1)                                   (:291-308)
//     xb = 0;   for t <= pos: for i: xb[i] += att[t] * v_t[i]   (position order)
// and softmax: max starts at 0 (NaN never wins), x = expf(x - max) summed in
// index order, then x /= sum.  Without FMA contraction every product and sum
// above is one rounding, so this kernel keeps each chain's order: a thread per
// position runs its 128-long score chain, the exponentials are the host libm's
// bits (q3_expf.h), one thread adds them in position order, and a thread per
// output element runs its value chain over the positions.  The scores and
// probabilities live in the caller's att buffer ([n_heads][seq_len], like the
// reference's RunState att), so any position up to seq_len is supported.
//
// One CTA per query head, 128 threads (one per element of the head).  Decode
// is latency-bound (a few microseconds per layer at short contexts); the
// position-order sum is the serial part and grows with pos.
#include "q3cu_internal.h"

namespace q3 {

constexpr int AT_HD = 128;

__global__ void __launch_bounds__(AT_HD) attn_decode_kernel(const float *__restrict__ q, const float *kc,
                                                            const float *vc, float *att, float *xb, int pos,
                                                            int kv_dim, int kv_mul, int seq_len) {
    __shared__ __align__(16) float qs[AT_HD];
    __shared__ ExpTab tab;
    __shared__ float red[AT_HD / 32];
    __shared__ float sum_sh;
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kvh = h / kv_mul;
    qs[tid] = q[int64_t(h) * AT_HD + tid];
    load_exp_table(tab);
    __syncthreads();
    float *a = att + int64_t(h) * seq_len;
    const float scale = __fsqrt_rn(float(AT_HD));            // sqrtf((float) head_dim)

    // scores: one thread per position, the dot product in index order
    float m = 0.0f;                                         // softmax's max starts at 0
    for (int t = tid; t <= pos; t += AT_HD) {
        const float *k = kc + int64_t(t) * kv_dim + kvh * AT_HD;
        float s = 0.0f;
#pragma unroll 8
        for (int i = 0; i < AT_HD; i += 4) {
            const float4 kv = *reinterpret_cast<const float4 *>(k + i);
            s = __fadd_rn(s, __fmul_rn(qs[i], kv.x));
            s = __fadd_rn(s, __fmul_rn(qs[i + 1], kv.y));
            s = __fadd_rn(s, __fmul_rn(qs[i + 2], kv.z));
            s = __fadd_rn(s, __fmul_rn(qs[i + 3], kv.w));
        }
        const float sc = __fdiv_rn(s, scale);
        a[t] = sc;
        m = fmaxf(m, sc);                                   // a NaN never replaces the max
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    // exp (the host libm's bits), then the sum in position order
    for (int t = tid; t <= pos; t += AT_HD) a[t] = expf_host(__fsub_rn(a[t], m), tab);
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        for (int t = 0; t <= pos; ++t) sum = __fadd_rn(sum, a[t]);
        sum_sh = sum;
    }
    __syncthreads();
    const float sum = sum_sh;
    for (int t = tid; t <= pos; t += AT_HD) a[t] = __fdiv_rn(a[t], sum);
    __syncthreads();
    // weighted values: one thread per element, positions in order
    const float *v = vc + kvh * AT_HD + tid;
    float acc = 0.0f;
#pragma unroll 4
    for (int t = 0; t <= pos; ++t) acc = __fadd_rn(acc, __fmul_rn(a[t], v[int64_t(t) * kv_dim]));
    xb[int64_t(h) * AT_HD + tid] = acc;
}

// Q/K RMSNorm + RoPE of one token (qwen3_original.c:361-393) with the
// rotation's cos/sin given by the host: the reference takes them from the C
// library (cosf/sinf of pos*freq, :368), so the host computing them with the
// same calls makes the rotation bit-exact.  One warp per head row (the n_heads
// query rows, then the n_kv key rows): lane 0 runs the row's sum of squares in
// index order (rmsnorm, :278-289), then every lane normalises and rotates four
// elements: x' = w*(ss*x), then (x, y) -> (x c - y s, x s + y c), each product
// and sum rounded once.
__global__ void __launch_bounds__(128) qk_norm_rope_tab_kernel(float *q, float *k, int n_heads, int n_kv,
                                                               const float *__restrict__ qn,
                                                               const float *__restrict__ kn, RopeTab tab,
                                                               float eps) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= n_heads + n_kv) return;                       // whole warps
    float *v = row < n_heads ? q + int64_t(row) * AT_HD : k + int64_t(row - n_heads) * AT_HD;
    const float *w = row < n_heads ? qn : kn;
    float ss = 0.0f;
    if (lane == 0) {
        for (int i = 0; i < AT_HD; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        ss = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(AT_HD)), eps)));
    }
    ss = __shfl_sync(FULL, ss, 0);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int j = lane + 32 * u;                         // pair (j, j + 64)
        const float x = __fmul_rn(w[j], __fmul_rn(ss, v[j]));
        const float y = __fmul_rn(w[j + 64], __fmul_rn(ss, v[j + 64]));
        const float c = tab.c[j], s = tab.s[j];
        v[j] = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
        v[j + 64] = __fadd_rn(__fmul_rn(x, s), __fmul_rn(y, c));
    }
}

cudaError_t launch_qk_norm_rope_tab(float *q, float *k, int n_heads, int n_kv, const float *qn, const float *kn,
                                    const RopeTab &tab, float eps, cudaStream_t stream) {
    qk_norm_rope_tab_kernel<<<(n_heads + n_kv + 3) / 4, 128, 0, stream>>>(q, k, n_heads, n_kv, qn, kn, tab, eps);
    return cudaGetLastError();
}

cudaError_t launch_attn_decode(const float *q, const float *kc, const float *vc, float *att, float *xb, int pos,
                               int n_heads, int kv_dim, int kv_mul, int seq_len, cudaStream_t stream) {
    attn_decode_kernel<<<n_heads, AT_HD, 0, stream>>>(q, kc, vc, att, xb, pos, kv_dim, kv_mul, seq_len);
    return cudaGetLastError();
}

}  // namespace q3
