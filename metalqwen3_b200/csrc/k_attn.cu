// k_attn.cu -- decode attention for one token, bit-exact with the reference.
//
// Reference: src/cpu/qwen3_original.c:395-428 (per query head h, kv head
// h / kv_mul, positions t = 0..pos):
//     score = 0; for i < head_dim: score += q[i] * k_t[i]      (index order)
//     att[t] = score / sqrtf(head_dim)
//     softmax(att, pos + 1)                                   (:291-308)
//     xb = 0;   for t <= pos: for i: xb[i] += att[t] * v_t[i]   (position order)
//     quantize(xq, xb, n_heads * head_dim)                    (:431, fused here)
// and softmax: max starts at 0 (NaN never wins), x = expf(x - max) summed in
// index order, then x /= sum.  Without FMA contraction every product and sum
// above is one rounding, so this kernel keeps each chain's order: a thread per
// position runs its 128-long score chain, the exponentials are the host libm's
// bits (q3_expf.h), one thread adds them in position order, and a thread per
// output element runs its value chain over the positions.  The scores and
// probabilities live in the caller's att buffer ([n_heads][seq_len], like the
// reference's RunState att), so any position up to seq_len is supported.
//
// One CTA per query head, 128 threads (one per element of the head).  K and V
// reach shared memory in chunks of 128 positions by cp.async, double-buffered
// (64 KB per chunk in flight, the next chunk loading while this one is used);
// K rows are padded to 528 B so a thread per position reads its row without
// bank conflicts.  The position-order probability sum is the serial part.
#include "q3cu_internal.h"

namespace q3 {

constexpr int AT_HD = 128;
constexpr int AT_CH = 128;                                  // positions per staged chunk
constexpr int AT_KROW = AT_HD * 4 + 16;                     // padded K row: 33 x 16 B, conflict-free float4 reads
constexpr size_t AT_BUF = size_t(AT_CH) * AT_KROW;          // 67,584 B per chunk buffer
constexpr size_t AT_SMEM = 2 * AT_BUF;                      // double-buffered

// Copies rows c0 .. c0+n-1 of a cache (this kv head's 128 floats of each) into
// buf with 16-byte cp.async pieces, `rowb` bytes apart; one commit group.
__device__ __forceinline__ void attn_stage(uint8_t *buf, const float *cache, int c0, int n, int kv_dim, int kvh,
                                           int rowb, int tid) {
    for (int f = tid; f < n * 32; f += AT_HD) {
        const int r = f >> 5, pc = f & 31;
        cp_async16(buf + r * rowb + pc * 16, cache + int64_t(c0 + r) * kv_dim + kvh * AT_HD + pc * 4);
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(AT_HD, 1) attn_decode_kernel(const float *__restrict__ q, const float *kc,
                                                               const float *vc, float *att, int8_t *xq, float *xs,
                                                               const StepParams *__restrict__ sp, int kv_dim,
                                                               int kv_mul, int seq_len) {
    extern __shared__ __align__(16) uint8_t tiles[];        // [2][AT_BUF]
    __shared__ __align__(16) float qs[AT_HD];
    __shared__ ExpTab tab;
    __shared__ float red[AT_HD / 32];
    __shared__ float sum_sh;
    __shared__ float gmax[2];
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kvh = h / kv_mul;
    const int pos = sp->pos;                                // this step's position (device memory)
    const int npos = pos + 1, nch = (npos + AT_CH - 1) / AT_CH;
    griddep_launch_dependents();                  // a dependent-launched successor may start its own prologue
    qs[tid] = q[int64_t(h) * AT_HD + tid];
    load_exp_table(tab);
    float *a = att + int64_t(h) * seq_len;
    const float scale = __fsqrt_rn(float(AT_HD));            // sqrtf((float) head_dim)

    // scores, chunk by chunk (the next chunk's K rows in flight): thread t
    // runs position c0 + t's dot product in index order from shared memory
    float m = 0.0f;                                         // softmax's max starts at 0
    attn_stage(tiles, kc, 0, npos < AT_CH ? npos : AT_CH, kv_dim, kvh, AT_KROW, tid);
    for (int c = 0; c < nch; ++c) {
        const int c0 = c * AT_CH, n = npos - c0 < AT_CH ? npos - c0 : AT_CH;
        if (c + 1 < nch) {
            const int n1 = npos - c0 - AT_CH < AT_CH ? npos - c0 - AT_CH : AT_CH;
            attn_stage(tiles + ((c + 1) & 1) * AT_BUF, kc, c0 + AT_CH, n1, kv_dim, kvh, AT_KROW, tid);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();                                     // chunk c landed (every thread's pieces)
        if (tid < n) {
            const float4 *kr = reinterpret_cast<const float4 *>(tiles + (c & 1) * AT_BUF + tid * AT_KROW);
            float s = 0.0f;
#pragma unroll 8
            for (int i4 = 0; i4 < AT_HD / 4; ++i4) {
                const float4 kv = kr[i4];
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4], kv.x));
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4 + 1], kv.y));
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4 + 2], kv.z));
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4 + 3], kv.w));
            }
            const float sc = __fdiv_rn(s, scale);
            a[c0 + tid] = sc;
            m = fmaxf(m, sc);                                // a NaN never replaces the max
        }
        __syncthreads();                                     // before the buffer is refilled
    }
    // the first V chunk streams in while the softmax runs
    attn_stage(tiles, vc, 0, npos < AT_CH ? npos : AT_CH, kv_dim, kvh, AT_HD * 4, tid);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    // exp (the host libm's bits), then the sum in position order
    for (int t = tid; t < npos; t += AT_HD) a[t] = expf_host(__fsub_rn(a[t], m), tab);
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        for (int t = 0; t < npos; ++t) sum = __fadd_rn(sum, a[t]);
        sum_sh = sum;
    }
    __syncthreads();
    const float sum = sum_sh;
    for (int t = tid; t < npos; t += AT_HD) a[t] = __fdiv_rn(a[t], sum);
    __syncthreads();
    // weighted values: thread i runs element i's chain over the positions in order
    float acc = 0.0f;
    for (int c = 0; c < nch; ++c) {
        const int c0 = c * AT_CH, n = npos - c0 < AT_CH ? npos - c0 : AT_CH;
        if (c + 1 < nch) {
            const int n1 = npos - c0 - AT_CH < AT_CH ? npos - c0 - AT_CH : AT_CH;
            attn_stage(tiles + ((c + 1) & 1) * AT_BUF, vc, c0 + AT_CH, n1, kv_dim, kvh, AT_HD * 4, tid);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *vt = reinterpret_cast<const float *>(tiles + (c & 1) * AT_BUF) + tid;
        const float *at = a + c0;
#pragma unroll 8
        for (int t = 0; t < n; ++t) acc = __fadd_rn(acc, __fmul_rn(at[t], vt[t * AT_HD]));
        __syncthreads();
    }
    // the quantize that follows (:431): the head's 128 outputs are Q8_0 groups
    // 2h and 2h+1 -- group absmax (strict >, from 0), scale = wmax / 127,
    // code = (int8) round(x / scale), the reference's operations exactly
    float gm = warp_max(fmaxf(0.0f, fabsf(acc)));           // from 0; a NaN never wins
    if (lane == 0) red[warp] = gm;
    __syncthreads();
    if (tid < 2) gmax[tid] = fmaxf(red[2 * tid], red[2 * tid + 1]);
    __syncthreads();
    const float qscale = q8_scale(gmax[tid >> 6]);
    xq[int64_t(h) * AT_HD + tid] = int8_t(q8_code(acc, qscale));
    if ((tid & 63) == 0) xs[int64_t(h) * 2 + (tid >> 6)] = qscale;
}

// Q/K RMSNorm + RoPE of one token (qwen3_original.c:361-393) with the
// rotation's cos/sin given by the host: the reference takes them from the C
// library (cosf/sinf of pos*freq, :367-368), so the host computing them with
// the same calls makes the rotation bit-exact; they reach the device in the
// step's parameters, with the position.  The Q|K|V matmul left this token's
// rows in qkv = [q | k | v]: one warp per head row normalises and rotates the
// n_heads query rows in place and the n_kv key rows into their cache row at
// pos (:349-350, keys rotated in the cache as the reference does), and n_kv
// more warps copy the value rows into theirs.  Lane 0 runs a row's sum of
// squares in index order (rmsnorm, :278-289); then every lane normalises and
// rotates four elements: x' = w*(ss*x), (x, y) -> (x c - y s, x s + y c), each
// product and sum rounded once.
__global__ void __launch_bounds__(128) qk_norm_rope_step_kernel(float *qkv, float *kc, float *vc, int n_heads, int n_kv,
                                                                const float *__restrict__ qn,
                                                                const float *__restrict__ kn,
                                                                const StepParams *__restrict__ sp, float eps) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= n_heads + 2 * n_kv) return;                  // whole warps
    const int kv_dim = n_kv * AT_HD, pos = sp->pos;
    if (row >= n_heads + n_kv) {                              // value row: copy into the cache
        const int r = row - n_heads - n_kv;
        const float *src = qkv + int64_t(n_heads) * AT_HD + kv_dim + r * AT_HD;
        float *dst = vc + int64_t(pos) * kv_dim + r * AT_HD;
        reinterpret_cast<float4 *>(dst)[lane] = reinterpret_cast<const float4 *>(src)[lane];
        return;
    }
    const bool isq = row < n_heads;
    const float *v = isq ? qkv + int64_t(row) * AT_HD : qkv + int64_t(n_heads) * AT_HD + (row - n_heads) * AT_HD;
    float *o = isq ? qkv + int64_t(row) * AT_HD : kc + int64_t(pos) * kv_dim + (row - n_heads) * AT_HD;
    const float *w = isq ? qn : kn;
    float ss = 0.0f;
    if (lane == 0) {
        for (int i = 0; i < AT_HD; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        ss = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(AT_HD)), eps)));
    }
    ss = __shfl_sync(FULL, ss, 0);
    float x[2], y[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {                            // read the row before any lane writes it
        const int j = lane + 32 * u;
        x[u] = __fmul_rn(w[j], __fmul_rn(ss, v[j]));
        y[u] = __fmul_rn(w[j + 64], __fmul_rn(ss, v[j + 64]));
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < 2; ++u) {                            // pair (j, j + 64)
        const int j = lane + 32 * u;
        const float c = sp->c[j], s = sp->s[j];
        o[j] = __fsub_rn(__fmul_rn(x[u], c), __fmul_rn(y[u], s));
        o[j + 64] = __fadd_rn(__fmul_rn(x[u], s), __fmul_rn(y[u], c));
    }
}

cudaError_t launch_qk_norm_rope_step(float *qkv, float *kc, float *vc, int n_heads, int n_kv, const float *qn,
                                     const float *kn, const StepParams *sp, float eps, cudaStream_t stream) {
    qk_norm_rope_step_kernel<<<(n_heads + 2 * n_kv + 3) / 4, 128, 0, stream>>>(qkv, kc, vc, n_heads, n_kv, qn, kn,
                                                                                 sp, eps);
    return cudaGetLastError();
}

__global__ void set_step_kernel(StepParams *sp, StepParams v) {
    reinterpret_cast<uint32_t *>(sp)[threadIdx.x] = reinterpret_cast<const uint32_t *>(&v)[threadIdx.x];
}

cudaError_t launch_set_step(StepParams *sp, const StepParams &v, cudaStream_t stream) {
    set_step_kernel<<<1, sizeof(StepParams) / 4, 0, stream>>>(sp, v);
    return cudaGetLastError();
}

cudaError_t launch_attn_decode(const float *q, const float *kc, const float *vc, float *att, int8_t *xq, float *xs,
                               const StepParams *sp, int n_heads, int kv_dim, int kv_mul, int seq_len,
                               cudaStream_t stream) {
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(attn_decode_kernel), AT_SMEM, 24);
    if (e != cudaSuccess) return e;
    attn_decode_kernel<<<n_heads, AT_HD, AT_SMEM, stream>>>(q, kc, vc, att, xq, xs, sp, kv_dim, kv_mul, seq_len);
    return cudaGetLastError();
}

}  // namespace q3
