// k_q8.cu -- Q8_0 kernels: activation quantize, dequantize, and the embedding
// row gather with dequant (+ optional re-quantize).
//
// All three are HBM streaming passes.  A Q8_0 group is 64 elements; one thread
// owns 16 bytes of input, so a group spans 16 lanes (f32), 8 lanes (bf16) or 4
// lanes (int8 codes) and its absmax is a short xor-shuffle inside that lane
// group.  Groups never straddle a row because every row length is a multiple
// of 64, so the row-major [rows][n] arrays are processed as one flat array of
// groups.
#include "q3cu_internal.h"

namespace q3 {

// ---------------------------------------------------------------------------
// quantize_q8: x [G*64] (f32 or bf16) -> q [G*64] int8, s [G] f32
// (src/cpu/qwen3_original.c:147-168)
// ---------------------------------------------------------------------------
template <typename T, int U>
__global__ void __launch_bounds__(256) quantize_q8_kernel(const T *__restrict__ x, int64_t groups,
                                                          int8_t *__restrict__ q, float *__restrict__ s) {
    constexpr int V = Vec<T>::N;              // elements per lane
    constexpr int LPG = GS / V;               // lanes per group
    constexpr int GPW = 32 / LPG;             // groups per warp step
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t steps = (groups + GPW - 1) / GPW;

    for (int64_t st0 = warp * U; st0 < steps; st0 += nwarps * U) {
        uint4 raw[U];
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int64_t g = (st0 + u) * GPW + lane / LPG;
            ok[u] = (st0 + u) < steps && g < groups;
            if (ok[u]) raw[u] = ld_nc_v4(reinterpret_cast<const uint8_t *>(x) + (g * GS + (lane % LPG) * V) * sizeof(T));
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if ((st0 + u) >= steps) break;                         // warp-uniform
            int64_t g = (st0 + u) * GPW + lane / LPG;
            float v[V];
            float m = 0.0f;
            if (ok[u]) {
                Vec<T>::widen(raw[u], v);
#pragma unroll
                for (int i = 0; i < V; ++i) m = amax_fold(m, v[i]);
            }
#pragma unroll
            for (int o = LPG / 2; o > 0; o >>= 1) m = amax_merge(m, __shfl_xor_sync(FULL, m, o));
            if (!ok[u]) continue;
            const Q8Scale gs = q8_prepare(m);
            int8_t *qp = q + g * GS + (lane % LPG) * V;
            if constexpr (V == 4) st_cs_u32(qp, q8_pack4(v, gs));
            else st_cs_v2(qp, make_uint2(q8_pack4(v, gs), q8_pack4(v + 4, gs)));
            if ((lane % LPG) == 0) st_cs_f32(s + g, gs.scale);
        }
    }
}

// ---------------------------------------------------------------------------
// dequantize: q [n] int8, s [n/64] -> x [n] f32 (qwen3_original.c:142-145)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) dequantize_kernel(const int8_t *__restrict__ q, const float *__restrict__ s,
                                                         int64_t n16, float *__restrict__ x) {
    const int64_t tid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = tid; i < n16; i += nthreads) {             // 16 codes per step
        uint4 c = ld_nc_v4(q + i * 16);
        float sc = __ldg(s + (i * 16) / GS);
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        float4 o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            o[k].x = __fmul_rn((float)(int8_t)(w[k] & 0xff), sc);
            o[k].y = __fmul_rn((float)(int8_t)((w[k] >> 8) & 0xff), sc);
            o[k].z = __fmul_rn((float)(int8_t)((w[k] >> 16) & 0xff), sc);
            o[k].w = __fmul_rn((float)(int8_t)(w[k] >> 24), sc);
        }
        float *xp = x + i * 16;
#pragma unroll
        for (int k = 0; k < 4; ++k) st_cs_v4(xp + 4 * k, f4_as_u4(o[k]));
    }
}

// ---------------------------------------------------------------------------
// embed_gather: one warp per lookup.  Lane owns 16 codes (one uint4) per step;
// a group is 4 lanes.  Writes f32 rows and/or Q8_0 rows.
// (dequantize qwen3_original.c:142-145 on the table row that the reference
//  copies at :342, then quantize :147-168)
// ---------------------------------------------------------------------------
template <bool F32, bool Q8>
__global__ void __launch_bounds__(256) embed_gather_kernel(const int8_t *__restrict__ tq, const float *__restrict__ ts,
                                                           int vocab, int dim, const int32_t *__restrict__ ids,
                                                           int64_t n, float *__restrict__ out, int8_t *__restrict__ oq,
                                                           float *__restrict__ os, uint32_t *status) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int steps = dim / 512;                       // full 512-code warp steps
    const int rem16 = (dim % 512) / 16;                // lanes active in the tail step
    for (int64_t i = warp; i < n; i += nwarps) {
        const int t = __ldg(ids + i);
        if (t < 0 || t >= vocab) {                     // out-of-range id: flag, skip row
            if (lane == 0) atomicOr(status, Q3CU_DEV_BAD_INDEX);
            continue;
        }
        const int8_t *row = tq + int64_t(t) * dim;
        const float *srow = ts + int64_t(t) * (dim / GS);
        const int nst = steps + (rem16 > 0 ? 1 : 0);    // warp steps of the row, the tail included
        // The codes and scales of EB steps are requested together, so the row's
        // loads wait out one latency per EB steps, not one per step.
        constexpr int EB = 4;
        for (int st0 = 0; st0 < nst; st0 += EB) {
            uint4 cb[EB];
            float sb[EB];
#pragma unroll
            for (int u = 0; u < EB; ++u) {
                const int st = st0 + u;
                const bool act = st < steps || (st == steps && lane < rem16);
                const int e = st * 512 + lane * 16;
                cb[u] = act ? ld_nc_v4(row + e) : make_uint4(0, 0, 0, 0);
                sb[u] = act ? __ldg(srow + e / GS) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < EB; ++u) {
                const int st = st0 + u;
                if (st >= nst) break;                  // warp-uniform
                const bool full = st < steps;
                const bool act = full || lane < rem16;
                const int e = st * 512 + lane * 16;    // element index of this lane
                const uint32_t w[4] = {cb[u].x, cb[u].y, cb[u].z, cb[u].w};
                const float sc = sb[u];
                float v[16];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    v[4 * k + 0] = __fmul_rn((float)(int8_t)(w[k] & 0xff), sc);
                    v[4 * k + 1] = __fmul_rn((float)(int8_t)((w[k] >> 8) & 0xff), sc);
                    v[4 * k + 2] = __fmul_rn((float)(int8_t)((w[k] >> 16) & 0xff), sc);
                    v[4 * k + 3] = __fmul_rn((float)(int8_t)(w[k] >> 24), sc);
                }
                if (F32 && act) {
                    float *op = out + i * dim + e;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        st_cs_v4(op + 4 * k, make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                                         __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3])));
                }
                if (Q8) {
                    float m = 0.0f;
#pragma unroll
                    for (int k = 0; k < 16; ++k) m = amax_fold(m, v[k]);
                    m = amax_merge(m, __shfl_xor_sync(FULL, m, 1));
                    m = amax_merge(m, __shfl_xor_sync(FULL, m, 2));
                    if (act) {
                        const Q8Scale gs = q8_prepare(m);
                        st_cs_v4(oq + i * dim + e, make_uint4(q8_pack4(v, gs), q8_pack4(v + 4, gs),
                                                              q8_pack4(v + 8, gs), q8_pack4(v + 12, gs)));
                        if ((lane & 3) == 0) st_cs_f32(os + i * (dim / GS) + e / GS, gs.scale);
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
cudaError_t launch_quantize_q8(const void *x, q3cu_dtype dt, int64_t elems, int8_t *q, float *s,
                               cudaStream_t stream, int sms) {
    const int64_t groups = elems / GS;
    if (groups == 0) return cudaSuccess;
    constexpr int U = 4;
    const int gpw = dt == Q3CU_F32 ? 2 : 4;
    const int64_t steps = (groups + gpw - 1) / gpw;
    const int64_t warps_needed = (steps + U - 1) / U;
    int64_t blocks = (warps_needed + 7) / 8;
    blocks = blocks < int64_t(sms) * 8 ? blocks : int64_t(sms) * 8;
    if (dt == Q3CU_F32)
        quantize_q8_kernel<float, U><<<unsigned(blocks), 256, 0, stream>>>(static_cast<const float *>(x), groups, q, s);
    else
        quantize_q8_kernel<bf16raw, U><<<unsigned(blocks), 256, 0, stream>>>(static_cast<const bf16raw *>(x), groups, q, s);
    return cudaGetLastError();
}

cudaError_t launch_dequantize_q8(const int8_t *q, const float *s, int64_t n, float *x, cudaStream_t stream, int sms) {
    const int64_t n16 = n / 16;
    if (n16 == 0) return cudaSuccess;
    int64_t blocks = (n16 + 255) / 256;
    blocks = blocks < int64_t(sms) * 8 ? blocks : int64_t(sms) * 8;
    dequantize_kernel<<<unsigned(blocks), 256, 0, stream>>>(q, s, n16, x);
    return cudaGetLastError();
}

cudaError_t launch_embed_gather(const int8_t *tq, const float *ts, int vocab, int dim, const int32_t *ids, int64_t n,
                                float *out, int8_t *oq, float *os, uint32_t *status, cudaStream_t stream, int sms) {
    if (n == 0) return cudaSuccess;
    int64_t blocks = (n + 7) / 8;                       // 8 warps per block, one lookup per warp
    blocks = blocks < int64_t(sms) * 16 ? blocks : int64_t(sms) * 16;
    const unsigned b = unsigned(blocks);
    if (out && oq)
        embed_gather_kernel<true, true><<<b, 256, 0, stream>>>(tq, ts, vocab, dim, ids, n, out, oq, os, status);
    else if (out)
        embed_gather_kernel<true, false><<<b, 256, 0, stream>>>(tq, ts, vocab, dim, ids, n, out, oq, os, status);
    else
        embed_gather_kernel<false, true><<<b, 256, 0, stream>>>(tq, ts, vocab, dim, ids, n, out, oq, os, status);
    return cudaGetLastError();
}

}  // namespace q3
