// k_swiglu.cu -- SwiGLU gate, in place or fused with the Q8_0 quantize that
// follows it in the FFN.
//
// Reference: src/cpu/qwen3_original.c:449-450 and :453
//     hb[i] *= hb2[i] * (1.0f / (1.0f + expf(-hb[i])));
//     quantize(&s->hq, s->hb, hidden_dim);
// (shaders/swiglu.metal:37-39 associates the product differently; the CPU
// order is the reference here.)  Every operator is one IEEE binary32 rounding
// and expf is q3_expf_tab, which returns the host libm's bits, so the float
// output and the Q8_0 codes/scales are bit-exact.
//
// Layout: [rows][hidden] with hidden % 64 == 0 is processed as a flat array of
// 64-element groups.  One lane owns 16 bytes of hb and of hb2 (4 f32 or 8
// bf16), a group spans 16 or 8 lanes, and each lane keeps U steps of loads in
// flight before computing.
#include "q3cu_internal.h"

namespace q3 {

template <typename T, int U, bool Q8>
__global__ void __launch_bounds__(256) swiglu_kernel(const T *hb, const T *__restrict__ hb2, int64_t elems,
                                                     T *out, int8_t *__restrict__ q, float *__restrict__ s) {
    constexpr int V = Vec<T>::N;
    constexpr int LPG = GS / V;
    constexpr int GPW = 32 / LPG;
    __shared__ uint64_t s_tab[32];
    load_exp_table(s_tab);
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t groups = (elems + GS - 1) / GS;       // a float-only tail group may be partial
    const int64_t steps = (groups + GPW - 1) / GPW;

    for (int64_t st0 = warp * U; st0 < steps; st0 += nwarps * U) {
        uint4 ra[U], rb[U];
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t g = (st0 + u) * GPW + lane / LPG;
            const int64_t e = g * GS + (lane % LPG) * V;
            ok[u] = (st0 + u) < steps && e < elems;
            if (ok[u]) {
                ra[u] = ld_v4(hb + e);           // coherent: out may alias hb
                rb[u] = ld_nc_v4(hb2 + e);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if ((st0 + u) >= steps) break;                        // warp-uniform
            const int64_t g = (st0 + u) * GPW + lane / LPG;
            const int64_t e = g * GS + (lane % LPG) * V;
            float o[V];
            if (ok[u]) {
                float a[V], b[V];
                Vec<T>::widen(ra[u], a);
                Vec<T>::widen(rb[u], b);
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    const float ex = q3_expf_tab(-a[i], s_tab);
                    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
                    o[i] = __fmul_rn(a[i], __fmul_rn(b[i], sig));
                }
            } else {
#pragma unroll
                for (int i = 0; i < V; ++i) o[i] = 0.0f;
            }
            if constexpr (Q8) {
                float m = 0.0f;
#pragma unroll
                for (int i = 0; i < V; ++i) m = amax_fold(m, o[i]);
#pragma unroll
                for (int k = LPG / 2; k > 0; k >>= 1) m = amax_merge(m, __shfl_xor_sync(FULL, m, k));
                if (!ok[u]) continue;
                const float scale = q8_scale(m);
                uint32_t cw[V / 4];
#pragma unroll
                for (int i = 0; i < V / 4; ++i)
                    cw[i] = q8_code(o[4 * i], scale) | (q8_code(o[4 * i + 1], scale) << 8) |
                            (q8_code(o[4 * i + 2], scale) << 16) | (q8_code(o[4 * i + 3], scale) << 24);
                if constexpr (V == 4) st_cs_u32(q + e, cw[0]);
                else st_cs_v2(q + e, make_uint2(cw[0], cw[1]));
                if ((lane % LPG) == 0) st_cs_f32(s + g, scale);
            } else {
                if (ok[u]) st_cs_v4(out + e, Vec<T>::narrow(o));
            }
        }
    }
}

template <typename T, bool Q8>
static cudaError_t launch_swiglu_t(const T *hb, const T *hb2, int64_t elems, T *out, int8_t *q, float *s,
                                   cudaStream_t stream, int sms) {
    constexpr int U = 2;
    constexpr int GPW = 32 / (GS / Vec<T>::N);
    const int64_t groups = (elems + GS - 1) / GS;
    const int64_t steps = (groups + GPW - 1) / GPW;
    const int64_t warps = (steps + U - 1) / U;
    int64_t blocks = (warps + 7) / 8;
    if (blocks > int64_t(sms) * 8) blocks = int64_t(sms) * 8;
    swiglu_kernel<T, U, Q8><<<unsigned(blocks), 256, 0, stream>>>(hb, hb2, elems, out, q, s);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(const void *hb, const void *hb2, q3cu_dtype dt, int64_t elems, void *out, int8_t *q,
                          float *s, cudaStream_t stream, int sms) {
    if (elems == 0) return cudaSuccess;
    const bool q8 = q != nullptr;
    if (dt == Q3CU_F32) {
        auto a = static_cast<const float *>(hb), b = static_cast<const float *>(hb2);
        auto o = static_cast<float *>(out);
        return q8 ? launch_swiglu_t<float, true>(a, b, elems, o, q, s, stream, sms)
                  : launch_swiglu_t<float, false>(a, b, elems, o, q, s, stream, sms);
    }
    auto a = static_cast<const bf16raw *>(hb), b = static_cast<const bf16raw *>(hb2);
    auto o = static_cast<bf16raw *>(out);
    return q8 ? launch_swiglu_t<bf16raw, true>(a, b, elems, o, q, s, stream, sms)
              : launch_swiglu_t<bf16raw, false>(a, b, elems, o, q, s, stream, sms);
}

}  // namespace q3
