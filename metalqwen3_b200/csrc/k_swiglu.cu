// k_swiglu.cu -- SwiGLU gate, in place or fused with the Q8_0 quantize that
// follows it in the FFN.
//
// Reference: src/cpu/qwen3_original.c:449-450 and :453
//     hb[i] *= hb2[i] * (1.0f / (1.0f + expf(-hb[i])));
//     quantize(&s->hq, s->hb, hidden_dim);
// (shaders/swiglu.metal:37-39 associates the product differently; the CPU
// order is the reference here.)  Every operator is one IEEE binary32 rounding
// and expf is q3_expf_fast, which returns the host libm's bits, so the float
// output and the Q8_0 codes/scales are bit-exact.
//
// Layout: [rows][hidden] with hidden % 64 == 0 is processed as one flat array
// (a float-only call may end in a partial group).  A warp step covers 32
// lanes x 16 bytes of hb and of hb2 (4 f32 or 8 bf16 per lane), so a 64-group
// spans 16 or 8 lanes; each lane keeps U steps of loads in flight before
// computing.  The rare exact-arithmetic paths (q3cu_device.cuh) are out of line.
#include "q3cu_internal.h"

namespace q3 {

template <typename T, int U, bool Q8>
__global__ void __launch_bounds__(256) swiglu_kernel(const T *hb, const T *__restrict__ hb2, int64_t elems,
                                                     T *out, int8_t *__restrict__ q, float *__restrict__ s) {
    constexpr int V = Vec<T>::N;                 // elements per lane per step (16 bytes)
    constexpr int LPG = GS / V;                  // lanes per Q8_0 group
    constexpr int STEP = 32 * V;                 // elements per warp step
    __shared__ ExpTab s_tab;
    load_exp_table(s_tab);
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t nsteps = (elems + STEP - 1) / STEP;

    for (int64_t st0 = warp * U; st0 < nsteps; st0 += nwarps * U) {
        const int64_t e0 = st0 * STEP + lane * V;        // this lane's first element in step st0
        uint4 ra[U], rb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t e = e0 + int64_t(u) * STEP;
            if (e < elems) {
                ra[u] = ld_v4(hb + e);                   // coherent: out may alias hb
                rb[u] = ld_nc_v4(hb2 + e);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (st0 + u >= nsteps) break;                // warp-uniform
            const int64_t e = e0 + int64_t(u) * STEP;
            const bool ok = e < elems;
            float o[V];
            if (ok) {
                float a[V], b[V];
                Vec<T>::widen(ra[u], a);
                Vec<T>::widen(rb[u], b);
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    const float ex = expf_host(-a[i], s_tab);
                    const float sig = rcp_rn_ge1(__fadd_rn(1.0f, ex));    // == 1.0f / (1.0f + ex), IEEE
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
                if (!ok) continue;
                const Q8Scale gs = q8_prepare(m);
                if constexpr (V == 4) st_cs_u32(q + e, q8_pack4(o, gs));
                else st_cs_v2(q + e, make_uint2(q8_pack4(o, gs), q8_pack4(o + 4, gs)));
                if ((lane % LPG) == 0) st_cs_f32(s + (e >> 6), gs.scale);
            } else {
                if (ok) st_cs_v4(out + e, Vec<T>::narrow(o));
            }
        }
    }
}

// Main kernel: 32 bytes of hb and hb2 per lane per step (8 f32 / 16 bf16), so a
// 64-group spans 8 / 4 lanes; the values by swiglu_lane (q3cu_device.cuh),
// codes from q8_encode_lane.
template <typename T, int U, bool Q8>
__global__ void __launch_bounds__(256, sizeof(T) == 4 ? 3 : 2) swiglu_v8_kernel(const T *hb, const T *__restrict__ hb2, int64_t elems,
                                                        T *out, int8_t *__restrict__ q, float *__restrict__ s) {
    constexpr int N = Wide<T>::N;
    constexpr int LPG = GS / N;
    constexpr int STEP = 32 * N;
    __shared__ ExpTab s_tab;
    griddep_launch_dependents();                  // a dependent-launched successor may start its own prologue
    load_exp_table(s_tab);
    griddep_wait();                               // hb / hb2 from the kernel before (a dependent launch)
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t nsteps = elems / STEP + ((elems % STEP) != 0);

    for (int64_t st0 = warp * U; st0 < nsteps; st0 += nwarps * U) {
        const int64_t e0 = st0 * STEP + lane * N;
        U8 ra[U], rb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t e = e0 + int64_t(u) * STEP;
            if (e < elems) {
                ra[u] = ld_v8(hb + e);               // coherent: out may alias hb
                rb[u] = ld_nc_v8(hb2 + e);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (st0 + u >= nsteps) break;            // warp-uniform
            const int64_t e = e0 + int64_t(u) * STEP;
            const bool ok = e < elems;
            float o[N];
            if (ok) {
                float a[N], b[N];
                Wide<T>::widen(ra[u], a);
                Wide<T>::widen(rb[u], b);
                swiglu_lane<N>(a, b, o, s_tab);
            } else {
#pragma unroll
                for (int i = 0; i < N; ++i) o[i] = 0.0f;
            }
            if constexpr (Q8) {
                uint32_t codes[N / 4];
                const float scale = q8_encode_lane<N, LPG>(o, codes);
                if (!ok) continue;
                if constexpr (N == 8) st_cs_v2(q + e, make_uint2(codes[0], codes[1]));
                else st_cs_v4(q + e, make_uint4(codes[0], codes[1], codes[2], codes[3]));
                if ((lane % LPG) == 0) st_cs_f32(s + (e >> 6), scale);
            } else {
                if (ok) st_cs_v8(out + e, Wide<T>::narrow(o));
            }
        }
    }
}

template <typename T, bool Q8>
static cudaError_t launch_swiglu_t(const T *hb, const T *hb2, int64_t elems, T *out, int8_t *q, float *s,
                                   cudaStream_t stream, int sms) {
    constexpr int U = 2;
    const bool v8 = (elems % Wide<T>::N) == 0 && (reinterpret_cast<uintptr_t>(hb) % 32) == 0 &&
                    (reinterpret_cast<uintptr_t>(hb2) % 32) == 0 &&
                    (Q8 ? (reinterpret_cast<uintptr_t>(q) % (Wide<T>::N)) == 0
                        : (reinterpret_cast<uintptr_t>(out) % 32) == 0);
    const int step = 32 * (v8 ? Wide<T>::N : Vec<T>::N);
    const int64_t steps = (elems + step - 1) / step;
    const int64_t warps = (steps + U - 1) / U;
    int64_t blocks = (warps + 7) / 8;
    const int per_sm = v8 ? (sizeof(T) == 4 ? 3 : 2) : 8;    // v8: one resident wave (its launch bounds)
    if (blocks > int64_t(sms) * per_sm) blocks = int64_t(sms) * per_sm;
    if (v8)
        return launch_dependent(swiglu_v8_kernel<T, U, Q8>, dim3(unsigned(blocks)), dim3(256), 0, stream, hb, hb2,
                                elems, out, q, s);
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
