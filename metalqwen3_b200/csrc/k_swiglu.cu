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

// Streaming kernel for large inputs: loads decoupled from the arithmetic.
// One CTA per SM, SW_WARPS warps; each warp owns a private ring of SW_K stages
// in shared memory and walks its own chunks (chunk c of the flat arrays:
// SW_CE<T> elements of hb and of hb2).  Lane 0 issues the two bulk copies of a
// chunk (cp.async.bulk, completing on the stage's mbarrier) SW_K - 1 chunks
// ahead of the one the warp computes, so every warp keeps a chunk of both
// inputs in flight while its lanes run the exp/reciprocal arithmetic from
// shared memory -- HBM never waits for the arithmetic and the arithmetic
// never waits for a load issued just before it.  A lane takes 32 bytes of each
// input per pass (8 f32 / 16 bf16 elements, 8 / 4 lanes per Q8_0 group).
constexpr int SW_WARPS = 16;
constexpr int SW_K = 2;                                      // stages per warp

// bf16 inputs: the gate RN(1 / RN(1 + expf(-a))) of the reference's expression
// (qwen3_original.c:450) depends only on the 16 bits of a, so a CTA tabulates
// it once, with the exact operations, over |a| in [2^-14, 2^8) (exponent
// fields 113..134, both signs: 5,632 entries, 22 KB of shared memory), and
// every element in that window takes its gate from the table: bit-identical by
// construction.  Elements outside the window (|a| < 2^-14, huge, inf, NaN,
// subnormal) take the exact path.
constexpr int SWT_E0 = 113;                                  // first exponent field in the table
constexpr int SWT_N = 22 * 128;                              // entries per sign
struct GateTab { float v[2 * SWT_N]; };
__device__ __forceinline__ void build_gate_table(GateTab &g, const ExpTab &tab) {
    for (int i = threadIdx.x; i < 2 * SWT_N; i += blockDim.x) {
        const uint32_t sign = i >= SWT_N ? 0x8000u : 0u;
        const uint32_t u = uint32_t(i % SWT_N) + (uint32_t(SWT_E0) << 7);
        const float a = bf16_to_f32(u | sign);
        g.v[i] = __frcp_rn(__fadd_rn(1.0f, expf_host(-a, tab)));      // 1.0f / (1.0f + expf(-a)), IEEE
    }
}
// SwiGLU of the 16 bf16 values of a lane (raw words wa, widened a, b):
// out = RN(a * RN(b * gate(a))), gate from the table where it covers a.
__device__ __forceinline__ void swiglu_lane_tab(const U8 &wa, const float *a, const float *b, float *o,
                                                const GateTab &g, const ExpTab &tab) {
    bool slow = false;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
        float sig[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t bits = h ? (wa.w[i / 2] >> 16) : (wa.w[i / 2] & 0xffffu);
            const uint32_t d = (bits & 0x7fffu) - (uint32_t(SWT_E0) << 7);
            const bool in = d < uint32_t(SWT_N);
            slow |= !in;
            sig[h] = g.v[(in ? d : 0u) + ((bits & 0x8000u) ? uint32_t(SWT_N) : 0u)];
        }
        up2(mul2(pk2(a[i], a[i + 1]), mul2(pk2(b[i], b[i + 1]), pk2(sig[0], sig[1]))), o[i], o[i + 1]);
    }
    if (__builtin_expect(slow, 0)) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const uint32_t bits = (i & 1) ? (wa.w[i / 2] >> 16) : (wa.w[i / 2] & 0xffffu);
            if ((bits & 0x7fffu) - (uint32_t(SWT_E0) << 7) >= uint32_t(SWT_N)) o[i] = swiglu_exact(a[i], b[i], tab);
        }
    }
}
template <typename T> struct SwCE { static constexpr int V = 3 * 32 * Wide<T>::N; };   // elements per chunk
constexpr int SW_STAGE = 2 * 3 * 32 * 32;                    // bytes per stage: hb + hb2, 3 passes of 32 B x 32 lanes
constexpr size_t SW_RING = size_t(SW_WARPS) * SW_K * SW_STAGE;   // 196,608 bytes

template <typename T, bool Q8>
__global__ void __launch_bounds__(SW_WARPS * 32, 1) swiglu_ring_kernel(const T *hb, const T *hb2, int64_t elems,
                                                                       T *out, int8_t *__restrict__ q,
                                                                       float *__restrict__ s, uint32_t *status) {
    constexpr int N = Wide<T>::N;
    constexpr int LPG = GS / N;
    constexpr int CE = SwCE<T>::V;                           // elements per chunk
    constexpr int HALF = SW_STAGE / 2;                       // bytes of one input per stage
    static_assert(CE * int(sizeof(T)) == HALF, "stage layout");
    constexpr bool TAB = sizeof(T) == 2;                    // bf16: the gate table
    extern __shared__ __align__(128) uint8_t sw_ring[];      // [SW_WARPS][SW_K][hb | hb2], then the gate table
    __shared__ __align__(8) uint64_t bar[SW_WARPS][SW_K];
    __shared__ ExpTab s_tab;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    GateTab &gtab = *reinterpret_cast<GateTab *>(sw_ring + size_t(SW_WARPS) * SW_K * SW_STAGE);
    load_exp_table(s_tab);
    if (lane == 0)
        for (int k = 0; k < SW_K; ++k) mbar_init(&bar[warp][k], 1);
    mbar_init_fence();
    __syncthreads();                                         // (also: the exp table)
    griddep_launch_dependents();                  // a dependent-launched successor may start its own prologue
    griddep_wait();                               // hb / hb2 from the kernel before (a dependent launch)

    const int64_t nch = (elems + CE - 1) / CE;
    const int64_t gw = int64_t(blockIdx.x) * SW_WARPS + warp, nw = int64_t(gridDim.x) * SW_WARPS;
    const int64_t mine = gw < nch ? (nch - 1 - gw) / nw + 1 : 0;   // chunks of this warp
    uint8_t *ring = sw_ring + size_t(warp) * SW_K * SW_STAGE;
    auto issue = [&](int64_t i) {                            // chunk gw + i * nw into stage i % SW_K
        const int64_t c0 = (gw + i * nw) * CE;
        const uint32_t bytes = uint32_t((elems - c0 < CE ? elems - c0 : CE) * int64_t(sizeof(T)));
        uint64_t *b = &bar[warp][i % SW_K];
        uint8_t *st = ring + size_t(i % SW_K) * SW_STAGE;
        mbar_arrive_expect_tx(b, 2 * bytes);
        bulk_g2s(st, hb + c0, bytes, b);
        bulk_g2s(st + HALF, hb2 + c0, bytes, b);
    };
    if (lane == 0)
        for (int64_t i = 0; i < SW_K && i < mine; ++i) issue(i);
    if constexpr (TAB) {                                     // while the first chunks land
        build_gate_table(gtab, s_tab);
        __syncthreads();
    }
    int64_t i = 0;
    for (; i < mine; ++i) {
        const int k = int(i % SW_K);
        if (!__all_sync(FULL, mbar_wait(&bar[warp][k], uint32_t(i / SW_K) & 1u, lane == 0 ? status : nullptr)))
            break;                                           // a copy did not land: stop (status set)
        const int64_t c0 = (gw + i * nw) * CE;
        const uint8_t *st = ring + size_t(k) * SW_STAGE;
#pragma unroll 1
        for (int p = 0; p < 3; ++p) {
            const int off = (p * 32 + lane) * N;             // element offset within the chunk
            const int64_t e = c0 + off;
            const bool ok = e < elems;
            float o[N];
            if (ok) {
                float a[N], b[N];
                const uint4 *pa = reinterpret_cast<const uint4 *>(st + off * sizeof(T));
                const uint4 *pb = reinterpret_cast<const uint4 *>(st + HALF + off * sizeof(T));
                const uint4 a0 = pa[0], a1 = pa[1];
                Vec<T>::widen(a0, a);
                Vec<T>::widen(a1, a + N / 2);
                Vec<T>::widen(pb[0], b);
                Vec<T>::widen(pb[1], b + N / 2);
                if constexpr (TAB) {
                    const U8 wa = {{a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w}};
                    swiglu_lane_tab(wa, a, b, o, gtab, s_tab);
                } else {
                    swiglu_lane<N>(a, b, o, s_tab);
                }
            } else {
#pragma unroll
                for (int j = 0; j < N; ++j) o[j] = 0.0f;
            }
            if constexpr (Q8) {
                uint32_t codes[N / 4];
                const float scale = q8_encode_lane<N, LPG>(o, codes);    // every lane (shuffles)
                if (!ok) continue;
                if constexpr (N == 8) st_cs_v2(q + e, make_uint2(codes[0], codes[1]));
                else st_cs_v4(q + e, make_uint4(codes[0], codes[1], codes[2], codes[3]));
                if ((lane % LPG) == 0) st_cs_f32(s + (e >> 6), scale);
            } else {
                if (!ok) continue;
                const U8 v = Wide<T>::narrow(o);
                st_cs_v4(out + e, make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]));
                st_cs_v4(out + e + N / 2, make_uint4(v.w[4], v.w[5], v.w[6], v.w[7]));
            }
        }
        __syncwarp();                                        // every lane is done with stage k
        if (lane == 0 && i + SW_K < mine) issue(i + SW_K);
    }
    // No copy may outlive the CTA: after a failed wait (i < mine), wait
    // (bounded) for the chunks this warp issued and did not consume, the
    // failed one included.
    if (lane == 0)
        for (int64_t d = i; d < mine && d < i + SW_K; ++d)
            mbar_wait(&bar[warp][d % SW_K], uint32_t(d / SW_K) & 1u, nullptr);
}

template <typename T, bool Q8>
static cudaError_t launch_swiglu_t(const T *hb, const T *hb2, int64_t elems, T *out, int8_t *q, float *s,
                                   uint32_t *status, cudaStream_t stream, int sms) {
    constexpr int U = 2;
    auto al = [](const void *p, uintptr_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; };
    // Large inputs (at least a quarter of a full grid's warps get a chunk): the streaming ring kernel.
    if (elems >= int64_t(sms) * (SW_WARPS / 4) * SwCE<T>::V && elems % Wide<T>::N == 0 && al(hb, 16) &&
        al(hb2, 16) && (Q8 ? al(q, sizeof(T) == 4 ? 8 : 16) : al(out, 16))) {
        const int slot = 20 + (sizeof(T) == 4 ? 0 : 2) + (Q8 ? 1 : 0);
        const size_t smem = SW_RING + (sizeof(T) == 2 ? sizeof(GateTab) : 0);
        cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(swiglu_ring_kernel<T, Q8>), smem, slot);
        if (e != cudaSuccess) return e;
        return launch_dependent(swiglu_ring_kernel<T, Q8>, dim3(sms), dim3(SW_WARPS * 32), smem, stream, hb, hb2,
                                elems, out, q, s, status);
    }
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
                          float *s, uint32_t *status, cudaStream_t stream, int sms) {
    if (elems == 0) return cudaSuccess;
    const bool q8 = q != nullptr;
    if (dt == Q3CU_F32) {
        auto a = static_cast<const float *>(hb), b = static_cast<const float *>(hb2);
        auto o = static_cast<float *>(out);
        return q8 ? launch_swiglu_t<float, true>(a, b, elems, o, q, s, status, stream, sms)
                  : launch_swiglu_t<float, false>(a, b, elems, o, q, s, status, stream, sms);
    }
    auto a = static_cast<const bf16raw *>(hb), b = static_cast<const bf16raw *>(hb2);
    auto o = static_cast<bf16raw *>(out);
    return q8 ? launch_swiglu_t<bf16raw, true>(a, b, elems, o, q, s, status, stream, sms)
              : launch_swiglu_t<bf16raw, false>(a, b, elems, o, q, s, status, stream, sms);
}

}  // namespace q3
