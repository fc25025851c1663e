// k_rmsnorm.cu -- RMSNorm, bit-exact with the reference, optionally fused with
// the Q8_0 quantize that follows it in the forward pass.
//
// Reference: src/cpu/qwen3_original.c:278-289
//     ss = sum_{j=0..n-1} x[j]*x[j]       (binary32, sequential, no FMA)
//     ss = 1.0f / sqrtf(ss/n + 1e-6f)
//     o[j] = w[j] * (ss * x[j])
// then quantize (:147-168) at :356/:443/:465.
//
// The sum is a chain of dependent adds in index order; changing the order
// changes the bits of ss and can move a Q8_0 scale or code.  So each row's sum
// is computed by one lane, in order, and the kernel gets its parallelism from
// many rows at once instead of from a tree reduction:
//
//   phase 1  warp 0 streams the CTA's R rows through shared memory in 1 KB
//            chunks with TMA bulk copies (cp.async.bulk + mbarrier, NS-stage
//            ring, padded rows so the R reader lanes hit distinct banks);
//            lane r folds row r's chunk into its running sum.
//   phase 2  all four warps re-read the rows (L2-resident: the row was read a
//            few microseconds earlier), apply w*(ss*x), and either store the
//            float row or quantize each 64-group (absmax by xor-shuffle) and
//            store int8 codes + one f32 scale per group.
//
// A CTA holds R <= 8 rows; many CTAs share an SM, so while some are in phase 1
// others stream their phase-2 output.  HBM traffic per row is one read of x
// plus the output; the chain costs ~4 cycles/element of latency, which the
// ~13 resident CTAs per SM (R=4) hide behind the memory time.
#include "q3cu_internal.h"

namespace q3 {

constexpr int RMS_CHUNK_BYTES = 1024;
constexpr int RMS_ROWB = RMS_CHUNK_BYTES + 16;   // padded smem row stride
constexpr int RMS_NS = 4;                        // ring stages
constexpr int RMS_THREADS = 128;

template <typename T>
__device__ __forceinline__ float chain_sum(float acc, const uint8_t *p, int elems) {
    // elems is a multiple of Vec<T>::N; 16-byte smem loads, adds in index order.
    constexpr int V = Vec<T>::N;
    const uint4 *p4 = reinterpret_cast<const uint4 *>(p);
    const int nv = elems / V;
#pragma unroll 8
    for (int k = 0; k < nv; ++k) {
        float v[V];
        Vec<T>::widen(p4[k], v);
#pragma unroll
        for (int i = 0; i < V; ++i) acc = __fadd_rn(acc, __fmul_rn(v[i], v[i]));
    }
    return acc;
}

template <typename T, int R, bool Q8>
__global__ void __launch_bounds__(RMS_THREADS) rmsnorm_kernel(const T *x, const float *__restrict__ w,
                                                              int64_t rows, int dim, int n_div, float eps, T *out,
                                                              int8_t *__restrict__ q, float *__restrict__ s,
                                                              uint32_t *status) {
    constexpr int ESZ = sizeof(T);
    constexpr int CW = RMS_CHUNK_BYTES / ESZ;    // elements per chunk
    constexpr int V = Vec<T>::N;                 // elements per 16-byte vector
    constexpr int LPG = GS / V;                  // lanes per Q8_0 group

    __shared__ __align__(128) uint8_t stage[RMS_NS][R][RMS_ROWB];
    __shared__ __align__(8) uint64_t bar[RMS_NS];
    __shared__ float s_ss[R];
    __shared__ int s_fail;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t r0 = int64_t(blockIdx.x) * R;
    const int rv = int(rows - r0 < R ? rows - r0 : R);
    const int nch = (dim + CW - 1) / CW;
    const uint8_t *xb = reinterpret_cast<const uint8_t *>(x) + r0 * int64_t(dim) * ESZ;

    if (tid == 0) {
        for (int i = 0; i < RMS_NS; ++i) mbar_init(&bar[i], 1);
        mbar_init_fence();
        s_fail = 0;
    }
    __syncthreads();

    // ---- phase 1: ordered sum of squares, one lane per row ----------------
    if (warp == 0) {
        int issued = 0;
        auto issue = [&](int c) {
            const int st = c % RMS_NS;
            const int el = dim - c * CW < CW ? dim - c * CW : CW;
            const uint32_t bytes = uint32_t(el) * ESZ;
            mbar_arrive_expect_tx(&bar[st], bytes * uint32_t(rv));
            for (int r = 0; r < rv; ++r)
                bulk_g2s(&stage[st][r][0], xb + (int64_t(r) * dim + int64_t(c) * CW) * ESZ, bytes, &bar[st]);
        };
        if (lane == 0)
            for (; issued < nch && issued < RMS_NS; ++issued) issue(issued);
        float acc = 0.0f;
        int c = 0;
        bool ok = true;
        for (; c < nch; ++c) {
            const int st = c % RMS_NS;
            ok = __all_sync(FULL, mbar_wait(&bar[st], uint32_t(c / RMS_NS) & 1u, lane == 0 ? status : nullptr));
            if (!ok) break;
            if (lane < rv) {
                const int el = dim - c * CW < CW ? dim - c * CW : CW;
                acc = chain_sum<T>(acc, &stage[st][lane][0], el);
            }
            __syncwarp();
            if (lane == 0 && c + RMS_NS < nch) { issue(c + RMS_NS); issued = c + RMS_NS + 1; }
        }
        if (!ok) {
            // Drain: wait (bounded) for copies still in flight before leaving.
            if (lane == 0) {
                for (int d = c; d < issued; ++d) mbar_wait(&bar[d % RMS_NS], uint32_t(d / RMS_NS) & 1u, nullptr);
                s_fail = 1;
            }
        } else if (lane < rv) {
            s_ss[lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, float(n_div)), eps)));
        }
    }
    __syncthreads();
    if (s_fail) return;

    // ---- phase 2: normalise, scale, store or quantize ----------------------
    // Thread t owns the column vectors f = t + 128*j of every row of the block,
    // so it loads each weight vector once and reuses it for the R rows; a warp
    // covers 32 consecutive vectors, so a Q8_0 group (LPG vectors) never
    // straddles warps.  JB column sweeps x R rows (8 loads) are issued before any
    // is consumed: the rows come back from L2 and the loads in flight hide its
    // latency.
    constexpr int JB = R >= 8 ? 1 : 8 / R;
    const int NV = dim / V;
    const int NJ = (NV + RMS_THREADS - 1) / RMS_THREADS;
    float ssr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) ssr[r] = r < rv ? s_ss[r] : 0.0f;
    for (int j0 = 0; j0 < NJ; j0 += JB) {
        uint4 xr[JB][R];
#pragma unroll
        for (int jj = 0; jj < JB; ++jj) {
            const int f = tid + RMS_THREADS * (j0 + jj);
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (j0 + jj < NJ && f < NV && r < rv)
                    xr[jj][r] = ld_v4(x + (r0 + r) * int64_t(dim) + int64_t(f) * V);   // coherent: out may alias x
        }
#pragma unroll
        for (int jj = 0; jj < JB; ++jj) {
            if (j0 + jj >= NJ) break;                                // uniform across the CTA
            const int f = tid + RMS_THREADS * (j0 + jj);
            const bool act = f < NV;
            float wv[V];
            if (act) {
                Vec<float>::widen(ld_nc_v4(w + f * V), wv);
                if constexpr (V == 8) Vec<float>::widen(ld_nc_v4(w + f * V + 4), wv + 4);
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (r >= rv) break;                                  // uniform across the CTA
                const int64_t e = (r0 + r) * int64_t(dim) + int64_t(f) * V;
                float o[V];
                if (act) {
                    float xv[V];
                    Vec<T>::widen(xr[jj][r], xv);
#pragma unroll
                    for (int i = 0; i < V; ++i) o[i] = __fmul_rn(wv[i], __fmul_rn(ssr[r], xv[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < V; ++i) o[i] = 0.0f;
                }
                if constexpr (Q8) {
                    float m = 0.0f;
#pragma unroll
                    for (int i = 0; i < V; ++i) m = amax_fold(m, o[i]);
#pragma unroll
                    for (int kk = LPG / 2; kk > 0; kk >>= 1) m = amax_merge(m, __shfl_xor_sync(FULL, m, kk));
                    if (act) {
                        const Q8Scale gs = q8_prepare(m);
                        if constexpr (V == 4) st_cs_u32(q + e, q8_pack4(o, gs));
                        else st_cs_v2(q + e, make_uint2(q8_pack4(o, gs), q8_pack4(o + 4, gs)));
                        if ((lane % LPG) == 0) st_cs_f32(s + e / GS, gs.scale);
                    }
                } else {
                    if (act) st_cs_v4(out + e, Vec<T>::narrow(o));
                }
            }
        }
    }
}

template <typename T, bool Q8>
static cudaError_t launch_rms_t(const T *x, const float *w, int64_t rows, int dim, int n_div, float eps, T *out, int8_t *q,
                                float *s, uint32_t *status, cudaStream_t stream, int sms) {
    // Rows per CTA: enough CTAs to keep every SM busy with several resident.
    int R = 1;
    if (rows >= int64_t(sms) * 64) R = 8;
    else if (rows >= int64_t(sms) * 16) R = 4;
    else if (rows >= int64_t(sms) * 4) R = 2;
    const int64_t blocks = (rows + R - 1) / R;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    const unsigned b = unsigned(blocks);
    switch (R) {
        case 8: rmsnorm_kernel<T, 8, Q8><<<b, RMS_THREADS, 0, stream>>>(x, w, rows, dim, n_div, eps, out, q, s, status); break;
        case 4: rmsnorm_kernel<T, 4, Q8><<<b, RMS_THREADS, 0, stream>>>(x, w, rows, dim, n_div, eps, out, q, s, status); break;
        case 2: rmsnorm_kernel<T, 2, Q8><<<b, RMS_THREADS, 0, stream>>>(x, w, rows, dim, n_div, eps, out, q, s, status); break;
        default: rmsnorm_kernel<T, 1, Q8><<<b, RMS_THREADS, 0, stream>>>(x, w, rows, dim, n_div, eps, out, q, s, status); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const void *x, q3cu_dtype dt, const float *w, int64_t rows, int dim, float eps, void *out,
                           int8_t *q, float *s, uint32_t *status, cudaStream_t stream, int sms) {
    if (rows == 0) return cudaSuccess;
    const bool q8 = (q != nullptr);
    if (dt == Q3CU_F32) {
        auto xx = static_cast<const float *>(x);
        auto oo = static_cast<float *>(out);
        return q8 ? launch_rms_t<float, true>(xx, w, rows, dim, dim, eps, oo, q, s, status, stream, sms)
                  : launch_rms_t<float, false>(xx, w, rows, dim, dim, eps, oo, q, s, status, stream, sms);
    }
    auto xx = static_cast<const bf16raw *>(x);
    auto oo = static_cast<bf16raw *>(out);
    return q8 ? launch_rms_t<bf16raw, true>(xx, w, rows, dim, dim, eps, oo, q, s, status, stream, sms)
              : launch_rms_t<bf16raw, false>(xx, w, rows, dim, dim, eps, oo, q, s, status, stream, sms);
}

// One f32 row stored with a zero tail up to `padded` (a multiple of 4): the sum
// runs over the padded row (adding +0 leaves it unchanged) and is divided by the
// true length `size`, as the reference divides by its `size` argument.
cudaError_t launch_rmsnorm_padded(const float *x, const float *w, int size, int padded, float *out, uint32_t *status,
                                  cudaStream_t stream, int sms) {
    return launch_rms_t<float, false>(x, w, 1, padded, size, 1e-6f, out, nullptr, nullptr, status, stream, sms);
}

}  // namespace q3
