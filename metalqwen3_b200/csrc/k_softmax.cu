// k_softmax.cu -- in-place softmax of ragged f32 rows.
//
// Reference: src/cpu/qwen3_original.c:291-308 (called per head with pos+1
// scores at :416):
//     max_val = 0; for i: if (x[i] > max_val) max_val = x[i];   // starts at 0
//     sum = 0;     for i: x[i] = expf(x[i] - max_val); sum += x[i];
//     for i: x[i] /= sum;
// The max is order-independent and exact.  Softmax owes the reference 1e-5
// relative, not its bits, so each exponential of d = x - max in [-80, 0] is
// exp_m80_0 (binary32 Cody-Waite reduction + ex2.approx, ~2^-22 relative); d
// below -80 or NaN takes the libm-identical expf, so the reference's underflow
// (a row entirely below -104 is 0/0 = NaN) is reproduced.  Each float4's four
// exponentials are added in binary32 and the partial sums accumulated in
// binary64 (per thread, then a tree): closer to the exact sum than the
// reference's sequential binary32 sum.  The tests bound the outputs (1e-5 rel /
// 1e-6 abs of a binary64 softmax, and no further from the oracle than the
// oracle is from it).
//
// Rows are bucketed by length into five kernels, each a grid-stride loop over
// all rows that skips rows outside its bucket:
//   len <= 512*NW (NW = 1, 2, 4, 8 warps): the row lives in registers (16
//       elements per thread) -> one HBM read, one HBM write;
//   len > 4096: 512 threads, three passes (max; exp stored in place + sum;
//       scale), the second and third reads served from L2.
// Rows start at arbitrary addresses (4-byte aligned): up to three leading
// elements reach a 16-byte boundary, the body moves in float4, the remainder is
// scalar.
#include "q3cu_internal.h"

namespace q3 {

constexpr int SMX_PER_THREAD = 16;            // register-resident elements per thread (body)
constexpr int SMX_LONG_THREADS = 512;

struct RowSplit {
    int a;      // leading scalar elements before the first 16-byte boundary
    int nb;     // float4 body count
    int tl;     // trailing scalar elements
};
// The split of the row starting at `row` (4-byte aligned): by its address, not
// its offset, since the API asks only 4-byte alignment of the buffer.
__device__ __forceinline__ RowSplit split_row(const float *row, int len) {
    RowSplit s;
    s.a = int(((16u - (uint32_t(reinterpret_cast<uintptr_t>(row)) & 15u)) & 15u) >> 2);
    if (s.a > len) s.a = len;
    s.nb = (len - s.a) >> 2;
    s.tl = len - s.a - 4 * s.nb;
    return s;
}
// scalar element handled by thread t (head then tail), or -1
__device__ __forceinline__ int scalar_index(const RowSplit &s, int t) {
    if (t < s.a) return t;
    if (t - s.a < s.tl) return s.a + 4 * s.nb + (t - s.a);
    return -1;
}

// The libm-identical exp, out of line: taken for d < -80 or NaN only, so the
// compiler branches around it instead of predicating it into every element.
static __device__ __noinline__ float smx_exp_slow(float d, const ExpTab *tab) { return expf_host(d, *tab); }
__device__ __forceinline__ float smx_exp(float d, const ExpTab &tab) {
    if (__builtin_expect(d >= -80.0f, 1)) return exp_m80_0(d);
    return smx_exp_slow(d, &tab);
}
__device__ __forceinline__ float4 smx_exp4(float4 v, float m, const ExpTab &tab) {
    return make_float4(smx_exp(__fsub_rn(v.x, m), tab), smx_exp(__fsub_rn(v.y, m), tab),
                       smx_exp(__fsub_rn(v.z, m), tab), smx_exp(__fsub_rn(v.w, m), tab));
}
__device__ __forceinline__ double sum4(float4 v) {
    return double(__fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w)));
}

template <int NW>
__device__ __forceinline__ float block_max(float v, float *sh) {
    v = warp_max(v);
    if constexpr (NW == 1) return v;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();                          // sh free from a previous reduction
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = lane < NW ? sh[lane] : 0.0f;
    return warp_max(r);
}
template <int NW>
__device__ __forceinline__ double block_sum(double v, double *sh) {
    v = warp_sum_d(v);
    if constexpr (NW == 1) return v;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    double r = lane < NW ? sh[lane] : 0.0;
    return warp_sum_d(r);
}

// ---- register-resident rows: lo < len <= hi ------------------------------
template <int NW>
__global__ void __launch_bounds__(NW * 32) softmax_reg_kernel(float *x, const int64_t *__restrict__ offs,
                                                              const int32_t *__restrict__ lens, int64_t rows,
                                                              int lo, int hi) {
    constexpr int NT = NW * 32;
    constexpr int NB = SMX_PER_THREAD / 4;    // float4 slots per thread
    __shared__ ExpTab s_tab;
    __shared__ float sh_f[NW];
    __shared__ double sh_d[NW];
    load_exp_table(s_tab);
    __syncthreads();
    const int t = threadIdx.x;

    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int len = __ldg(lens + r);
        if (len <= lo || len > hi) continue;                    // block-uniform
        const int64_t off = __ldg(offs + r);
        float *row = x + off;
        const RowSplit sp = split_row(row, len);
        float4 *body = reinterpret_cast<float4 *>(row + sp.a);

        float4 v[NB];
        float m = 0.0f;                                         // the reference's max starts at 0
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const int bi = t + j * NT;
            if (bi < sp.nb) {
                v[j] = u4_as_f4(ld_v4(body + bi));
                m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
            }
        }
        const int si = scalar_index(sp, t);
        float xs = 0.0f;
        if (si >= 0) { xs = row[si]; m = fmaxf(m, xs); }
        m = block_max<NW>(m, sh_f);

        double sum = 0.0;
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            if (t + j * NT < sp.nb) {
                v[j] = smx_exp4(v[j], m, s_tab);
                sum += sum4(v[j]);
            }
        }
        if (si >= 0) { xs = smx_exp(__fsub_rn(xs, m), s_tab); sum += double(xs); }
        sum = block_sum<NW>(sum, sh_d);
        const float inv = float(1.0 / sum);

#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const int bi = t + j * NT;
            if (bi < sp.nb) {
                float4 o = make_float4(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv), __fmul_rn(v[j].z, inv),
                                       __fmul_rn(v[j].w, inv));
                st_cs_v4(body + bi, f4_as_u4(o));
            }
        }
        if (si >= 0) row[si] = __fmul_rn(xs, inv);
    }
}

// ---- long rows (len > lo): three passes -----------------------------------
__global__ void __launch_bounds__(SMX_LONG_THREADS) softmax_long_kernel(float *x, const int64_t *__restrict__ offs,
                                                                        const int32_t *__restrict__ lens,
                                                                        int64_t rows, int lo) {
    constexpr int NW = SMX_LONG_THREADS / 32;
    constexpr int NT = SMX_LONG_THREADS;
    __shared__ ExpTab s_tab;
    __shared__ float sh_f[NW];
    __shared__ double sh_d[NW];
    load_exp_table(s_tab);
    __syncthreads();
    const int t = threadIdx.x;

    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int len = __ldg(lens + r);
        if (len <= lo) continue;
        const int64_t off = __ldg(offs + r);
        float *row = x + off;
        const RowSplit sp = split_row(row, len);
        float4 *body = reinterpret_cast<float4 *>(row + sp.a);
        const int si = scalar_index(sp, t);

        // pass A: max
        float m = 0.0f;
#pragma unroll 4
        for (int bi = t; bi < sp.nb; bi += NT) {
            const float4 v = u4_as_f4(ld_v4(body + bi));
            m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
        }
        if (si >= 0) m = fmaxf(m, row[si]);
        m = block_max<NW>(m, sh_f);

        // pass B: exponentials in place, binary64 sum
        double sum = 0.0;
#pragma unroll 4
        for (int bi = t; bi < sp.nb; bi += NT) {
            const float4 v = smx_exp4(u4_as_f4(ld_v4(body + bi)), m, s_tab);
            sum += sum4(v);
            *reinterpret_cast<uint4 *>(body + bi) = f4_as_u4(v);
        }
        if (si >= 0) {
            const float e = smx_exp(__fsub_rn(row[si], m), s_tab);
            row[si] = e;
            sum += double(e);
        }
        sum = block_sum<NW>(sum, sh_d);      // its barriers also order pass B's stores before pass C
        const float inv = float(1.0 / sum);

        // pass C: scale
#pragma unroll 4
        for (int bi = t; bi < sp.nb; bi += NT) {
            const float4 v = u4_as_f4(ld_v4(body + bi));
            st_cs_v4(body + bi, f4_as_u4(make_float4(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv),
                                                     __fmul_rn(v.z, inv), __fmul_rn(v.w, inv))));
        }
        if (si >= 0) row[si] = __fmul_rn(row[si], inv);
        __syncthreads();
    }
}

cudaError_t launch_softmax_rows(float *x, const int64_t *off, const int32_t *len, int64_t rows, cudaStream_t stream,
                                int sms) {
    if (rows == 0) return cudaSuccess;
    auto grid = [&](int per_sm) {
        int64_t g = int64_t(sms) * per_sm;
        return unsigned(rows < g ? rows : g);
    };
    softmax_reg_kernel<1><<<grid(32), 32, 0, stream>>>(x, off, len, rows, 0, 512);
    softmax_reg_kernel<2><<<grid(16), 64, 0, stream>>>(x, off, len, rows, 512, 1024);
    softmax_reg_kernel<4><<<grid(8), 128, 0, stream>>>(x, off, len, rows, 1024, 2048);
    softmax_reg_kernel<8><<<grid(4), 256, 0, stream>>>(x, off, len, rows, 2048, 4096);
    softmax_long_kernel<<<grid(4), SMX_LONG_THREADS, 0, stream>>>(x, off, len, rows, 4096);
    return cudaGetLastError();
}

}  // namespace q3
