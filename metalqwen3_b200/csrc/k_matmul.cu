// k_matmul.cu -- Q8_0 x Q8_0 matrix-vector products, bit-exact with the
// reference's matmul, for a few token rows at a time (decode).
//
// Reference: src/cpu/qwen3_original.c:310-331, W (d,n) @ x (n,) -> xout (d,):
//     for i < d:  val = 0
//                 for each 64-group j (in order):
//                     ival = sum_k x.q[j+k] * w.q[i*n+j+k]          (int32, exact)
//                     val += ((float) ival) * w.s[(i*n+j)/64] * x.s[j/64]
//                 xout[i] = val
// Built without FMA contraction, the group term is RN(RN(float(ival) * ws) * xs)
// and val is a sequential binary32 sum over the groups, in group order.
//
// Layout: W codes [d][n] int8 and scales [d][n/64] f32 (row-major [out][in],
// as the reference stores them); x codes [B][n] and scales [B][n/64]; out
// [B][d] f32.  The int8 dot products are exact in any order, so they are
// spread over lanes: a warp job is a tile of RB output rows x TB tokens, and
// in each pass over 32 consecutive groups lane g takes group g of every row of
// the tile -- two 32-byte loads of the row's codes per lane, so the warp reads
// 2 KB of the row contiguously -- and forms the TB group terms with dp4a.  The
// terms go to a padded shared-memory transpose, and lane s = (row, token) then
// adds its 32 terms to its running val in group order: the reference's
// accumulation, so the outputs are its bits.  The codes of the lane's group for
// the TB tokens stay in registers across the rows of the tile.  Rows with
// fewer than 32 groups share a pass: GL lanes per row (the group count
// rounded up to a power of two), 32 / GL rows side by side, and U rows' loads
// are in flight per lane.
//
// With `pdl`, the launch may overlap its predecessor (programmatic dependent
// launch): every warp requests its first rows of W, then waits for the
// predecessor (griddep_wait) before it reads x or add or writes anything.
//
// With `add` set, out = RN(add + val): the residual update that follows the
// wo and w2 matmuls in the forward pass (x[i] += xb[i], :434 and :457), one
// rounding as there; out may equal add.
//
// Cost: W is read once per block of TB tokens (TB <= 4), so for one to four
// tokens the kernel streams W at HBM speed; larger batches re-read W per block
// (a tensor-core path for prefill-sized batches is not part of this file).
#include "q3cu_internal.h"

namespace q3 {

constexpr int MM_WARPS = 8;
constexpr int MM_THREADS = MM_WARPS * 32;

__device__ __forceinline__ int dot64(const U8 &a0, const U8 &a1, const U8 &b0, const U8 &b1) {
    int acc = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc = __dp4a(int(a0.w[k]), int(b0.w[k]), acc);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc = __dp4a(int(a1.w[k]), int(b1.w[k]), acc);
    return acc;
}

// Shared-memory layout of a fused input: codes [n], scales [n / 64] (padded to
// 16 bytes), then for PRO_RMS the row and its squares [n] each.
__host__ __device__ constexpr int pro_scales_bytes(int n) { return ((n / GS) * 4 + 15) & ~15; }
__host__ __device__ constexpr int pro_smem_bytes(int pro, int n) {
    return n + pro_scales_bytes(n) + (pro == PRO_RMS ? 8 * n : 0);
}
constexpr int PRO_RMS_MAXN = 16384, PRO_SWIGLU_MAXN = 32768;

// The fused input (B = 1) by every thread of the CTA; ends with a barrier.
template <int PRO>
__device__ __forceinline__ void mm_prologue(const MmPro &pro, int n, uint8_t *psm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int8_t *xq_s = reinterpret_cast<int8_t *>(psm);
    float *xs_s = reinterpret_cast<float *>(psm + n);
    const int units = n / 8;                        // 8 values per lane; a group is 8 lanes (n % 64 == 0)
    if constexpr (PRO == PRO_RMS) {
        __shared__ float ss_sh;
        float *row = reinterpret_cast<float *>(psm + n + pro_scales_bytes(n));
        float *sq = row + n;
        for (int i = tid; i < n / 4; i += MM_THREADS) {
            const float4 v = u4_as_f4(ld_v4(pro.a + 4 * i));
            reinterpret_cast<float4 *>(row)[i] = v;
            reinterpret_cast<float4 *>(sq)[i] =
                make_float4(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y), __fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w));
        }
        __syncthreads();
        if (tid == 0)                                 // ss = 1 / sqrt(sum / n + eps), the sum in index order
            ss_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ordered_sum_smem(0.0f, sq, n), float(n)), pro.eps)));
        __syncthreads();
        const f2 ss2 = pk2(ss_sh, ss_sh);
        for (int u0 = warp * 32; u0 < units; u0 += MM_THREADS) {
            const int u = u0 + lane;
            const bool act = u < units;                 // whole groups of 8 lanes
            float o[8];
            if (act) {
                float xv[8], wv[8];
                Vec<float>::widen(*reinterpret_cast<const uint4 *>(row + 8 * u), xv);
                Vec<float>::widen(*reinterpret_cast<const uint4 *>(row + 8 * u + 4), xv + 4);
                Vec<float>::widen(ld_l1_v4(pro.w + 8 * u), wv);
                Vec<float>::widen(ld_l1_v4(pro.w + 8 * u + 4), wv + 4);
#pragma unroll
                for (int i = 0; i < 8; i += 2)            // w * (ss * x)
                    up2(mul2(pk2(wv[i], wv[i + 1]), mul2(ss2, pk2(xv[i], xv[i + 1]))), o[i], o[i + 1]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = 0.0f;
            }
            uint32_t codes[2];
            const float scale = q8_encode_lane<8, 8>(o, codes);
            if (act) {
                *reinterpret_cast<uint2 *>(xq_s + 8 * u) = make_uint2(codes[0], codes[1]);
                if ((lane & 7) == 0) xs_s[u >> 3] = scale;
            }
        }
    } else {
        __shared__ ExpTab tab;
        load_exp_table(tab);
        __syncthreads();
        for (int u0 = warp * 32; u0 < units; u0 += MM_THREADS) {
            const int u = u0 + lane;
            const bool act = u < units;
            float o[8];
            if (act) {
                const U8 ra = ld_v8(pro.a + 8 * u), rb = ld_v8(pro.b + 8 * u);
                float a[8], b[8];
                Wide<float>::widen(ra, a);
                Wide<float>::widen(rb, b);
                swiglu_lane<8>(a, b, o, tab);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = 0.0f;
            }
            uint32_t codes[2];
            const float scale = q8_encode_lane<8, 8>(o, codes);
            if (act) {
                *reinterpret_cast<uint2 *>(xq_s + 8 * u) = make_uint2(codes[0], codes[1]);
                if ((lane & 7) == 0) xs_s[u >> 3] = scale;
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ U8 ld_shared_v8(const int8_t *p) {
    const uint4 lo = *reinterpret_cast<const uint4 *>(p), hi = *reinterpret_cast<const uint4 *>(p + 16);
    return U8{{lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w}};
}

// PRO = 0: x codes / scales from global memory.  PRO_RMS / PRO_SWIGLU (TB = 1):
// every CTA computes x into shared memory first (mm_prologue), after asking L2
// for its warps' first rows of W and waiting for the kernel that wrote pro.a.
template <int TB, int U, int PRO>
__global__ void __launch_bounds__(MM_THREADS) matmul_q8_kernel(const int8_t *__restrict__ xq,
                                                               const float *__restrict__ xs, int B,
                                                               const int8_t *__restrict__ wq,
                                                               const float *__restrict__ ws, int n, int d, int RB,
                                                               const float *add, MmOut out, MmPro pro) {
    static_assert(PRO == 0 || TB == 1, "a fused input is one token");
    __shared__ float terms[MM_WARPS][32][33];      // [slot = row * TB + token][group of the pass], padded
    extern __shared__ __align__(16) uint8_t psm[]; // the fused input (PRO != 0)
    // No early griddep_launch_dependents(): the successor starts when this grid
    // completes.  Triggering at the start let the chain of dependent launches
    // run ahead (each of them triggers early) and cost 0.12 ms per decode token.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = n / GS;                           // groups per row
    // A pass covers GL consecutive groups (G rounded up to a power of two, at
    // most 32) of RP = 32 / GL rows at once: lane = sub * GL + gi.
    int GL = 1;
    while (GL < G && GL < 32) GL <<= 1;
    const int RP = 32 / GL, sub = lane / GL, gi = lane % GL;
    const int tiles = (d + RB - 1) / RB;
    const int ntb = (B + TB - 1) / TB;
    const int64_t jobs = int64_t(tiles) * ntb;
    const int slots = RB * TB;                      // (row, token) pairs of a tile, <= 32
    float(*tw)[33] = terms[warp];
    bool waited = false;                            // griddep_wait done (before the first read of x / add)
    if constexpr (PRO != 0) {
        const int64_t j0 = int64_t(blockIdx.x) * MM_WARPS + warp;
        if (lane == 0 && j0 < jobs) {               // this warp's first tile of W, into L2
            const int i0 = int(j0 % tiles) * RB, rm = d - i0 < RB ? d - i0 : RB;
            const int8_t *pw = wq + int64_t(i0) * n;
            const float *ps = ws + int64_t(i0) * G;
            if ((reinterpret_cast<uintptr_t>(pw) & 15) == 0) prefetch_l2_bulk(pw, uint32_t(rm) * uint32_t(n));
            if ((reinterpret_cast<uintptr_t>(ps) & 15) == 0 && (rm * G) % 4 == 0)
                prefetch_l2_bulk(ps, uint32_t(rm * G) * 4u);
        }
        griddep_wait();                             // pro.a / pro.b / add from the kernel before
        waited = true;
        mm_prologue<PRO>(pro, n, psm);
    }

    for (int64_t job = int64_t(blockIdx.x) * MM_WARPS + warp; job < jobs; job += int64_t(gridDim.x) * MM_WARPS) {
        const int tile = int(job % tiles), tb = int(job / tiles);
        const int i0 = tile * RB, t0 = tb * TB;
        const int rmax = d - i0 < RB ? d - i0 : RB;
        float val = 0.0f;                           // lane s < slots: row i0 + s / TB, token t0 + s % TB
        for (int g0 = 0; g0 < G; g0 += GL) {
            const int g = g0 + gi;
            const bool gl = g < G;
            U8 wa[U], wb[U];
            float wsc[U];
            bool ok[U];
            auto load_w = [&](int r) {                  // U rows' codes and scales in flight
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int rr = r + u * RP + sub;
                    ok[u] = gl && rr < rmax;
                    if (ok[u]) {
                        const int64_t row = i0 + rr;
                        wa[u] = ld_nc_v8(wq + row * n + int64_t(g) * GS);
                        wb[u] = ld_nc_v8(wq + row * n + int64_t(g) * GS + 32);
                        wsc[u] = ws[row * G + g];
                    }
                }
            };
            // the first rows' weights are constant data: they are requested before
            // the wait for the kernel that produced x (programmatic dependent launch)
            load_w(0);
            if (!waited) {
                griddep_wait();
                waited = true;
            }
            U8 xa[TB], xb[TB];
            float xsc[TB];
#pragma unroll
            for (int t = 0; t < TB; ++t) {
                if (PRO != 0 && gl) {
                    const int8_t *sp = reinterpret_cast<const int8_t *>(psm) + int64_t(g) * GS;
                    xa[t] = ld_shared_v8(sp);
                    xb[t] = ld_shared_v8(sp + 32);
                    xsc[t] = reinterpret_cast<const float *>(psm + n)[g];
                } else if (gl && t0 + t < B) {
                    const int8_t *xp = xq + int64_t(t0 + t) * n + int64_t(g) * GS;
                    xa[t] = ld_nc_v8(xp);
                    xb[t] = ld_nc_v8(xp + 32);
                    xsc[t] = xs[int64_t(t0 + t) * G + g];
                } else {
#pragma unroll
                    for (int k = 0; k < 8; ++k) xa[t].w[k] = xb[t].w[k] = 0u;
                    xsc[t] = 0.0f;
                }
            }
            for (int r = 0; r < rmax; r += RP * U) {
                if (r > 0) load_w(r);
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int rr = r + u * RP + sub;
                    if (rr < rmax) {
#pragma unroll
                        for (int t = 0; t < TB; ++t) {
                            float f = 0.0f;
                            if (ok[u])
                                f = __fmul_rn(__fmul_rn(__int2float_rn(dot64(wa[u], wb[u], xa[t], xb[t])), wsc[u]),
                                              xsc[t]);
                            tw[rr * TB + t][gi] = f;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane < slots) {
                const int gc = G - g0 < GL ? G - g0 : GL;
                const float *row = tw[lane];
#pragma unroll 8
                for (int j = 0; j < gc; ++j) val = __fadd_rn(val, row[j]);   // group order
            }
            __syncwarp();
        }
        if (lane < slots) {
            const int i = i0 + lane / TB, t = t0 + lane % TB;
            if (i < d && t < B) {
                // output rows [0, e0) -> p0, [e0, e1) -> p1, [e1, d) -> p2, each segment [B][len]
                float *p;
                int64_t o;
                if (i < out.e0) {
                    p = out.p0; o = int64_t(t) * out.e0 + i;
                } else if (i < out.e1) {
                    p = out.p1; o = int64_t(t) * (out.e1 - out.e0) + (i - out.e0);
                } else {
                    p = out.p2; o = int64_t(t) * (d - out.e1) + (i - out.e1);
                }
                p[o] = add ? __fadd_rn(add[o], val) : val;        // residual: x[i] += xb[i] (:434, :457)
            }
        }
    }
}

template <int TB>
static cudaError_t launch_mm_t(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n,
                               int d, const float *add, const MmOut &out, cudaStream_t stream, int sms, bool pdl) {
    const int ntb = (B + TB - 1) / TB;
    // Rows per tile: enough jobs for ~16 warps per SM, at most 32 / TB (one lane
    // per (row, token)); one token: at most 16 (the 151,936-row classifier
    // streams faster as 1,187 CTAs of 8 warps x 16 rows than as 594 x 32 rows).
    const int64_t want = int64_t(sms) * 16;
    int64_t rb = (int64_t(d) * ntb + want - 1) / want;
    if (rb < 1) rb = 1;
    if (rb > (TB == 1 ? 16 : 32 / TB)) rb = TB == 1 ? 16 : 32 / TB;
    const int RB = int(rb);
    const int64_t jobs = int64_t((d + RB - 1) / RB) * ntb;
    int64_t grid = (jobs + MM_WARPS - 1) / MM_WARPS;
    if (grid > int64_t(sms) * 8) grid = int64_t(sms) * 8;
    if (!pdl) {
        matmul_q8_kernel<TB, TB == 1 ? 4 : 2, 0><<<unsigned(grid), MM_THREADS, 0, stream>>>(xq, xs, B, wq, ws, n, d,
                                                                                           RB, add, out, MmPro{});
        return cudaGetLastError();
    }
    return launch_dependent(matmul_q8_kernel<TB, TB == 1 ? 4 : 2, 0>, dim3(unsigned(grid)), dim3(MM_THREADS), 0,
                            stream, xq, xs, B, wq, ws, n, d, RB, add, out, MmPro{});
}

// Tiles as launch_mm_t<1> sizes them; always a dependent launch.
template <int PRO>
static cudaError_t launch_mm_pro(const MmPro &pro, int n, const int8_t *wq, const float *ws, int d, const float *add,
                                 const MmOut &out, cudaStream_t stream, int sms) {
    const int64_t want = int64_t(sms) * 16;
    int64_t rb = (int64_t(d) + want - 1) / want;
    if (rb < 1) rb = 1;
    if (rb > 32) rb = 32;
    const int RB = int(rb);
    const int64_t jobs = (d + RB - 1) / RB;
    int64_t grid = (jobs + MM_WARPS - 1) / MM_WARPS;
    if (grid > int64_t(sms) * 8) grid = int64_t(sms) * 8;
    const int cap = pro_smem_bytes(PRO, PRO == PRO_RMS ? PRO_RMS_MAXN : PRO_SWIGLU_MAXN);
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(matmul_q8_kernel<1, 4, PRO>), size_t(cap),
                                     PRO == PRO_RMS ? 27 : 28);
    if (e != cudaSuccess) return e;
    return launch_dependent(matmul_q8_kernel<1, 4, PRO>, dim3(unsigned(grid)), dim3(MM_THREADS),
                            size_t(pro_smem_bytes(PRO, n)), stream, static_cast<const int8_t *>(nullptr),
                            static_cast<const float *>(nullptr), 1, wq, ws, n, d, RB, add, out, pro);
}

cudaError_t launch_matmul_q8_pro(MmProKind kind, const MmPro &pro, int n, const int8_t *wq, const float *ws, int d,
                                 const MmOut &out, cudaStream_t stream, int sms, const float *add) {
    if (d == 0) return cudaSuccess;
    if (n <= 0 || n % GS != 0 || (kind == PRO_RMS ? n > PRO_RMS_MAXN : n > PRO_SWIGLU_MAXN)) return cudaErrorInvalidValue;
    return kind == PRO_RMS ? launch_mm_pro<PRO_RMS>(pro, n, wq, ws, d, add, out, stream, sms)
                           : launch_mm_pro<PRO_SWIGLU>(pro, n, wq, ws, d, add, out, stream, sms);
}

cudaError_t launch_matmul_q8(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n,
                             int d, float *out, cudaStream_t stream, int sms, const float *add) {
    return launch_matmul_q8_seg(xq, xs, B, wq, ws, n, d, MmOut{out, out, out, d, d}, stream, sms, add, false);
}

cudaError_t launch_matmul_q8_seg(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n,
                                 int d, const MmOut &out, cudaStream_t stream, int sms, const float *add, bool pdl) {
    if (B == 0 || d == 0) return cudaSuccess;
    if (B == 1) return launch_mm_t<1>(xq, xs, B, wq, ws, n, d, add, out, stream, sms, pdl);
    if (B == 2) return launch_mm_t<2>(xq, xs, B, wq, ws, n, d, add, out, stream, sms, pdl);
    return launch_mm_t<4>(xq, xs, B, wq, ws, n, d, add, out, stream, sms, pdl);
}

}  // namespace q3
