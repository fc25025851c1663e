// k_gemm.cu -- the Q8_0 matmul of a prefill batch on the 5th-generation tensor
// cores (tcgen05, int8 MMA into tensor memory), bit-exact with the reference.
//
// Reference: src/cpu/qwen3_original.c:310-331, for each token row b:
//     for i < d:  val = 0
//                 for each 64-group j (in order):
//                     ival = sum_k xq[b][j*64+k] * wq[i][j*64+k]          (int32, exact)
//                     val += ((float) ival) * ws[i][j] * xs[b][j]         (three roundings)
//                 out[b][i] = val
// The group's integer dot is exact in any order, so the tensor cores compute
// it; the float part is the reference's chain, one rounding per operator, in
// group order: after every group the dot is read out of tensor memory and
// folded in as RN(acc + RN(RN(float(dot) * ws) * xs)).
//
// Tiles of 128 tokens (MMA M, tensor-memory lane = token) by 128 output rows
// (MMA N, column = output row), one CTA per SM over the tiles; 10 warps:
//   warp 0   TMA producer: per K-stage of 128 bytes (two groups), a 128 x 128 B
//            box of the token codes and of the weight codes, 128-byte swizzled
//            (the K-major operand layout), into a 4-stage ring;
//   warp 1   allocates all 512 tensor-memory columns (4 accumulators of 128)
//            and issues the MMAs (one elected lane): per group two
//            tcgen05.mma.kind::i8 of K = 32 into accumulator g % 4, committed
//            to that accumulator's `full` barrier; per stage a commit that
//            releases the stage;
//   warps 2-9 fold: warp w reads tensor-memory lanes 32*(w%4).. (its 32
//            tokens) and half of the 128 columns.  Per group: tcgen05.ld of the
//            64 dots, the accumulator re-armed, the 64 folds (products in packed
//            f32x2 arithmetic, the accumulate scalar), and after the tile's last
//            group the 64 sums stored.
// float(dot) costs one add: every accumulator starts at the integer 0x4B400000
// (the MMA adds the dot to it, enable-input-d always on), whose bit pattern
// read as a float is 1.5 * 2^23 + dot for |dot| < 2^22 (here |dot| <= 64 *
// 127 * 128 < 2^20), so float(dot) = that float - 1.5 * 2^23, exactly.  The
// fold re-arms the accumulator by storing 0x4B400000 back (tcgen05.st).
// Every wait is bounded; on a timeout the kernel records Q3CU_DEV_TIMEOUT,
// waits (bounded) for its own copies and MMAs, frees tensor memory and returns.
#include "q3cu_internal.h"
#include "q3cu_tma.h"

namespace q3 {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 128;        // tokens, output rows, K bytes per stage
constexpr int TC_NS = 4;                                     // smem stages
constexpr int TC_NACC = 4;                                   // tensor-memory accumulators (128 columns each)
constexpr int TC_WARPS = 10, TC_THREADS = TC_WARPS * 32, TC_EPI = 8;
constexpr int TC_TILE_B = TC_BM * TC_BK;                     // 16 KB per operand per stage
constexpr int TC_STAGE_B = 2 * TC_TILE_B;
constexpr size_t TC_SMEM = size_t(TC_NS) * TC_STAGE_B + 1024 + size_t(TC_EPI) * 64 * 4;   // ring + align + ws staging
constexpr uint32_t TC_MAGIC = 0x4B400000u;                   // 1.5 * 2^23 as a float
// Instruction descriptor: int32 accumulator, signed int8 A and B, both K-major,
// N = 128 (bits 17-22: N / 8), M = 128 (bits 24-28: M / 16).
constexpr uint32_t TC_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(TC_BN / 8) << 17) | (uint32_t(TC_BM / 16) << 24);

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled operand:
// start address / 16, leading offset 1 (unused with the swizzle), stride 1024 B
// between 8-row groups (/16), descriptor version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t tc_sdesc(uint32_t smem_addr) {
    return uint64_t((smem_addr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(1u) : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tc_st32_magic(uint32_t taddr) {
    const uint32_t m = TC_MAGIC;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};"
        :: "r"(taddr), "r"(m) : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(TC_THREADS, 1) q8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmx,
                                                                   const __grid_constant__ CUtensorMap tmw,
                                                                   const float *__restrict__ xs,
                                                                   const float *__restrict__ ws, float *out,
                                                                   int T, int d, int n, uint32_t *status) {
    extern __shared__ uint8_t tc_dyn[];
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_dyn) + 1023) & ~uintptr_t(1023));
    float *ws_stage = reinterpret_cast<float *>(ring + size_t(TC_NS) * TC_STAGE_B);      // [TC_EPI][64]
    __shared__ __align__(8) uint64_t full[TC_NS], empty[TC_NS], acc_full[TC_NACC], acc_empty[TC_NACC], drain;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = n / GS, KB = n / TC_BK;                    // groups per row, K-stages per tile
    const int mt = (T + TC_BM - 1) / TC_BM, ntl = (d + TC_BN - 1) / TC_BN;
    const int tiles = mt * ntl;
    const int my_tiles = tiles > int(blockIdx.x) ? (tiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < TC_NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < TC_NACC; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], TC_EPI);
        }
        mbar_init(&drain, 1);
        mbar_init_fence();
        abort_sh = 0;
    }
    if (warp == 1) {                                          // all 512 columns (one CTA per SM)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_addr(&tmem_base_sh)), "r"(512) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base_sh;

    if (warp == 0) {
        // ---- TMA producer -------------------------------------------------------
        if (lane == 0) {
            int it = 0;
            for (int t = 0; t < my_tiles && !*static_cast<volatile int *>(&abort_sh); ++t) {
                const int tile = int(blockIdx.x) + t * int(gridDim.x);
                const int m0 = (tile % mt) * TC_BM, n0 = (tile / mt) * TC_BN;
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int s = it % TC_NS;
                    if (it >= TC_NS && !mbar_wait(&empty[s], uint32_t(it / TC_NS - 1) & 1u, status)) {
                        abort_sh = 1;
                        break;
                    }
                    uint8_t *st = ring + size_t(s) * TC_STAGE_B;
                    mbar_arrive_expect_tx(&full[s], TC_STAGE_B);
                    tma_load_2d(st, &tmx, kb * TC_BK, m0, &full[s]);
                    tma_load_2d(st + TC_TILE_B, &tmw, kb * TC_BK, n0, &full[s]);
                }
            }
            // no copy may outlive the CTA: the last stages issued have landed (bounded)
            for (int d2 = it > TC_NS ? it - TC_NS : 0; d2 < it; ++d2)
                mbar_wait(&full[d2 % TC_NS], uint32_t(d2 / TC_NS) & 1u, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer ---------------------------------------------------------
        if (lane == 0) {
            int it = 0, g = 0;
            bool ok = true;
            for (int t = 0; t < my_tiles && ok; ++t) {
                for (int kb = 0; kb < KB && ok; ++kb, ++it) {
                    const int s = it % TC_NS;
                    if (!(ok = mbar_wait(&full[s], uint32_t(it / TC_NS) & 1u, status))) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(ring + size_t(s) * TC_STAGE_B), b_addr = a_addr + TC_TILE_B;
                    for (int h = 0; h < 2; ++h, ++g) {            // the stage's two 64-groups
                        const int acc = g % TC_NACC;
                        if (!(ok = mbar_wait(&acc_empty[acc], uint32_t(g / TC_NACC) & 1u, status))) break;
                        tc_fence_after();
                        const uint32_t tmem_d = tbase + uint32_t(acc * TC_BN);
                        for (int k = 0; k < 2; ++k) {             // K = 32 bytes each
                            const uint32_t off = uint32_t((2 * h + k) * 32);
                            tc_mma(tmem_d, tc_sdesc(a_addr + off), tc_sdesc(b_addr + off));
                        }
                        tc_commit(&acc_full[acc]);
                    }
                    if (ok) tc_commit(&empty[s]);              // the stage is free once these MMAs have read it
                }
            }
            if (!ok) abort_sh = 1;
            // every MMA issued has completed before tensor memory is released (bounded)
            tc_commit(&drain);
            mbar_wait(&drain, 0, nullptr);
        }
        __syncwarp();
    } else {
        // ---- fold warps ---------------------------------------------------------
        const int e = warp - 2;                               // 0..7
        const int q = warp & 3, half = e >> 2;                // tensor-memory lane quarter, column half
        const uint32_t lane_addr = tbase + (uint32_t(32 * q) << 16) + uint32_t(64 * half);
        float *wsb = ws_stage + e * 64;
        // arm every accumulator with the bias, then hand them to the MMA warp
        for (int a = 0; a < TC_NACC; ++a) {
            tc_st32_magic(lane_addr + uint32_t(a * TC_BN));
            tc_st32_magic(lane_addr + uint32_t(a * TC_BN + 32));
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int a = 0; a < TC_NACC; ++a) mbar_arrive(&acc_empty[a]);
        const f2 NEG_M = pk2(-12582912.0f, -12582912.0f);
        int g = 0;
        bool ok = true;
        for (int t = 0; t < my_tiles && ok; ++t) {
            const int tile = int(blockIdx.x) + t * int(gridDim.x);
            const int m0 = (tile % mt) * TC_BM, n0 = (tile / mt) * TC_BN;
            const int row = m0 + 32 * q + lane;               // this thread's token
            const int col0 = n0 + 64 * half;                  // this warp's first output row
            const float *xs_row = xs + int64_t(row < T ? row : 0) * G;
            float accv[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) accv[i] = 0.0f;
            for (int j = 0; j < G; ++j, ++g) {
                // this group's weight scales for the warp's 64 output rows, staged for broadcast reads
                const int c0 = col0 + lane, c1 = col0 + 32 + lane;
                wsb[lane] = c0 < d ? __ldg(ws + int64_t(c0) * G + j) : 0.0f;
                wsb[32 + lane] = c1 < d ? __ldg(ws + int64_t(c1) * G + j) : 0.0f;
                const float xsv = row < T ? __ldg(xs_row + j) : 0.0f;
                const f2 xs2 = pk2(xsv, xsv);
                __syncwarp();
                const int acc = g % TC_NACC;
                if (!(ok = __all_sync(FULL, mbar_wait(&acc_full[acc], uint32_t(g / TC_NACC) & 1u,
                                                      lane == 0 ? status : nullptr))))
                    break;
                tc_fence_after();
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t v[32];
                    const uint32_t ta = lane_addr + uint32_t(acc * TC_BN + 32 * hh);
                    tc_ld32(ta, v);
                    tc_wait_ld();
                    tc_st32_magic(ta);                        // re-arm (after the read above completed)
                    const float4 *w4 = reinterpret_cast<const float4 *>(wsb + 32 * hh);
#pragma unroll
                    for (int c = 0; c < 32; c += 4) {
                        const float4 wv = w4[c / 4];
                        const f2 f01 = add2(pk2(__uint_as_float(v[c]), __uint_as_float(v[c + 1])), NEG_M);
                        const f2 f23 = add2(pk2(__uint_as_float(v[c + 2]), __uint_as_float(v[c + 3])), NEG_M);
                        const f2 t01 = mul2(mul2(f01, pk2(wv.x, wv.y)), xs2);     // RN(RN(dot * ws) * xs)
                        const f2 t23 = mul2(mul2(f23, pk2(wv.z, wv.w)), xs2);
                        float t[4];
                        up2(t01, t[0], t[1]);
                        up2(t23, t[2], t[3]);
                        // the add is scalar: a packed add after packed multiplies was measured to be
                        // contracted into a fused multiply-add (one rounding fewer than the reference)
#pragma unroll
                        for (int u = 0; u < 4; ++u) accv[32 * hh + c + u] = __fadd_rn(accv[32 * hh + c + u], t[u]);
                    }
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();                                 // wsb reads done before the next group's writes
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
            }
            if (!ok) break;
            // the tile's sums: 64 consecutive output rows of this token
            if (row < T) {
                float *o = out + int64_t(row) * d + col0;
                if (col0 + 64 <= d && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                    for (int i = 0; i < 64; i += 4)
                        st_cs_v4(o + i, make_uint4(__float_as_uint(accv[i]), __float_as_uint(accv[i + 1]),
                                                   __float_as_uint(accv[i + 2]), __float_as_uint(accv[i + 3])));
                } else {
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (col0 + i < d) o[i] = accv[i];
                }
            }
        }
        if (!ok) abort_sh = 1;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tbase), "r"(512) : "memory");
}

bool matmul_q8_tc_supported(int B, int n, int d) {
    return B >= TC_BM && n % TC_BK == 0 && d >= 1 && n >= TC_BK;
}

cudaError_t launch_matmul_q8_tc(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n,
                                int d, float *out, uint32_t *status, cudaStream_t stream, int sms) {
    CUtensorMap mx, mw;
    if (!encode_rows_2d_map(&mx, xq, uint64_t(B), uint64_t(n), TC_BM) ||
        !encode_rows_2d_map(&mw, wq, uint64_t(d), uint64_t(n), TC_BN))
        return cudaErrorInvalidValue;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(q8_gemm_tc_kernel), TC_SMEM, 29);
    if (e != cudaSuccess) return e;
    const int tiles = ((B + TC_BM - 1) / TC_BM) * ((d + TC_BN - 1) / TC_BN);
    const int grid = tiles < sms ? tiles : sms;
    q8_gemm_tc_kernel<<<grid, TC_THREADS, TC_SMEM, stream>>>(mx, mw, xs, ws, out, B, d, n, status);
    return cudaGetLastError();
}

}  // namespace q3
