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
// (MMA N, column = output row), one CTA per SM over the tiles; 18 warps:
//   warp 0   TMA producer: per K-stage of 128 bytes (two groups), a 128 x 128 B
//            box of the token codes and of the weight codes, 128-byte swizzled
//            (the K-major operand layout), into a 4-stage ring;
//   warp 1   allocates all 512 tensor-memory columns (4 accumulators of 128)
//            and issues the MMAs (one elected lane): per group two
//            tcgen05.mma.kind::i8 of K = 32 into accumulator g % 4, committed
//            to that accumulator's `full` barrier; per stage a commit that
//            releases the stage;
//   warps 2-17 fold: warp w reads tensor-memory lanes 32*(w%4).. (its 32
//            tokens) and a quarter of the 128 columns.  Each warp stages the
//            weight scales of its own 32 output rows, 16 groups at a time, by
//            coalesced asynchronous copies and an in-warp transpose to
//            [group][row], into a private double buffer (no barrier between
//            warps); its token's scale is read two groups ahead.  Per group:
//            tcgen05.ld of the 32 dots (the second 16 read while the first are
//            folded), the accumulator handed back to the MMA warp, the 32 folds
//            (products in packed f32x2 arithmetic, the accumulate scalar);
//            after the tile's last group the 32 sums go out through shared
//            memory as two tensor stores (plain stores when d % 4 != 0).
// Measured on the 4096 x 2560 -> 9728 product (Qwen3-4B W1 of a 4096-token
// prefill): ~470 us.  The fold issues ~190 instructions per warp and group
// (issue ~70% busy), each group's accumulator makes a round trip fold -> MMA
// -> fold through four tensor-memory buffers, and the MMA thread still waits
// ~500-650 cycles per stage for its operands: the tensor pipe is ~12% busy.
// Each group's first MMA overwrites its accumulator (the second adds to it),
// so no accumulator needs clearing; the fold converts the int32 dot to float
// exactly (|dot| <= 64 * 128 * 128 < 2^24).
// Every wait is bounded; on a timeout the kernel records Q3CU_DEV_TIMEOUT,
// waits (bounded) for its own copies and MMAs, frees tensor memory and returns.
#include "q3cu_internal.h"
#include "q3cu_tma.h"

namespace q3 {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 128;        // tokens, output rows, K bytes per stage
constexpr int TC_NS = 4;                                     // smem stages
constexpr int TC_NACC = 4;                                   // tensor-memory accumulators (128 columns each)
constexpr int TC_EPI = 16;                                   // fold warps: 4 per tensor-memory lane quarter
constexpr int TC_WARPS = 2 + TC_EPI, TC_THREADS = TC_WARPS * 32;
constexpr int TC_TILE_B = TC_BM * TC_BK;                     // 16 KB per operand per stage
constexpr int TC_STAGE_B = 2 * TC_TILE_B;
constexpr int TC_CG = 16;                                    // groups of weight scales staged at a time
constexpr int TC_WCH = TC_CG * 32;                           // floats of one warp's staged chunk ([group][32 rows])
constexpr int TC_OST = 32 * 16;                              // floats of one warp's output staging (32 x 16)
constexpr size_t TC_SMEM = size_t(TC_NS) * TC_STAGE_B + 1024 +
                           size_t(TC_EPI) * (2 * TC_WCH + TC_OST) * 4;   // ring, align, per warp: 2 chunks + staging
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
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The wait, with the loaded registers as operands: nothing that reads them can
// be scheduled before it.
__device__ __forceinline__ void tc_wait_ld16(uint32_t (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
                 :: "memory");
}
// 16-byte asynchronous copy global -> shared; src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16z(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
// 4-byte asynchronous copy global -> shared (any destination: it transposes);
// src_bytes 0 writes a zero.
__device__ __forceinline__ void cp_async4(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" :: "r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

// acc[c] = RN(acc[c] + RN(RN(float(dot_c) * ws[c]) * xs)) for 16 consecutive
// columns.  Products in packed f32x2 arithmetic; the add is scalar, because a
// packed add after packed multiplies was measured to be contracted into a fused
// multiply-add (one rounding fewer than the reference).
__device__ __forceinline__ void fold16(float *acc, const uint32_t (&v)[16], const float *w, f2 xs2) {
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
#pragma unroll
    for (int c = 0; c < 16; c += 4) {
        const float4 wv = w4[c / 4];                              // the same address in every lane
        const f2 f01 = pk2(__int2float_rn(int(v[c])), __int2float_rn(int(v[c + 1])));
        const f2 f23 = pk2(__int2float_rn(int(v[c + 2])), __int2float_rn(int(v[c + 3])));
        const f2 t01 = mul2(mul2(f01, pk2(wv.x, wv.y)), xs2);
        const f2 t23 = mul2(mul2(f23, pk2(wv.z, wv.w)), xs2);
        float tt[4];
        up2(t01, tt[0], tt[1]);
        up2(t23, tt[2], tt[3]);
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[c + u] = __fadd_rn(acc[c + u], tt[u]);
    }
}

// The producer's and the MMA thread's bounded wait: it naps 64 ns between
// polls, so the two waiting warps take few issue slots from the fold warps
// that share their SM sub-partitions (measured ~1.5% faster than spinning on
// the 4096 x 2560 -> 9728 product).
__device__ __forceinline__ bool tc_wait_nap(uint64_t *bar, uint32_t parity, uint32_t *status) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < WAIT_POLLS; ++i) {
        __nanosleep(64);
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 15u) == 15u && global_ns() - t0 > WAIT_NS) break;
    }
    if (status) atomicOr(status, Q3CU_DEV_TIMEOUT);
    return false;
}

// Tile order: the output tile varies fastest (measured a few per cent faster
// than token-tile-fastest and than blocked orders on the 4096 x 2560 -> 9728
// product), so the CTAs running at one time share each token tile.
__device__ __forceinline__ void tc_tile(int tile, int mt, int ntl, int &m0, int &n0) {
    (void)mt;
    m0 = (tile / ntl) * TC_BM;
    n0 = (tile % ntl) * TC_BN;
}

__global__ void __launch_bounds__(TC_THREADS, 1) q8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmx,
                                                                   const __grid_constant__ CUtensorMap tmw,
                                                                   const __grid_constant__ CUtensorMap tmo,
                                                                   int tma_out,
                                                                   const float *__restrict__ xs,
                                                                   const float *__restrict__ ws, float *out,
                                                                   int T, int d, int n, uint32_t *status) {
    extern __shared__ uint8_t tc_dyn[];
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_dyn) + 1023) & ~uintptr_t(1023));
    // per fold warp: two weight-scale chunks [TC_CG][32] and an output staging [32][16]
    float *fw_s = reinterpret_cast<float *>(ring + size_t(TC_NS) * TC_STAGE_B);
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
                int m0, n0;
                tc_tile(tile, mt, ntl, m0, n0);
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int s = it % TC_NS;
                    if (it >= TC_NS && !tc_wait_nap(&empty[s], uint32_t(it / TC_NS - 1) & 1u, status)) {
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
                    if (!(ok = tc_wait_nap(&full[s], uint32_t(it / TC_NS) & 1u, status))) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(ring + size_t(s) * TC_STAGE_B), b_addr = a_addr + TC_TILE_B;
                    for (int h = 0; h < 2; ++h, ++g) {            // the stage's two 64-groups
                        const int acc = g % TC_NACC;
                        if (!(ok = tc_wait_nap(&acc_empty[acc], uint32_t(g / TC_NACC) & 1u, status))) break;
                        tc_fence_after();
                        const uint32_t tmem_d = tbase + uint32_t(acc * TC_BN);
                        for (int k = 0; k < 2; ++k) {             // K = 32 bytes each
                            const uint32_t off = uint32_t((2 * h + k) * 32);
                            tc_mma(tmem_d, tc_sdesc(a_addr + off), tc_sdesc(b_addr + off), uint32_t(k));
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
        const int e = warp - 2;                               // 0..15
        const int q = warp & 3, part = e >> 2;                // tensor-memory lane quarter, column quarter
        const uint32_t lane_addr = tbase + (uint32_t(32 * q) << 16) + uint32_t(32 * part);
        float *wbuf = fw_s + e * (2 * TC_WCH + TC_OST);       // this warp's two chunks, then its staging
        float *ost = wbuf + 2 * TC_WCH;
        // every accumulator starts free
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int a = 0; a < TC_NACC; ++a) mbar_arrive(&acc_empty[a]);
        // The weight scales of this warp's 32 output rows, TC_CG groups at a time,
        // transposed to [group][row] by 4-byte asynchronous copies (lane = row) into
        // buffer k % 2; chunk k + 1 is copied while chunk k is folded.  The token
        // scale of this thread's token is read from global memory two groups ahead.
        auto tile_org = [&](int t, int &m0, int &n0) {
            const int tile = int(blockIdx.x) + t * int(gridDim.x);
            tc_tile(tile, mt, ntl, m0, n0);
        };
        // With G % 4 == 0 (every 16-byte piece of a row's chunk aligned) the chunk is
        // copied coalesced, 16 bytes at a time, into `raw` as [32 rows][TC_CG groups]
        // and transposed by the warp once it has landed; otherwise 4 bytes at a time
        // straight to [group][row].
        const bool vec = (G & 3) == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0;
        float *raw = ost;                                     // free between a tile's stores and its next chunk
        auto stage_ws = [&](int t, int j0, int b) {
            int m0, n0;
            tile_org(t, m0, n0);
            const int cg = G - j0 < TC_CG ? G - j0 : TC_CG;
            if (vec) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {                 // 128 pieces: row 8i + lane / 4, piece lane % 4
                    const int rr = 8 * i + (lane >> 2), c4 = 4 * (lane & 3), r = n0 + 32 * part + rr;
                    const bool v = r < d && c4 < cg;
                    cp_async16z(raw + rr * TC_CG + c4, ws + (v ? int64_t(r) * G + j0 + c4 : 0), v ? 16u : 0u);
                }
            } else {
                const int r = n0 + 32 * part + lane;
                const bool v = r < d;
                const float *src = ws + (v ? int64_t(r) * G + j0 : 0);
                float *dst = wbuf + b * TC_WCH + lane;
                for (int jj = 0; jj < cg; ++jj) cp_async4(dst + jj * 32, src + (v ? jj : 0), v ? 4u : 0u);
            }
            cp_async_commit();
        };
        // the staged chunk into buffer b: wait for the copies, transpose `raw` (vec)
        auto land_ws = [&](int b) {
            cp_async_wait<0>();
            __syncwarp();
            if (vec) {
                // lane = row; its 16 groups read as 4 float4 in a lane-rotated order
                // (conflict-free), written as [group][row] (conflict-free)
                float *dst = wbuf + b * TC_WCH + lane;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int ci = (c + (lane >> 1)) & 3;
                    const float4 v4 = *reinterpret_cast<const float4 *>(raw + lane * TC_CG + 4 * ci);
                    dst[(4 * ci + 0) * 32] = v4.x;
                    dst[(4 * ci + 1) * 32] = v4.y;
                    dst[(4 * ci + 2) * 32] = v4.z;
                    dst[(4 * ci + 3) * 32] = v4.w;
                }
                __syncwarp();
            }
        };
        // token-scale prefetch cursor: tile pf_t, group pf_j, this thread's row of xs (or null)
        int pf_t = 0, pf_j = 0;
        const float *pf_row = nullptr;
        auto pf_seek = [&]() {
            pf_row = nullptr;
            if (pf_t < my_tiles) {
                int m0, n0;
                tile_org(pf_t, m0, n0);
                const int row = m0 + 32 * q + lane;
                if (row < T) pf_row = xs + int64_t(row) * G;
            }
        };
        auto xs_next = [&]() -> float {                       // the cursor's scale, then advance
            const float v = pf_row ? __ldg(pf_row + pf_j) : 0.0f;
            if (++pf_j == G) {
                pf_j = 0;
                ++pf_t;
                pf_seek();
            }
            return v;
        };
        int g = 0, k = 0;
        bool ok = true;
        if (my_tiles > 0) {
            stage_ws(0, 0, 0);
            land_ws(0);
        }
        pf_seek();
        float xs_n1 = xs_next(), xs_n2 = xs_next();           // the next two groups' token scales
        for (int t = 0; t < my_tiles && ok; ++t) {
            int m0, n0;
            tile_org(t, m0, n0);
            const int col0 = n0 + 32 * part;                  // this warp's first output row
            float accv[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) accv[i] = 0.0f;
            for (int j0 = 0; j0 < G && ok; j0 += TC_CG, ++k) {
                const int b = k & 1, cg = G - j0 < TC_CG ? G - j0 : TC_CG;
                const bool more = j0 + TC_CG < G || t + 1 < my_tiles;   // a next chunk exists
                const float *wch = wbuf + b * TC_WCH;
                // Per group: the second half of the dots is read while the first is folded;
                // the accumulator is released before the second half is folded.
                for (int jj = 0; jj < cg && ok; ++jj, ++g) {
                    const int acc = g % TC_NACC;
                    const uint32_t ta = lane_addr + uint32_t(acc * TC_BN);
                    const float xsv = xs_n1;
                    xs_n1 = xs_n2;
                    xs_n2 = xs_next();
                    if (!(ok = __all_sync(FULL, mbar_wait(&acc_full[acc], uint32_t(g / TC_NACC) & 1u,
                                                          lane == 0 ? status : nullptr))))
                        break;
                    tc_fence_after();
                    uint32_t va[16], vb[16];
                    tc_ld16(ta, va);                          // columns 0-15 of this warp's 32
                    tc_wait_ld16(va);
                    tc_ld16(ta + 16, vb);                     // columns 16-31, read during the first fold
                    const f2 xs2 = pk2(xsv, xsv);
                    const float *wrow = wch + jj * 32;
                    fold16(accv, va, wrow, xs2);
                    tc_wait_ld16(vb);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[acc]);   // the MMA warp may reuse it now
                    fold16(accv + 16, vb, wrow + 16, xs2);
                    if (jj == 0 && more) {
                        // the next chunk's copies, once the previous tile's tensor stores have
                        // read their staging (`raw` and the other buffer)
                        if (lane == 0) bulk_wait_read();
                        __syncwarp();
                        if (j0 + TC_CG < G) stage_ws(t, j0 + TC_CG, b ^ 1);
                        else stage_ws(t + 1, 0, b ^ 1);
                    }
                }
                if (ok && more) land_ws(b ^ 1);               // the next chunk, ready in the other buffer
            }
            if (!ok) break;
            // the tile's sums: 32 consecutive output rows of this token
            if (tma_out) {
                // through shared memory as two tensor stores of 32 tokens x 16 outputs: the
                // first half staged in `ost`, the second in the chunk buffer just folded (the
                // next chunk's copies wait for these stores); rows past T and columns past d
                // are clipped by the copy
                if (lane == 0) bulk_wait_read();          // the previous tile's stores have read `ost`
                __syncwarp();
                float *half[2] = {ost, wbuf + ((k - 1) & 1) * TC_WCH};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float4 *dst = reinterpret_cast<float4 *>(half[h] + lane * 16);
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        dst[c] = make_float4(accv[16 * h + 4 * c], accv[16 * h + 4 * c + 1], accv[16 * h + 4 * c + 2],
                                             accv[16 * h + 4 * c + 3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && m0 + 32 * q < T) {               // boxes wholly outside: none
                    for (int h = 0; h < 2; ++h)
                        if (col0 + 16 * h < d) tma_store_2d(&tmo, col0 + 16 * h, m0 + 32 * q, half[h]);
                    bulk_commit();
                }
            } else {
                const int row = m0 + 32 * q + lane;           // this thread's token
                if (row < T) {
                    float *o = out + int64_t(row) * d + col0;
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (col0 + i < d) o[i] = accv[i];
                }
            }
        }
        cp_async_wait<0>();                                   // no copy outlives the CTA
        if (lane == 0) bulk_wait_all();                       // the tensor stores are complete
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
    CUtensorMap mx, mw, mo;
    if (!encode_rows_2d_map(&mx, xq, uint64_t(B), uint64_t(n), TC_BM) ||
        !encode_rows_2d_map(&mw, wq, uint64_t(d), uint64_t(n), TC_BN))
        return cudaErrorInvalidValue;
    // outputs by tensor stores where the rows allow a map (d % 4 == 0, 16-byte aligned), else plain stores
    const int tma_out = encode_f32_2d_map(&mo, out, uint64_t(B), uint64_t(d), 16, 32, false) ? 1 : 0;
    if (!tma_out) mo = mx;                                    // unused
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(q8_gemm_tc_kernel), TC_SMEM, 29);
    if (e != cudaSuccess) return e;
    const int tiles = ((B + TC_BM - 1) / TC_BM) * ((d + TC_BN - 1) / TC_BN);
    const int grid = tiles < sms ? tiles : sms;
    q8_gemm_tc_kernel<<<grid, TC_THREADS, TC_SMEM, stream>>>(mx, mw, mo, tma_out, xs, ws, out, B, d, n, status);
    return cudaGetLastError();
}

}  // namespace q3
