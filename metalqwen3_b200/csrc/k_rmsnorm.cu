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
// is run by one lane, in order, and parallelism comes from many rows at once:
// one warp carries up to 32 row chains, one per lane (about 5 cycles per element
// of latency; 28 chains keep pace with an SM's share of HBM for f32 rows).
//
// Persistent CTA per SM over blocks of R <= 32 rows (the same number of rows
// per SM): 16 compute warps and one producer warp.  All data moves through one
// ring of NS = 3 stages of 32 rows x 2 KB in shared memory (an mbarrier per
// stage, rows padded so the chain lanes read distinct banks), so two stages
// are in flight while the chain consumes the third.  Per block:
//   phase 1  the row chunks in order; chain-warp lane r folds row r's chunk into
//            its running sum.  The first nch - NS chunks are released as soon
//            as the chain has read them; the last NS stay in their stages.
//   phase 2  all 16 warps normalise the resident chunks from shared memory,
//            then the released chunks again (second copies, served from L2:
//            they were streamed a few microseconds earlier), apply w*(ss*x)
//            and store the float rows or quantize each 64-group (absmax by
//            xor-shuffle) into int8 codes + f32 scales.
// For a 2560-wide f32 row (5 chunks) only 2 of the 5 chunks are read twice.
// The copies form one stream per CTA (first reads, then second reads, block
// after block).  The first NS items are copied by every thread (cp.async);
// then the producer warp issues item it into stage it % NS, one bulk copy per
// row, once the consumers have released item it - NS (an "empty" mbarrier per
// stage), so the ring runs across phases and blocks, and the ~1 us it takes
// to issue a stage's row copies is spent by a warp with nothing else to do.
#include "q3cu_internal.h"
#include "q3cu_tma.h"

namespace q3 {

constexpr int RMS_CWARPS = 16;                   // compute warps; warp RMS_CWARPS is the producer
constexpr int RMS_CTHREADS = RMS_CWARPS * 32;
constexpr int RMS_THREADS = RMS_CTHREADS + 32;
constexpr int RMS_CHAIN = 1;                     // chain warp: not on the producer's SMSP (warp % 4)
constexpr int RMS_MAXR = 32;                     // rows per block = lanes of the chain warp
constexpr int RMS_CB = 2048;                     // bytes per row per stage
constexpr int RMS_ROWB = RMS_CB + 16;            // padded smem row stride
constexpr int RMS_NS = 3;                        // ring stages
constexpr size_t RMS_SMEM = size_t(RMS_NS) * RMS_MAXR * RMS_ROWB;   // 198,144 bytes

// One 16-byte vector's squares folded into the chain, in index order.
//   * f32: each square rounded, then added (scalar: measured faster than
//     packed squares with the adds between them, 27.9 against 28.6 us on the
//     4096 x 2560 prefill rows);
//   * bf16: squares by packed multiplies, then the adds;
//   * bf16 with FUSE: acc = fma(v, v, acc).  A bf16 value has an 8-bit
//     significand, so v*v has at most 16 significant bits and is exact in
//     binary32 unless it falls below 2^-126, i.e. unless 0 < |v| < 2^-63; for
//     every other v the fused step rounds once where the reference rounds the
//     exact square (no-op) and then the sum: the same bits.  Callers that use
//     it check the row for such values and redo the chain without it.
template <typename T, bool FUSE>
__device__ __forceinline__ void fold_vec(float &acc, uint4 u) {
    constexpr int V = Vec<T>::N;
    static_assert(!FUSE || sizeof(T) == 2, "the fused square is exact for bf16 inputs only");
    float v[V];
    Vec<T>::widen(u, v);
    if constexpr (FUSE) {
#pragma unroll
        for (int i = 0; i < V; ++i) acc = __fmaf_rn(v[i], v[i], acc);
    } else if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int i = 0; i < V; ++i) acc = __fadd_rn(acc, __fmul_rn(v[i], v[i]));
    } else {
        float sq[V];
#pragma unroll
        for (int i = 0; i < V; i += 2) up2(mul2(pk2(v[i], v[i + 1]), pk2(v[i], v[i + 1])), sq[i], sq[i + 1]);
#pragma unroll
        for (int i = 0; i < V; ++i) acc = __fadd_rn(acc, sq[i]);
    }
}

template <typename T, bool FUSE = false>
__device__ __forceinline__ float chain_sum(float acc, const uint8_t *p, int elems) {
    // 16-byte smem loads in batches of 8, the next batch loaded before the
    // current one is folded in; the squares added in index order.
    constexpr int V = Vec<T>::N;
    const uint4 *p4 = reinterpret_cast<const uint4 *>(p);
    const int nv = elems / V, nb8 = nv / 8;
    if (nb8 > 0) {
        uint4 cur[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) cur[j] = p4[j];
        for (int b = 0; b < nb8; ++b) {
            uint4 nxt[8];
            const int kn = (b + 1 < nb8 ? b + 1 : b) * 8;          // the last batch reloads itself
#pragma unroll
            for (int j = 0; j < 8; ++j) nxt[j] = p4[kn + j];
#pragma unroll
            for (int j = 0; j < 8; ++j) fold_vec<T, FUSE>(acc, cur[j]);
#pragma unroll
            for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
        }
    }
    for (int k = nb8 * 8; k < nv; ++k) fold_vec<T, FUSE>(acc, p4[k]);
    return acc;
}

// The same fold over one full 2 KB chunk, fully unrolled: two register batches
// of 8 vectors alternate, so the next batch is in flight while the current one
// is folded in and no copies between them are needed.  (With a run-time trip
// count the loop stays rolled and the batch copies slow the chain by ~40%.)
template <typename T, bool FUSE = false>
__device__ __forceinline__ float chain_full(float acc, const uint8_t *p) {
    constexpr int NB = RMS_CB / 16 / 8;                     // 16 batches of 8 vectors
    const uint4 *p4 = reinterpret_cast<const uint4 *>(p);
    uint4 buf[2][8];
#pragma unroll
    for (int j = 0; j < 8; ++j) buf[0][j] = p4[j];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b + 1 < NB) {
#pragma unroll
            for (int j = 0; j < 8; ++j) buf[(b + 1) & 1][j] = p4[(b + 1) * 8 + j];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) fold_vec<T, FUSE>(acc, buf[b & 1][j]);
    }
    return acc;
}

template <typename T, bool Q8>
__global__ void __launch_bounds__(RMS_THREADS, 1) rmsnorm_kernel(const T *x, const float *__restrict__ w, int64_t rows,
                                                                 int dim, int n_div, float eps, int R, T *out,
                                                                 int8_t *__restrict__ q, float *__restrict__ s,
                                                                 uint32_t *status) {
    constexpr int ESZ = sizeof(T);
    constexpr int V = Vec<T>::N;                 // elements per 16-byte vector
    constexpr int NLPG = GS / V;                 // lanes per Q8_0 group
    extern __shared__ __align__(128) uint8_t stage[];          // [RMS_NS][RMS_MAXR][RMS_ROWB]
    __shared__ __align__(8) uint64_t bar[RMS_NS];             // full: the stage's copies landed
    __shared__ __align__(8) uint64_t empty[RMS_NS];           // the stage's item was released
    __shared__ float ss_sh[RMS_MAXR];
    __shared__ int fail_sh;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t nblocks = (rows + R - 1) / R;
    const int nb = int((nblocks - 1 - blockIdx.x) / gridDim.x) + 1;   // blocks of this CTA (grid <= nblocks)
    const int64_t row_bytes = int64_t(dim) * ESZ;
    const int nch = int((row_bytes + RMS_CB - 1) / RMS_CB);
    const int nre = nch > RMS_NS ? nch - RMS_NS : 0;    // chunks read twice; chunks nre.. stay resident
    const int per_block = nch + nre;                    // stream items per block
    const int total = nb * per_block;

    if (tid == 0) {
        for (int i = 0; i < RMS_NS; ++i) {
            mbar_init(&bar[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init_fence();
        fail_sh = 0;
    }
    __syncthreads();
    griddep_launch_dependents();                  // a dependent-launched successor may start its own prologue
    griddep_wait();                               // x from the kernel before (a dependent launch)

    auto block_rows = [&](int k, int64_t &r0, int &rv) {
        const int64_t b = blockIdx.x + int64_t(k) * gridDim.x;
        r0 = b * R;
        rv = int(rows - r0 < R ? rows - r0 : R);
    };
    auto chunk_bytes = [&](int c) {
        const int64_t off = int64_t(c) * RMS_CB;
        return int(row_bytes - off < RMS_CB ? row_bytes - off : RMS_CB);
    };
    // Item it: block it / per_block; j = it % per_block is the first read of
    // chunk j (j < nch) or the second read of chunk j - nch.  Stage it % NS.
    // Every stage barrier expects one plain arrival per item.
    //
    // The first NS items are copied by every thread with 16-byte cp.async
    // pieces (a warp instruction moves 512 contiguous bytes of one row), so the
    // first chunk lands within about a microsecond; each copying thread attaches
    // its pieces to the stage barrier (a balanced arrival: the pending count
    // rises now and falls when they land), and after a CTA barrier thread 0
    // makes the item's one arrival.
    const int first_items = total < RMS_NS ? total : RMS_NS;
    auto copy_item = [&](int it, int t0, int nthr) {
        const int kb = it / per_block, j = it % per_block, c = j < nch ? j : j - nch, st = it % RMS_NS;
        int64_t r0; int rv;
        block_rows(kb, r0, rv);
        const int vpr = chunk_bytes(c) / 16;            // 16-byte vectors per row
        const uint8_t *src = reinterpret_cast<const uint8_t *>(x) + r0 * row_bytes + int64_t(c) * RMS_CB;
        uint8_t *dst = stage + size_t(st) * RMS_MAXR * RMS_ROWB;
        for (int f = t0; f < rv * vpr; f += nthr) {
            const int r = f / vpr, v = f - (f / vpr) * vpr;
            cp_async16(dst + r * RMS_ROWB + v * 16, src + r * row_bytes + v * 16);
        }
        cp_async_track(&bar[st]);
    };
    // Item 0 by every thread, published as soon as every piece is attached.
    // Items 1.. by the compute warps other than the chain warp (an SM keeps
    // only ~50 KB of cp.async in flight, so issuing them stalls their issuers
    // until earlier pieces land; the chain warp starts on item 0 meanwhile).
    copy_item(0, tid, RMS_THREADS);
    __syncthreads();
    if (tid == 0) mbar_arrive(&bar[0]);
    if (first_items > 1 && warp < RMS_CWARPS && warp != RMS_CHAIN) {
        const int ft = tid - (warp > RMS_CHAIN ? 32 : 0);        // 0 .. RMS_CTHREADS - 33
        for (int it = 1; it < first_items; ++it) copy_item(it, ft, RMS_CTHREADS - 32);
        named_sync(2, RMS_CTHREADS - 32);
        if (ft == 0)
            for (int it = 1; it < first_items; ++it) mbar_arrive(&bar[it]);
    }
    // Later items: the producer warp, one bulk copy per row (lane r copies row
    // r's piece); the expect-tx arrival is the item's one arrival.  Bulk copies
    // do not count against the SM's cap on outstanding cp.async bytes (~50 KB),
    // so two stages can be in flight while the chain reads the third.
    auto issue = [&](int it) {
        const int k = it / per_block, j = it % per_block, c = j < nch ? j : j - nch, st = it % RMS_NS;
        int64_t r0; int rv;
        block_rows(k, r0, rv);
        const uint32_t bytes = uint32_t(chunk_bytes(c));
        if (lane == 0) mbar_arrive_expect_tx(&bar[st], bytes * uint32_t(rv));
        __syncwarp();
        if (lane < rv)
            bulk_g2s(stage + (size_t(st) * RMS_MAXR + lane) * RMS_ROWB,
                     reinterpret_cast<const uint8_t *>(x) + (r0 + lane) * row_bytes + int64_t(c) * RMS_CB, bytes,
                     &bar[st]);
    };
    // ---- producer warp -----------------------------------------------------
    // Items are released in stream order (one arrival on empty[] each), so the
    // u-th completion of empty[st] is the release of item st + u * NS.  The
    // producer only reads fail_sh: the compute warps' exits must not depend on
    // a write that can land between their reads.
    if (warp == RMS_CWARPS) {
        int issued = first_items;
        for (; issued < total; ++issued) {
            const int st = issued % RMS_NS;
            if (__any_sync(FULL, fail_sh != 0)) break;
            if (!__all_sync(FULL, mbar_wait(&empty[st], uint32_t(issued / RMS_NS - 1) & 1u, lane == 0 ? status : nullptr)))
                break;                             // the consumers' own waits report the failure
            issue(issued);
        }
        // Before the CTA may exit, every copy has landed: the producer's own
        // cp.async pieces, and (bounded wait) the at most NS bulk-copied items
        // that may still be in flight after a failure (normally the consumers
        // have seen them all).
        cp_async_wait<0>();
        if (lane == 0)
            for (int d = issued > first_items + RMS_NS ? issued - RMS_NS : first_items; d < issued; ++d)
                mbar_wait(&bar[d % RMS_NS], uint32_t(d / RMS_NS) & 1u, nullptr);
        return;
    }
    auto wait_item = [&](int i) {
        return __all_sync(FULL, mbar_wait(&bar[i % RMS_NS], uint32_t(i / RMS_NS) & 1u, lane == 0 ? status : nullptr));
    };
    // The norm weights are re-read by every phase-2 step: while the chain warp runs the
    // chains, the other warps pull them into L1.
    if (warp != RMS_CHAIN)
        for (int64_t off = int64_t(tid - (warp > RMS_CHAIN ? 32 : 0)) * 32; off < int64_t(dim); off += int64_t(RMS_CTHREADS - 32) * 32)
            prefetch_l1(w + off);

    for (int k = 0, base = 0; k < nb && !fail_sh; ++k, base += per_block) {
        int64_t r0; int rv;
        block_rows(k, r0, rv);
        // ---- phase 1: the chain warp runs the chains -------------------------
        if (warp == RMS_CHAIN) {
            float acc = 0.0f;
            bool ok = true;
            for (int c = 0; c < nch; ++c) {
                ok = wait_item(base + c);
                if (!ok) break;
                if (lane < rv) {
                    const uint8_t *rp = stage + (size_t((base + c) % RMS_NS) * RMS_MAXR + lane) * RMS_ROWB;
                    const int cb = chunk_bytes(c);
                    acc = cb == RMS_CB ? chain_full<T>(acc, rp) : chain_sum<T>(acc, rp, cb / ESZ);
                }
                __syncwarp();
                if (c < nre && lane == 0) mbar_arrive(&empty[(base + c) % RMS_NS]);   // resident chunks: phase 2
            }
            if (lane < rv) ss_sh[lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, float(n_div)), eps)));
            if (!ok && lane == 0) fail_sh = 1;
        }
        named_sync(1, RMS_CTHREADS);               // ss visible to every compute warp
        if (fail_sh) break;
        // ---- phase 2: every warp, from shared memory -----------------------
        // Step j handles item base + nre + j: the resident chunks nre..nch-1,
        // then the second reads of chunks 0..nre-1.
        for (int j = 0; j < nch; ++j) {
            const int i = base + nre + j;
            const int c = j < nch - nre ? nre + j : j - (nch - nre);
            if (!wait_item(i)) fail_sh = 1;        // benign race: every writer stores 1
            const bool live = __all_sync(FULL, !fail_sh);
            const int cb = chunk_bytes(c);
            const uint8_t *sb = stage + size_t(i % RMS_NS) * RMS_MAXR * RMS_ROWB;
            const int64_t col0 = int64_t(c) * (RMS_CB / ESZ);     // first element of the chunk
            if (cb == RMS_CB) {
                // Full chunk.  Threads tid / 64 + 8p take row r, and the 64 threads of a row
                // take its 8 (f32) or 16 (bf16) groups, LPG2 consecutive lanes per group; a lane
                // holds two 16-byte vectors of its group, at element li*V of the group's first
                // and second half, so each quarter-warp's shared-memory reads cover 128
                // contiguous bytes (odd bf16 groups load their second half first, to take the
                // other 16 banks).  Rows are whole warps, so every branch below is warp-uniform.
                constexpr int LPG2 = GS / (2 * V), RPP = RMS_CTHREADS / 64;
                constexpr int G = ESZ == 4 ? 4 : 1;          // passes in flight (bf16: register limit)
                const int u = tid % 64, rr = tid / 64, gi = u / LPG2, li = u % LPG2;
                const int h0 = ESZ == 2 ? (gi & 1) : 0;
                const int eo0 = gi * GS + h0 * (GS / 2) + li * V, eo1 = gi * GS + (1 - h0) * (GS / 2) + li * V;
                float wv[2 * V];
#pragma unroll
                for (int k4 = 0; k4 < V / 4; ++k4) {
                    Vec<float>::widen(ld_l1_v4(w + col0 + eo0 + 4 * k4), wv + 4 * k4);
                    Vec<float>::widen(ld_l1_v4(w + col0 + eo1 + 4 * k4), wv + V + 4 * k4);
                }
                for (int p0 = 0; p0 * RPP < rv; p0 += G) {
                    float o[G][2 * V];
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const int r = rr + (p0 + g) * RPP;
                        if (!(live && r < rv)) continue;
                        const uint8_t *row = sb + size_t(r) * RMS_ROWB;
                        float xv[2 * V];
                        Vec<T>::widen(*reinterpret_cast<const uint4 *>(row + eo0 * ESZ), xv);
                        Vec<T>::widen(*reinterpret_cast<const uint4 *>(row + eo1 * ESZ), xv + V);
                        const float ssr = ss_sh[r];
                        const f2 ss2 = pk2(ssr, ssr);
#pragma unroll
                        for (int e = 0; e < 2 * V; e += 2)
                            up2(mul2(pk2(wv[e], wv[e + 1]), mul2(ss2, pk2(xv[e], xv[e + 1]))), o[g][e], o[g][e + 1]);
                    }
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const int r = rr + (p0 + g) * RPP;
                        if (!(live && r < rv)) continue;
                        const int64_t e = (r0 + r) * int64_t(dim) + col0;    // chunk start in the row
                        if constexpr (Q8) {
                            uint32_t codes[2 * V / 4];
                            const float scale = q8_encode_lane<2 * V, LPG2>(o[g], codes);
                            if constexpr (V == 4) {
                                st_cs_u32(q + e + eo0, codes[0]);
                                st_cs_u32(q + e + eo1, codes[1]);
                            } else {
                                st_cs_v2(q + e + eo0, make_uint2(codes[0], codes[1]));
                                st_cs_v2(q + e + eo1, make_uint2(codes[2], codes[3]));
                            }
                            if (li == 0) st_cs_f32(s + ((e + gi * GS) >> 6), scale);
                        } else {
                            st_cs_v4(out + e + eo0, Vec<T>::narrow(o[g]));
                            st_cs_v4(out + e + eo1, Vec<T>::narrow(o[g] + V));
                        }
                    }
                }
            } else {
                // Partial last chunk: thread t handles 16-byte
                // vectors f = t + RMS_CTHREADS*i of the [rv][vpr] chunk, U at a time.  vpr is a
                // multiple of the group width (the chunk holds whole 64-groups), so one warp
                // covers whole groups.
                constexpr int U = 4;
                const int vpr = cb / 16;           // 16-byte vectors per row in this chunk
                const int nvec = rv * vpr;
                for (int f0 = 0; f0 < nvec; f0 += RMS_CTHREADS * U) {
                    float o[U][V];
                    int64_t e[U];
                    bool act[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int f = f0 + u * RMS_CTHREADS + tid;
                        act[u] = f < nvec && live;
                        const int r = act[u] ? f / vpr : 0, v = act[u] ? f - (f / vpr) * vpr : 0;
                        e[u] = (r0 + r) * int64_t(dim) + col0 + int64_t(v) * V;
                        if (act[u]) {
                            float wv[V], xv[V];
                            Vec<float>::widen(ld_l1_v4(w + col0 + v * V), wv);
                            if constexpr (V == 8) Vec<float>::widen(ld_l1_v4(w + col0 + v * V + 4), wv + 4);
                            Vec<T>::widen(*reinterpret_cast<const uint4 *>(sb + size_t(r) * RMS_ROWB + v * 16), xv);
                            const float ssr = ss_sh[r];
#pragma unroll
                            for (int i2 = 0; i2 < V; ++i2) o[u][i2] = __fmul_rn(wv[i2], __fmul_rn(ssr, xv[i2]));
                        } else {
#pragma unroll
                            for (int i2 = 0; i2 < V; ++i2) o[u][i2] = 0.0f;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        if constexpr (Q8) {
                            uint32_t codes[V / 4];
                            const float scale = q8_encode_lane<V, NLPG>(o[u], codes);
                            if (act[u]) {
                                if constexpr (V == 4) st_cs_u32(q + e[u], codes[0]);
                                else st_cs_v2(q + e[u], make_uint2(codes[0], codes[1]));
                                if ((lane % NLPG) == 0) st_cs_f32(s + (e[u] >> 6), scale);
                            }
                        } else {
                            if (act[u]) st_cs_v4(out + e[u], Vec<T>::narrow(o[u]));
                        }
                    }
                }
            }
            named_sync(1, RMS_CTHREADS);           // item i consumed by every compute warp
            if (tid == 0) mbar_arrive(&empty[i % RMS_NS]);
        }
    }
}

// ---------------------------------------------------------------------------
// Few rows (decode): one CTA of 256 threads per row.  Every thread copies its
// 16-byte pieces of the row into shared memory with cp.async, attaching each
// to the barrier of its 2 KB chunk; lane 0 of warp 0 folds the chunks into the
// chain as they land (the same fold, in index order, as the persistent
// kernel); then all threads normalise and quantize from shared memory, a lane
// per 8 consecutive elements, 8 lanes per Q8_0 group.  No producer warp, ring
// or block loop: the latency is the first chunk, the chain, and one pass.
constexpr int RSM_THREADS = 256;
constexpr int RSM_CB = 2048;                     // chunk bytes
constexpr int RSM_MAXCH = 32;                    // rows of up to 64 KB
constexpr int RSM_PPC = RSM_CB / 16;             // 16-byte pieces per chunk

template <typename T, bool Q8>
__global__ void __launch_bounds__(RSM_THREADS) rmsnorm_row_kernel(const T *x, const float *__restrict__ w, int dim,
                                                                 int n_div, float eps, T *out,
                                                                 int8_t *__restrict__ q, float *__restrict__ s,
                                                                 uint32_t *status) {
    constexpr int ESZ = sizeof(T);
    extern __shared__ __align__(128) uint8_t rbuf[];
    __shared__ __align__(8) uint64_t bar[RSM_MAXCH];
    __shared__ float ss_sh;
    griddep_launch_dependents();                  // a dependent-launched successor may start its own prologue
    const int tid = threadIdx.x;
    const int64_t row = blockIdx.x;
    const int row_bytes = dim * ESZ;
    const int nch = (row_bytes + RSM_CB - 1) / RSM_CB;
    const uint8_t *src = reinterpret_cast<const uint8_t *>(x) + row * int64_t(row_bytes);
    if (tid == 0) {
        for (int c = 0; c < nch; ++c) mbar_init(&bar[c], 1);
        mbar_init_fence();
    }
    griddep_wait();                               // x from the kernel before (a dependent launch)
    __syncthreads();
    for (int f = tid; f < row_bytes / 16; f += RSM_THREADS) {
        cp_async16(rbuf + f * 16, src + f * 16);
        cp_async_track(&bar[f / RSM_PPC]);
    }
    __syncthreads();                              // every piece attached before the arrivals
    if (tid == 0)
        for (int c = 0; c < nch; ++c) mbar_arrive(&bar[c]);
    // bf16 rows: the chain folds each square with a fused multiply-add (exact
    // unless the row holds a value with 0 < |v| < 2^-63, see fold_vec); the
    // other warps look for such values while it runs, and if there is one the
    // chain is folded again the reference's way.  Measured on 256 x 8192 bf16
    // rows: 42 -> 31 us per launch.
    constexpr bool FUSE = ESZ == 2;
    auto rsqrt_ss = [&](float acc) { return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, float(n_div)), eps))); };
    bool ok = true;
    int tiny = 0;
    if (tid < 32) {
        float acc = 0.0f;
        for (int c = 0; c < nch && ok; ++c) {
            ok = __all_sync(FULL, mbar_wait(&bar[c], 0, tid == 0 ? status : nullptr));
            if (ok && tid == 0) {
                const int cb = row_bytes - c * RSM_CB < RSM_CB ? row_bytes - c * RSM_CB : RSM_CB;
                acc = cb == RSM_CB ? chain_full<T, FUSE>(acc, rbuf + c * RSM_CB)
                                   : chain_sum<T, FUSE>(acc, rbuf + c * RSM_CB, cb / ESZ);
            }
            __syncwarp();
        }
        if (tid == 0) ss_sh = ok ? rsqrt_ss(acc) : __int_as_float(0x7fc00000);
    } else if constexpr (FUSE) {
        for (int f = tid - 32; f < row_bytes / 16; f += RSM_THREADS - 32) {
            if (!mbar_wait(&bar[f / RSM_PPC], 0, nullptr)) {
                tiny = 1;
                break;
            }
            const uint4 u = *reinterpret_cast<const uint4 *>(rbuf + f * 16);
            const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                tiny |= int(((wd[i] & 0x7fffu) - 1u) < 0x1fffu) | int((((wd[i] >> 16) & 0x7fffu) - 1u) < 0x1fffu);
        }
    }
    if constexpr (FUSE) {
        if (__syncthreads_or(tiny)) {                // block-uniform
            if (tid == 0 && ok) {
                float acc = 0.0f;
                for (int c = 0; c < nch; ++c) {
                    const int cb = row_bytes - c * RSM_CB < RSM_CB ? row_bytes - c * RSM_CB : RSM_CB;
                    acc = cb == RSM_CB ? chain_full<T, false>(acc, rbuf + c * RSM_CB)
                                       : chain_sum<T, false>(acc, rbuf + c * RSM_CB, cb / ESZ);
                }
                ss_sh = rsqrt_ss(acc);
            }
            __syncthreads();
        }
    } else {
        __syncthreads();
    }
    const float ss = ss_sh;
    const f2 ss2 = pk2(ss, ss);
    const int64_t e0 = row * int64_t(dim);
    for (int u = tid; u * 8 < dim; u += RSM_THREADS) {   // 8 elements per lane; dim % 8 == 0 (host)
        float xv[8], wv[8], o[8];
        if constexpr (ESZ == 4) {
            Vec<float>::widen(*reinterpret_cast<const uint4 *>(rbuf + u * 32), xv);
            Vec<float>::widen(*reinterpret_cast<const uint4 *>(rbuf + u * 32 + 16), xv + 4);
        } else {
            Vec<T>::widen(*reinterpret_cast<const uint4 *>(rbuf + u * 16), xv);
        }
        Vec<float>::widen(ld_l1_v4(w + u * 8), wv);
        Vec<float>::widen(ld_l1_v4(w + u * 8 + 4), wv + 4);
#pragma unroll
        for (int i = 0; i < 8; i += 2)
            up2(mul2(pk2(wv[i], wv[i + 1]), mul2(ss2, pk2(xv[i], xv[i + 1]))), o[i], o[i + 1]);
        if constexpr (Q8) {
            uint32_t codes[2];
            const float scale = q8_encode_lane<8, 8>(o, codes);
            st_cs_u32(q + e0 + u * 8, codes[0]);
            st_cs_u32(q + e0 + u * 8 + 4, codes[1]);
            if ((tid & 7) == 0) st_cs_f32(s + ((e0 + u * 8) >> 6), scale);
        } else if constexpr (ESZ == 4) {
            st_cs_v4(out + e0 + u * 8, Vec<float>::narrow(o));
            st_cs_v4(out + e0 + u * 8 + 4, Vec<float>::narrow(o + 4));
        } else {
            st_cs_v4(out + e0 + u * 8, Vec<T>::narrow(o));
        }
    }
    cp_async_wait<0>();                           // (all landed already; no copy outlives the CTA)
}

// ---------------------------------------------------------------------------
// Many rows (prefill): the rows stream in by TMA, each row's chain is a lane,
// and the normalise + encode pass re-reads the rows from L2.
//
// One CTA per SM owns blocks of R <= 64 consecutive rows (the same number of
// rows per SM).  Warp roles: chain warps 0..ncw-1 (ncw = ceil(R/32); lane l of
// chain warp j runs the Sum x^2 chain of row 32j + l, in index order), the
// producer (the last warp), and the other warps, which normalise and encode.
//   * Producer: one tiled tensor copy per stage -- L lines (128 B each, L odd)
//     of all R rows of a block, [R][L][128 B] with the 128-byte swizzle, so a
//     chain lane reading 16-byte chunk c of its own line i finds it at chunk
//     c ^ (i % 8): lanes r..r+7 hit 8 different bank groups because L is odd.
//     RT_NS stages ring ahead of the chains across blocks (full / empty
//     mbarriers), so HBM streams while the chains add.
//   * Chains: per stage, the row's L lines folded in order (two register sets
//     alternate, one line loaded while the previous is added), then the stage
//     is released.  After the block's last stage each lane publishes
//     ss = 1/sqrtf(sum/n + eps) in a double-buffered slot (ssfull / ssempty
//     mbarriers) and moves on to the next block's stages.
//   * Normalise + encode: the block's rows are read again from global memory
//     (the copy left them in L2 a few microseconds earlier) in 32-byte pieces
//     per lane, the next pieces loading while these are encoded, and w*(ss*x) is stored as floats or
//     encoded into Q8_0 (8 or 4 lanes per 64-group).  This overlaps the next
//     block's chains; in the CTA's last block the chain warps join it.
// Every wait is bounded (mbar_wait); a timeout sets Q3CU_DEV_TIMEOUT and the
// CTA stops after waiting (bounded) for the copies it issued.
constexpr int RT_WARPS = 16;
constexpr int RT_THREADS = RT_WARPS * 32;
constexpr int RT_PRODUCER = RT_WARPS - 1;
constexpr int RT_MAXR = 64;
constexpr int RT_NS = 6;                          // ring stages
constexpr int RT_STAGE_TARGET = 28672;            // bytes of one stage (before 1024-byte rounding)
constexpr int RT_STAGE_MAX = 29696;
constexpr size_t RT_SMEM = size_t(RT_NS) * RT_STAGE_MAX + 1024;   // + alignment of the ring to 1024 B
constexpr int RT_U_F32 = 4;                       // normalise/encode pieces in flight per lane (f32;
constexpr int RT_U_BF16 = 2;                      // bf16 pieces hold twice the elements): two sets of half

// One 128-byte line (8 swizzled 16-byte chunks) folded into the chain: each
// square one rounding, each add one rounding, in index order.  (Scalar
// squares: with the adds between them they schedule better than packed pairs.)
template <typename T>
__device__ __forceinline__ void rt_fold(float &acc, const uint4 (&buf)[8]) {
    constexpr int V = Vec<T>::N;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        float v[V];
        Vec<T>::widen(buf[c], v);
#pragma unroll
        for (int i = 0; i < V; ++i) acc = __fadd_rn(acc, __fmul_rn(v[i], v[i]));     // in index order
    }
}
// Line l of `row` in a swizzled stage: smem line row*L + l, 16-byte chunk c at c ^ (line % 8).
__device__ __forceinline__ void rt_load(uint4 (&buf)[8], const uint8_t *stage, int row, int L, int l) {
    const int line = row * L + l;
    const uint8_t *p = stage + line * 128;
    const int sw = line & 7;
#pragma unroll
    for (int c = 0; c < 8; ++c) buf[c] = *reinterpret_cast<const uint4 *>(p + ((c ^ sw) << 4));
}
// A whole stage of LL lines, LL known at compile time: fully unrolled, the next
// line in flight while this one is added (about 5.7 cycles per element against
// 6.9 with a run-time line count, measured on this B200).
template <typename T, int LL>
__device__ __forceinline__ float rt_chain_fixed(float acc, const uint8_t *stage, int row) {
    uint4 buf[2][8];
    rt_load(buf[0], stage, row, LL, 0);
#pragma unroll
    for (int l = 0; l < LL; ++l) {
        if (l + 1 < LL) rt_load(buf[(l + 1) & 1], stage, row, LL, l + 1);
        rt_fold<T>(acc, buf[l & 1]);
    }
    return acc;
}
// Any line count (the partial last stage of a row): two register sets alternate.
template <typename T>
__device__ __forceinline__ float rt_chain(float acc, const uint8_t *stage, int row, int L, int nlines) {
    uint4 a[8], b[8];
    rt_load(a, stage, row, L, 0);
    int l = 0;
    for (; l + 2 <= nlines; l += 2) {
        rt_load(b, stage, row, L, l + 1);
        rt_fold<T>(acc, a);
        if (l + 2 < nlines) rt_load(a, stage, row, L, l + 2);
        rt_fold<T>(acc, b);
    }
    if (l < nlines) rt_fold<T>(acc, a);
    return acc;
}
template <typename T>
__device__ __forceinline__ float rt_chain_stage(float acc, const uint8_t *stage, int row, int L, int nlines) {
    if (nlines == L) {
        switch (L) {
            case 3: return rt_chain_fixed<T, 3>(acc, stage, row);
            case 5: return rt_chain_fixed<T, 5>(acc, stage, row);
            case 7: return rt_chain_fixed<T, 7>(acc, stage, row);
            case 15: return rt_chain_fixed<T, 15>(acc, stage, row);
            case 31: return rt_chain_fixed<T, 31>(acc, stage, row);
            default: break;
        }
    }
    return rt_chain<T>(acc, stage, row, L, nlines);
}

// One 32-byte piece of a row in the normalise + encode pass.
template <typename T>
struct RtPiece {
    float x[Wide<T>::N], w[Wide<T>::N];
    int64_t e;            // element offset of the piece in x / out / q
    int r;                // row within the block
    bool ok;
};

template <typename T, bool Q8>
__global__ void __launch_bounds__(RT_THREADS, 1) rmsnorm_tma_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                    const T *x, const float *__restrict__ w,
                                                                    int64_t rows, int dim, int n_div, float eps, int R,
                                                                    int L, int stage_b, T *out,
                                                                    int8_t *__restrict__ q, float *__restrict__ s,
                                                                    uint32_t *status) {
    constexpr int N = Wide<T>::N;                    // elements per lane per piece (32 bytes)
    constexpr int LPG = GS / N;                      // lanes per Q8_0 group
    constexpr int STEP = 32 * N;                     // elements per warp piece
    extern __shared__ uint8_t rt_dyn[];
    __shared__ __align__(8) uint64_t full[RT_NS], empty[RT_NS], ssfull[2], ssempty[2];
    __shared__ float ss_sh[2][RT_MAXR];
    __shared__ int fail_sh;
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(rt_dyn) + 1023) & ~uintptr_t(1023));

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ncw = (R + 31) / 32, np2 = RT_WARPS - 1 - ncw;
    const int64_t nblocks = (rows + R - 1) / R;
    const int nb = int((nblocks - 1 - blockIdx.x) / gridDim.x) + 1;   // blocks of this CTA (grid <= nblocks)
    const int64_t row_bytes = int64_t(dim) * sizeof(T);
    const int nl = int(row_bytes / 128);                              // lines per row
    const int spb = (nl + L - 1) / L;                                 // stages per block
    const int total = nb * spb;
    const uint32_t box_bytes = uint32_t(128) * uint32_t(L) * uint32_t(R);

    if (tid == 0) {
        for (int i = 0; i < RT_NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], ncw);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ssfull[i], ncw);
            mbar_init(&ssempty[i], np2);
        }
        mbar_init_fence();
        fail_sh = 0;
    }
    __syncthreads();
    griddep_launch_dependents();                  // a dependent-launched successor may start its own prologue
    griddep_wait();                               // x from the kernel before (a dependent launch)

    auto block_rows = [&](int k, int64_t &r0, int &rv) {
        const int64_t b = blockIdx.x + int64_t(k) * gridDim.x;
        r0 = b * R;
        rv = int(rows - r0 < R ? rows - r0 : R);
    };

    // ---- producer ------------------------------------------------------------
    if (warp == RT_PRODUCER) {
        int issued = 0;
        if (lane == 0) {
            tma_prefetch_desc(&tmap);
            for (; issued < total; ++issued) {
                const int slot = issued % RT_NS;
                if (issued >= RT_NS &&
                    !mbar_wait(&empty[slot], uint32_t(issued / RT_NS - 1) & 1u, status)) {
                    fail_sh = 1;
                    break;
                }
                if (*static_cast<volatile int *>(&fail_sh)) break;
                const int kb = issued / spb, j = issued % spb;
                int64_t r0; int rv;
                block_rows(kb, r0, rv);
                mbar_arrive_expect_tx(&full[slot], box_bytes);
                tma_load_3d(ring + size_t(slot) * stage_b, &tmap, 0, j * L, int(r0), &full[slot]);
            }
            // no copy may outlive the CTA: wait (bounded) for the ones still in flight
            for (int d = issued > RT_NS ? issued - RT_NS : 0; d < issued; ++d)
                mbar_wait(&full[d % RT_NS], uint32_t(d / RT_NS) & 1u, nullptr);
        }
        __syncwarp();
        return;
    }

    // ---- chain warps ---------------------------------------------------------
    if (warp < ncw) {
        const int row = warp * 32 + lane;
        for (int k = 0; k < nb; ++k) {
            int64_t r0; int rv;
            block_rows(k, r0, rv);
            float acc = 0.0f;
            bool ok = true;
            for (int j = 0; j < spb; ++j) {
                const int it = k * spb + j, slot = it % RT_NS;
                ok = __all_sync(FULL, mbar_wait(&full[slot], uint32_t(it / RT_NS) & 1u, lane == 0 ? status : nullptr));
                if (!ok) break;
                if (row < rv) {
                    const int nlines = nl - j * L < L ? nl - j * L : L;
                    acc = rt_chain_stage<T>(acc, ring + size_t(slot) * stage_b, row, L, nlines);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            if (ok && k >= 2)
                ok = __all_sync(FULL, mbar_wait(&ssempty[k & 1], uint32_t((k >> 1) - 1) & 1u,
                                                lane == 0 ? status : nullptr));
            if (!ok) {
                fail_sh = 1;
                break;
            }
            if (row < rv) ss_sh[k & 1][row] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, float(n_div)), eps)));
            __syncwarp();
            if (lane == 0) mbar_arrive(&ssfull[k & 1]);
        }
        if (fail_sh) return;
    }

    // ---- normalise + encode (the other warps; in the last block also the chain warps)
    // A block's pieces (row r, 32-byte piece p) are numbered piece-major,
    // it = p * rv + r, and each participant takes a contiguous range of them;
    // UU pieces are loaded one set ahead of the set being encoded (two register
    // sets alternate), so the L2 latency of the re-read is covered.
    constexpr int UU = sizeof(T) == 4 ? RT_U_F32 / 2 : RT_U_BF16 / 2;
    const bool chain = warp < ncw;
    const int spr = (dim + STEP - 1) / STEP;                        // pieces per row
    for (int k = chain ? nb - 1 : 0; k < nb; ++k) {
        // (the warps that only normalise wait the whole first block's chain: they sleep meanwhile)
        const bool got = chain ? mbar_wait(&ssfull[k & 1], uint32_t(k >> 1) & 1u, lane == 0 ? status : nullptr)
                               : mbar_wait_idle(&ssfull[k & 1], uint32_t(k >> 1) & 1u, lane == 0 ? status : nullptr);
        if (!__all_sync(FULL, got)) {
            fail_sh = 1;
            return;
        }
        int64_t r0; int rv;
        block_rows(k, r0, rv);
        const bool last = k == nb - 1;
        const int P = last ? np2 + ncw : np2;                       // participants
        const int pi = chain ? np2 + warp : warp - ncw;
        const int items = rv * spr;
        const int per = (items + P - 1) / P;
        const int ib = pi * per, ie = ib + per < items ? ib + per : items;
        const float *ssk = ss_sh[k & 1];

        const float inv_rv = 1.0f / float(rv);
        auto load = [&](RtPiece<T> &pc, int it) {
            // p = it / rv from a float reciprocal, off by at most one for it < 2^24: corrected
            int p = __float2int_rz(__fmul_rn(float(it), inv_rv)), r = it - p * rv;
            if (r < 0) { --p; r += rv; } else if (r >= rv) { ++p; r -= rv; }
            const int col = p * STEP + lane * N;
            pc.ok = it < ie && col < dim;
            pc.r = pc.ok ? r : 0;
            pc.e = (r0 + pc.r) * int64_t(dim) + (pc.ok ? col : 0);
            if (pc.ok) {
                // one 32-byte load per lane (x is 32-byte aligned): each L2 sector is requested once
                const U8 xr = Q8 ? ld_nc_v8(x + pc.e) : ld_v8(x + pc.e);      // out may alias x: coherent
                Wide<T>::widen(xr, pc.x);
#pragma unroll
                for (int k4 = 0; k4 < N / 4; ++k4) Vec<float>::widen(ld_l1_v4(w + col + 4 * k4), pc.w + 4 * k4);
            }
        };
        auto encode = [&](const RtPiece<T> &pc, bool active) {      // `active`: warp-uniform
            if (!active) return;
            float o[N];
            if (pc.ok) {
                const float ssr = ssk[pc.r];
                const f2 ss2 = pk2(ssr, ssr);
#pragma unroll
                for (int i = 0; i < N; i += 2)
                    up2(mul2(pk2(pc.w[i], pc.w[i + 1]), mul2(ss2, pk2(pc.x[i], pc.x[i + 1]))), o[i], o[i + 1]);
            } else {
#pragma unroll
                for (int i = 0; i < N; ++i) o[i] = 0.0f;
            }
            if constexpr (Q8) {
                uint32_t codes[N / 4];
                const float scale = q8_encode_lane<N, LPG>(o, codes);      // every lane (shuffles)
                if (!pc.ok) return;
                if constexpr (N == 8) st_cs_v2(q + pc.e, make_uint2(codes[0], codes[1]));
                else st_cs_v4(q + pc.e, make_uint4(codes[0], codes[1], codes[2], codes[3]));
                if ((lane % LPG) == 0) st_cs_f32(s + (pc.e >> 6), scale);
            } else {
                if (!pc.ok) return;
                const U8 v = Wide<T>::narrow(o);
                st_cs_v4(out + pc.e, make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]));
                st_cs_v4(out + pc.e + N / 2, make_uint4(v.w[4], v.w[5], v.w[6], v.w[7]));
            }
        };
        RtPiece<T> A[UU], B[UU];
#pragma unroll
        for (int u = 0; u < UU; ++u) load(A[u], ib + u);
        for (int it = ib; it < ie;) {
#pragma unroll
            for (int u = 0; u < UU; ++u) load(B[u], it + UU + u);
#pragma unroll
            for (int u = 0; u < UU; ++u) encode(A[u], it + u < ie);
            it += UU;
            if (it >= ie) break;
#pragma unroll
            for (int u = 0; u < UU; ++u) load(A[u], it + UU + u);
#pragma unroll
            for (int u = 0; u < UU; ++u) encode(B[u], it + u < ie);
            it += UU;
        }
        __syncwarp();
        if (!chain && !last && lane == 0) mbar_arrive(&ssempty[k & 1]);
    }
}

template <typename T, bool Q8>
static cudaError_t launch_rms_t(const T *x, const float *w, int64_t rows, int dim, int n_div, float eps, T *out,
                                int8_t *q, float *s, uint32_t *status, cudaStream_t stream, int sms) {
    // Equal rows per SM: blocks of R <= 32 rows, the same number per SM, one CTA per SM.
    const int64_t rows_per_sm = (rows + sms - 1) / sms;
    const int64_t bps = (rows_per_sm + RMS_MAXR - 1) / RMS_MAXR;
    const int R = int((rows_per_sm + bps - 1) / bps);
    const int64_t nblocks = (rows + R - 1) / R;
    const unsigned grid = unsigned(nblocks < sms ? nblocks : sms);
    const int64_t row_bytes = int64_t(dim) * sizeof(T);
    if (rows <= int64_t(sms) * 4 && row_bytes <= int64_t(RSM_CB) * RSM_MAXCH && dim % 8 == 0) {
        const int rslot = 12 + (sizeof(T) == 4 ? 0 : 2) + (Q8 ? 1 : 0);
        cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(rmsnorm_row_kernel<T, Q8>),
                                         size_t(RSM_CB) * RSM_MAXCH, rslot);
        if (e != cudaSuccess) return e;
        return launch_dependent(rmsnorm_row_kernel<T, Q8>, dim3(unsigned(rows)), dim3(RSM_THREADS), size_t(row_bytes),
                                stream, x, w, dim, n_div, eps, out, q, s, status);
    }
    // More rows per SM than one chain warp holds (so each SM has several blocks
    // whose normalise + encode pass overlaps the next block's chains), whole
    // 128-byte lines per row: the TMA-fed kernel, blocks of up to 64 rows (the
    // same number per SM), L odd lines per stage.  With one block per SM the
    // pass cannot overlap anything, and the persistent kernel below, which
    // normalises the block's last chunks straight from its ring, measured
    // faster (4096 x 2560 f32: 28.9 against 36 us).  For f32 rows the ring
    // kernel also wins up to two blocks per SM (8192 x 2560: 47.1 against
    // 51.2 us; 20011 x 1024, 135 rows per SM: the same); bf16 rows stream at
    // half the bytes per chain element and take the TMA kernel (16384 x 5120:
    // 135 against 166 us).
    if (rows_per_sm > RMS_MAXR && (sizeof(T) == 2 || rows_per_sm > 2 * RMS_MAXR) && row_bytes % 128 == 0 &&
        reinterpret_cast<uintptr_t>(x) % 32 == 0 &&
        (Q8 ? reinterpret_cast<uintptr_t>(q) % 16 == 0 : reinterpret_cast<uintptr_t>(out) % 16 == 0)) {
        const int64_t bps2 = (rows_per_sm + RT_MAXR - 1) / RT_MAXR;
        const int R2 = int((rows_per_sm + bps2 - 1) / bps2);
        // L: the largest odd line count the chain has an unrolled form for (conflict-free reads need L odd)
        int L = 1;
        for (int c : {31, 15, 7, 5, 3})
            if (128 * c * R2 <= RT_STAGE_TARGET && c <= row_bytes / 128) { L = c; break; }
        const int stage_b = (128 * L * R2 + 1023) & ~1023;
        const int64_t nb2 = (rows + R2 - 1) / R2;
        CUtensorMap map;
        if (stage_b <= RT_STAGE_MAX && encode_row_lines_map(&map, x, uint64_t(rows), uint64_t(row_bytes), L, R2)) {
            const int tslot = 16 + (sizeof(T) == 4 ? 0 : 2) + (Q8 ? 1 : 0);
            cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(rmsnorm_tma_kernel<T, Q8>), RT_SMEM, tslot);
            if (e != cudaSuccess) return e;
            const unsigned g2 = unsigned(nb2 < sms ? nb2 : sms);
            return launch_dependent(rmsnorm_tma_kernel<T, Q8>, dim3(g2), dim3(RT_THREADS), RT_SMEM, stream, map, x, w,
                                    rows, dim, n_div, eps, R2, L, stage_b, out, q, s, status);
        }
    }
    const int slot = 2 + (sizeof(T) == 4 ? 0 : 2) + (Q8 ? 1 : 0);
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(rmsnorm_kernel<T, Q8>), RMS_SMEM, slot);
    if (e != cudaSuccess) return e;
    return launch_dependent(rmsnorm_kernel<T, Q8>, dim3(grid), dim3(RMS_THREADS), RMS_SMEM, stream, x, w, rows, dim,
                            n_div, eps, R, out, q, s, status);
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
