// k_softmax.cu -- in-place softmax of ragged f32 rows.
//
// Reference: src/cpu/qwen3_original.c:291-308 (called per head with pos+1
// scores at :416):
//     max_val = 0; for i: if (x[i] > max_val) max_val = x[i];   // starts at 0
//     sum = 0;     for i: x[i] = expf(x[i] - max_val); sum += x[i];
//     for i: x[i] /= sum;
// The max is order-independent and exact.  Softmax owes the reference 1e-5
// relative, not its bits, so each exponential of d = x - max in [-80, 0] is
// exp_m80_0 (2^(d*log2 e) from ex2.approx with the product's rounding error
// restored, ~2^-22 relative); a float4 with any d below -80 takes the
// libm-identical expf, so subnormal results and the reference's underflow (a
// row entirely below -104 is 0/0 = NaN) are reproduced.  Each float4's four
// exponentials are added in binary32 (at most 4*U of them per thread and
// step) and the partial sums accumulated in binary64 (per thread, then a
// fixed tree): closer to the exact sum than the reference's sequential
// binary32 sum, and deterministic.  The tests bound the
// outputs (1e-5 rel / 1e-6 abs of a binary64 softmax, and no further from the
// oracle than the oracle is from it).
//
// One launch for every row length.  A persistent CTA per SM streams whole rows
// through a 220 KB shared-memory ring, so HBM sees each score read once and
// written once, with up to the whole ring in flight per SM:
//
//   producer warp   takes units of `unit` consecutive rows from a device
//                   counter (dynamic balance across SMs) and cuts them into
//                   batches: one long row (> SMX_WMAX scores), or a run of
//                   short rows of at most 48 KB.  For each batch it reserves
//                   ring space and row descriptors in order, fills the
//                   descriptors (offset, length, ring position, the up-to-six
//                   scalars outside the row's 16-byte-aligned body) and bulk-
//                   copies the bodies (cp.async.bulk, completing on the batch's
//                   mbarrier);
//   15 consumer     walk the batches in order.  A short row belongs to one warp
//   warps           (round-robin); a long row is shared by all 15, whose two
//                   reductions meet on mbarriers (bounded waits, no unbounded
//                   bar.sync).  A row too long for the ring is read from and
//                   written to global memory in three passes.  Max, then exp
//                   written back over the staged scores with the sum, then the
//                   scaled scores stored straight to HBM.  Every warp arrives
//                   once per batch on its `empty` barrier.
//
// Batches are reclaimed in order (the producer waits for the oldest batch's
// release), so a batch's ring bytes and descriptors are reused only after all
// 15 warps are done with it; the parity waits stay exact because every
// consumer warp waits on every batch in sequence.  The counter pair {next unit,
// finished CTAs} is reset by the last CTA to finish, so it is zero for the next
// launch on that pair.
#include "q3cu_internal.h"

namespace q3 {

constexpr int SMX_CW = 15;                       // consumer warps (16 warps in all: 128 registers each)
constexpr int SMX_CT = SMX_CW * 32;              // consumer threads
constexpr int SMX_THREADS = SMX_CT + 32;         // + the producer warp
constexpr int SMX_NB = 16;                       // batch slots per CTA
constexpr int SMX_NDESC = 128;                   // row descriptors per CTA
constexpr uint32_t SMX_RING = 220u * 1024u;      // ring bytes: rows of up to 56320 scores are staged
constexpr uint32_t SMX_BATCH16 = 3072;           // a batch of short rows holds at most 48 KB (in float4)
constexpr int SMX_WMAX = 4096;                   // rows up to this length: one warp
constexpr int SMX_UNIT_MAX = 32;                 // rows per unit taken from the counter (lanes of the producer)

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

struct SmxDesc {
    int64_t off;      // first score of the row in x
    int32_t len;
    int32_t sidx;     // float4 index of the staged body in the ring; -1: not staged (global)
    int32_t nb;       // float4 body count
    int16_t a, tl;    // leading / trailing scalar counts (<= 3 each)
    float sc[6];      // sc[0..a) leading scalars, sc[3..3+tl) trailing scalars
};
static_assert(sizeof(SmxDesc) == 48, "descriptor layout");

// A batch: one long row (all consumer warps), or a run of short rows (one
// warp each), or the end of the sequence.
enum : uint16_t { SMX_SHORT = 0, SMX_LONG = 1, SMX_END = 2 };
struct SmxBatch {
    uint32_t d0;      // first descriptor (monotonic; slot d0 % SMX_NDESC)
    uint16_t n;       // rows
    uint16_t kind;
};

// exp(v - m) of four scores: exp_m80_0 when every d = v - m is in [-80, 0]
// (RN(min v - m) is the smallest d; NaN scores are skipped by the min and come
// out NaN).  Returns false otherwise (a score far below the max, or -inf), and
// the caller recomputes the four with smx_exp4_exact (the libm-identical expf
// below -80), a branch that is cold in practice and kept out of the hot loop's
// register allocation.
__device__ __forceinline__ bool smx_exp4(float4 &v, float m) {
    const bool ok = __fsub_rn(fminf(fminf(v.x, v.y), fminf(v.z, v.w)), m) >= -80.0f;
    const f2 mm = pk2(m, m);
    up2(exp2_m80_0(sub2(pk2(v.x, v.y), mm)), v.x, v.y);
    up2(exp2_m80_0(sub2(pk2(v.z, v.w), mm)), v.z, v.w);
    return ok;
}
static __device__ __noinline__ float smx_exp_slow(float d, const ExpTab *tab) { return expf_host(d, *tab); }
__device__ __forceinline__ float smx_exp1(float d, const ExpTab &tab) {
    return d >= -80.0f ? exp_m80_0(d) : smx_exp_slow(d, &tab);
}
__device__ __forceinline__ float4 smx_exp4_exact(float4 v, float m, const ExpTab &tab) {
    return make_float4(smx_exp1(__fsub_rn(v.x, m), tab), smx_exp1(__fsub_rn(v.y, m), tab),
                       smx_exp1(__fsub_rn(v.z, m), tab), smx_exp1(__fsub_rn(v.w, m), tab));
}

__device__ __forceinline__ float max4(float m, float4 v) {
    return fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
}
__device__ __forceinline__ float4 scale4(float4 v, float inv) {      // packed f32x2 products
    const f2 s = pk2(inv, inv);
    float4 r;
    up2(mul2(pk2(v.x, v.y), s), r.x, r.y);
    up2(mul2(pk2(v.z, v.w), s), r.z, r.w);
    return r;
}
// Orders this thread's earlier generic-proxy shared-memory writes before the
// bulk copies the producer issues into the same bytes after the release.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One row by NT threads (t = 0..NT-1): a warp (NT = 32) or the 15 consumer
// warps (NT = 480, reductions on the two mbarriers of `red`).  Returns false
// if a reduction wait gave up (status recorded).
template <int NT, int U, bool STAGED>
__device__ __forceinline__ bool smx_row(float *x, float4 *ring, const SmxDesc &d, int t, const ExpTab &tab,
                                        uint64_t *red, uint32_t red_par, float *red_f, double *red_d,
                                        uint32_t *status) {
    const int lane = t & 31, w = t >> 5;
    float *row = x + d.off;
    const int a = d.a, tl = d.tl, nb = d.nb;
    float4 *sb = STAGED ? ring + d.sidx : nullptr;
    float4 *gb = reinterpret_cast<float4 *>(row + a);
    // scalar handled by thread t: head t (t < a) or tail t - a
    const int si = t < a ? t : (t - a < tl ? 3 + (t - a) : -1);
    const int64_t spos = t < a ? t : a + 4 * int64_t(nb) + (t - a);

    // Each pass moves U float4 per thread per step: all U loads are issued
    // before their uses (the asm loads and stores are ordered).
    auto load4 = [&](int j0, float4 *v) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u * NT;
            if (j < nb) v[u] = STAGED ? sb[j] : u4_as_f4(ld_v4(gb + j));
        }
    };
    float m = 0.0f;                               // the reference's max starts at 0
    for (int j0 = t; j0 < nb; j0 += U * NT) {
        float4 v[U];
        load4(j0, v);
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (j0 + u * NT < nb) m = max4(m, v[u]);
    }
    float xs = 0.0f;
    if (si >= 0) { xs = d.sc[si]; m = fmaxf(m, xs); }
    m = warp_max(m);
    if constexpr (NT > 32) {
        if (lane == 0) red_f[w] = m;
        __syncwarp();
        if (lane == 0) mbar_arrive(&red[0]);
        if (!__all_sync(FULL, mbar_wait(&red[0], red_par, lane == 0 ? status : nullptr))) return false;
        m = warp_max(lane < NT / 32 ? red_f[lane] : 0.0f);
    }

    double s = 0.0;
    for (int j0 = t; j0 < nb; j0 += U * NT) {
        float4 v[U];
        load4(j0, v);
        float4 e[U];
        bool ok = true;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            e[u] = v[u];
            if (j0 + u * NT < nb) ok &= smx_exp4(e[u], m);
        }
        if (__builtin_expect(!ok, 0)) {
#pragma unroll
            for (int u = 0; u < U; ++u) e[u] = smx_exp4_exact(v[u], m, tab);
        }
        f2 part = pk2(0.0f, 0.0f);                    // this step's exponentials, binary32 pairs
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u * NT;
            if (j < nb) {
                if constexpr (STAGED) sb[j] = e[u];
                else *reinterpret_cast<uint4 *>(gb + j) = f4_as_u4(e[u]);
                part = add2(part, add2(pk2(e[u].x, e[u].y), pk2(e[u].z, e[u].w)));
            }
        }
        float p0, p1;
        up2(part, p0, p1);
        s += double(__fadd_rn(p0, p1));
    }
    if (si >= 0) { xs = smx_exp1(__fsub_rn(xs, m), tab); s += double(xs); }
    s = warp_sum_d(s);
    if constexpr (NT > 32) {
        if (lane == 0) red_d[w] = s;
        __syncwarp();
        if (lane == 0) mbar_arrive(&red[1]);
        if (!__all_sync(FULL, mbar_wait(&red[1], red_par, lane == 0 ? status : nullptr))) return false;
        s = warp_sum_d(lane < NT / 32 ? red_d[lane] : 0.0);
    }
    const float inv = float(1.0 / s);

    for (int j0 = t; j0 < nb; j0 += U * NT) {
        float4 v[U];
        load4(j0, v);
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (j0 + u * NT < nb) st_cs_v4(gb + j0 + u * NT, f4_as_u4(scale4(v[u], inv)));
    }
    if (si >= 0) row[spos] = __fmul_rn(xs, inv);
    return true;
}

__global__ void __launch_bounds__(SMX_THREADS, 1)
softmax_ring_kernel(float *x, const int64_t *__restrict__ offs, const int32_t *__restrict__ lens, int64_t rows,
                    int unit, uint32_t *sched, uint32_t *status) {
    extern __shared__ __align__(128) float4 ring[];
    __shared__ ExpTab s_tab;
    __shared__ __align__(8) uint64_t full[SMX_NB], empty[SMX_NB], red[2];
    __shared__ SmxBatch hdr[SMX_NB];
    __shared__ uint32_t s_end[SMX_NB], s_dend[SMX_NB];   // ring (float4) and descriptor ends of each batch
    __shared__ SmxDesc desc[SMX_NDESC];
    __shared__ float red_f[SMX_CW];
    __shared__ double red_d[SMX_CW];
    __shared__ int fail_sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    load_exp_table(s_tab);
    if (tid == 0) {
        for (int i = 0; i < SMX_NB; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], SMX_CW);
        }
        mbar_init(&red[0], SMX_CW);
        mbar_init(&red[1], SMX_CW);
        fail_sh = 0;
        mbar_init_fence();
    }
    __syncthreads();

    // ---- producer warp -----------------------------------------------------
    // Ring positions count 16-byte units (float4): `alloc` (monotonic) is the
    // end of the newest batch's bytes, `head` its offset in the ring, `freed`
    // the end of the newest reclaimed batch; [freed, alloc) spans every live
    // byte (plus a tail skipped when a batch would cross the ring's end).
    // Descriptors likewise ([dfreed, dalloc)).  Batches are reclaimed in
    // sequence order.  A batch is the first pending row of the unit if it is
    // long, else the run of short rows that follows it: an exclusive scan of
    // their sizes places every row that fits (slot, descriptor and ring space
    // free, no crossing, at most SMX_BATCH16 after the first) and those lanes
    // write their descriptors and issue their copies together.
    if (warp == SMX_CW) {
        constexpr uint32_t R16 = SMX_RING / 16u;
        const uint64_t units = (uint64_t(rows) + unit - 1) / unit;
        const uint32_t lt = (1u << lane) - 1u;       // lanes below this one
        uint32_t alloc = 0, head = 0, freed = 0, dalloc = 0, dfreed = 0;
        uint32_t k = 0, oldest = 0;                   // next batch; oldest not yet reclaimed
        bool ok = true;
        auto take = [&]() {
            freed = s_end[oldest % SMX_NB];
            dfreed = s_dend[oldest % SMX_NB];
            ++oldest;
        };
        auto reclaim_ready = [&]() {                  // every released batch, without waiting (warp-uniform)
            while (oldest != k && __all_sync(FULL, mbar_test_wait(&empty[oldest % SMX_NB], (oldest / SMX_NB) & 1u)))
                take();
            if (oldest == k) freed = alloc;           // nothing live: a skipped tail is free too
        };
        auto reclaim_one = [&]() -> bool {            // the oldest batch, bounded wait
            if (__any_sync(FULL, fail_sh != 0)) return false;
            if (!__all_sync(FULL, mbar_wait(&empty[oldest % SMX_NB], (oldest / SMX_NB) & 1u,
                                            lane == 0 ? status : nullptr)))
                return false;
            take();
            return true;
        };
        uint8_t *ring_b = reinterpret_cast<uint8_t *>(ring);

        uint32_t cur = 0;
        if (lane == 0) cur = atomicAdd(&sched[0], 1u);
        cur = __shfl_sync(FULL, cur, 0);
        int len = 0;
        int64_t off = 0;
        auto load_unit = [&](uint32_t b) {
            const int64_t r = int64_t(b) * unit + lane;
            const bool valid = b < units && lane < unit && r < rows;
            len = valid ? __ldg(lens + r) : 0;
            off = valid ? __ldg(offs + r) : 0;
        };
        load_unit(cur);
        while (ok && cur < units) {
            uint32_t nxt = 0;
            if (lane == 0) nxt = atomicAdd(&sched[0], 1u);      // the next unit, in flight meanwhile
            float *row = x + off;
            RowSplit sp{0, 0, 0};
            if (len > 0) sp = split_row(row, len);
            const bool is_long = len > SMX_WMAX;
            const bool staged = len > 0 && (!is_long || uint32_t(sp.nb) <= R16);
            const uint32_t b16 = staged ? uint32_t(sp.nb) : 0u;
            float sc[6];
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                sc[i] = i < sp.a ? row[i] : 0.0f;
                sc[3 + i] = i < sp.tl ? row[sp.a + 4 * int64_t(sp.nb) + i] : 0.0f;
            }
            const int my_len = len;
            const int64_t my_off = off;
            cur = __shfl_sync(FULL, nxt, 0);
            load_unit(cur);                           // the next unit's lengths and offsets, in flight meanwhile

            uint32_t pend = __ballot_sync(FULL, my_len > 0);
            const uint32_t longs = __ballot_sync(FULL, my_len > 0 && is_long);
            while (pend) {
                reclaim_ready();
                const int f = __ffs(pend) - 1;
                uint32_t cand;
                if ((longs >> f) & 1u) {
                    cand = 1u << f;
                } else {
                    const uint32_t lb = longs & pend;             // long rows after f end the run
                    cand = lb ? pend & ((1u << (__ffs(lb) - 1)) - 1u) : pend;
                }
                const bool in_c = (cand >> lane) & 1u;
                uint32_t incl = in_c ? b16 : 0u;                  // inclusive scan, lane order
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t v = __shfl_up_sync(FULL, incl, o);
                    if (lane >= o) incl += v;
                }
                const uint32_t rank = __popc(cand & lt);
                const bool fits = k < oldest + SMX_NB && head + incl <= R16 && alloc + incl - freed <= R16 &&
                                  (rank == 0 || incl <= SMX_BATCH16) && dalloc + rank + 1 - dfreed <= SMX_NDESC;
                const uint32_t bad = __ballot_sync(FULL, in_c && !fits);
                const uint32_t go = bad ? cand & ((1u << (__ffs(bad) - 1)) - 1u) : cand;
                if (go) {
                    const int n = __popc(go);
                    const uint32_t used = __shfl_sync(FULL, incl, 31 - __clz(go));
                    const uint32_t sl = k % SMX_NB;
                    const bool mine = (go >> lane) & 1u;
                    const uint32_t at = head + incl - b16;        // float4 index in the ring
                    if (mine) {
                        SmxDesc &d = desc[(dalloc + rank) % SMX_NDESC];
                        d.off = my_off;
                        d.len = my_len;
                        d.sidx = staged ? int32_t(at) : -1;
                        d.nb = sp.nb;
                        d.a = int16_t(sp.a);
                        d.tl = int16_t(sp.tl);
#pragma unroll
                        for (int i = 0; i < 6; ++i) d.sc[i] = sc[i];
                    }
                    if (lane == 0) {
                        hdr[sl].d0 = dalloc;
                        hdr[sl].n = uint16_t(n);
                        hdr[sl].kind = ((longs >> f) & 1u) ? SMX_LONG : SMX_SHORT;
                        s_end[sl] = alloc + used;
                        s_dend[sl] = dalloc + uint32_t(n);
                        if (used) mbar_expect_tx(&full[sl], used * 16u);
                    }
                    __syncwarp();
                    if (mine && b16) bulk_g2s(ring_b + size_t(at) * 16u, row + sp.a, b16 * 16u, &full[sl]);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[sl]);        // descriptors and header published
                    ++k;
                    alloc += used;
                    head += used;
                    if (head == R16) head = 0;
                    dalloc += uint32_t(n);
                    pend &= ~go;
                    continue;
                }
                // The first row of the batch does not fit.
                const uint32_t bf = __shfl_sync(FULL, b16, f);
                if (head + bf > R16) {                // skip the ring's tail
                    alloc += R16 - head;
                    head = 0;
                    continue;
                }
                if (oldest == k) {                    // cannot happen: nothing is live and the row fits
                    if (lane == 0) atomicOr(status, Q3CU_DEV_TIMEOUT);
                    ok = false;
                    break;
                }
                if (!reclaim_one()) { ok = false; break; }
            }
        }
        if (ok) {                                     // end of the sequence
            while (k >= oldest + SMX_NB)
                if (!reclaim_one()) { ok = false; break; }
            if (ok) {
                if (lane == 0) {
                    hdr[k % SMX_NB].kind = SMX_END;
                    hdr[k % SMX_NB].n = 0;
                    mbar_arrive(&full[k % SMX_NB]);
                }
                ++k;
            }
        }
        if (!ok) {
            // After a failure, no copy may still be landing when the CTA exits:
            // bounded wait for every batch not yet reclaimed.
            if (lane == 0)
                for (uint32_t q = oldest; q < k; ++q)
                    mbar_wait(&full[q % SMX_NB], (q / SMX_NB) & 1u, nullptr);
        }
        // The last CTA to finish resets the counter pair for the next launch.
        if (lane == 0) {
            __threadfence();
            if (atomicAdd(&sched[1], 1u) == gridDim.x - 1) {
                sched[0] = 0;
                sched[1] = 0;
                __threadfence();
            }
        }
        return;
    }

    // ---- consumer warps ----------------------------------------------------
    // Every warp waits on every batch in order and arrives once on its
    // `empty` barrier.  Short rows: row i of a batch goes to warp
    // (rot + i) % SMX_CW, rot counting the short rows of earlier batches.
    uint32_t rot = 0, cc = 0;
    for (uint32_t k = 0;; ++k) {
        const int s = int(k % SMX_NB);
        if (__any_sync(FULL, fail_sh != 0)) break;
        if (!__all_sync(FULL, mbar_wait(&full[s], (k / SMX_NB) & 1u, lane == 0 ? status : nullptr))) {
            fail_sh = 1;
            break;
        }
        const SmxBatch h = hdr[s];
        if (h.kind == SMX_END) break;
        bool ok = true, wrote = false;
        if (h.kind == SMX_LONG) {
            const SmxDesc &d = desc[h.d0 % SMX_NDESC];
            ok = d.sidx >= 0 ? smx_row<SMX_CT, 2, true>(x, ring, d, tid, s_tab, red, cc & 1u, red_f, red_d, status)
                             : smx_row<SMX_CT, 1, false>(x, ring, d, tid, s_tab, red, cc & 1u, red_f, red_d, status);
            ++cc;
            wrote = true;
        } else {
            for (int i = (warp + SMX_CW - int(rot % SMX_CW)) % SMX_CW; i < h.n; i += SMX_CW) {
                smx_row<32, 4, true>(x, ring, desc[(h.d0 + i) % SMX_NDESC], lane, s_tab, nullptr, 0, nullptr, nullptr,
                                     status);
                wrote = true;
            }
            rot += h.n;
        }
        if (wrote) fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (!ok) {
            fail_sh = 1;
            break;
        }
    }
}

// ---- few rows (a decode token's heads) -------------------------------------
// One CTA of SMS_THREADS per row, no ring: a row of at most SMS_THREADS * 16
// scores is held in registers (one read, one write); a longer row takes three
// passes over global memory (max; exponentials in place + sum; scale).  Same
// arithmetic as the ring kernel: max from 0, exp_m80_0 with the exact expf
// below -80, binary32 float4 partials summed in binary64 over a fixed tree.
constexpr int SMS_THREADS = 256;
constexpr int SMS_REG = 4;                       // float4 per thread held in registers

__device__ __forceinline__ float sms_block_max(float v, float *sh) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();                              // sh free from the previous reduction
    if (lane == 0) sh[w] = v;
    __syncthreads();
    return warp_max(lane < SMS_THREADS / 32 ? sh[lane] : 0.0f);
}
__device__ __forceinline__ double sms_block_sum(double v, double *sh) {
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    return warp_sum_d(lane < SMS_THREADS / 32 ? sh[lane] : 0.0);
}

__global__ void __launch_bounds__(SMS_THREADS) softmax_small_kernel(float *x, const int64_t *__restrict__ offs,
                                                                    const int32_t *__restrict__ lens) {
    __shared__ ExpTab s_tab;
    __shared__ float sh_f[SMS_THREADS / 32];
    __shared__ double sh_d[SMS_THREADS / 32];
    load_exp_table(s_tab);
    const int t = threadIdx.x;
    const int len = __ldg(lens + blockIdx.x);
    float *row = x + __ldg(offs + blockIdx.x);
    __syncthreads();
    if (len <= 0) return;                         // block-uniform
    const RowSplit sp = split_row(row, len);
    float4 *gb = reinterpret_cast<float4 *>(row + sp.a);
    const int si = t < sp.a ? t : (t - sp.a < sp.tl ? sp.a + 4 * sp.nb + (t - sp.a) : -1);
    float xs = si >= 0 ? row[si] : 0.0f;
    if (sp.nb <= SMS_THREADS * SMS_REG) {
        float4 v[SMS_REG];
        float m = 0.0f;                           // the reference's max starts at 0
#pragma unroll
        for (int u = 0; u < SMS_REG; ++u) {
            const int j = t + u * SMS_THREADS;
            if (j < sp.nb) { v[u] = u4_as_f4(ld_v4(gb + j)); m = max4(m, v[u]); }
        }
        if (si >= 0) m = fmaxf(m, xs);
        m = sms_block_max(m, sh_f);
        double s = 0.0;
        f2 part = pk2(0.0f, 0.0f);
#pragma unroll
        for (int u = 0; u < SMS_REG; ++u) {
            if (t + u * SMS_THREADS < sp.nb) {
                const float4 v0 = v[u];
                if (!smx_exp4(v[u], m)) v[u] = smx_exp4_exact(v0, m, s_tab);
                part = add2(part, add2(pk2(v[u].x, v[u].y), pk2(v[u].z, v[u].w)));
            }
        }
        float p0, p1;
        up2(part, p0, p1);
        s = double(__fadd_rn(p0, p1));
        if (si >= 0) { xs = smx_exp1(__fsub_rn(xs, m), s_tab); s += double(xs); }
        const float inv = float(1.0 / sms_block_sum(s, sh_d));
#pragma unroll
        for (int u = 0; u < SMS_REG; ++u) {
            const int j = t + u * SMS_THREADS;
            if (j < sp.nb) st_cs_v4(gb + j, f4_as_u4(scale4(v[u], inv)));
        }
        if (si >= 0) row[si] = __fmul_rn(xs, inv);
        return;
    }
    float m = 0.0f;
    for (int j = t; j < sp.nb; j += SMS_THREADS) m = max4(m, u4_as_f4(ld_v4(gb + j)));
    if (si >= 0) m = fmaxf(m, xs);
    m = sms_block_max(m, sh_f);
    double s = 0.0;
    for (int j = t; j < sp.nb; j += SMS_THREADS) {
        float4 v = u4_as_f4(ld_v4(gb + j));
        const float4 v0 = v;
        if (!smx_exp4(v, m)) v = smx_exp4_exact(v0, m, s_tab);
        *reinterpret_cast<uint4 *>(gb + j) = f4_as_u4(v);
        s += double(__fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w)));
    }
    if (si >= 0) { xs = smx_exp1(__fsub_rn(xs, m), s_tab); s += double(xs); }
    const float inv = float(1.0 / sms_block_sum(s, sh_d));
    for (int j = t; j < sp.nb; j += SMS_THREADS)
        st_cs_v4(gb + j, f4_as_u4(scale4(u4_as_f4(ld_v4(gb + j)), inv)));
    if (si >= 0) row[si] = __fmul_rn(xs, inv);
}

constexpr int SMX_SMEM_SLOT = 8;

cudaError_t launch_softmax_rows(float *x, const int64_t *off, const int32_t *len, int64_t rows, uint32_t *sched,
                                uint32_t *status, cudaStream_t stream, int sms) {
    if (rows <= 0) return cudaSuccess;
    if (rows <= int64_t(sms) * 2) {               // a decode token's heads: one CTA per row
        softmax_small_kernel<<<unsigned(rows), SMS_THREADS, 0, stream>>>(x, off, len);
        return cudaGetLastError();
    }
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(softmax_ring_kernel), SMX_RING, SMX_SMEM_SLOT);
    if (e != cudaSuccess) return e;
    // Units small enough that every SM takes about 16 of them (balance), at
    // most one row per producer lane.
    int64_t unit = rows / (int64_t(sms) * 16);
    unit = unit < 1 ? 1 : (unit > SMX_UNIT_MAX ? SMX_UNIT_MAX : unit);
    const int64_t units = (rows + unit - 1) / unit;
    if (units > int64_t(0x7fffffff)) return cudaErrorInvalidValue;     // the unit counter is 32-bit
    const unsigned grid = unsigned(units < sms ? units : sms);
    softmax_ring_kernel<<<grid, SMX_THREADS, SMX_RING, stream>>>(x, off, len, rows, int(unit), sched, status);
    return cudaGetLastError();
}

}  // namespace q3
