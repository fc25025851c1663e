// k_rope.cu -- per-head QK-RMSNorm followed by rotate-half RoPE, in place.
//
// Reference: src/cpu/qwen3_original.c:361-393.  For every query head (n_heads)
// and key head (n_kv_heads) of a token at position pos:
//     rmsnorm(v, v, norm_w, hd)                       (:365, :382; :278-289)
//     for j < hd/2: freq = powf(1e6, -(float)j/(hd/2))  (:367, :384)
//                   c = cosf(pos*freq), s = sinf(pos*freq)
//                   (x, y) = (v[j], v[j+hd/2])
//                   v[j] = x*c - y*s;  v[j+hd/2] = x*s + y*c
//
// q [T][n_heads][128] and k [T][n_kv][128] are flat lists of 128-element head
// rows.  A warp owns a tile of 32 consecutive head rows of one tensor, one row
// per lane:
//   * a copy warp per CTA copies every compute warp's tiles (one contiguous
//     16 KB / 8 KB range each) with one bulk copy per tile (cp.async.bulk,
//     completing on the buffer's mbarrier); two buffers per compute warp with
//     full/empty mbarriers (bounded waits), so the next tile streams in while
//     this one is processed.  Bulk copies are not held to the ~50 KB of
//     16-byte cp.async an SM keeps in flight, which capped the earlier
//     per-piece copies near 25 GB/s per SM.  The tile lands dense; the compute
//     warp then moves it in place into 32 padded row slots (coalesced 16-byte
//     reads, conflict-free 16-byte writes; the back half of the rows first,
//     so no row is overwritten before it is read);
//   * lane i runs row i's sum of squares in index order (the reference's
//     rounding sequence, so the normalised values are bit-exact);
//   * the warp fills a table with cos/sin of every token the tile touches
//     (two sincosf per lane per token), then lane i normalises and rotates
//     its own row in place: 64 independent pairs per lane, 16-byte shared
//     memory accesses (the row padding puts the 32 lanes on different banks;
//     table and weight reads are broadcasts);
//   * the warp writes the tile back to HBM with coalesced 16-byte stores.
// freq_j comes from the host (the C library's powf, the reference's own
// call); the angle pos*freq_j is the same binary32 product; cos/sin are CUDA's
// sincosf (a few ulp from the host's cosf/sinf, inside the 1e-5 tolerance).
#include "q3cu_internal.h"

namespace q3 {

constexpr int HD = 128;
constexpr int ROPE_TILE = 32;                    // head rows per warp tile (one per lane)
constexpr int ROPE_TOKS = 8;                     // tokens in a warp's cos/sin table (32 rows / 4 heads)
constexpr int ROPE_TABB = 2 * (HD / 2) * 4 + 16; // one token: cos[64], sin[64], padding
template <typename T> __host__ __device__ constexpr int rope_rowb() { return HD * int(sizeof(T)) + 16; }
template <typename T> __host__ __device__ constexpr int rope_warp_bytes() {
    return 2 * ROPE_TILE * rope_rowb<T>() + ROPE_TOKS * ROPE_TABB;
}
// Warps per CTA (one CTA per SM): 6 x 38,016 B (f32), 10 x 21,632 B (bf16).
template <typename T> __host__ __device__ constexpr int rope_warps() { return sizeof(T) == 4 ? 6 : 10; }

// Normalises and rotates one head row in place (lane-private).  Same operation
// order as the reference: x' = w_lo*(ss*x), y' = w_hi*(ss*y),
// x'' = x'c - y's, y'' = x's + y'c, each product and sum rounded once.
template <typename T>
__device__ __forceinline__ void rotate_row(uint8_t *row, const float *w, const float *cs, float ss) {
    constexpr int P = Vec<T>::N;                 // pairs per 16-byte access (4 f32, 8 bf16)
    constexpr int ESZ = sizeof(T);
    const f2 ss2 = pk2(ss, ss);
#pragma unroll 2
    for (int j = 0; j < HD / 2; j += P) {
        uint4 *px = reinterpret_cast<uint4 *>(row + j * ESZ);
        uint4 *py = reinterpret_cast<uint4 *>(row + (HD / 2 + j) * ESZ);
        float x[P], y[P], wl[P], wh[P], c[P], s[P], a[P], b[P];
        Vec<T>::widen(*px, x);
        Vec<T>::widen(*py, y);
#pragma unroll
        for (int i = 0; i < P; i += 4) {
            Vec<float>::widen(*reinterpret_cast<const uint4 *>(w + j + i), wl + i);
            Vec<float>::widen(*reinterpret_cast<const uint4 *>(w + HD / 2 + j + i), wh + i);
            Vec<float>::widen(*reinterpret_cast<const uint4 *>(cs + j + i), c + i);
            Vec<float>::widen(*reinterpret_cast<const uint4 *>(cs + HD / 2 + j + i), s + i);
        }
#pragma unroll
        for (int i = 0; i < P; i += 2) {
            const f2 xn = mul2(pk2(wl[i], wl[i + 1]), mul2(ss2, pk2(x[i], x[i + 1])));
            const f2 yn = mul2(pk2(wh[i], wh[i + 1]), mul2(ss2, pk2(y[i], y[i + 1])));
            const f2 c2 = pk2(c[i], c[i + 1]), s2 = pk2(s[i], s[i + 1]);
            up2(sub2(mul2(xn, c2), mul2(yn, s2)), a[i], a[i + 1]);
            up2(add2(mul2(xn, s2), mul2(yn, c2)), b[i], b[i + 1]);
        }
        *px = Vec<T>::narrow(a);
        *py = Vec<T>::narrow(b);
    }
}

template <typename T>
__global__ void __launch_bounds__((rope_warps<T>() + 1) * 32, 1) qk_norm_rope_kernel(
    T *q, T *k, const int32_t *__restrict__ pos, int64_t q_rows, int64_t k_rows, int n_heads, int n_kv,
    const float *__restrict__ q_norm, const float *__restrict__ k_norm, InvFreq invf, float eps, uint32_t *status) {
    constexpr int ESZ = sizeof(T);
    constexpr int RW = rope_warps<T>();
    constexpr int ROWBYTES = HD * ESZ;
    constexpr int ROWB = rope_rowb<T>();                // padded: lane-per-row accesses hit distinct banks
    constexpr int CPR = ROWBYTES / 16;                  // 16-byte chunks per row (32 / 16)
    constexpr int V = Vec<T>::N;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(16) float wsh[2][HD];          // q_norm, k_norm
    __shared__ __align__(8) uint64_t full[RW][2];       // a compute warp's buffer holds its next tile
    __shared__ __align__(8) uint64_t empty[RW][2];      // ... and was written back
    __shared__ int fail_sh;

    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int w = 0; w < RW; ++w)
            for (int b = 0; b < 2; ++b) {
                mbar_init(&full[w][b], 1);
                mbar_init(&empty[w][b], 1);
            }
        fail_sh = 0;
        mbar_init_fence();
    }
    __syncthreads();
    griddep_launch_dependents();                  // a dependent-launched successor may start its own prologue
    griddep_wait();                               // q / k from the kernel before (a dependent launch)

    const int64_t q_tiles = (q_rows + ROPE_TILE - 1) / ROPE_TILE;
    const int64_t k_tiles = (k_rows + ROPE_TILE - 1) / ROPE_TILE;
    const int64_t ntiles = q_tiles + k_tiles;
    const int64_t GW = int64_t(gridDim.x) * RW;

    // per-lane frequencies for j = 2*lane, 2*lane+1
    const float f0 = invf.v[2 * lane], f1 = invf.v[2 * lane + 1];

    auto tile_info = [&](int64_t t, T *&base, int64_t &row0, int &nvalid, int &heads) {
        const bool isq = t < q_tiles;
        base = isq ? q : k;
        row0 = (isq ? t : t - q_tiles) * ROPE_TILE;
        const int64_t left = (isq ? q_rows : k_rows) - row0;
        nvalid = left < ROPE_TILE ? int(left) : ROPE_TILE;
        heads = isq ? n_heads : n_kv;
    };
    // Compute warp w's tiles are t = blockIdx.x * RW + w + kk * GW, kk = 0, 1, ...,
    // in buffer kk & 1.  The copy warp (wid == RW) copies them all, in kk order,
    // one bulk copy per tile into the start of the buffer (the expect-tx
    // arrival is the buffer's one arrival); the compute warp releases the
    // buffer on `empty` after its write-back.
    if (wid == RW) {
        int64_t last[RW];                       // the last round whose tile was copied, per compute warp
#pragma unroll
        for (int w = 0; w < RW; ++w) last[w] = -1;
        bool ok = true;
        for (int64_t kk = 0; ok; ++kk) {
            bool any = false;
            for (int w = 0; w < RW && ok; ++w) {
                const int64_t t = int64_t(blockIdx.x) * RW + w + kk * GW;
                if (t >= ntiles) continue;
                any = true;
                const int b = int(kk & 1);
                if (kk >= 2 && !__all_sync(FULL, mbar_wait(&empty[w][b], uint32_t(((kk >> 1) - 1) & 1),
                                                           lane == 0 ? status : nullptr))) {
                    ok = false;
                    break;
                }
                T *base; int64_t row0; int nvalid, heads;
                tile_info(t, base, row0, nvalid, heads);
                if (lane == 0) {
                    const uint32_t bytes = uint32_t(nvalid) * ROWBYTES;
                    mbar_arrive_expect_tx(&full[w][b], bytes);
                    bulk_g2s(smem + size_t(w) * rope_warp_bytes<T>() + size_t(b) * ROPE_TILE * ROWB,
                             base + row0 * HD, bytes, &full[w][b]);
                }
                __syncwarp();
                last[w] = kk;
            }
            if (!any || !ok || __any_sync(FULL, fail_sh != 0)) break;
        }
        // No copy may still be landing when the CTA exits.  Normally every compute
        // warp has waited for all of its tiles; after a failure, wait (bounded) for
        // the latest copy into each buffer.
        if (lane == 0)
#pragma unroll
            for (int w = 0; w < RW; ++w)
                for (int64_t kk = last[w] > 0 ? last[w] - 1 : 0; kk <= last[w]; ++kk)
                    mbar_wait(&full[w][int(kk & 1)], uint32_t((kk >> 1) & 1), nullptr);
        return;
    }

    // The compute warps load the norm weights while the copy warp starts.
    for (int i = threadIdx.x; i < HD; i += RW * 32) {
        wsh[0][i] = q_norm[i];
        wsh[1][i] = k_norm[i];
    }
    named_sync(1, RW * 32);
    uint8_t *buf0 = smem + size_t(wid) * rope_warp_bytes<T>();
    uint8_t *tab = buf0 + 2 * ROPE_TILE * ROWB;
    for (int64_t kk = 0;; ++kk) {
        const int64_t t = int64_t(blockIdx.x) * RW + wid + kk * GW;
        if (t >= ntiles) break;
        const int b = int(kk & 1);
        // positions of the tile's tokens (lane l: token tok0 + l), loaded while the tile lands
        int pv = 0;
        {
            T *pb; int64_t pr0; int pnv, phe;
            tile_info(t, pb, pr0, pnv, phe);
            const int64_t ptok0 = pr0 / phe;
            if (lane <= int((pr0 + pnv - 1) / phe - ptok0)) pv = __ldg(pos + ptok0 + lane);
        }
        if (!__all_sync(FULL, mbar_wait(&full[wid][b], uint32_t((kk >> 1) & 1), lane == 0 ? status : nullptr))) {
            fail_sh = 1;
            break;
        }
        T *base; int64_t row0; int nvalid, heads;
        tile_info(t, base, row0, nvalid, heads);
        const float *w = wsh[t < q_tiles ? 0 : 1];
        uint8_t *tb = buf0 + size_t(b) * ROPE_TILE * ROWB;
        uint8_t *row = tb + size_t(lane) * ROWB;
        // dense [32][ROWBYTES] -> padded [32][ROWB], in place: rows 16..31, then 0..15
        // (a half's padded range overlaps only dense bytes of that half or of rows
        // already moved); rows past nvalid move garbage that is never used
#pragma unroll
        for (int h = 1; h >= 0; --h) {
            constexpr int NC = ROPE_TILE / 2 * CPR / 32;         // 16-byte chunks per lane per half
            uint4 v[NC];
#pragma unroll
            for (int i = 0; i < NC; ++i)
                v[i] = *reinterpret_cast<const uint4 *>(tb + size_t(h * (ROPE_TILE / 2) * CPR + i * 32 + lane) * 16);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < NC; ++i) {
                const int c = i * 32 + lane, r = h * (ROPE_TILE / 2) + c / CPR;
                *reinterpret_cast<uint4 *>(tb + size_t(r) * ROWB + (c % CPR) * 16) = v[i];
            }
            __syncwarp();
        }

        // ordered sum of squares of head row `lane`: batches of 8 16-byte vectors,
        // the next batch loaded while this one is added (two register sets
        // alternate), so the chain runs at the add latency
        float acc = 0.0f;
        if (lane < nvalid) {
            constexpr int NV = HD / V, BT = 8, NBT = NV / BT;
            const uint4 *p4 = reinterpret_cast<const uint4 *>(row);
            uint4 buf[2][BT];
#pragma unroll
            for (int j = 0; j < BT; ++j) buf[0][j] = p4[j];
#pragma unroll
            for (int bt = 0; bt < NBT; ++bt) {
                if (bt + 1 < NBT) {
#pragma unroll
                    for (int j = 0; j < BT; ++j) buf[(bt + 1) & 1][j] = p4[(bt + 1) * BT + j];
                }
#pragma unroll
                for (int j = 0; j < BT; ++j) {
                    float v[V], sq[V];
                    Vec<T>::widen(buf[bt & 1][j], v);
#pragma unroll
                    for (int i = 0; i < V; i += 2) up2(mul2(pk2(v[i], v[i + 1]), pk2(v[i], v[i + 1])), sq[i], sq[i + 1]);
#pragma unroll
                    for (int i = 0; i < V; ++i) acc = __fadd_rn(acc, sq[i]);     // in index order
                }
            }
        }
        const float ss = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, float(HD)), eps)));

        // tokens of the tile's rows, ROPE_TOKS at a time (one pass for >= 4 heads)
        const int64_t tok0 = row0 / heads;
        const int my_tok = int((row0 + lane) / heads - tok0);
        const int ntok = int((row0 + nvalid - 1) / heads - tok0) + 1;
        for (int tt0 = 0; tt0 < ntok; tt0 += ROPE_TOKS) {
            const int nt = ntok - tt0 < ROPE_TOKS ? ntok - tt0 : ROPE_TOKS;
            for (int tt = 0; tt < nt; ++tt) {
                const float p = float(__shfl_sync(FULL, pv, tt0 + tt));   // a tile spans <= 32 tokens
                float c0, s0, c1, s1;
                sincosf(__fmul_rn(p, f0), &s0, &c0);
                sincosf(__fmul_rn(p, f1), &s1, &c1);
                float *ct = reinterpret_cast<float *>(tab + tt * ROPE_TABB);
                *reinterpret_cast<float2 *>(ct + 2 * lane) = make_float2(c0, c1);
                *reinterpret_cast<float2 *>(ct + HD / 2 + 2 * lane) = make_float2(s0, s1);
            }
            __syncwarp();
            const int slot = my_tok - tt0;
            if (lane < nvalid && slot >= 0 && slot < nt)
                rotate_row<T>(row, w, reinterpret_cast<const float *>(tab + slot * ROPE_TABB), ss);
            __syncwarp();                          // table reuse / rows complete
        }
        // coalesced write-back of the tile
        uint8_t *dst = reinterpret_cast<uint8_t *>(base + row0 * HD);
        for (int c = lane; c < nvalid * CPR; c += 32)
            st_cs_v4(dst + size_t(c) * 16, *reinterpret_cast<const uint4 *>(tb + (c / CPR) * ROWB + (c % CPR) * 16));
        // this warp's shared-memory writes to buffer b are ordered before the bulk copy
        // (async proxy) that refills it; all reads of it are done
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[wid][b]);
    }
}

template <typename T>
static cudaError_t launch_rope_t(T *q, T *k, const int32_t *pos, int64_t rows, int nh, int nkv, const float *qn,
                                 const float *kn, const InvFreq &invf, float eps, uint32_t *status,
                                 cudaStream_t stream, int sms) {
    constexpr int RW = rope_warps<T>();
    constexpr size_t SMEM = size_t(RW) * rope_warp_bytes<T>();
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(qk_norm_rope_kernel<T>), SMEM,
                                     sizeof(T) == 4 ? 0 : 1);
    if (e != cudaSuccess) return e;
    const int64_t qr = rows * nh, kr = rows * nkv;
    const int64_t tiles = (qr + ROPE_TILE - 1) / ROPE_TILE + (kr + ROPE_TILE - 1) / ROPE_TILE;
    int64_t blocks = (tiles + RW - 1) / RW;                      // one CTA per SM (shared memory)
    if (blocks > sms) blocks = sms;
    return launch_dependent(qk_norm_rope_kernel<T>, dim3(unsigned(blocks)), dim3((RW + 1) * 32), SMEM, stream, q, k,
                            pos, qr, kr, nh, nkv, qn, kn, invf, eps, status);
}

cudaError_t launch_qk_norm_rope(void *q, void *k, q3cu_dtype dt, const int32_t *pos, int64_t rows, int n_heads,
                                int n_kv, const float *q_norm, const float *k_norm, const InvFreq &inv_freq,
                                float eps, uint32_t *status, cudaStream_t stream, int sms) {
    if (rows == 0) return cudaSuccess;
    if (dt == Q3CU_F32)
        return launch_rope_t<float>(static_cast<float *>(q), static_cast<float *>(k), pos, rows, n_heads, n_kv,
                                    q_norm, k_norm, inv_freq, eps, status, stream, sms);
    return launch_rope_t<bf16raw>(static_cast<bf16raw *>(q), static_cast<bf16raw *>(k), pos, rows, n_heads, n_kv,
                                  q_norm, k_norm, inv_freq, eps, status, stream, sms);
}

}  // namespace q3
