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
// rows.  A warp owns a tile of 16 consecutive head rows of one tensor:
//   * lane i bulk-copies head row i into a padded shared-memory slot (TMA,
//     one mbarrier per buffer; two buffers per warp so the next tile streams
//     in while this one is processed);
//   * lane i runs row i's sum of squares in index order (the reference's
//     rounding sequence, so the normalised values are bit-exact);
//   * then the warp walks the 16 rows: lane l rotates the pairs (2l, 2l+64)
//     and (2l+1, 2l+65), reading the row from shared memory and writing it
//     back to HBM with coalesced stores.
// freq_j comes from the host (the C library's powf, the reference's own
// call); the angle pos*freq_j is the same binary32 product; cos/sin are CUDA's
// sincosf (a few ulp from the host's cosf/sinf, inside the 1e-5 tolerance).
#include "q3cu_internal.h"

namespace q3 {

constexpr int HD = 128;
constexpr int ROPE_WARPS = 12;                   // 12 warps x 2 tiles of 16 rows: 203 KB (f32), 104 KB (bf16)
constexpr int ROPE_TILE = 16;

template <typename T>
__device__ __forceinline__ void load_pair(const uint8_t *rowp, int j, float &a, float &b) {
    if constexpr (sizeof(T) == 4) {
        const float2 v = *reinterpret_cast<const float2 *>(rowp + j * 4);
        a = v.x; b = v.y;
    } else {
        const uint32_t v = *reinterpret_cast<const uint32_t *>(rowp + j * 2);
        a = bf16_to_f32(v & 0xffffu); b = bf16_to_f32(v >> 16);
    }
}

template <typename T>
__device__ __forceinline__ void store_pair(T *p, float a, float b) {
    if constexpr (sizeof(T) == 4) {
        st_cs_v2(p, make_uint2(__float_as_uint(a), __float_as_uint(b)));
    } else {
        st_cs_u32(p, f32_to_bf16(a) | (f32_to_bf16(b) << 16));
    }
}

template <typename T>
__global__ void __launch_bounds__(ROPE_WARPS * 32) qk_norm_rope_kernel(
    T *q, T *k, const int32_t *__restrict__ pos, int64_t q_rows, int64_t k_rows, int n_heads, int n_kv,
    const float *__restrict__ q_norm, const float *__restrict__ k_norm, InvFreq invf, float eps, uint32_t *status) {
    constexpr int ESZ = sizeof(T);
    constexpr int ROWBYTES = HD * ESZ;
    constexpr int ROWB = ROWBYTES + 16;                 // padded: lanes hit distinct banks
    constexpr int V = Vec<T>::N;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[ROPE_WARPS][2];

    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    uint8_t *buf0 = smem + size_t(wid) * 2 * ROPE_TILE * ROWB;
    uint64_t *bar = bars[wid];
    if (lane == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init_fence();
    }
    __syncwarp();

    const int64_t q_tiles = (q_rows + ROPE_TILE - 1) / ROPE_TILE;
    const int64_t k_tiles = (k_rows + ROPE_TILE - 1) / ROPE_TILE;
    const int64_t ntiles = q_tiles + k_tiles;
    const int64_t gw = int64_t(blockIdx.x) * ROPE_WARPS + wid;
    const int64_t GW = int64_t(gridDim.x) * ROPE_WARPS;

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
    auto issue = [&](int64_t t, int b) {
        T *base; int64_t row0; int nvalid, heads;
        tile_info(t, base, row0, nvalid, heads);
        if (lane == 0) mbar_arrive_expect_tx(&bar[b], uint32_t(nvalid) * ROWBYTES);
        __syncwarp();
        if (lane < nvalid)
            bulk_g2s(buf0 + size_t(b) * ROPE_TILE * ROWB + size_t(lane) * ROWB,
                     reinterpret_cast<const uint8_t *>(base) + (row0 + lane) * ROWBYTES, ROWBYTES, &bar[b]);
    };

    if (gw < ntiles) issue(gw, 0);
    int64_t kk = 0;
    for (int64_t t = gw; t < ntiles; t += GW, ++kk) {
        const int b = int(kk & 1);
        const int64_t tn = t + GW;
        if (tn < ntiles) issue(tn, b ^ 1);
        const bool ok = __all_sync(FULL, mbar_wait(&bar[b], uint32_t(kk >> 1) & 1u, lane == 0 ? status : nullptr));
        if (!ok) {
            // drain the prefetch (bounded) and leave; the rows stay unmodified
            if (tn < ntiles) mbar_wait(&bar[b ^ 1], uint32_t((kk + 1) >> 1) & 1u, nullptr);
            return;
        }
        T *base; int64_t row0; int nvalid, heads;
        tile_info(t, base, row0, nvalid, heads);
        const float *nw = (t < q_tiles) ? q_norm : k_norm;
        const uint8_t *tb = buf0 + size_t(b) * ROPE_TILE * ROWB;

        // ordered sum of squares of head row `lane`
        float acc = 0.0f;
        if (lane < nvalid) {
            const uint4 *p4 = reinterpret_cast<const uint4 *>(tb + size_t(lane) * ROWB);
#pragma unroll
            for (int c = 0; c < HD / V; ++c) {
                float v[V];
                Vec<T>::widen(p4[c], v);
#pragma unroll
                for (int i = 0; i < V; ++i) acc = __fadd_rn(acc, __fmul_rn(v[i], v[i]));
            }
        }
        const float ssl = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, float(HD)), eps)));

        const float2 wlo = *reinterpret_cast<const float2 *>(nw + 2 * lane);
        const float2 whi = *reinterpret_cast<const float2 *>(nw + 64 + 2 * lane);
        // token of each head row, tracked incrementally (one division per tile)
        int64_t tok = row0 / heads;
        int hin = int(row0 - tok * heads);
        float c0 = 0.f, s0 = 0.f, c1 = 0.f, s1 = 0.f;
        for (int i = 0; i < nvalid; ++i) {
            const float ss = __shfl_sync(FULL, ssl, i);
            const int64_t hr = row0 + i;
            if (i == 0 || hin == 0) {                      // warp-uniform: a new token
                const float p = float(__ldg(pos + tok));
                sincosf(__fmul_rn(p, f0), &s0, &c0);
                sincosf(__fmul_rn(p, f1), &s1, &c1);
            }
            if (++hin == heads) { hin = 0; ++tok; }
            const uint8_t *rp = tb + size_t(i) * ROWB;
            float x0, x1, y0, y1;
            load_pair<T>(rp, 2 * lane, x0, x1);
            load_pair<T>(rp, 64 + 2 * lane, y0, y1);
            x0 = __fmul_rn(wlo.x, __fmul_rn(ss, x0));
            x1 = __fmul_rn(wlo.y, __fmul_rn(ss, x1));
            y0 = __fmul_rn(whi.x, __fmul_rn(ss, y0));
            y1 = __fmul_rn(whi.y, __fmul_rn(ss, y1));
            const float a0 = __fsub_rn(__fmul_rn(x0, c0), __fmul_rn(y0, s0));
            const float b0 = __fadd_rn(__fmul_rn(x0, s0), __fmul_rn(y0, c0));
            const float a1 = __fsub_rn(__fmul_rn(x1, c1), __fmul_rn(y1, s1));
            const float b1 = __fadd_rn(__fmul_rn(x1, s1), __fmul_rn(y1, c1));
            T *dst = base + hr * HD;
            store_pair<T>(dst + 2 * lane, a0, a1);
            store_pair<T>(dst + 64 + 2 * lane, b0, b1);
        }
        __syncwarp();          // all reads of buffer b done before it is refilled
    }
}

template <typename T>
static cudaError_t launch_rope_t(T *q, T *k, const int32_t *pos, int64_t rows, int nh, int nkv, const float *qn,
                                 const float *kn, const InvFreq &invf, float eps, uint32_t *status,
                                 cudaStream_t stream, int sms) {
    constexpr int ROWB = HD * int(sizeof(T)) + 16;
    constexpr size_t SMEM = size_t(ROPE_WARPS) * 2 * ROPE_TILE * ROWB;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(qk_norm_rope_kernel<T>), SMEM,
                                     sizeof(T) == 4 ? 0 : 1);
    if (e != cudaSuccess) return e;
    const int64_t qr = rows * nh, kr = rows * nkv;
    const int64_t tiles = (qr + ROPE_TILE - 1) / ROPE_TILE + (kr + ROPE_TILE - 1) / ROPE_TILE;
    const int per_sm = (sizeof(T) == 4) ? 1 : 2;                // CTAs that fit an SM's shared memory
    int64_t blocks = (tiles + ROPE_WARPS - 1) / ROPE_WARPS;
    const int64_t cap = int64_t(sms) * per_sm;
    if (blocks > cap) blocks = cap;
    qk_norm_rope_kernel<T><<<unsigned(blocks), ROPE_WARPS * 32, SMEM, stream>>>(q, k, pos, qr, kr, nh, nkv, qn, kn,
                                                                              invf, eps, status);
    return cudaGetLastError();
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
