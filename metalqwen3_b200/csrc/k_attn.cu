// k_attn.cu -- decode attention for one token, bit-exact with the reference.
//
// Reference: src/cpu/qwen3_original.c:395-428 (per query head h, kv head
// h / kv_mul, positions t = 0..pos):
//     score = 0; for i < head_dim: score += q[i] * k_t[i]      (index order)
//     att[t] = score / sqrtf(head_dim)
//     softmax(att, pos + 1)                                   (:291-308)
//     xb = 0;   for t <= pos: for i: xb[i] += att[t] * v_t[i]   (position order)
//     quantize(xq, xb, n_heads * head_dim)                    (:431, fused here)
// and softmax: max starts at 0 (NaN never wins), x = expf(x - max) summed in
// index order, then x /= sum.  Without FMA contraction every product and sum
// above is one rounding, so this kernel keeps each chain's order: a thread per
// position runs its 128-long score chain, the exponentials are the host libm's
// bits (q3_expf.h), one thread adds them in position order, and a thread per
// output element runs its value chain over the positions.  The scores and
// probabilities live in the caller's att buffer ([n_heads][seq_len], like the
// reference's RunState att), so any position up to seq_len is supported.
//
// Two launches that spread over the GPU (below).  K and V reach shared memory
// in chunks of 128 positions by cp.async; K rows are padded to 528 B so a
// thread per position reads its row without bank conflicts.  The
// position-order probability sum is the serial part.
#include "q3cu_internal.h"

namespace q3 {

constexpr int AT_HD = 128;
constexpr int AT_CH = 128;                                  // positions per staged chunk
constexpr int AT_KROW = AT_HD * 4 + 16;                     // padded K row: 33 x 16 B, conflict-free float4 reads
constexpr size_t AT_BUF = size_t(AT_CH) * AT_KROW;          // 67,584 B per chunk buffer

// Copies rows c0 .. c0+n-1 of a cache (this kv head's 128 floats of each) into
// buf with 16-byte cp.async pieces, `rowb` bytes apart; one commit group.
__device__ __forceinline__ void attn_stage(uint8_t *buf, const float *cache, int c0, int n, int kv_dim, int kvh,
                                           int rowb, int tid) {
    for (int f = tid; f < n * 32; f += AT_HD) {
        const int r = f >> 5, pc = f & 31;
        cp_async16(buf + r * rowb + pc * 16, cache + int64_t(c0 + r) * kv_dim + kvh * AT_HD + pc * 4);
    }
    cp_async_commit();
}

// The attention in two launches that spread over the GPU (one CTA per head
// would run on only n_heads SMs and stream 512 B per cached position through
// each):
//   attn_scores_kernel: a CTA per (head, chunk of 128 positions) work item,
//     grid-stride over the items of this position -- the chunk's K rows staged
//     by cp.async (padded, as above), a thread per position runs its score
//     chain and writes att;
//   attn_values_kernel: a CTA per (head, half-head = 64 elements = one Q8_0
//     group) -- two warps take the row max, the libm-identical exponentials
//     into shared memory, their sum in position order by one thread, the
//     division, then a thread per element runs its value chain over the
//     positions, while the other two warps stream V half-rows through an
//     AV_NST-deep cp.async ring; the CTA quantizes its group.
// Both halves of a head compute the same probabilities (the same operations on
// the same scores), so every chain keeps the reference's order and bits.  Both
// kernels read the position from device memory and size their work from it,
// so a captured graph serves every position.  Each is launched as a
// programmatic dependent of the kernel before it and waits for it
// (griddep_wait) before reading anything that kernel or an earlier one wrote.
constexpr int AV_COLS = 64;                                  // elements per values CTA
constexpr int AV_ROWB = AV_COLS * 4;                         // staged V half-row
constexpr size_t AV_BUF = size_t(AT_CH) * AV_ROWB;           // 32 KB per chunk
constexpr int AV_NST = 4;                                    // ring depth (three chunks in flight)
constexpr int AV_MAXPOS = 16384;                             // probabilities in shared memory up to here
constexpr int AS_PER_SM = 3;                                 // resident scores CTAs per SM (67.5 KB each)

// QK-RMSNorm + RoPE of one head row (:361-393) by one warp: v the row in
// global memory, w its norm weight; the rotated row to out (shared or global
// memory; out may be v, which is read whole before any lane writes).  Lane 0
// runs the sum of squares in index order from shared memory; rows / sq are
// this warp's 128-float scratch.
__device__ __forceinline__ void norm_rope_row(const float *v, const float *__restrict__ w,
                                              const StepParams *__restrict__ sp, float eps, float *rows, float *sq,
                                              float *out, int lane) {
    const float4 r4 = reinterpret_cast<const float4 *>(v)[lane];
    reinterpret_cast<float4 *>(rows)[lane] = r4;
    reinterpret_cast<float4 *>(sq)[lane] =
        make_float4(__fmul_rn(r4.x, r4.x), __fmul_rn(r4.y, r4.y), __fmul_rn(r4.z, r4.z), __fmul_rn(r4.w, r4.w));
    __syncwarp();
    float ss = 0.0f;
    if (lane == 0) {
        ss = ordered_sum_smem(0.0f, sq, AT_HD);
        ss = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(AT_HD)), eps)));
    }
    ss = __shfl_sync(FULL, ss, 0);
#pragma unroll
    for (int u = 0; u < 2; ++u) {                            // pair (j, j + 64)
        const int j = lane + 32 * u;
        const float x = __fmul_rn(w[j], __fmul_rn(ss, rows[j]));
        const float y = __fmul_rn(w[j + 64], __fmul_rn(ss, rows[j + 64]));
        const float c = sp->c[j], s = sp->s[j];
        out[j] = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
        out[j + 64] = __fadd_rn(__fmul_rn(x, s), __fmul_rn(y, c));
    }
    __syncwarp();                                            // out written, scratch free
}

// Scores with the step's QK-norm + RoPE folded in (ROT): qkv holds this
// token's raw [q | k | v] rows.  Each work item normalizes and rotates its
// head's q into shared memory (warp 0).  The item holding position pos also
// rotates the kv head's k straight into its tile row (warp 1) and, once per kv
// head (the first of its query heads), writes that k row and the v row into the
// caches for the values kernel and later steps (warps 1 and 2).  Without ROT,
// qkv is the already rotated q [n_heads][128] and the caches already hold row
// pos (MetalContext::executeAttention's inputs).  The position is *pos_p (the
// step's parameters) or, with pos_p NULL, pos_v.
template <bool ROT>
__global__ void __launch_bounds__(AT_HD) attn_scores_kernel(const float *qkv, float *kc, float *vc, float *att,
                                                            const float *__restrict__ qn,
                                                            const float *__restrict__ kn,
                                                            const StepParams *__restrict__ sp, int pos_v, float eps,
                                                            int n_heads, int kv_dim, int kv_mul, int seq_len) {
    extern __shared__ __align__(16) uint8_t tile[];          // [AT_CH][AT_KROW]
    __shared__ __align__(16) float qs[AT_HD];
    __shared__ __align__(16) float scr[2][2][AT_HD];
    griddep_launch_dependents();
    griddep_wait();                                          // qkv from the matmul before
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pos = sp ? sp->pos : pos_v, npos = pos + 1, items = (npos + AT_CH - 1) / AT_CH * n_heads;
    const int qdim = n_heads * AT_HD;
    for (int w = blockIdx.x; w < items; w += gridDim.x) {
        const int h = w % n_heads, c0 = (w / n_heads) * AT_CH, kvh = h / kv_mul;
        const int n = npos - c0 < AT_CH ? npos - c0 : AT_CH;
        const bool last = ROT && c0 + n == npos;             // this chunk holds position pos (rotated here)
        __syncthreads();                                     // the previous item's reads of tile / qs are done
        attn_stage(tile, kc, c0, last ? n - 1 : n, kv_dim, kvh, AT_KROW, tid);   // cached rows (below pos)
        if (!ROT) {
            if (warp == 0)
                reinterpret_cast<float4 *>(qs)[lane] = reinterpret_cast<const float4 *>(qkv + int64_t(h) * AT_HD)[lane];
        } else if (warp == 0) {
            norm_rope_row(qkv + int64_t(h) * AT_HD, qn, sp, eps, scr[0][0], scr[0][1], qs, lane);
        } else if (warp == 1 && last) {
            float *kr = reinterpret_cast<float *>(tile + (n - 1) * AT_KROW);
            norm_rope_row(qkv + qdim + kvh * AT_HD, kn, sp, eps, scr[1][0], scr[1][1], kr, lane);
            if (h % kv_mul == 0)
                reinterpret_cast<float4 *>(kc + int64_t(pos) * kv_dim + kvh * AT_HD)[lane] =
                    reinterpret_cast<const float4 *>(kr)[lane];
        } else if (warp == 2 && last && h % kv_mul == 0) {
            reinterpret_cast<float4 *>(vc + int64_t(pos) * kv_dim + kvh * AT_HD)[lane] =
                reinterpret_cast<const float4 *>(qkv + qdim + kv_dim + kvh * AT_HD)[lane];
        }
        cp_async_wait<0>();
        __syncthreads();
        if (tid < n) {
            const float4 *kr = reinterpret_cast<const float4 *>(tile + tid * AT_KROW);
            float s = 0.0f;
#pragma unroll 8
            for (int i4 = 0; i4 < AT_HD / 4; ++i4) {
                const float4 kv = kr[i4];
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4], kv.x));
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4 + 1], kv.y));
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4 + 2], kv.z));
                s = __fadd_rn(s, __fmul_rn(qs[4 * i4 + 3], kv.w));
            }
            att[int64_t(h) * seq_len + c0 + tid] = __fdiv_rn(s, __fsqrt_rn(float(AT_HD)));
        }
    }
}

// acc + p[0] v[0] + p[1] v[AV_COLS] + ... over n positions in order (one
// rounding per product and per add, as the reference's loop): p 16-byte aligned
// shared memory (broadcast), v this thread's column of a staged chunk.  The
// next 8 positions' operands are loaded while the current 8 are added.
__device__ __forceinline__ float value_chain(float acc, const float *p, const float *v, int n) {
    const float4 *p4 = reinterpret_cast<const float4 *>(p);
    const int nb = n >> 3;
    // two register sets, A and B, alternate: one batch is loaded while the
    // other is added, with no copies between them
    auto add8 = [&](const float4 &pa, const float4 &pb, const float *x) {
        acc = __fadd_rn(acc, __fmul_rn(pa.x, x[0]));
        acc = __fadd_rn(acc, __fmul_rn(pa.y, x[1]));
        acc = __fadd_rn(acc, __fmul_rn(pa.z, x[2]));
        acc = __fadd_rn(acc, __fmul_rn(pa.w, x[3]));
        acc = __fadd_rn(acc, __fmul_rn(pb.x, x[4]));
        acc = __fadd_rn(acc, __fmul_rn(pb.y, x[5]));
        acc = __fadd_rn(acc, __fmul_rn(pb.z, x[6]));
        acc = __fadd_rn(acc, __fmul_rn(pb.w, x[7]));
    };
    if (nb > 0) {
        float4 a0 = p4[0], b0 = p4[1];
        float x0[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x0[i] = v[i * AV_COLS];
        int b = 0;
        for (; b + 2 <= nb; b += 2) {
            const int k1 = b + 1;                                  // < nb
            const float4 a1 = p4[2 * k1], b1 = p4[2 * k1 + 1];
            float x1[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) x1[i] = v[(k1 * 8 + i) * AV_COLS];
            add8(a0, b0, x0);                                      // batch b
            const int k2 = b + 2 < nb ? b + 2 : k1;                // past the end: reload (unused)
            a0 = p4[2 * k2];
            b0 = p4[2 * k2 + 1];
#pragma unroll
            for (int i = 0; i < 8; ++i) x0[i] = v[(k2 * 8 + i) * AV_COLS];
            add8(a1, b1, x1);                                      // batch b + 1
        }
        if (b < nb) add8(a0, b0, x0);                              // odd count: the last batch
    }
    for (int t = nb << 3; t < n; ++t) acc = __fadd_rn(acc, __fmul_rn(p[t], v[t * AV_COLS]));
    return acc;
}

// Copies columns [col0, col0 + 64) of V rows c0 .. c0+n-1 of kv head kvh into
// buf, by threads t = 0 .. nthr-1 of the copying warps.
__device__ __forceinline__ void attn_stage_half(uint8_t *buf, const float *vc, int c0, int n, int kv_dim, int kvh,
                                                int col0, int t, int nthr) {
    for (int f = t; f < n * (AV_ROWB / 16); f += nthr) {
        const int r = f / (AV_ROWB / 16), pc = f % (AV_ROWB / 16);
        cp_async16(buf + r * AV_ROWB + pc * 16, vc + int64_t(c0 + r) * kv_dim + kvh * AT_HD + col0 + pc * 4);
    }
    cp_async_commit();
}

// Above AV_MAXPOS positions the probabilities do not fit next to the V ring:
// the kernel then keeps none of them.  It takes the row max from the scores in
// global memory, adds the exponentials in position order chunk by chunk (each
// chunk's exponentials computed in parallel into a buffer, then summed by one
// thread), and recomputes each V chunk's probabilities, with the same
// operations and therefore the same bits, just before that chunk's value
// chains.  Any context length; one more exponential per position.
constexpr int AV_ECH = 4096;                                 // exponentials per sum chunk (long mode)

// Outputs: Q8_0 codes/scales of the head (xq, xs; the decode step) and/or the
// float head outputs xb [n_heads][128] and the probabilities into probs (the
// first half's CTA only; executeAttention).  probs must not be att: the other
// half's CTA may still be reading the scores.  Position from *sp or, with sp
// NULL, pos_v.
__global__ void __launch_bounds__(AT_HD, 1) attn_values_kernel(float *att, const float *vc, int8_t *xq, float *xs,
                                                               float *xb, float *probs,
                                                               const StepParams *__restrict__ sp, int pos_v,
                                                               int kv_dim, int kv_mul, int seq_len, int res_cap) {
    extern __shared__ __align__(16) uint8_t dyn[];          // [AV_NST][AV_BUF] V ring, then the probabilities
    float *pr = reinterpret_cast<float *>(dyn + AV_NST * AV_BUF);
    __shared__ ExpTab tab;
    __shared__ float red[AT_HD / 32];
    __shared__ float sum_sh;
    griddep_launch_dependents();
    const int h = blockIdx.x, part = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kvh = h / kv_mul, col0 = part * AV_COLS;
    // Warps 0-1 run the value chains (thread = element); warps 2-3 copy V.  An
    // SM holds only ~50 KB of cp.async in flight, so issuing a chunk can stall
    // its issuer: only the copying warps issue, while the chains run.
    const bool producer = tid >= AV_COLS;
    const int pt = tid - AV_COLS;
    load_exp_table(tab);
    griddep_wait();                                          // att (and the caches, written two kernels back)
    const int npos = (sp ? sp->pos : pos_v) + 1, nch = (npos + AT_CH - 1) / AT_CH;
    // every probability kept in shared memory, if the launch's allocation holds them (res_cap floats)
    const bool resident = npos <= res_cap;
    float *a = att + int64_t(h) * seq_len;
    float *ech = pr + AT_CH;                                 // long mode: pr = one chunk, ech = AV_ECH exponentials
    auto stage = [&](int c) {                                // chunk c into slot c % AV_NST, or an empty group
        if (c < nch) {
            const int c0 = c * AT_CH;
            attn_stage_half(dyn + (c % AV_NST) * AV_BUF, vc, c0, npos - c0 < AT_CH ? npos - c0 : AT_CH, kv_dim, kvh,
                            col0, pt, AT_HD - AV_COLS);
        } else {
            cp_async_commit();
        }
    };
    float m = 0.0f;
    if (producer) {                                          // the first chunks stream in during the softmax
        for (int c = 0; c < AV_NST - 1; ++c) stage(c);
    } else {                                                 // the softmax by the chain warps (named barrier 1)
        for (int t = tid; t < npos; t += AV_COLS) m = fmaxf(m, a[t]);   // max from 0; a NaN never replaces it
        m = warp_max(m);
        if (lane == 0) red[warp] = m;
        named_sync(1, AV_COLS);                               // (also: the exp table is loaded)
        m = fmaxf(red[0], red[1]);
        if (resident) {
            for (int t = tid; t < npos; t += AV_COLS) pr[t] = expf_host(__fsub_rn(a[t], m), tab);
            named_sync(1, AV_COLS);
            if (tid == 0) sum_sh = ordered_sum_smem(0.0f, pr, npos);
            named_sync(1, AV_COLS);
            const float sum = sum_sh;
            for (int t = tid; t < npos; t += AV_COLS) pr[t] = __fdiv_rn(pr[t], sum);
        } else {
            float sum = 0.0f;                                 // thread 0's running sum, in position order
            for (int e0 = 0; e0 < npos; e0 += AV_ECH) {
                const int ne = npos - e0 < AV_ECH ? npos - e0 : AV_ECH;
                for (int t = tid; t < ne; t += AV_COLS) ech[t] = expf_host(__fsub_rn(a[e0 + t], m), tab);
                named_sync(1, AV_COLS);
                if (tid == 0) sum = ordered_sum_smem(sum, ech, ne);
                named_sync(1, AV_COLS);                       // ech is free again
            }
            if (tid == 0) sum_sh = sum;
        }
    }
    // value chains: thread j < 64 runs element col0 + j over the positions in
    // order.  Iteration c: chunk c has landed (the copiers' wait, then the
    // barrier), the copiers refill slot (c + AV_NST - 1) % AV_NST -- chunk
    // c - 1's, which every chain finished before this barrier -- while the
    // chains run c.  (Long mode: the chunk's probabilities first, into pr.)
    float acc = 0.0f;
    for (int c = 0; c < nch; ++c) {
        if (producer) cp_async_wait<AV_NST - 2>();            // chunks c .. c + AV_NST - 2 were pending
        __syncthreads();                                      // chunk c visible; (c == 0) the softmax is done
        const int c0 = c * AT_CH, n = npos - c0 < AT_CH ? npos - c0 : AT_CH;
        if (producer) {
            stage(c + AV_NST - 1);
        } else {
            const float *pc = pr + c0;
            if (!resident) {                                  // this chunk's probabilities, recomputed
                const float sum = sum_sh;
                for (int t = tid; t < n; t += AV_COLS) pr[t] = __fdiv_rn(expf_host(__fsub_rn(a[c0 + t], m), tab), sum);
                named_sync(1, AV_COLS);
                pc = pr;
            }
            if (probs && part == 0)
                for (int t = tid; t < n; t += AV_COLS) probs[int64_t(h) * seq_len + c0 + t] = pc[t];
            acc = value_chain(acc, pc, reinterpret_cast<const float *>(dyn + (c % AV_NST) * AV_BUF) + tid, n);
            if (!resident) named_sync(1, AV_COLS);            // every chain is done with pr before it is refilled
        }
    }
    if (producer) cp_async_wait<0>();                         // nothing in flight at exit
    if (xb && tid < AV_COLS) xb[int64_t(h) * AT_HD + col0 + tid] = acc;
    if (!xq) return;                                          // (uniform over the CTA)
    // the quantize of this group (:431): absmax from 0, scale = wmax / 127, codes
    const float gm = warp_max(tid < AV_COLS ? fmaxf(0.0f, fabsf(acc)) : 0.0f);
    if (lane == 0) red[warp] = gm;
    __syncthreads();
    const float qscale = q8_scale(fmaxf(red[0], red[1]));
    if (tid < AV_COLS) xq[int64_t(h) * AT_HD + col0 + tid] = int8_t(q8_code(acc, qscale));
    if (tid == 0) xs[int64_t(h) * 2 + part] = qscale;
}

cudaError_t launch_attention_step(float *qkv, float *kc, float *vc, float *att, int8_t *xq, float *xs,
                                  const StepParams *sp, int n_heads, int n_kv, const float *qn, const float *kn,
                                  float eps, int seq_len, cudaStream_t stream, int sms) {
    const int kv_dim = n_kv * AT_HD, kv_mul = n_heads / n_kv;
    // two launches, (head, chunk) / (head, half), any context length; the values
    // launch keeps all probabilities in shared memory while they fit (res_cap)
    const int res_cap = seq_len <= AV_MAXPOS ? seq_len : AT_CH + AV_ECH;
    const size_t vsm = AV_NST * AV_BUF + size_t(res_cap) * 4;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(attn_scores_kernel<true>), AT_BUF, 25);
    if (e == cudaSuccess) e = ensure_smem_attr(reinterpret_cast<const void *>(attn_values_kernel),
                                               AV_NST * AV_BUF + size_t(AV_MAXPOS) * 4, 26);
    if (e != cudaSuccess) return e;
    const int64_t items = int64_t(n_heads) * ((seq_len + AT_CH - 1) / AT_CH);
    const int grid = int(items < int64_t(AS_PER_SM) * sms ? items : int64_t(AS_PER_SM) * sms);
    e = launch_dependent(attn_scores_kernel<true>, dim3(grid), dim3(AT_HD), AT_BUF, stream, qkv, kc, vc, att, qn, kn,
                         sp, 0, eps, n_heads, kv_dim, kv_mul, seq_len);
    if (e != cudaSuccess) return e;
    return launch_dependent(attn_values_kernel, dim3(n_heads, 2), dim3(AT_HD), vsm, stream, att, vc, xq, xs,
                            static_cast<float *>(nullptr), static_cast<float *>(nullptr), sp, 0, kv_dim, kv_mul,
                            seq_len, res_cap);
}

cudaError_t launch_attention_rows(const float *q, const float *kc, const float *vc, float *att, float *probs, float *xb,
                                  int pos, int n_heads, int kv_dim, int kv_mul, int att_stride, cudaStream_t stream,
                                  int sms) {
    const int npos = pos + 1;
    const int res_cap = npos <= AV_MAXPOS ? npos : AT_CH + AV_ECH;
    const size_t vsm = AV_NST * AV_BUF + size_t(res_cap) * 4;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(attn_scores_kernel<false>), AT_BUF, 24);
    if (e == cudaSuccess) e = ensure_smem_attr(reinterpret_cast<const void *>(attn_values_kernel),
                                               AV_NST * AV_BUF + size_t(AV_MAXPOS) * 4, 26);
    if (e != cudaSuccess) return e;
    const int64_t items = int64_t(n_heads) * ((npos + AT_CH - 1) / AT_CH);
    const int grid = int(items < int64_t(AS_PER_SM) * sms ? items : int64_t(AS_PER_SM) * sms);
    e = launch_dependent(attn_scores_kernel<false>, dim3(grid), dim3(AT_HD), AT_BUF, stream, q,
                         const_cast<float *>(kc), const_cast<float *>(vc), att, static_cast<const float *>(nullptr),
                         static_cast<const float *>(nullptr), static_cast<const StepParams *>(nullptr), pos, 0.0f,
                         n_heads, kv_dim, kv_mul, att_stride);
    if (e != cudaSuccess) return e;
    return launch_dependent(attn_values_kernel, dim3(n_heads, 2), dim3(AT_HD), vsm, stream, att, vc,
                            static_cast<int8_t *>(nullptr), static_cast<float *>(nullptr), xb, probs,
                            static_cast<const StepParams *>(nullptr), pos, kv_dim, kv_mul, att_stride, res_cap);
}

__global__ void set_step_kernel(StepParams *sp, StepParams v) {
    reinterpret_cast<uint32_t *>(sp)[threadIdx.x] = reinterpret_cast<const uint32_t *>(&v)[threadIdx.x];
}

cudaError_t launch_set_step(StepParams *sp, const StepParams &v, cudaStream_t stream) {
    set_step_kernel<<<1, sizeof(StepParams) / 4, 0, stream>>>(sp, v);
    return cudaGetLastError();
}


}  // namespace q3
