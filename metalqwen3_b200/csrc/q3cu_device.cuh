// q3cu_device.cuh -- device helpers shared by the sm_100a kernels.
//
// Numerics: the library is compiled with --fmad=false and without -ftz, so a
// float expression rounds once per operator and denormals are kept, as in the
// reference CPU engine built without -ffast-math.  Where the reference's
// rounding points matter the code also spells them with __fmul_rn/__fadd_rn.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3_expf.h"
#include "q3cu.h"

namespace q3 {

constexpr int GS = 64;                         // Q8_0 group size
constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------------------
// bf16 <-> f32 (bit patterns; f32 -> bf16 rounds to nearest even)
// ---------------------------------------------------------------------------
struct bf16raw { uint16_t b; };

__device__ __forceinline__ float bf16_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ uint32_t f32_to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (u >> 16) | 0x40u;
    return (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
}

// ---------------------------------------------------------------------------
// global memory: 16-byte vector loads/stores
// ---------------------------------------------------------------------------
// Read-once inputs of a kernel that does not write them: non-coherent path,
// no L1 allocation.
__device__ __forceinline__ uint4 ld_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
// Read-only data that a CTA re-reads many times (norm weights): non-coherent
// path, cached in L1.
__device__ __forceinline__ uint4 ld_l1_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
// Asks L2 to fetch [p, p + bytes) (p 16-byte aligned, bytes a multiple of 16);
// nothing waits for it.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}
// Coherent load (data the same kernel may have written).
__device__ __forceinline__ uint4 ld_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}
// Streaming stores (evict-first): outputs are not re-read by the kernel.
__device__ __forceinline__ void st_cs_v4(void *p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void st_cs_v2(void *p, uint2 v) {
    asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" :: "l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void st_cs_u32(void *p, uint32_t v) {
    asm volatile("st.global.cs.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cs_f32(float *p, float v) {
    asm volatile("st.global.cs.f32 [%0], %1;" :: "l"(p), "f"(v) : "memory");
}

// Programmatic dependent launch (sm_90+).  A kernel launched with the
// programmatic-serialization attribute may start before its predecessor
// finishes; griddep_wait() blocks until the predecessor has completed and its
// writes are visible (it returns at once for an ordinary launch).
// griddep_launch_dependents() lets such a successor be scheduled now; it
// changes nothing for ordinary successors.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float4 u4_as_f4(uint4 u) {
    return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
}
__device__ __forceinline__ uint4 f4_as_u4(float4 f) {
    return make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z), __float_as_uint(f.w));
}

// Loads 16 bytes = VEC elements of T and widens them to float.
template <typename T> struct Vec;
template <> struct Vec<float> {
    static constexpr int N = 4;
    __device__ __forceinline__ static void widen(uint4 u, float *o) {
        o[0] = __uint_as_float(u.x); o[1] = __uint_as_float(u.y);
        o[2] = __uint_as_float(u.z); o[3] = __uint_as_float(u.w);
    }
    __device__ __forceinline__ static uint4 narrow(const float *o) {
        return make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]),
                          __float_as_uint(o[2]), __float_as_uint(o[3]));
    }
};
template <> struct Vec<bf16raw> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void widen(uint4 u, float *o) {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[2 * i] = bf16_to_f32(w[i] & 0xffffu);
            o[2 * i + 1] = bf16_to_f32(w[i] >> 16);
        }
    }
    __device__ __forceinline__ static uint4 narrow(const float *o) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = f32_to_bf16(o[2 * i]) | (f32_to_bf16(o[2 * i + 1]) << 16);
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};

// ---------------------------------------------------------------------------
// Q8_0 code semantics (src/cpu/qwen3_original.c:147-168)
// ---------------------------------------------------------------------------
// |v| folded into a running max with the reference's strict `>` (a NaN never
// replaces the max; the max starts at 0).
__device__ __forceinline__ float amax_fold(float m, float v) {
    float a = fabsf(v);
    return a > m ? a : m;
}
__device__ __forceinline__ float amax_merge(float m, float o) { return o > m ? o : m; }

// Round half away from zero, exactly (C `round` of a binary32 value).
__device__ __forceinline__ float round_half_away(float v) {
    float t = truncf(v);
    float d = __fsub_rn(v, t);                 // exact: the fractional part
    if (fabsf(d) >= 0.5f) t = __fadd_rn(t, copysignf(1.0f, v));
    return t;
}

// `(int8_t) round(x / scale)` as the x86-64 build of the reference executes it:
// IEEE division, round half away, truncation to int32 whose invalid result
// (NaN, inf, |r| >= 2^31) is INT_MIN, then the low byte.
__device__ __forceinline__ uint32_t q8_code(float v, float scale) {
    float r = round_half_away(__fdiv_rn(v, scale));
    if (!(fabsf(r) < 2147483648.0f)) return 0u;
    return (uint32_t)__float2int_rz(r) & 0xffu;
}

__device__ __forceinline__ float q8_scale(float wmax) { return __fdiv_rn(wmax, 127.0f); }

// 1/x within 1 ulp, for x whose reciprocal is a normal binary32 number (every
// caller: 1 <= x < 2^120, or a Q8_0 scale in [2^-97, 2^93]; a group outside
// that range takes the exact path and ignores this value).  The .ftz form is
// the bare hardware approximation; without .ftz the compiler wraps it in a
// subnormal rescaling (compare, two selects, two multiplies per call) that
// these operands never need.
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Correctly rounded 1/d for d >= 1 by Newton-Raphson from the 1-ulp seed
// followed by Markstein's correction step (Markstein, IBM J. Res. Dev. 34(1),
// 1990): e = 1 - d*y and y + y*e with fused multiply-adds.  Equal to the IEEE
// reciprocal (__frcp_rn) for every binary32 d in [1, 2^120), which
// tests/test_device_math.py checks exhaustively on the GPU; larger d, inf and
// NaN use __frcp_rn.
// Rare paths are kept out of line so the compiler branches around them
// instead of predicating them into every element's instruction stream.
static __device__ __noinline__ float rcp_rn_slow(float d) { return __frcp_rn(d); }

__device__ __forceinline__ float rcp_rn_ge1(float d) {
    if (!(d < 0x1p120f)) return rcp_rn_slow(d);
    const float y0 = rcp_approx(d);
    const float y1 = __fmaf_rn(y0, __fmaf_rn(-d, y0, 1.0f), y0);
    return __fmaf_rn(y1, __fmaf_rn(-d, y1, 1.0f), y1);
}

// One correction step is enough on [1, 2^120): the rcp.approx seed is within
// one ulp of 1/d there, and y0 + y0*(1 - d*y0) (two fused multiply-adds) is
// then equal to __frcp_rn(d) for every binary32 d in that range (exhaustive
// check in tests/test_device_math.py).  The caller guarantees the range.
__device__ __forceinline__ float rcp_rn_1to2p120(float d) {
    const float y0 = rcp_approx(d);
    return __fmaf_rn(y0, __fmaf_rn(-d, y0, 1.0f), y0);
}

// Per-group state for the fast code path.
//  * scale = RN(wmax/127): one multiply by RN(1/127) = 0x1.020408p-7 and one
//    FMA-based correction (Markstein); equal to the IEEE quotient for every
//    wmax in [2^-100, 2^100] (exhaustive check in tests/test_device_math.py).
//    Groups outside [2^-90, 2^100] (zero, tiny, huge, inf) use the division.
//  * codes: q8_code needs one IEEE division per element, but the code depends
//    on that quotient only through round-half-away.  So multiply by an
//    approximate reciprocal (rcp.approx, within 1 ulp) and fall back to the
//    exact division when the product lies within 2^-14 of a tie k + 1/2.  For
//    |v| <= wmax, |v*inv - v/scale| <= 127.0001 * (2^-23 + 2^-24) < 2.3e-5 and
//    the IEEE quotient is within half an ulp (< 3.9e-6) of v/scale, so outside
//    the window both round to the same integer.
struct Q8Scale {
    float scale, inv;
    bool exact;
};
static __device__ __noinline__ float q8_scale_slow(float wmax) { return q8_scale(wmax); }
static __device__ __noinline__ uint32_t q8_code_slow(float v, float scale) { return q8_code(v, scale); }

__device__ __forceinline__ Q8Scale q8_prepare(float wmax) {
    Q8Scale g;
    const float c = 0x1.020408p-7f;
    const float s0 = __fmul_rn(wmax, c);
    g.scale = __fmaf_rn(__fmaf_rn(-s0, 127.0f, wmax), c, s0);
    g.exact = !(wmax >= 0x1p-90f && wmax <= 0x1p+100f);
    if (g.exact) g.scale = q8_scale_slow(wmax);
    g.inv = g.exact ? 0.0f : rcp_approx(g.scale);
    return g;
}
__device__ __forceinline__ uint32_t q8_code_g(float v, const Q8Scale &g) {
    const float qa = __fmul_rn(v, g.inv);
    const float t = __fadd_rn(qa, 12582912.0f);          // 1.5*2^23: round to nearest integer (|qa| < 2^22)
    const float d = fabsf(__fsub_rn(qa, __fsub_rn(t, 12582912.0f)));   // exact distance to it
    if (g.exact || !(d <= 0.49993896484375f))            // exact group, near a tie, or NaN
        return q8_code_slow(v, g.scale);
    return uint32_t(__float_as_int(t) - 0x4B400000) & 0xffu;
}
// Four codes packed little-endian into one word.
__device__ __forceinline__ uint32_t q8_pack4(const float *o, const Q8Scale &g) {
    return q8_code_g(o[0], g) | (q8_code_g(o[1], g) << 8) | (q8_code_g(o[2], g) << 16) | (q8_code_g(o[3], g) << 24);
}

// ---------------------------------------------------------------------------
// 32-byte vectors (one 256-bit access per lane; sm_100) and packed f32 pairs
// ---------------------------------------------------------------------------
struct U8 { uint32_t w[8]; };

__device__ __forceinline__ U8 ld_nc_v8(const void *p) {
    U8 v;
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                   "=r"(v.w[6]), "=r"(v.w[7]) : "l"(p));
    return v;
}
__device__ __forceinline__ U8 ld_v8(const void *p) {
    U8 v;
    asm volatile("ld.global.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                   "=r"(v.w[6]), "=r"(v.w[7]) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_cs_v8(void *p, const U8 &v) {
    asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 :: "l"(p), "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]),
                    "r"(v.w[6]), "r"(v.w[7]) : "memory");
}

// 32 bytes of T widened to float (8 f32 or 16 bf16), and back.
template <typename T> struct Wide;
template <> struct Wide<float> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void widen(const U8 &u, float *o) {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(u.w[i]);
    }
    __device__ __forceinline__ static U8 narrow(const float *o) {
        U8 u;
#pragma unroll
        for (int i = 0; i < 8; ++i) u.w[i] = __float_as_uint(o[i]);
        return u;
    }
};
template <> struct Wide<bf16raw> {
    static constexpr int N = 16;
    __device__ __forceinline__ static void widen(const U8 &u, float *o) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[2 * i] = bf16_to_f32(u.w[i] & 0xffffu);
            o[2 * i + 1] = bf16_to_f32(u.w[i] >> 16);
        }
    }
    __device__ __forceinline__ static U8 narrow(const float *o) {
        U8 u;
#pragma unroll
        for (int i = 0; i < 8; ++i) u.w[i] = f32_to_bf16(o[2 * i]) | (f32_to_bf16(o[2 * i + 1]) << 16);
        return u;
    }
};

// Packed pairs of binary32 (sm_100 add/sub/mul/fma.rn.f32x2): each half is an
// independent IEEE operation with round-to-nearest, as the scalar forms.
typedef uint64_t f2;
__device__ __forceinline__ f2 pk2(float a, float b) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void up2(f2 p, float &a, float &b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(p)); }
__device__ __forceinline__ f2 add2(f2 a, f2 b) { f2 r; asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b)); return r; }
__device__ __forceinline__ f2 sub2(f2 a, f2 b) { f2 r; asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b)); return r; }
__device__ __forceinline__ f2 mul2(f2 a, f2 b) { f2 r; asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b)); return r; }
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// Q8_0 codes of the N values one lane holds of a 64-group that spans LPG lanes
// (N * LPG == 64).  The fast path is the one of q8_prepare/q8_code_g, done on
// pairs, with the code read from the low byte of (q + 1.5*2^23): for
// |k| < 2^22 that float's bit pattern is 0x4B400000 + k.  Lanes whose group
// needs the exact division (tiny/huge/zero scale) or that have a quotient near
// a tie redo their codes with q8_code afterwards (lane-local, rare).
// Returns the group scale; codes[] receives N/4 little-endian words.
template <int N, int LPG>
__device__ __forceinline__ float q8_encode_lane(const float *o, uint32_t *codes) {
    static_assert(N * LPG == GS, "a group is 64 values");
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) m = fmaxf(m, fabsf(o[i]));           // NaN never wins; starts at 0
#pragma unroll
    for (int k = LPG / 2; k > 0; k >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, k));
    const float c = 0x1.020408p-7f;
    const float s0 = __fmul_rn(m, c);
    float scale = __fmaf_rn(__fmaf_rn(-s0, 127.0f, m), c, s0);
    const bool exact_group = !(m >= 0x1p-90f && m <= 0x1p+100f);
    if (__builtin_expect(exact_group, 0)) scale = q8_scale(m);
    const float inv = rcp_approx(scale);
    const f2 inv2 = pk2(inv, inv), M2 = pk2(12582912.0f, 12582912.0f);
    bool fix = exact_group;
    uint32_t tb[N];
#pragma unroll
    for (int i = 0; i < N; i += 2) {
        const f2 qa = mul2(pk2(o[i], o[i + 1]), inv2);
        const f2 t = add2(qa, M2);
        const f2 d = sub2(qa, sub2(t, M2));
        float d0, d1, t0, t1;
        up2(d, d0, d1);
        up2(t, t0, t1);
        fix |= !(fabsf(d0) <= 0.49993896484375f) | !(fabsf(d1) <= 0.49993896484375f);
        tb[i] = __float_as_uint(t0);
        tb[i + 1] = __float_as_uint(t1);
    }
#pragma unroll
    for (int w = 0; w < N / 4; ++w)
        codes[w] = __byte_perm(__byte_perm(tb[4 * w], tb[4 * w + 1], 0x0040),
                               __byte_perm(tb[4 * w + 2], tb[4 * w + 3], 0x0040), 0x5410);
    if (__builtin_expect(fix, 0)) {
#pragma unroll
        for (int w = 0; w < N / 4; ++w)
            codes[w] = q8_code(o[4 * w], scale) | (q8_code(o[4 * w + 1], scale) << 8) |
                       (q8_code(o[4 * w + 2], scale) << 16) | (q8_code(o[4 * w + 3], scale) << 24);
    }
    return scale;
}

// ---------------------------------------------------------------------------
// expf with the host libm's bits (q3_expf.h); the table lives in shared memory
// ---------------------------------------------------------------------------
static __constant__ uint64_t c_exp_tab[32] = Q3_EXP2_TAB32_INIT;

__device__ __forceinline__ void load_exp_table(uint64_t *s_tab) {
    if (threadIdx.x < 32) s_tab[threadIdx.x] = c_exp_tab[threadIdx.x];
}
// High and low 32-bit words in separate arrays, for q3_expf_fast.
struct ExpTab {
    uint32_t hi[32], lo[32];
};
__device__ __forceinline__ void load_exp_table(ExpTab &t) {
    if (threadIdx.x < 32) {
        const uint64_t v = c_exp_tab[threadIdx.x];
        t.hi[threadIdx.x] = uint32_t(v >> 32);
        t.lo[threadIdx.x] = uint32_t(v);
    }
}
__device__ __forceinline__ float expf_host(float x, const ExpTab &t) { return q3_expf_fast(x, t.hi, t.lo); }
__device__ __forceinline__ float expf_core(float x, const ExpTab &t) { return q3_expf_core(x, t.hi, t.lo); }

// SwiGLU of one element by the reference's chain (:449-450), exactly:
// a * (b * (1 / (1 + expf(-a)))), expf with the host libm's bits.
__device__ __forceinline__ float swiglu_exact(float a, float b, const ExpTab &tab) {
    const float ex = expf_host(-a, tab);
    return __fmul_rn(a, __fmul_rn(b, __frcp_rn(__fadd_rn(1.0f, ex))));
}

// SwiGLU of the N (even) values a lane holds, bit-identical to swiglu_exact.
// Per element: the expf core (binary64, branch free), then 1/(1+e) by a
// rcp.approx seed and one Markstein correction step (correctly rounded for
// 1 <= d < 2^120, checked against __frcp_rn on every such d), and the two
// products, element pairs in packed f32x2 arithmetic.  |a| < 83 keeps -a off
// expf's special inputs (|x| >= 88, NaN, inf) and d = 1 + e^-a inside
// [1, 2^120); nd = -1 - e is -d exactly (round-to-nearest is symmetric), so
// d's negation costs nothing.  A lane holding an |a| >= 83 (or NaN) recomputes
// its values with swiglu_exact.
template <int N>
__device__ __forceinline__ void swiglu_lane(const float *a, const float *b, float *o, const ExpTab &tab) {
    bool slow = false;
    const f2 NEG1 = pk2(-1.0f, -1.0f), ONE = pk2(1.0f, 1.0f);
#pragma unroll
    for (int i = 0; i < N; i += 2) {
        slow |= !(fabsf(a[i]) < 83.0f) | !(fabsf(a[i + 1]) < 83.0f);
        const f2 nd = sub2(NEG1, pk2(expf_core(-a[i], tab), expf_core(-a[i + 1], tab)));
        float nd0, nd1;
        up2(nd, nd0, nd1);
        const f2 y0 = pk2(rcp_approx(-nd0), rcp_approx(-nd1));
        const f2 y = fma2(y0, fma2(nd, y0, ONE), y0);      // y0 + y0*(1 - d*y0)
        up2(mul2(pk2(a[i], a[i + 1]), mul2(pk2(b[i], b[i + 1]), y)), o[i], o[i + 1]);
    }
    if (__builtin_expect(slow, 0)) {
#pragma unroll
        for (int i = 0; i < N; ++i) o[i] = swiglu_exact(a[i], b[i], tab);
    }
}

// exp(d) for -80 <= d <= 0, where only accuracy is required (softmax: 1e-5
// relative), in binary32 without the binary64 core: exp(d) = 2^t, t = d*log2(e).
// t is carried as th + tl: th = RN(d*L) with L = RN(log2 e), and tl = the
// product's rounding error, exact by fused multiply-add (the TwoProduct of
// Ogita, Rump & Oishi, "Accurate sum and dot product", 2005), plus d*(log2 e - L).
// Then 2^th from ex2.approx (th in [-115.5, 0]: a normal result) and the factor
// 2^tl = 1 + tl*ln2 to first order (|tl| < 6e-6, so the dropped term is below
// 2^-36).  Relative error about 2^-22 over the whole range
// (tests/test_device_math.py sweeps every binary32 d in [-80, 0] against the
// binary64 exp).  NaN gives NaN; d = -inf does not belong here (tl is NaN).
__device__ __forceinline__ float ex2_approx_ftz(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
constexpr float EXP_L = 1.44269502162933349609375f;      // RN(log2 e)
constexpr float EXP_L_LO = 1.925963033500011079e-8f;     // RN(log2 e - EXP_L)
constexpr float EXP_LN2 = 0.693147182464599609375f;      // RN(ln 2)
__device__ __forceinline__ float exp_m80_0(float d) {
    const float th = __fmul_rn(d, EXP_L);
    const float tl = __fmaf_rn(d, EXP_L_LO, __fmaf_rn(d, EXP_L, -th));
    const float e = ex2_approx_ftz(th);
    return __fmaf_rn(__fmul_rn(e, EXP_LN2), tl, e);
}
// exp_m80_0 of an element pair in packed f32x2 arithmetic, the same roundings in
// the same order (bit-identical: -th = RN(d*(-L)) is the exact negation of
// RN(d*L), round-to-nearest being symmetric).
__device__ __forceinline__ f2 exp2_m80_0(f2 d) {
    const f2 nth = mul2(d, pk2(-EXP_L, -EXP_L));
    const f2 tl = fma2(d, pk2(EXP_L_LO, EXP_L_LO), fma2(d, pk2(EXP_L, EXP_L), nth));
    float n0, n1;
    up2(nth, n0, n1);
    const f2 e = pk2(ex2_approx_ftz(-n0), ex2_approx_ftz(-n1));
    return fma2(mul2(e, pk2(EXP_LN2, EXP_LN2)), tl, e);
}

// ---------------------------------------------------------------------------
// TMA bulk copies (cp.async.bulk, no tensor map, no multicast) and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Raises the barrier's expected transaction bytes without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_addr(bar)) : "memory");
}
// Barrier `id` (1..15) over the first `threads` threads of the CTA (a multiple of 32).
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void prefetch_l1(const void *p) {
    asm volatile("prefetch.global.L1 [%0];" :: "l"(p));
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Non-blocking probe: true if the phase with parity `parity` has completed.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Global -> shared bulk copy completing on `bar` (16-byte aligned addresses,
// size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Per-thread asynchronous 16-byte global -> shared copies (cp.async, L2 only).
// Both addresses 16-byte aligned.  A thread's copies are grouped by commit;
// wait<N> blocks until at most N of its groups are still in flight (a hardware
// wait for outstanding loads, not a polling loop).  Other threads see the data
// after a barrier that follows their wait.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_addr(dst)), "l"(src) : "memory");
}
// Makes `bar`'s current phase wait for all of this thread's earlier cp.async
// copies: the pending count rises by one now and falls by one when they have
// landed (no net arrival, so the barrier's expected count is unaffected).
__device__ __forceinline__ void cp_async_track(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Every wait is bounded: after ~2 s (or 2^26 polls) it records
// Q3CU_DEV_TIMEOUT in the status word and returns false; callers then skip
// their remaining work for the affected rows.
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr uint32_t WAIT_POLLS = 1u << 26;

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < WAIT_POLLS; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && global_ns() - t0 > WAIT_NS) break;
    }
    if (status) atomicOr(status, Q3CU_DEV_TIMEOUT);
    return false;
}

// The same bounded wait for warps that expect a long wait (microseconds) and
// share their SM with a latency-bound warp: between polls the warp sleeps
// (nanosleep), so it takes no issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t *bar, uint32_t parity, uint32_t *status) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < WAIT_POLLS; ++i) {
        if (mbar_test_wait(bar, parity)) return true;
        __nanosleep(200);
        if ((i & 15u) == 15u && global_ns() - t0 > WAIT_NS) break;
    }
    if (status) atomicOr(status, Q3CU_DEV_TIMEOUT);
    return false;
}

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
// acc + p[0] + p[1] + ... + p[n-1] by one thread, in index order with one
// binary32 rounding per add (the reference's serial loops).  p is 16-byte
// aligned shared memory; 16 values are loaded while the previous 16 are added,
// so the chain runs at the add latency, not the load latency.
__device__ __forceinline__ float ordered_sum_smem(float acc, const float *p, int n) {
    const float4 *p4 = reinterpret_cast<const float4 *>(p);
    const int nb = n >> 4;
    if (nb > 0) {
        float4 cur[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) cur[j] = p4[j];
        for (int b = 0; b < nb; ++b) {
            float4 nxt[4];
            const int kn = (b + 1 < nb ? b + 1 : b) * 4;               // the last batch reloads itself
#pragma unroll
            for (int j = 0; j < 4; ++j) nxt[j] = p4[kn + j];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc = __fadd_rn(acc, cur[j].x);
                acc = __fadd_rn(acc, cur[j].y);
                acc = __fadd_rn(acc, cur[j].z);
                acc = __fadd_rn(acc, cur[j].w);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) cur[j] = nxt[j];
        }
    }
    for (int t = nb << 4; t < n; ++t) acc = __fadd_rn(acc, p[t]);
    return acc;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

}  // namespace q3
