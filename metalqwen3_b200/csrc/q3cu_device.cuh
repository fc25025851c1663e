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

// ---------------------------------------------------------------------------
// expf with the host libm's bits (q3_expf.h); the table lives in shared memory
// ---------------------------------------------------------------------------
static __constant__ uint64_t c_exp_tab[32] = Q3_EXP2_TAB32_INIT;

__device__ __forceinline__ void load_exp_table(uint64_t *s_tab) {
    if (threadIdx.x < 32) s_tab[threadIdx.x] = c_exp_tab[threadIdx.x];
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
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
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

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
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
