// Exhaustive / sweeping checks of the fast device arithmetic in
// metalqwen3_b200/csrc/q3cu_device.cuh against the exact forms it replaces.
// Built and run by tests/test_device_math.py; prints the counts and the bound.
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "q3cu_device.cuh"

using namespace q3;

// (1) rcp_rn_ge1(d) == __frcp_rn(d) for every binary32 d in [1, 2^120) (and a
//     few beyond, which take the library path)
__global__ void check_rcp(uint32_t lo, uint32_t hi, unsigned long long *bad) {
    unsigned long long n = 0;
    for (uint64_t u = lo + uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < hi;
         u += uint64_t(gridDim.x) * blockDim.x) {
        const float d = __uint_as_float(uint32_t(u));
        if (__float_as_uint(rcp_rn_ge1(d)) != __float_as_uint(__frcp_rn(d))) ++n;
    }
    if (n) atomicAdd(bad, n);
}

// (1b) the one-step form on [1, 2^120)
__global__ void check_rcp1(uint32_t lo, uint32_t hi, unsigned long long *bad) {
    unsigned long long n = 0;
    for (uint64_t u = lo + uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < hi;
         u += uint64_t(gridDim.x) * blockDim.x) {
        const float d = __uint_as_float(uint32_t(u));
        if (__float_as_uint(rcp_rn_1to2p120(d)) != __float_as_uint(__frcp_rn(d))) ++n;
    }
    if (n) atomicAdd(bad, n);
}

// (1c) exp_m80_0 (softmax's binary32 exp) on every binary32 d in [-80, 0]:
//      largest relative error against the binary64 exp, in units of 1e-12
__global__ void check_exp80(unsigned long long *worst) {
    unsigned long long w = 0;
    const uint32_t lo = 0x80000000u, hi = 0xc2a00000u;             // -0 .. -80 (bit patterns ascend)
    for (uint64_t u = lo + uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; u <= hi;
         u += uint64_t(gridDim.x) * blockDim.x) {
        const float d = __uint_as_float(uint32_t(u));
        const double ref = exp(double(d));
        const double rel = fabs(double(exp_m80_0(d)) - ref) / ref;
        const unsigned long long e = (unsigned long long)(rel * 1e12);
        if (e > w) w = e;
    }
    atomicMax(worst, w);
}

// (1d) the packed pair form exp2_m80_0 returns exp_m80_0's bits, on every
//      binary32 d in [-80, 0] (each d paired with its neighbour)
__global__ void check_exp80_pair(unsigned long long *bad) {
    unsigned long long n = 0;
    const uint32_t lo = 0x80000000u, hi = 0xc2a00000u;
    for (uint64_t u = lo + uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; u <= hi;
         u += uint64_t(gridDim.x) * blockDim.x) {
        const float d0 = __uint_as_float(uint32_t(u)), d1 = __uint_as_float(uint32_t(u == hi ? u : u + 1));
        float r0, r1;
        up2(exp2_m80_0(pk2(d0, d1)), r0, r1);
        if (__float_as_uint(r0) != __float_as_uint(exp_m80_0(d0)) || __float_as_uint(r1) != __float_as_uint(exp_m80_0(d1))) ++n;
    }
    if (n) atomicAdd(bad, n);
}

// (2) scale and codes of the fast path == the exact path
//     q8_scale (IEEE m/127) and q8_code (IEEE division + round half away)
__device__ __forceinline__ uint32_t hash32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352du; x ^= x >> 15; x *= 0x846ca68bu; x ^= x >> 16;
    return x;
}
__global__ void check_q8(uint32_t nm, unsigned long long *bad_scale, unsigned long long *bad_code) {
    unsigned long long bs = 0, bc = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nm; i += gridDim.x * blockDim.x) {
        // wmax: random sign-free binary32 across the whole exponent range
        const uint32_t h = hash32(i * 2654435761u + 12345u);
        const float m = __uint_as_float(h & 0x7f7fffffu);
        const Q8Scale g = q8_prepare(m);
        const float exact_scale = q8_scale(m);
        if (__float_as_uint(g.scale) != __float_as_uint(exact_scale)) ++bs;
        // values whose quotient lands on and around every tie k + 1/2 and integer,
        // plus random ones in [-m, m]
        for (int k = -127; k <= 127; ++k) {
            for (int t = 0; t < 4; ++t) {
                const float target = float(k) + (t < 2 ? 0.5f : 0.0f) * (k < 0 ? -1.0f : 1.0f);
                float v = __fmul_rn(target, exact_scale);
                const int32_t step = (t & 1) ? 1 : -1;
                for (int s = 0; s < 3; ++s) {
                    if (fabsf(v) <= m && q8_code_g(v, g) != q8_code(v, exact_scale)) ++bc;
                    v = __int_as_float(__float_as_int(v) + step);
                }
            }
        }
        for (int r = 0; r < 64; ++r) {
            const uint32_t hr = hash32(h ^ (r * 0x9e3779b9u));
            const float v = __fmul_rn(m, __fmul_rn(float(int32_t(hr)), 0x1p-31f));
            if (q8_code_g(v, g) != q8_code(v, exact_scale)) ++bc;
        }
    }
    if (bs) atomicAdd(bad_scale, bs);
    if (bc) atomicAdd(bad_code, bc);
}

int main() {
    unsigned long long *d;
    cudaMalloc(&d, 6 * sizeof(unsigned long long));
    cudaMemset(d, 0, 6 * sizeof(unsigned long long));
    check_rcp<<<148 * 16, 256>>>(0x3f800000u, 0x7f800001u, d);           // [1, +inf]
    check_q8<<<148 * 8, 128>>>(1u << 20, d + 1, d + 2);
    check_rcp1<<<148 * 16, 256>>>(0x3f800000u, 0x7b800000u, d + 3);     // [1, 2^120)
    check_exp80<<<148 * 16, 256>>>(d + 4);                                 // [-80, 0]
    check_exp80_pair<<<148 * 16, 256>>>(d + 5);
    cudaError_t e = cudaDeviceSynchronize();
    unsigned long long h[6] = {~0ull, ~0ull, ~0ull, ~0ull, ~0ull, ~0ull};
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) { printf("cuda error %s\n", cudaGetErrorString(e)); return 1; }
    printf("%llu %llu %llu %llu %llu %llu\n", h[0], h[1], h[2], h[3], h[4], h[5]);
    return 0;
}
