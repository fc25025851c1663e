// q3cu_tma.h -- tensor maps (TMA descriptors) for the kernels that stage rows
// through shared memory with cp.async.bulk.tensor, and the device-side copy.
//
// Host: the driver's cuTensorMapEncodeTiled is looked up once through the
// runtime (cudaGetDriverEntryPoint), so the library does not link libcuda.
// Device: one tiled 3-D load per call, completing on an mbarrier; no multicast
// (the maps only ever describe this GPU's own memory).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q3 {

// A row-major [rows][row_bytes] byte array viewed as 3-D for TMA: dim 0 = the
// 128 bytes of one line, dim 1 = the line within a row (stride 128 B), dim 2 =
// the row (stride row_bytes).  Box = {128, L, R}: L consecutive lines of R
// consecutive rows, landing in shared memory as [R][L][128 B] with the 128-byte
// swizzle (16-byte chunk c of smem line i is stored at chunk c ^ (i % 8); the
// destination must be 1024-byte aligned).  Out-of-range lines and rows are
// filled with zeros.  Requires base 16-byte aligned and row_bytes % 128 == 0.
// Returns false (and leaves *map undefined) if the driver rejects it.
// The map depends only on the arguments, so the last few are kept per host
// thread and reused (encode_row_lines_map_uncached always encodes).
bool encode_row_lines_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes, uint32_t L,
                          uint32_t R);
bool encode_row_lines_map_uncached(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes,
                                   uint32_t L, uint32_t R);

// A row-major [rows][row_bytes] byte array as 2-D for TMA: box = {128 bytes,
// box_rows rows}, landing as box_rows x 128 B with the 128-byte swizzle (the
// K-major operand layout of the tensor-core MMA).  Cached like the above.
bool encode_rows_2d_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows);

// A row-major [rows][cols] fp32 matrix as 2-D for TMA stores: box = {box_cols,
// box_rows}; shared memory holds the box row-major, with the 128-byte swizzle
// when swizzle128 (box_cols == 32; 16-byte chunk c of box row r at c ^ (r % 8),
// 1024-byte aligned).  Requires base 16-byte aligned, cols % 4 == 0 and
// box_cols * 4 a multiple of 16.  Cached.
bool encode_f32_2d_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                       uint32_t box_rows, bool swizzle128);

#if defined(__CUDACC__)
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(reinterpret_cast<uint64_t>(map)), "r"(x),
           "r"(y), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}
// Tiled 3-D tensor load of the box at (x, y, z) into shared memory at dst,
// completing on `bar` (the caller has armed it with the box's bytes).  x is
// the byte offset within the line and is always 0 here (16-byte aligned).
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(reinterpret_cast<uint64_t>(map)), "r"(x),
           "r"(y), "r"(z), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}
// Tiled 2-D tensor store of the box at (x, y) from shared memory at src, in the
// thread's bulk async-group (the caller commits it).  Out-of-range parts of the
// box are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, const void *src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 :: "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
                    "r"(static_cast<uint32_t>(__cvta_generic_to_shared(src)))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until the thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
#endif

}  // namespace q3
