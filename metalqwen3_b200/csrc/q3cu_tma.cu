// q3cu_tma.cu -- host side of the tensor maps (q3cu_tma.h).
#include "q3cu_tma.h"

#include <mutex>

namespace q3 {

namespace {
typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}
}  // namespace

namespace {
// The last few encoded maps of this host thread: a launcher called again on the
// same buffer with the same shape (every step of a loop) skips the encode.
struct MapKey {
    const void *base;
    uint64_t rows, row_bytes;
    uint32_t L, R;                       // L == 0: the 2-D map of encode_rows_2d_map
    bool operator==(const MapKey &o) const {
        return base == o.base && rows == o.rows && row_bytes == o.row_bytes && L == o.L && R == o.R;
    }
};
constexpr int kMapCache = 8;
thread_local MapKey t_keys[kMapCache];
thread_local CUtensorMap t_maps[kMapCache];
thread_local int t_used = 0, t_next = 0;
}  // namespace

static bool cache_lookup(const MapKey &key, CUtensorMap *map) {
    for (int i = 0; i < t_used; ++i)
        if (t_keys[i] == key) {
            *map = t_maps[i];
            return true;
        }
    return false;
}
static void cache_store(const MapKey &key, const CUtensorMap &map) {
    t_keys[t_next] = key;
    t_maps[t_next] = map;
    t_next = (t_next + 1) % kMapCache;
    if (t_used < kMapCache) ++t_used;
}

bool encode_row_lines_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes, uint32_t L,
                          uint32_t R) {
    const MapKey key{base, rows, row_bytes, L, R};
    if (cache_lookup(key, map)) return true;
    if (!encode_row_lines_map_uncached(map, base, rows, row_bytes, L, R)) return false;
    cache_store(key, *map);
    return true;
}

bool encode_rows_2d_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
    const MapKey key{base, rows, row_bytes, 0, box_rows};
    if (cache_lookup(key, map)) return true;
    EncodeTiled enc = encoder();
    if (!enc || rows == 0 || row_bytes % 128 || (reinterpret_cast<uintptr_t>(base) % 16) || box_rows == 0 ||
        box_rows > 256)
        return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {128, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    cache_store(key, *map);
    return true;
}

bool encode_f32_2d_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                       uint32_t box_rows, bool swizzle128) {
    // keyed apart from the byte maps: L = box_cols | 1 << 31 (| 1 << 30 swizzled) never occurs there
    const MapKey key{base, rows, cols, box_cols | 0x80000000u | (swizzle128 ? 0x40000000u : 0u), box_rows};
    if (cache_lookup(key, map)) return true;
    EncodeTiled enc = encoder();
    if (!enc || rows == 0 || cols % 4 || (reinterpret_cast<uintptr_t>(base) % 16) || box_cols == 0 ||
        (box_cols * 4) % 16 || box_cols > 256 || box_rows == 0 || box_rows > 256 || (swizzle128 && box_cols != 32))
        return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    cache_store(key, *map);
    return true;
}

bool encode_row_lines_map_uncached(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes,
                                   uint32_t L, uint32_t R) {
    EncodeTiled enc = encoder();
    if (!enc || rows == 0 || row_bytes % 128 || (reinterpret_cast<uintptr_t>(base) % 16) || L == 0 || L > 256 ||
        R == 0 || R > 256)
        return false;
    const cuuint64_t dims[3] = {128, row_bytes / 128, rows};
    const cuuint64_t strides[2] = {128, row_bytes};
    const cuuint32_t box[3] = {128, L, R};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace q3
