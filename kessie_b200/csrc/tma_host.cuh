// tma_host.cuh -- host-side TMA descriptor encoding through the driver entry point
// (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string.h>

namespace kessie {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// Tensor map over the paged K (or V) cache of one layer, viewed as the 5-D
// tensor [d_lo 64][token ps][d_hi D/64][head H][page P] (innermost first).
// One box = one 16-token slice of one head of one page:
// {64, 16, D/64, 1, 1} elements, 128-byte swizzled rows in shared memory
// (row r = d_hi*16 + token, so ldmatrix row groups never share a bank set).
// Returns CUDA_SUCCESS or the driver's error.
inline CUresult encode_kv_tile_map(CUtensorMap* map, const void* base, bool bf16, int head_dim, int page_size,
                                   int num_heads, int num_pages, int64_t token_stride, int64_t head_stride,
                                   int64_t page_stride) {
    auto enc = tensor_map_encoder();
    if (!enc) return CUDA_ERROR_NOT_SUPPORTED;
    const int dhi = head_dim / 64;
    cuuint64_t dims[5] = {64, (cuuint64_t)page_size, (cuuint64_t)dhi, (cuuint64_t)num_heads, (cuuint64_t)num_pages};
    cuuint64_t strides[4] = {(cuuint64_t)token_stride * 2, 128, (cuuint64_t)head_stride * 2, (cuuint64_t)page_stride * 2};
    cuuint32_t box[5] = {64, 16, (cuuint32_t)dhi, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
               const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// encode_kv_tile_map through a small cache of the last 8 distinct argument
// sets: the encode is pure host work, but a per-call cost of a decode step.
inline CUresult encode_kv_tile_map_cached(CUtensorMap* map, const void* base, bool bf16, int head_dim, int page_size,
                                          int num_heads, int num_pages, int64_t token_stride, int64_t head_stride,
                                          int64_t page_stride) {
    struct Entry { bool used; const void* base; int64_t key[8]; CUtensorMap map; };
    static Entry cache[8];
    static int next = 0;
    static std::mutex mu;
    const int64_t key[8] = {bf16 ? 1 : 0, head_dim, page_size, num_heads, num_pages, token_stride, head_stride,
                            page_stride};
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Entry& e : cache)
            if (e.used && e.base == base && memcmp(e.key, key, sizeof(key)) == 0) {
                *map = e.map;
                return CUDA_SUCCESS;
            }
    }
    const CUresult r = encode_kv_tile_map(map, base, bf16, head_dim, page_size, num_heads, num_pages, token_stride,
                                          head_stride, page_stride);
    if (r == CUDA_SUCCESS) {
        std::lock_guard<std::mutex> lock(mu);
        Entry& e = cache[next];
        next = (next + 1) % 8;
        e.used = true;
        e.base = base;
        memcpy(e.key, key, sizeof(key));
        e.map = *map;
    }
    return r;
}

// Generic 5-D tiled tensor map with 128-byte swizzle (16-bit elements).
// strides_bytes: dims 1..4.  Returns the driver's result.
inline CUresult encode_tiled_5d_sw128(CUtensorMap* map, const void* base, bool bf16, const cuuint64_t dims[5],
                                      const cuuint64_t strides_bytes[4], const cuuint32_t box[5]) {
    auto enc = tensor_map_encoder();
    if (!enc) return CUDA_ERROR_NOT_SUPPORTED;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
               const_cast<void*>(base), dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Tensor map over an fp32 K (or V) cache for the fp32 decode: one box = 8
// tokens of one head, all of head_dim, as rows of 32 floats (128 bytes,
// 128-byte swizzled); row d_hi * 8 + token holds dims [32 d_hi, 32 d_hi + 32).
// Paged (num_pages > 0): the 5-D tensor [32][page_size][D/32][heads][pages],
// coordinates (0, token in page, 0, head, page).  Dense (num_pages == 0): the
// 4-D tensor [32][tokens][D/32][heads], coordinates (0, token, 0, head); rows
// past `tokens` read as zeros.  Strides in elements.
inline CUresult encode_f32_kv_map(CUtensorMap* map, const void* base, int head_dim, int tokens, int num_heads,
                                  int num_pages, int64_t token_stride, int64_t head_stride, int64_t page_stride) {
    auto enc = tensor_map_encoder();
    if (!enc) return CUDA_ERROR_NOT_SUPPORTED;
    const int rank = num_pages > 0 ? 5 : 4;
    cuuint64_t dims[5] = {32, (cuuint64_t)tokens, (cuuint64_t)(head_dim / 32), (cuuint64_t)num_heads,
                          (cuuint64_t)(num_pages > 0 ? num_pages : 1)};
    cuuint64_t strides[4] = {(cuuint64_t)token_stride * 4, 128, (cuuint64_t)head_stride * 4,
                             (cuuint64_t)page_stride * 4};
    cuuint32_t box[5] = {32, 8, (cuuint32_t)(head_dim / 32), 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace kessie
