// Host-side encoding of TMA tensor maps.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "tensormap.h"

namespace slc {
namespace k {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

bool encode_tensor_map_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                          uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                          uint32_t box_inner, uint32_t box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                       uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                       uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tensor_map_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                          const uint64_t dims[3], const uint64_t strides_bytes[2],
                          const uint32_t box[3]) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    const cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
    const cuuint32_t bx[3] = {box[0], box[1], box[2]};
    const cuuint32_t elem[3] = {1, 1, 1};
    return fn(map, dtype, 3, const_cast<void *>(base), d, st, bx, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace k
}  // namespace slc
