// Host-side encoding of TMA tensor maps (driver entry point resolved once
// through the runtime, so the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace slc {
namespace k {

// A 2-D row-major tensor [rows][inner] of `dtype`, rows `row_stride_bytes`
// apart, copied in boxes of [box_rows][box_inner] without swizzle; elements
// outside the tensor read as zero. Returns false when the driver refuses.
bool encode_tensor_map_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                          uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                          uint32_t box_inner, uint32_t box_rows);

// The same with an optional 128-byte swizzle (box_inner * element size must
// then be at most 128 bytes; the shared destination 1024-byte aligned).
bool encode_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                       uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                       uint32_t box_inner, uint32_t box_rows, bool swizzle128);

// A 3-D tensor [dims[2]][dims[1]][dims[0]] of `dtype` (dims[0] contiguous;
// strides_bytes[0] between dim-1 entries, strides_bytes[1] between dim-2
// entries), copied in boxes of box[0] x box[1] x box[2] without swizzle.
bool encode_tensor_map_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                          const uint64_t dims[3], const uint64_t strides_bytes[2],
                          const uint32_t box[3]);

}  // namespace k
}  // namespace slc
