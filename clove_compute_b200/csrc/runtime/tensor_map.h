// tensor_map.h -- CUtensorMap encoding for the TMA-fed kernels.
#pragma once

#include <cuda.h>
#include <cstdint>

namespace clove {
namespace rt {

// Encodes a 2D row-major tensor [outer, inner] (inner contiguous, rows
// row_stride_bytes apart) for tiled TMA with a box of [box_outer, box_inner]
// elements and the given swizzle width in bytes (0 = none, 32, 64, 128).
// Out-of-bounds box elements read as zero and are clipped on store.
// Returns CLOVE_OK or an error code with the message recorded.
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_outer, int swizzle_bytes);

// As encode_tmap_2d for a stack of `depth` such matrices, plane_stride_bytes apart
// (a batch): a 3D tensor [depth, outer, inner] with a box one plane deep, so that
// out-of-bounds rows of one matrix never read or write its neighbour.
int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t depth, uint64_t row_stride_bytes,
                   uint64_t plane_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   int swizzle_bytes);

// A 4D tensor [d3, d2, d1, d0] (d0 contiguous) with arbitrary byte strides of the
// three outer dimensions, for a box [1, 1, box_outer, box_inner]: e.g. attention
// operands [batch, heads, seq, head_dim] or [batch, seq, heads, head_dim] viewed as
// (head_dim, seq, heads, batch) with the matching strides.
int encode_tmap_4d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   const uint64_t dims[4], const uint64_t strides_bytes[3], uint32_t box_inner,
                   uint32_t box_outer, int swizzle_bytes);

}  // namespace rt
}  // namespace clove
