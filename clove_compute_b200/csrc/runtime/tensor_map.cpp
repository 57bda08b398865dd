// tensor_map.cpp -- CUtensorMap encoding through the driver entry point (no -lcuda).
#include "tensor_map.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "internal.h"

namespace clove {
namespace rt {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

void resolve_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

namespace {
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                int rank, const uint64_t* dims_in, const uint64_t* strides_in, uint32_t box_inner,
                uint32_t box_outer, int swizzle_bytes) {
  std::call_once(g_encode_once, resolve_encode);
  if (g_encode == nullptr)
    return fail(CLOVE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(CLOVE_ERR_UNSUPPORTED, "TMA needs a 16-byte aligned base");
  for (int i = 0; i + 1 < rank; ++i)
    if ((strides_in[i] & 15u) != 0)
      return fail(CLOVE_ERR_UNSUPPORTED, "TMA needs 16-byte multiple strides");
  if (static_cast<uint64_t>(box_inner) * elem_bytes % 16 != 0)
    return fail(CLOVE_ERR_UNSUPPORTED, "TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return fail(CLOVE_ERR_INVALID_ARG, "bad swizzle width %d", swizzle_bytes);
  }
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  const cuuint32_t box[4] = {box_inner, box_outer, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) dims[i] = static_cast<cuuint64_t>(dims_in[i]);
  for (int i = 0; i + 1 < rank; ++i) strides[i] = static_cast<cuuint64_t>(strides_in[i]);
  const CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(CLOVE_ERR_UNSUPPORTED,
                "cuTensorMapEncodeTiled failed (%d): rank %d dims %llu x %llu x %llu box %u x %u sw %d",
                static_cast<int>(r), rank, static_cast<unsigned long long>(dims_in[0]),
                static_cast<unsigned long long>(dims_in[1]),
                static_cast<unsigned long long>(rank > 2 ? dims_in[2] : 1), box_inner, box_outer,
                swizzle_bytes);
  return CLOVE_OK;
}
}  // namespace

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_outer, int swizzle_bytes) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_stride_bytes};
  return encode_tmap(map, dtype, elem_bytes, base, 2, dims, strides, box_inner, box_outer,
                     swizzle_bytes);
}

int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t depth, uint64_t row_stride_bytes,
                   uint64_t plane_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   int swizzle_bytes) {
  const uint64_t dims[3] = {inner, outer, depth};
  const uint64_t strides[2] = {row_stride_bytes, plane_stride_bytes};
  return encode_tmap(map, dtype, elem_bytes, base, 3, dims, strides, box_inner, box_outer,
                     swizzle_bytes);
}

int encode_tmap_4d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   const uint64_t dims[4], const uint64_t strides_bytes[3], uint32_t box_inner,
                   uint32_t box_outer, int swizzle_bytes) {
  return encode_tmap(map, dtype, elem_bytes, base, 4, dims, strides_bytes, box_inner, box_outer,
                     swizzle_bytes);
}

}  // namespace rt
}  // namespace clove
