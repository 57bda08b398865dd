// gemm_int4_sm100.cu -- INT4 tensor-core GEMM (kind::i8 with in-smem nibble unpack).
// Placeholder TU: the tensor-core path is not yet enabled, so every large INT4
// shape reports ineligible and the dispatcher uses the GEMV or SIMT kernels.
#include "sm100_ptx.cuh"
#include "../runtime/internal.h"

namespace clove {
namespace rt {

CLOVE_DEFINE_ERROR_READER(read_clear_error_int4)

bool gemm_int4_tc_eligible(const uint8_t*, const void*, const void*, const uint8_t*, const void*,
                           const void*, const void*, int, int, int) {
  return false;
}

int launch_gemm_int4_tc(const uint8_t*, const void*, const void*, const uint8_t*, const void*,
                        const void*, void*, int, int, int, const DeviceInfo&, cudaStream_t) {
  return fail(CLOVE_ERR_UNSUPPORTED, "int4 tensor-core kernel not built");
}

}  // namespace rt
}  // namespace clove
