// gemm_int8_noalloc.cu -- clove_gemm_int8_noalloc: the int8 GEMM (reference
// signature) with no device-memory allocation at all.
//
// Why: clove_gemm_int8 with non-zero zero points needs int32 row sums of A and
// column sums of B, which it keeps in stream-ordered scratch from
// cudaMallocAsync. Some callers cannot let a library allocate: serving runtimes
// that reserve all of HBM up front for their own pools (a stray allocation can
// fail with out-of-memory in the middle of serving), and hosts that budget every
// device byte at start-up. This entry point keeps those sums in a fixed array
// compiled into the library instead.
//
// The array is a file-scope `static __device__` object of kNoAllocMaxSums int32
// entries (256 KiB), present on every GPU that loads the library until the
// process exits. A call needs M + N entries; larger shapes are rejected with
// CLOVE_ERR_UNSUPPORTED. Host code cannot use the array's name as a device
// address, so the first call on each device asks the runtime for the address
// (cudaGetSymbolAddress, with that device current) and caches it; make that first
// call before any stream capture. All calls share the one array: every entry a
// call reads is written earlier in the same call, and calls whose kernels overlap
// on the GPU (two streams, or two host threads) race on it.
#include <cuda_runtime.h>

#include <mutex>

#include "../kernels/params.h"
#include "internal.h"

namespace clove {
namespace rt {
namespace {

constexpr int kNoAllocMaxSums = CLOVE_NOALLOC_MAX_SUMS;  // int32 entries: M + N
static __device__ __align__(256) int32_t g_noalloc_sums[kNoAllocMaxSums];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int32_t* g_sums_on_device[kMaxDevices] = {};

// Device address of g_noalloc_sums on the current device (looked up once per device).
int sums_address(int device, int32_t** out) {
  if (device < 0 || device >= kMaxDevices) return fail(CLOVE_ERR_DEVICE, "device ordinal %d", device);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sums_on_device[device] == nullptr) {
    void* p = nullptr;
    const int rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_sums),
                              "cudaGetSymbolAddress(no-alloc scratch)");
    if (rc) return rc;
    g_sums_on_device[device] = static_cast<int32_t*>(p);
  }
  *out = g_sums_on_device[device];
  return CLOVE_OK;
}

}  // namespace
}  // namespace rt
}  // namespace clove

using namespace clove;
using namespace clove::rt;

extern "C" int clove_gemm_int8_noalloc(const int8_t* A_q, const int8_t* B_q, void* C, int M,
                                       int N, int K, float A_scale, int8_t A_zero, float B_scale,
                                       int8_t B_zero, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative size");
  if (M == 0 || N == 0) return CLOVE_OK;
  if (A_q == nullptr || B_q == nullptr || C == nullptr)
    return fail(CLOVE_ERR_INVALID_ARG, "null matrix pointer");
  // The kernel family clove_gemm_int8 would pick for this shape (its automatic
  // dispatch and the test override alike), so both entry points run the same
  // kernel and give the same bits.
  const char* family = nullptr;
  int rc = int8_route(A_q, B_q, C, M, N, K, &family);
  if (rc) return rc;
  // Without zero points, or on the GEMV / SIMT kernels (which keep their sums in
  // registers), the ordinary entry point allocates nothing.
  const bool tile = family[0] == 't';
  if ((A_zero == 0 && B_zero == 0) || !tile)
    return clove_gemm_int8(A_q, B_q, C, M, N, K, A_scale, A_zero, B_scale, B_zero, stream);
  if (static_cast<long long>(M) + N > kNoAllocMaxSums)
    return fail(CLOVE_ERR_UNSUPPORTED,
                "clove_gemm_int8_noalloc: M + N = %lld exceeds the %d-entry static scratch "
                "(use clove_gemm_int8)",
                static_cast<long long>(M) + N, kNoAllocMaxSums);
  DeviceInfo dev;
  rc = current_device(&dev);
  if (rc) return rc;
  int32_t* sums = nullptr;
  rc = sums_address(dev.device, &sums);
  if (rc) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Row sums of A (for the B zero point) at [0, M), column sums of B at [M, M+N);
  // each is rewritten by this call before the GEMM reads it.
  if (B_zero != 0) rc = launch_int8_row_sums(A_q, sums, M, K, s);
  if (!rc && A_zero != 0) rc = launch_int8_col_sums(B_q, sums + M, K, N, s);
  if (rc) return rc;
  const TcPlan plan = plan_tc(M, N, K, 1, dev.num_sms);
  kern::EpiParams ep{};
  ep.mode = kern::kEpiI8Tensor;
  ep.scale = A_scale * B_scale;
  ep.za = A_zero;
  ep.zb = B_zero;
  ep.row_sum = sums;
  ep.col_sum = sums + M;
  // CTA pairs with whole-K tiles only: the stream-K schedule would need a
  // workspace. Its sums are the same (exact int32), so results do not change.
  if (family[2] == '2')
    return launch_gemm_tc2(kTcI8, A_q, B_q, C, M, N, K, ep, dev, s, nullptr, nullptr, false);
  return launch_gemm_tc(kTcI8, plan.bn, plan.split, 2, A_q, B_q, C, M, N, K, ep, dev, s);
}
