// gemm_int4_sm100.cu -- host launcher of the INT4 tcgen05 kernel (gemm_int4_sm100.cuh).
#include <atomic>

#include "gemm_int4_sm100.cuh"
#include "../runtime/internal.h"
#include "../runtime/tensor_map.h"

namespace clove {
namespace rt {

CLOVE_DEFINE_ERROR_READER(read_clear_error_int4)

}  // namespace rt
}  // namespace clove

#ifdef CLOVE_TRACE
// Development builds only: trace slots of the INT4 kernel.
extern "C" int clove_trace_read_int4(unsigned long long* out) {
  return static_cast<int>(cudaMemcpyFromSymbol(out, g_clove_trace, sizeof(unsigned long long) * 256));
}
extern "C" int clove_trace_write_int4(const unsigned long long* in) {
  return static_cast<int>(cudaMemcpyToSymbol(g_clove_trace, in, sizeof(unsigned long long) * 256));
}
#endif

namespace clove {
namespace rt {

namespace {
std::atomic<uint64_t> g_attr_set[4];
inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

// Codes and C go through TMA: 16-byte row strides (K/2 bytes of codes, K % 32;
// N fp16 of C, N % 8) and aligned bases. Scales and zero points go through TMA
// too when their rows (K/128 fp16) are 16-byte multiples (K % 1024) and their
// bases are aligned; otherwise the transform warps read them directly, which
// needs only K % 128 and 2-byte alignment.
namespace {
bool meta_by_tma(const void* As, const void* Az, const void* Bs, const void* Bz, int K) {
  return K % 1024 == 0 && a16(As) && a16(Az) && a16(Bs) && a16(Bz);
}
inline bool a2(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 1u) == 0; }
}  // namespace

bool gemm_int4_tc_eligible(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                           const void* Bs, const void* Bz, const void* C, int M, int N, int K) {
  return M > 0 && N > 0 && K > 0 && K % 128 == 0 && N % 8 == 0 && a16(Aq) && a16(Bq) &&
         a16(C) && a2(As) && a2(Az) && a2(Bs) && a2(Bz);
}

int launch_gemm_int4_tc(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                        const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int M, int N,
                        int K, const DeviceInfo& dev, cudaStream_t stream,
                        const PeerTargets* peer_targets) {
  using S = kern::I4Shape;
  const int NG = K / 128;
  CUtensorMap tAq, tBq, tAs, tAz, tBs, tBz, tC;
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc;
  if ((rc = encode_tmap_2d(&tAq, U8, 1, Aq, K / 2, M, K / 2, 64, 128, 64))) return rc;
  if ((rc = encode_tmap_2d(&tBq, U8, 1, Bq, K / 2, N, K / 2, 64, 128, 64))) return rc;
  const bool tmeta = meta_by_tma(As, Az, Bs, Bz, K);
  if (tmeta) {
    if ((rc = encode_tmap_2d(&tAs, F16, 2, As, NG, M, NG * 2ull, 8, 128, 0))) return rc;
    if ((rc = encode_tmap_2d(&tAz, F16, 2, Az, NG, M, NG * 2ull, 8, 128, 0))) return rc;
    if ((rc = encode_tmap_2d(&tBs, F16, 2, Bs, NG, N, NG * 2ull, 8, 128, 0))) return rc;
    if ((rc = encode_tmap_2d(&tBz, F16, 2, Bz, NG, N, NG * 2ull, 8, 128, 0))) return rc;
  } else {
    tAs = tAz = tBs = tBz = tAq;  // unused by the direct-load variant
  }
  if ((rc = encode_tmap_2d(&tC, F16, 2, C, N, M, N * 2ull, 64, 32, 128))) return rc;
  const bool dbg = Gdbg != nullptr;
  const int variant = (dbg ? 1 : 0) | (tmeta ? 2 : 0);
  decltype(&kern::gemm_int4_tc_kernel<false, true>) kernel = nullptr;
  switch (variant) {
    case 0: kernel = kern::gemm_int4_tc_kernel<false, false>; break;
    case 1: kernel = kern::gemm_int4_tc_kernel<true, false>; break;
    case 2: kernel = kern::gemm_int4_tc_kernel<false, true>; break;
    default: kernel = kern::gemm_int4_tc_kernel<true, true>; break;
  }
  const uint64_t bit = 1ull << (dev.device & 63);
  if ((g_attr_set[variant].load(std::memory_order_acquire) & bit) == 0) {
    // The kernel moves registers between its warpgroups with setmaxnreg, planned for
    // a launch allocation of S::REGS_LAUNCH per thread: with fewer, an increase
    // would wait forever, so such a build is refused here rather than launched.
    cudaFuncAttributes fa{};
    rc = check_cuda(cudaFuncGetAttributes(&fa, kernel), "cudaFuncGetAttributes(int4)");
    if (rc) return rc;
    if (fa.numRegs != S::REGS_LAUNCH)
      return fail(CLOVE_ERR_UNSUPPORTED,
                  "gemm_int4_tc: built with %d registers per thread, its register plan needs %d",
                  fa.numRegs, S::REGS_LAUNCH);
    rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::SMEM_BYTES),
                    "cudaFuncSetAttribute(int4 smem)");
    if (rc) return rc;
    g_attr_set[variant].fetch_or(bit, std::memory_order_acq_rel);
  }
  kern::I4Meta meta = {static_cast<const __half*>(As), static_cast<const __half*>(Az),
                       static_cast<const __half*>(Bs), static_cast<const __half*>(Bz)};
  kern::PeerOut peer = {};
  if (peer_targets != nullptr) {
    rc = encode_peer_maps(*peer_targets, M, N, 64, 128, &peer);
    if (rc) return rc;
  }
  const dim3 grid((N + S::BN - 1) / S::BN, (M + S::BM - 1) / S::BM, 1);
  kernel<<<grid, S::THREADS, S::SMEM_BYTES, stream>>>(tAq, tBq, tAs, tAz, tBs, tBz, tC, M, N, K,
                                                      Gdbg, peer, meta);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kernel);
    return fail(CLOVE_ERR_CUDA,
                "gemm_int4_tc launch: %s (regs %d, max threads %d, dyn smem %d of %d)",
                cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, S::SMEM_BYTES,
                fa.maxDynamicSharedSizeBytes);
  }
  return CLOVE_OK;
}

}  // namespace rt
}  // namespace clove
