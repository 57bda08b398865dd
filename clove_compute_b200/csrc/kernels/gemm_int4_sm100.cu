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
#endif

namespace clove {
namespace rt {

namespace {
std::atomic<uint64_t> g_attr_set[2];
inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

// TMA needs 16-byte row strides: K/2 bytes of codes (K % 32) and K/128 fp16 of
// scales / zero points (K % 1024); C rows of N fp16 (N % 8); aligned bases.
bool gemm_int4_tc_eligible(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                           const void* Bs, const void* Bz, const void* C, int M, int N, int K) {
  return M > 0 && N > 0 && K > 0 && K % 1024 == 0 && N % 8 == 0 && a16(Aq) && a16(Bq) &&
         a16(As) && a16(Az) && a16(Bs) && a16(Bz) && a16(C);
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
  if ((rc = encode_tmap_2d(&tAs, F16, 2, As, NG, M, NG * 2ull, 8, 128, 0))) return rc;
  if ((rc = encode_tmap_2d(&tAz, F16, 2, Az, NG, M, NG * 2ull, 8, 128, 0))) return rc;
  if ((rc = encode_tmap_2d(&tBs, F16, 2, Bs, NG, N, NG * 2ull, 8, 128, 0))) return rc;
  if ((rc = encode_tmap_2d(&tBz, F16, 2, Bz, NG, N, NG * 2ull, 8, 128, 0))) return rc;
  if ((rc = encode_tmap_2d(&tC, F16, 2, C, N, M, N * 2ull, 64, 32, 128))) return rc;
  const bool dbg = Gdbg != nullptr;
  auto kernel = dbg ? kern::gemm_int4_tc_kernel<true> : kern::gemm_int4_tc_kernel<false>;
  const uint64_t bit = 1ull << (dev.device & 63);
  if ((g_attr_set[dbg].load(std::memory_order_acquire) & bit) == 0) {
    rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::SMEM_BYTES),
                    "cudaFuncSetAttribute(int4 smem)");
    if (rc) return rc;
    g_attr_set[dbg].fetch_or(bit, std::memory_order_acq_rel);
  }
  kern::PeerOut peer = {};
  if (peer_targets != nullptr) {
    rc = encode_peer_maps(*peer_targets, M, N, 64, 128, &peer);
    if (rc) return rc;
  }
  const dim3 grid((N + S::BN - 1) / S::BN, (M + S::BM - 1) / S::BM, 1);
  kernel<<<grid, S::THREADS, S::SMEM_BYTES, stream>>>(tAq, tBq, tAs, tAz, tBs, tBz, tC, M, N, K,
                                                      Gdbg, peer);
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
