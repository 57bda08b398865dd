// ref_shim.cu -- C entry points onto the reference's own GEMM host functions, so the
// test harness can run the unmodified reference kernels (compiled from the
// reference tree by oracle/Makefile, target `ref`) and record their outputs as
// golden vectors. Test infrastructure only.
//
// gemm_int8 is deliberately not exposed: the reference int8 kernel reads shared
// memory out of bounds (gemm_int8.cu:77,84 index 128-wide rows of 68-byte tiles)
// and is never run.
#include <clove/kernels/gemm.cuh>

extern "C" int clove_ref_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K,
                                   float alpha, float beta, void* stream) {
  clove::gemm_fp16(static_cast<const half*>(A), static_cast<const half*>(B),
                   static_cast<half*>(C), M, N, K, alpha, beta,
                   static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}

extern "C" int clove_ref_gemm_int4(const void* A_q, const void* A_scale, const void* A_zero,
                                   const void* B_q, const void* B_scale, const void* B_zero,
                                   void* C, int M, int N, int K, void* stream) {
  clove::gemm_int4(static_cast<const uint8_t*>(A_q), static_cast<const half*>(A_scale),
                   static_cast<const half*>(A_zero), static_cast<const uint8_t*>(B_q),
                   static_cast<const half*>(B_scale), static_cast<const half*>(B_zero),
                   static_cast<half*>(C), M, N, K, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}
