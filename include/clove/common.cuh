// clove/common.cuh -- helpers the GEMM boundary header needs (the subset of the
// reference's include/clove/common.cuh:11-53 used on the GEMM path).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

namespace clove {

// Print and exit on a CUDA error, as the reference's macros do (common.cuh:11-27).
#define CLOVE_CHECK_CUDA(call)                                                   \
  do {                                                                           \
    cudaError_t clove_err_ = (call);                                             \
    if (clove_err_ != cudaSuccess) {                                             \
      fprintf(stderr, "CUDA error at %s:%d: %s\n", __FILE__, __LINE__,           \
              cudaGetErrorString(clove_err_));                                   \
      exit(EXIT_FAILURE);                                                        \
    }                                                                            \
  } while (0)

#define CLOVE_CHECK_LAST() CLOVE_CHECK_CUDA(cudaGetLastError())

#define CLOVE_SYNC_CHECK()                         \
  do {                                             \
    CLOVE_CHECK_CUDA(cudaDeviceSynchronize());     \
    CLOVE_CHECK_LAST();                            \
  } while (0)

constexpr int cdiv(int a, int b) { return (a + b - 1) / b; }

enum class DType { FP32, FP16, BF16, INT8, INT4 };

inline size_t dtype_size(DType dtype) {
  switch (dtype) {
    case DType::FP32: return 4;
    case DType::FP16: return 2;
    case DType::BF16: return 2;
    case DType::INT8: return 1;
    case DType::INT4: return 0;  // two values per byte
  }
  return 0;
}

}  // namespace clove
