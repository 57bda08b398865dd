// clove/common.cuh -- the clove common header: error macros, cdiv, DType, element
// traits, half vectors and warp / block reductions, with the names and behaviour of
// the reference's include/clove/common.cuh:1-121, so that this include/ can be put
// ahead of the reference's and the reference's other kernels (layernorm, softmax,
// activations, rope, attention) still compile against it.
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

// Element-type traits used by the reference's kernel templates (common.cuh:55-60).
template <typename T>
struct CudaType;
template <>
struct CudaType<float> {
  using type = float;
  static constexpr DType dtype = DType::FP32;
};
template <>
struct CudaType<half> {
  using type = half;
  static constexpr DType dtype = DType::FP16;
};
template <>
struct CudaType<int8_t> {
  using type = int8_t;
  static constexpr DType dtype = DType::INT8;
};

// Four and eight binary16 values, laid out as consecutive halves with the natural
// 2-byte alignment (the reference's half4 / half8, common.cuh:62-67).
struct half4 {
  half x, y, z, w;
};
struct half8 {
  half4 lo, hi;
};

#ifdef __CUDACC__
// Device helpers of the reference's common.cuh:64-119. They are compiled only by
// nvcc, so host-only translation units (.cpp) can include this header too.

__device__ __forceinline__ half4 make_half4(half a, half b, half c, half d) {
  half4 r;
  r.x = a;
  r.y = b;
  r.z = c;
  r.w = d;
  return r;
}

// Sum / max over the 32 lanes of a fully active warp; every lane gets the result.
// The sum folds lanes at XOR distances 16, 8, 4, 2, 1, so kernels written against
// the reference header round exactly as before.
__device__ __forceinline__ float warp_reduce_sum(float v) {
  for (int d = 16; d >= 1; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

__device__ __forceinline__ float warp_reduce_max(float v) {
  for (int d = 16; d >= 1; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

namespace detail {
// Per-warp partials -> warp 0. Every thread of the block must call it (it has
// block barriers). The leading barrier lets a kernel call the reductions back to
// back: no warp overwrites the partials before warp 0 has read the previous ones.
template <int BLOCK_SIZE, bool MAX>
__device__ __forceinline__ float block_reduce(float v) {
  static_assert(BLOCK_SIZE % 32 == 0 && BLOCK_SIZE <= 1024, "whole warps, at most 1024 threads");
  __shared__ float partial[32];
  const float pad = MAX ? __int_as_float(0xff800000) : 0.0f;  // -inf or 0
  const int lane = static_cast<int>(threadIdx.x & 31u);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  v = MAX ? warp_reduce_max(v) : warp_reduce_sum(v);
  __syncthreads();
  if (lane == 0) partial[warp] = v;
  __syncthreads();
  // Warp 0 folds the BLOCK_SIZE / 32 partials; the other warps return the pad value.
  v = static_cast<int>(threadIdx.x) < BLOCK_SIZE / 32 ? partial[lane] : pad;
  if (warp == 0) v = MAX ? warp_reduce_max(v) : warp_reduce_sum(v);
  return v;
}
}  // namespace detail

// Block-wide sum / max of one float per thread (BLOCK_SIZE threads). The result
// is valid in warp 0 (every lane of it); the other warps get 0 / -inf.
template <int BLOCK_SIZE>
__device__ __forceinline__ float block_reduce_sum(float v) {
  return detail::block_reduce<BLOCK_SIZE, false>(v);
}

template <int BLOCK_SIZE>
__device__ __forceinline__ float block_reduce_max(float v) {
  return detail::block_reduce<BLOCK_SIZE, true>(v);
}
#endif  // __CUDACC__

}  // namespace clove
