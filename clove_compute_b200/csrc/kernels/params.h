// params.h -- plain parameter structs shared by the kernels and the host launchers.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace clove {
namespace kern {

enum EpiMode : int {
  kEpiF16AlphaBeta = 0,  // C = half(alpha*acc + beta*C)
  kEpiI8Tensor = 1,      // C = half(float(acc') * scale)
  kEpiI8RowCol = 2,      // C = half(float(acc) * row_scale[m] * col_scale[n])
  kEpiI32Raw = 3,        // C(int32) = acc'  (acc' = zero-point corrected acc)
};

// Epilogue of the tensor-core tile kernels.
struct EpiParams {
  int mode;
  float alpha, beta;        // kEpiF16AlphaBeta
  const __half* c_in;       // beta source, row-major [M,N] (may alias C)
  float scale;              // kEpiI8Tensor: A_scale * B_scale
  const float* row_scale;   // kEpiI8RowCol
  const float* col_scale;
  int za, zb;               // int8 zero points
  const int32_t* row_sum;   // sum_k A[m,k]   (required when zb != 0)
  const int32_t* col_sum;   // sum_k B[k,n]   (required when za != 0)
  void* c_out;              // C itself (split-K tiles store rows directly)
};

// Epilogue of the int8 GEMV (modes as EpiMode 1..3).
struct GemvI8Epi {
  int mode;
  float scale;
  const float* row_scale;   // [rows]
  const float* col_scale;   // [NC]
  int za, zb;
};

// Epilogue of the SIMT fallback (modes as EpiMode 0..3).
struct SimtEpi {
  int mode;
  float alpha, beta;
  float scale;
  const float* row_scale;
  const float* col_scale;
  int za, zb;
};

}  // namespace kern
}  // namespace clove
