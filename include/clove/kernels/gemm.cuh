// clove/kernels/gemm.cuh -- drop-in GEMM boundary for the clove runtime, B200 build.
//
// Same namespace, names, argument order, default arguments and row-major layouts as
// the reference header include/clove/kernels/gemm.cuh:41-101, so the runtime's
// linear layers (src/runtime/inference.cu:139-194) link against this library
// unchanged. The functions forward to the C ABI in clove/capi.h. Like the
// reference (common.cuh:11-21 via CLOVE_CHECK_LAST), a failure prints a message
// and exits; callers that want status codes use the clove_* C functions.
#pragma once

#include <clove/common.cuh>
#include <clove/capi.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace clove {

// C = alpha * A @ B + beta * C ; A [M,K], B [K,N], C [M,N] row-major fp16,
// fp32 accumulation on tcgen05 tensor cores (gemm.cuh:37-49).
void gemm_fp16(const half* A, const half* B, half* C, int M, int N, int K, float alpha = 1.0f,
               float beta = 0.0f, cudaStream_t stream = 0);

// C = (A_q - A_zero) * A_scale @ (B_q - B_zero) * B_scale ; per-tensor quantisation,
// A_q [M,K], B_q [K,N] int8 row-major, int32 accumulation (gemm.cuh:55-65).
void gemm_int8(const int8_t* A_q, const int8_t* B_q, half* C, int M, int N, int K, float A_scale,
               int8_t A_zero, float B_scale, int8_t B_zero, cudaStream_t stream = 0);

// Per-row / per-column scaled variant (extension; zero points 0).
void gemm_int8_rowcol(const int8_t* A_q, const int8_t* B_q, half* C, int M, int N, int K,
                      const float* A_row_scale, const float* B_col_scale,
                      cudaStream_t stream = 0);

constexpr int INT4_GROUP_SIZE = 128;  // gemm.cuh:72

// INT4 group-wise GEMM. Layout (K-packed on both operands):
//   A_q [M, K/2], A_scale / A_zero [M, K/128]
//   B_q [N, K/2], B_scale / B_zero [N, K/128]
// element 2j of a row in the high nibble of byte j; codes 0..15; zero points are
// integer codes. C[m,n] = sum_g sA*sB*sum_{k in g}(a-za)(b-zb). (The reference
// header's comment gives B as [K, N/2]; see clove/capi.h for the exact contract.)
void gemm_int4(const uint8_t* A_q, const half* A_scale, const half* A_zero, const uint8_t* B_q,
               const half* B_scale, const half* B_zero, half* C, int M, int N, int K,
               cudaStream_t stream = 0);

// Batched: A [B,M,K], B [B,K,N], C [B,M,N] (gemm.cuh:93-101).
void gemm_fp16_batched(const half* A, const half* B, half* C, int batch, int M, int N, int K,
                       float alpha = 1.0f, float beta = 0.0f, cudaStream_t stream = 0);

// The reference declares swiglu_fused in include/clove/kernels/activations.cuh:37-46
// (with `stream = 0`) and never defines it; this library defines it (one CTA-pair
// GEMM computing both projections, silu(gate) * up in the epilogue). Declared here
// without a default argument so that both headers can be included together.
void swiglu_fused(const half* input, const half* W_gate, const half* W_up, half* output,
                  int batch_seq, int hidden_dim, int intermediate_dim, cudaStream_t stream);

}  // namespace clove
