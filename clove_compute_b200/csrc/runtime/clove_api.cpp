// clove_api.cpp -- the reference's C++ entry points (include/clove/kernels/gemm.cuh),
// forwarding to the C ABI. As in the reference (CLOVE_CHECK_LAST, common.cuh:11-21)
// a failure prints the reason and exits the process.
#include <cstdio>
#include <cstdlib>

#include "clove/kernels/attention_tc.cuh"
#include "clove/kernels/gemm.cuh"

namespace clove {

namespace {
void die_on_error(int rc, const char* what) {
  if (rc != CLOVE_OK) {
    fprintf(stderr, "clove::%s failed (%d): %s\n", what, rc, clove_last_error_string());
    exit(EXIT_FAILURE);
  }
}
}  // namespace

void gemm_fp16(const half* A, const half* B, half* C, int M, int N, int K, float alpha,
               float beta, cudaStream_t stream) {
  die_on_error(clove_gemm_fp16(A, B, C, M, N, K, alpha, beta, stream), "gemm_fp16");
}

void gemm_int8(const int8_t* A_q, const int8_t* B_q, half* C, int M, int N, int K, float A_scale,
               int8_t A_zero, float B_scale, int8_t B_zero, cudaStream_t stream) {
  die_on_error(clove_gemm_int8(A_q, B_q, C, M, N, K, A_scale, A_zero, B_scale, B_zero, stream),
               "gemm_int8");
}

void gemm_int8_rowcol(const int8_t* A_q, const int8_t* B_q, half* C, int M, int N, int K,
                      const float* A_row_scale, const float* B_col_scale, cudaStream_t stream) {
  die_on_error(
      clove_gemm_int8_rowcol(A_q, B_q, C, M, N, K, A_row_scale, B_col_scale, stream),
      "gemm_int8_rowcol");
}

void gemm_int4(const uint8_t* A_q, const half* A_scale, const half* A_zero, const uint8_t* B_q,
               const half* B_scale, const half* B_zero, half* C, int M, int N, int K,
               cudaStream_t stream) {
  die_on_error(
      clove_gemm_int4(A_q, A_scale, A_zero, B_q, B_scale, B_zero, C, M, N, K, stream),
      "gemm_int4");
}

void gemm_fp16_batched(const half* A, const half* B, half* C, int batch, int M, int N, int K,
                       float alpha, float beta, cudaStream_t stream) {
  die_on_error(clove_gemm_fp16_batched(A, B, C, batch, M, N, K, alpha, beta, stream),
               "gemm_fp16_batched");
}

void swiglu_fused(const half* input, const half* W_gate, const half* W_up, half* output,
                  int batch_seq, int hidden_dim, int intermediate_dim, cudaStream_t stream) {
  die_on_error(clove_swiglu_fused(input, W_gate, W_up, output, batch_seq, hidden_dim,
                                  intermediate_dim, stream),
               "swiglu_fused");
}

void flash_attention_tc(const half* Q, const half* K, const half* V, half* O, int batch,
                        int num_heads, int seq_len, int head_dim, float scale, bool causal,
                        cudaStream_t stream) {
  die_on_error(clove_flash_attention(Q, K, V, O, batch, num_heads, num_heads, seq_len, head_dim,
                                     scale, causal ? 1 : 0, 0, stream),
               "flash_attention_tc");
}

void flash_attention_tc_bshd(const half* Q, const half* K, const half* V, half* O, int batch,
                             int num_heads, int num_kv_heads, int seq_len, int head_dim,
                             float scale, bool causal, cudaStream_t stream) {
  die_on_error(clove_flash_attention(Q, K, V, O, batch, num_heads, num_kv_heads, seq_len,
                                     head_dim, scale, causal ? 1 : 0, 1, stream),
               "flash_attention_tc_bshd");
}

}  // namespace clove
