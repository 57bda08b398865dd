// clove/kernels/attention_tc.cuh -- tensor-core attention for the clove runtime.
//
// The reference declares clove::flash_attention (include/clove/kernels/attention.cuh:44-56)
// and defines it in src/kernels/attention.cu beside apply_rope and flash_attention_rope,
// so a library cannot take over that one symbol without the rest of that file. These
// functions keep its argument list and meaning under their own names; a runtime swaps
// the call (`flash_attention(...)` -> `flash_attention_tc(...)`), and the reference's
// other attention code stays as it is.
#pragma once

#include <clove/capi.h>
#include <clove/common.cuh>
#include <cuda_fp16.h>

namespace clove {

// Q, K, V, O: [batch, num_heads, seq_len, head_dim] (the reference's flash_attention).
// head_dim 128. Prints and exits on failure, as the reference's CLOVE_CHECK_LAST.
void flash_attention_tc(const half* Q, const half* K, const half* V, half* O, int batch,
                        int num_heads, int seq_len, int head_dim, float scale, bool causal,
                        cudaStream_t stream = 0);

// Q, O: [batch, seq_len, num_heads, head_dim]; K, V: [batch, seq_len, num_kv_heads,
// head_dim] -- the runtime's q/k/v projection outputs (inference.cu:138-161), after
// RoPE. num_heads a multiple of num_kv_heads (grouped-query attention).
void flash_attention_tc_bshd(const half* Q, const half* K, const half* V, half* O, int batch,
                             int num_heads, int num_kv_heads, int seq_len, int head_dim,
                             float scale, bool causal, cudaStream_t stream = 0);

}  // namespace clove
