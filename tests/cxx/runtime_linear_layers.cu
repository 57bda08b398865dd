// Compile-and-link check of the drop-in C++ boundary: the call forms the
// reference runtime's linear layers use (src/runtime/inference.cu:139-194), plus
// the other entry points of clove/kernels/gemm.cuh, built against this library's
// headers and linked against its shared library. The CPU test suite compiles and
// links it; running it needs a GPU (it then checks one status and exits 0).
#include <clove/kernels/gemm.cuh>

#include <cstdio>

namespace {
// A transformer block's projections as the reference runtime issues them.
void block_forward(const half* X, const half* Wq, const half* Wk, const half* Wv, const half* Wo,
                   const half* W_gate, const half* W_up, const half* W_down, half* q, half* k,
                   half* v, half* attn, half* hidden, half* mlp, int T, int H, int I,
                   cudaStream_t stream_) {
  clove::gemm_fp16(X, Wq, q, T, H, H, 1.0f, 0.0f, stream_);
  clove::gemm_fp16(X, Wk, k, T, H, H, 1.0f, 0.0f, stream_);
  clove::gemm_fp16(X, Wv, v, T, H, H, 1.0f, 0.0f, stream_);
  clove::gemm_fp16(attn, Wo, hidden, T, H, H, 1.0f, 1.0f, stream_);  // residual, C in place
  clove::swiglu_fused(hidden, W_gate, W_up, mlp, T, H, I, stream_);
  clove::gemm_fp16(mlp, W_down, hidden, T, H, I, 1.0f, 1.0f, stream_);
}
}  // namespace

int main() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    std::printf("no GPU: link check only\n");
    return 0;
  }
  const int T = 128, H = 256, I = 512;
  half *X, *W, *out;
  cudaMalloc(&X, sizeof(half) * T * I);
  cudaMalloc(&W, sizeof(half) * I * I * 8);
  cudaMalloc(&out, sizeof(half) * T * I * 8);
  cudaMemset(X, 0, sizeof(half) * T * I);
  cudaMemset(W, 0, sizeof(half) * I * I * 8);
  block_forward(X, W, W, W, W, W, W, W, out, out + T * I, out + 2 * T * I, X, out + 3 * T * I,
                out + 4 * T * I, T, H, I, 0);
  clove::gemm_fp16(X, W, out, T, H, H);  // the default arguments
  clove::gemm_int8(reinterpret_cast<const int8_t*>(X), reinterpret_cast<const int8_t*>(W), out,
                   T, 64, 256, 0.01f, 0, 0.02f, 0);
  clove::gemm_fp16_batched(X, W, out, 2, 64, 64, 64);
  const int rc = cudaDeviceSynchronize();
  std::printf("status %d\n", rc);
  cudaFree(X);
  cudaFree(W);
  cudaFree(out);
  return rc == 0 ? 0 : 1;
}
