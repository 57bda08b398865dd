// fallback_simt.cu -- host launchers for the CUDA-core fallback kernels.
#include "fallback_simt.cuh"
#include "../runtime/internal.h"

namespace clove {
namespace rt {

CLOVE_DEFINE_ERROR_READER(read_clear_error_simt)

int launch_simt_f16(const void* A, const void* B, void* C, int batch, int M, int N, int K,
                    float alpha, float beta, cudaStream_t stream) {
  const dim3 block(kern::kSimtTile, kern::kSimtTile);
  const dim3 grid((N + kern::kSimtTile - 1) / kern::kSimtTile,
                  (M + kern::kSimtTile - 1) / kern::kSimtTile, batch);
  kern::gemm_f16_simt_kernel<<<grid, block, 0, stream>>>(
      static_cast<const __half*>(A), static_cast<const __half*>(B), static_cast<__half*>(C), M, N,
      K, alpha, beta, static_cast<long long>(M) * K, static_cast<long long>(K) * N,
      static_cast<long long>(M) * N);
  return check_cuda(cudaGetLastError(), "simt fp16 launch");
}

int launch_simt_i8(const int8_t* A, const int8_t* B, void* C, int M, int N, int K,
                   const kern::SimtEpi& ep, cudaStream_t stream) {
  const dim3 block(kern::kSimtTile, kern::kSimtTile);
  const dim3 grid((N + kern::kSimtTile - 1) / kern::kSimtTile,
                  (M + kern::kSimtTile - 1) / kern::kSimtTile);
  kern::gemm_i8_simt_kernel<<<grid, block, 0, stream>>>(A, B, C, M, N, K, ep);
  return check_cuda(cudaGetLastError(), "simt int8 launch");
}

int launch_simt_i4(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                   const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int M, int N, int K,
                   cudaStream_t stream) {
  const long long total = static_cast<long long>(M) * N;
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  kern::gemm_i4_simt_kernel<<<grid, 256, 0, stream>>>(
      Aq, static_cast<const __half*>(As), static_cast<const __half*>(Az), Bq,
      static_cast<const __half*>(Bs), static_cast<const __half*>(Bz), static_cast<__half*>(C),
      Gdbg, M, N, K);
  return check_cuda(cudaGetLastError(), "simt int4 launch");
}

int launch_int8_row_sums(const int8_t* A, int32_t* out, int M, int K, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((M + 7) / 8);
  kern::int8_row_sums_kernel<<<grid, 256, 0, stream>>>(A, out, M, K);
  return check_cuda(cudaGetLastError(), "int8 row sums launch");
}

int launch_int8_col_sums(const int8_t* B, int32_t* out, int K, int N, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((N + 255) / 256);
  kern::int8_col_sums_kernel<<<grid, 256, 0, stream>>>(B, out, K, N);
  return check_cuda(cudaGetLastError(), "int8 col sums launch");
}

// out = silu(g) * u elementwise (the unfused SwiGLU: the reference's swiglu,
// src/kernels/activations.cu:76-121, with silu(x) = x / (1 + exp(-x)), :9-11).
__global__ void swiglu_f16_kernel(const __half* __restrict__ g, const __half* __restrict__ u,
                                  __half* __restrict__ out, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float x = __half2float(g[i]);
    out[i] = __float2half_rn(x / (1.0f + expf(-x)) * __half2float(u[i]));
  }
}

int launch_swiglu_f16(const void* g, const void* u, void* out, long long n, cudaStream_t stream) {
  if (n <= 0) return CLOVE_OK;
  long long blocks = (n + 255) / 256;
  if (blocks > 65535LL * 8) blocks = 65535LL * 8;
  swiglu_f16_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const __half*>(g), static_cast<const __half*>(u), static_cast<__half*>(out), n);
  return check_cuda(cudaGetLastError(), "swiglu launch");
}

int launch_scale_f16(void* C, long long n, float beta, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((n + 255) / 256);
  kern::scale_f16_kernel<<<grid, 256, 0, stream>>>(static_cast<__half*>(C), n, beta);
  return check_cuda(cudaGetLastError(), "scale fp16 launch");
}

}  // namespace rt
}  // namespace clove

namespace clove {
namespace rt {

// timeout_ns 0: the product bound (2 s).
int launch_peer_signal_wait(int nranks, int rank, unsigned long long* epoch,
                            unsigned long long* const* flags, unsigned long long timeout_ns,
                            cudaStream_t stream) {
  if (nranks > kern::kMaxPeers) return fail(CLOVE_ERR_UNSUPPORTED, "too many ranks");
  kern::PeerSync ps = {};
  ps.nranks = nranks;
  ps.rank = rank;
  ps.timeout_ns = timeout_ns ? timeout_ns : dev::kWaitTimeoutNs;
  ps.epoch = epoch;
  for (int q = 0; q < nranks; ++q) ps.flags[q] = flags[q];
  kern::peer_signal_wait_kernel<<<1, 32, 0, stream>>>(ps);
  return check_cuda(cudaGetLastError(), "peer signal launch");
}

int launch_relayout_columns(const void* staging, void* C, int M, int N, int P, int Nmax,
                            int elem_bytes, cudaStream_t stream) {
  if (elem_bytes != 2) return fail(CLOVE_ERR_UNSUPPORTED, "relayout: 16-bit elements only");
  const long long total = static_cast<long long>(M) * N;
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  kern::relayout_columns_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(staging),
                                                          static_cast<uint16_t*>(C), M, N, P, Nmax);
  return check_cuda(cudaGetLastError(), "relayout launch");
}

}  // namespace rt
}  // namespace clove
