// fallback_simt.cuh -- CUDA-core GEMMs for shapes the TMA / vector paths cannot take
// (row strides that are not 16-byte multiples, misaligned pointers, K == 0, tiny
// tiles). Correctness path only: 32x32 output tile per CTA, operands staged in
// shared memory, fp32 / int32 accumulation in increasing k. Same arithmetic as
// the fast paths (and as the reference's naive kernel, gemm_fp16.cu:223-271).
#pragma once

#include "params.h"
#include "sm100_ptx.cuh"

namespace clove {
namespace kern {

constexpr int kSimtTile = 32;

__global__ void __launch_bounds__(kSimtTile * kSimtTile)
    gemm_f16_simt_kernel(const __half* __restrict__ A, const __half* __restrict__ B,
                         __half* __restrict__ C, int M, int N, int K, float alpha, float beta,
                         long long sA, long long sB, long long sC) {
  __shared__ float As[kSimtTile][kSimtTile + 1];
  __shared__ float Bs[kSimtTile][kSimtTile + 1];
  const int b = blockIdx.z;
  A += b * sA;
  B += b * sB;
  C += b * sC;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int row = blockIdx.y * kSimtTile + ty;
  const int col = blockIdx.x * kSimtTile + tx;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += kSimtTile) {
    const int ka = k0 + tx, kb = k0 + ty;
    As[ty][tx] = (row < M && ka < K) ? __half2float(A[static_cast<size_t>(row) * K + ka]) : 0.f;
    Bs[ty][tx] = (kb < K && col < N) ? __half2float(B[static_cast<size_t>(kb) * N + col]) : 0.f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kSimtTile; ++k) acc = fmaf(As[ty][k], Bs[k][tx], acc);
    __syncthreads();
  }
  if (row < M && col < N) {
    float out = alpha * acc;
    __half* c = C + static_cast<size_t>(row) * N + col;
    if (beta != 0.f) out += beta * __half2float(*c);
    *c = __float2half_rn(out);
  }
}

__global__ void __launch_bounds__(kSimtTile * kSimtTile)
    gemm_i8_simt_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ B,
                        void* __restrict__ Cout, int M, int N, int K, SimtEpi ep) {
  __shared__ int As[kSimtTile][kSimtTile + 1];
  __shared__ int Bs[kSimtTile][kSimtTile + 1];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int row = blockIdx.y * kSimtTile + ty;
  const int col = blockIdx.x * kSimtTile + tx;
  uint32_t acc = 0;
  for (int k0 = 0; k0 < K; k0 += kSimtTile) {
    const int ka = k0 + tx, kb = k0 + ty;
    As[ty][tx] = (row < M && ka < K) ? static_cast<int>(A[static_cast<size_t>(row) * K + ka]) - ep.za : 0;
    Bs[ty][tx] = (kb < K && col < N) ? static_cast<int>(B[static_cast<size_t>(kb) * N + col]) - ep.zb : 0;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kSimtTile; ++k)
      acc += static_cast<uint32_t>(As[ty][k]) * static_cast<uint32_t>(Bs[k][tx]);
    __syncthreads();
  }
  if (row < M && col < N) {
    const size_t o = static_cast<size_t>(row) * N + col;
    const int32_t a = static_cast<int32_t>(acc);
    if (ep.mode == 3) {
      reinterpret_cast<int32_t*>(Cout)[o] = a;
    } else {
      const float f = ep.mode == 1 ? static_cast<float>(a) * ep.scale
                                   : (static_cast<float>(a) * ep.row_scale[row]) * ep.col_scale[col];
      reinterpret_cast<__half*>(Cout)[o] = __float2half_rn(f);
    }
  }
}

// One thread per output element; groups of 128 codes unpacked on the fly.
__global__ void __launch_bounds__(256)
    gemm_i4_simt_kernel(const uint8_t* __restrict__ Aq, const __half* __restrict__ As,
                        const __half* __restrict__ Az, const uint8_t* __restrict__ Bq,
                        const __half* __restrict__ Bs, const __half* __restrict__ Bz,
                        __half* __restrict__ C, int32_t* __restrict__ Gdbg, int M, int N, int K) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(M) * N) return;
  const int m = static_cast<int>(idx / N);
  const int n = static_cast<int>(idx - static_cast<long long>(m) * N);
  const int NG = K / 128;
  const uint8_t* a = Aq + static_cast<size_t>(m) * (K / 2);
  const uint8_t* b = Bq + static_cast<size_t>(n) * (K / 2);
  float acc = 0.f;
  for (int g = 0; g < NG; ++g) {
    const int za = __half2int_rn(Az[static_cast<size_t>(m) * NG + g]);
    const int zb = __half2int_rn(Bz[static_cast<size_t>(n) * NG + g]);
    int s = 0;
    for (int j = g * 64; j < g * 64 + 64; ++j) {
      const int a_hi = a[j] >> 4, a_lo = a[j] & 0xf;
      const int b_hi = b[j] >> 4, b_lo = b[j] & 0xf;
      s += (a_hi - za) * (b_hi - zb) + (a_lo - za) * (b_lo - zb);
    }
    const float sc = __half2float(As[static_cast<size_t>(m) * NG + g]) *
                     __half2float(Bs[static_cast<size_t>(n) * NG + g]);
    acc += static_cast<float>(s) * sc;
    if (Gdbg != nullptr) Gdbg[(static_cast<size_t>(m) * N + n) * NG + g] = s;
  }
  C[static_cast<size_t>(m) * N + n] = __float2half_rn(acc);
}

// Row sums of A [M,K] and column sums of B [K,N] (int8), for zero-point corrections.
__global__ void int8_row_sums_kernel(const int8_t* __restrict__ A, int32_t* __restrict__ out,
                                     int M, int K) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const int lane = threadIdx.x & 31;
  int s = 0;
  for (int k = lane; k < K; k += 32) s += A[static_cast<size_t>(row) * K + k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[row] = s;
}

__global__ void int8_col_sums_kernel(const int8_t* __restrict__ B, int32_t* __restrict__ out,
                                     int K, int N) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= N) return;
  int s = 0;
  for (int k = 0; k < K; ++k) s += B[static_cast<size_t>(k) * N + col];
  out[col] = s;
}

// C = beta * C (K == 0 with a tensor-core-eligible shape never reaches here; used
// by the dispatcher when K == 0).
__global__ void scale_f16_kernel(__half* __restrict__ C, long long n, float beta) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) C[i] = __float2half_rn(beta == 0.f ? 0.f : beta * __half2float(C[i]));
}

}  // namespace kern
}  // namespace clove

namespace clove {
namespace kern {

// N-split all-gather re-layout: staging holds P slots [M, Nmax] (slot p = the
// C columns of rank p, padded to Nmax); scatter them into row-major C [M, N].
// Rank p owns columns [p*base + min(p, extra), ...), base = N/P, extra = N%P.
__global__ void relayout_columns_kernel(const uint16_t* __restrict__ staging,
                                        uint16_t* __restrict__ C, int M, int N, int P, int Nmax) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(M) * N) return;
  const int m = static_cast<int>(idx / N);
  const int n = static_cast<int>(idx - static_cast<long long>(m) * N);
  const int base = N / P, extra = N % P;
  const int wide = extra * (base + 1);
  int p, j;
  if (n < wide) {
    p = n / (base + 1);
    j = n - p * (base + 1);
  } else {
    p = extra + (n - wide) / base;
    j = n - (p * base + extra);
  }
  C[idx] = staging[(static_cast<size_t>(p) * M + m) * Nmax + j];
}

// Cross-rank completion signal after a replicated-output GEMM (PeerOut). Rank r
// bumps its device-side epoch e, then stores e into slot r of every rank's flag
// array (system-scope release, after a system fence, so the GEMM's remote stores
// that preceded this kernel on the stream are visible first) and waits until
// every other rank's slot in its own array holds >= e (system-scope acquire).
// All ranks make the same calls in the same order, so the epochs agree, also
// when the kernel is replayed from a CUDA graph. The wait gives up after
// timeout_ns (2 s in the product) and records a timeout instead of hanging.
struct PeerSync {
  int nranks, rank;
  unsigned long long timeout_ns;
  unsigned long long* epoch;                    // this rank's counter
  unsigned long long* flags[kMaxPeers];         // flags[q]: rank q's array [nranks]
};

__global__ void peer_signal_wait_kernel(PeerSync ps) {
  const int lane = static_cast<int>(threadIdx.x);
  unsigned long long e = 0;
  if (lane == 0) {
    e = *ps.epoch + 1;
    *ps.epoch = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  __threadfence_system();
  if (lane < ps.nranks) dev::st_release_sys_u64(ps.flags[lane] + ps.rank, e);
  if (lane < ps.nranks && lane != ps.rank)
    dev::wait_flag_geq(ps.flags[ps.rank] + lane, e, ps.timeout_ns);
  __syncwarp();
}

}  // namespace kern
}  // namespace clove
