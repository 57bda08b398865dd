// gemv_sm100.cuh -- HBM-bound skinny GEMMs (N <= 8 columns of C) for decode.
//
// The big operand A [rows, K] is streamed once with 128-bit non-coherent loads, a
// warp per row pair, every load of a row pair issued before any math so that each
// SM keeps tens of KB in flight. The skinny operand (N <= 8 vectors) is unpacked
// once per CTA into shared memory in the lane order the stream needs.
//
// Replaces, for decode shapes, the reference's naive fallback
// (src/kernels/gemm_fp16.cu:223-271) and the SIMT int8 / int4 kernels
// (gemm_int8.cu:16-117, gemm_int4.cu:45-193).
//
// INT4 (north-star layout, both operands [rows, K/2] nibbles + [rows, K/128] fp16
// scale / zero point): four consecutive lanes hold one 128-element group (64 bytes);
// each lane dots its 32 codes against (b - zB) with dp4a, the quad reduces to the
// group's exact int32 sum D, and G = D - zA * sum(b - zB) is the exact group
// accumulator sum_k (a - zA)(b - zB). C = sum_g float(G) * sA * sB in fp32.
#pragma once

#include "params.h"
#include "sm100_ptx.cuh"

namespace clove {
namespace kern {

constexpr int kGemvThreads = 256;  // 8 warps
constexpr int kGemvRowsPerWarp = 2;

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i32(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// INT4
// ---------------------------------------------------------------------------
// Shared memory (dynamic), per B vector n:
//   bp  [K/32 chunks][8 words]  (b - zB) as packed int8x4; for the 4 A words of a
//                               16-byte chunk, word 2w holds the 4 even-k codes
//                               (high nibbles), word 2w+1 the 4 odd-k codes.
//   sb  [K/128] float scale, zs [K/128] int sum over the group of (b - zB).
__host__ __device__ constexpr size_t gemv_int4_smem_bytes(int nc, int K) {
  return static_cast<size_t>(nc) * (static_cast<size_t>(K) + 2 * 4 * (K / 128));
}

template <int NC>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_int4_kernel(const uint8_t* __restrict__ Aq, const __half* __restrict__ As,
                     const __half* __restrict__ Az, const uint8_t* __restrict__ Bq,
                     const __half* __restrict__ Bs, const __half* __restrict__ Bz,
                     __half* __restrict__ C, int32_t* __restrict__ Gdbg, int rows, int K,
                     long long ldc_row, long long ldc_col, long long ldg_row, long long ldg_col) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int NG = K >> 7;          // groups per row
  const int NCH = K >> 5;         // 16-byte chunks per row
  const int KB = K >> 1;          // bytes per row
  uint32_t* bp = reinterpret_cast<uint32_t*>(smem);                    // [NC][NCH*8]
  float* sb = reinterpret_cast<float*>(smem + static_cast<size_t>(NC) * K);  // [NC][NG]
  int* zs = reinterpret_cast<int*>(sb + NC * NG);                            // [NC][NG]

  // ---- unpack the B vectors (tiny: NC * K/2 bytes)
  for (int idx = threadIdx.x; idx < NC * NCH * 8; idx += blockDim.x) {
    const int n = idx / (NCH * 8);
    const int r = idx - n * NCH * 8;
    const int ch = r >> 3;         // chunk
    const int w = (r >> 1) & 3;    // A word within the chunk
    const int odd = r & 1;         // 0: high nibbles (even k), 1: low nibbles (odd k)
    const int byte0 = ch * 16 + w * 4;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(Bq + static_cast<size_t>(n) * KB + byte0);
    const int zb = __half2int_rn(Bz[static_cast<size_t>(n) * NG + (byte0 * 2) / 128]);
    uint32_t packed = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t byte = (word >> (8 * t)) & 0xffu;
      const int code = odd ? static_cast<int>(byte & 0xfu) : static_cast<int>(byte >> 4);
      packed |= (static_cast<uint32_t>(code - zb) & 0xffu) << (8 * t);
    }
    bp[n * NCH * 8 + r] = packed;
  }
  for (int idx = threadIdx.x; idx < NC * NG; idx += blockDim.x) {
    const int n = idx / NG;
    const int g = idx - n * NG;
    const uint8_t* row = Bq + static_cast<size_t>(n) * KB + g * 64;
    const int zb = __half2int_rn(Bz[static_cast<size_t>(n) * NG + g]);
    int s = 0;
    for (int j = 0; j < 64; ++j) s += (row[j] >> 4) + (row[j] & 0xf);
    zs[idx] = s - 128 * zb;
    sb[idx] = __half2float(Bs[static_cast<size_t>(n) * NG + g]);
  }
  __syncthreads();

  const int lane = static_cast<int>(dev::lane_idx());
  const int gwarp = static_cast<int>(blockIdx.x * (blockDim.x >> 5) + dev::warp_idx());
  const int nwarps = static_cast<int>(gridDim.x * (blockDim.x >> 5));
  const int passes = (NCH + 31) >> 5;  // 512-byte windows per row

  for (int row0 = gwarp * kGemvRowsPerWarp; row0 < rows; row0 += nwarps * kGemvRowsPerWarp) {
    float acc[kGemvRowsPerWarp][NC];
#pragma unroll
    for (int r = 0; r < kGemvRowsPerWarp; ++r)
#pragma unroll
      for (int n = 0; n < NC; ++n) acc[r][n] = 0.f;

    for (int p0 = 0; p0 < passes; p0 += 4) {
      // Issue every load of this window for both rows first.
      uint4 v[kGemvRowsPerWarp][4];
      __half2 zsA[kGemvRowsPerWarp][4];
#pragma unroll
      for (int r = 0; r < kGemvRowsPerWarp; ++r) {
        const int m = row0 + r;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = (p0 + j) * 32 + lane;
          if (m < rows && p0 + j < passes && ch < NCH) {
            v[r][j] = dev::ld_nc_v4(Aq + static_cast<size_t>(m) * KB + static_cast<size_t>(ch) * 16);
            const size_t gi = static_cast<size_t>(m) * NG + (ch >> 2);
            zsA[r][j] = __halves2half2(Az[gi], As[gi]);
          } else {
            v[r][j] = make_uint4(0u, 0u, 0u, 0u);
            zsA[r][j] = __halves2half2(__float2half(0.f), __float2half(0.f));
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kGemvRowsPerWarp; ++r) {
        const int m = row0 + r;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (p0 + j >= passes) continue;  // warp-uniform
          const int ch = (p0 + j) * 32 + lane;
          const bool valid = ch < NCH;
          const int chc = valid ? ch : 0;
          const uint32_t w[4] = {v[r][j].x, v[r][j].y, v[r][j].z, v[r][j].w};
#pragma unroll
          for (int n = 0; n < NC; ++n) {
            const uint4* b4 = reinterpret_cast<const uint4*>(bp + n * NCH * 8 + chc * 8);
            const uint4 b0 = b4[0];
            const uint4 b1 = b4[1];
            int d = 0;
            d = __dp4a(static_cast<int>((w[0] >> 4) & 0x0f0f0f0fu), static_cast<int>(b0.x), d);
            d = __dp4a(static_cast<int>(w[0] & 0x0f0f0f0fu), static_cast<int>(b0.y), d);
            d = __dp4a(static_cast<int>((w[1] >> 4) & 0x0f0f0f0fu), static_cast<int>(b0.z), d);
            d = __dp4a(static_cast<int>(w[1] & 0x0f0f0f0fu), static_cast<int>(b0.w), d);
            d = __dp4a(static_cast<int>((w[2] >> 4) & 0x0f0f0f0fu), static_cast<int>(b1.x), d);
            d = __dp4a(static_cast<int>(w[2] & 0x0f0f0f0fu), static_cast<int>(b1.y), d);
            d = __dp4a(static_cast<int>((w[3] >> 4) & 0x0f0f0f0fu), static_cast<int>(b1.z), d);
            d = __dp4a(static_cast<int>(w[3] & 0x0f0f0f0fu), static_cast<int>(b1.w), d);
            if (!valid) d = 0;
            // The 4 lanes of a group (lane & ~3 .. +3) hold its 4 chunks.
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            if (valid && (lane & 3) == 0 && m < rows) {
              const int g = ch >> 2;
              const float2 zsa = __half22float2(zsA[r][j]);
              const int za = __half2int_rn(__low2half(zsA[r][j]));
              const int G = d - za * zs[n * NG + g];
              acc[r][n] += static_cast<float>(G) * (zsa.y * sb[n * NG + g]);
              if (Gdbg != nullptr)
                Gdbg[m * ldg_row + n * ldg_col + g] = G;
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kGemvRowsPerWarp; ++r) {
      const int m = row0 + r;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const float s = warp_sum_f32(acc[r][n]);
        if (lane == 0 && m < rows) C[m * ldc_row + n * ldc_col] = __float2half_rn(s);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// INT8: A int8 [rows, K] streamed, B int8 [K, NC] row-major (reference layout).
// ---------------------------------------------------------------------------
__host__ __device__ constexpr size_t gemv_int8_smem_bytes(int nc, int K) {
  return static_cast<size_t>(nc) * K + 4 * 8;
}

template <int NC>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_int8_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ B,
                     void* __restrict__ Cout, int rows, int K, GemvI8Epi ep) {
  extern __shared__ __align__(16) uint8_t smem[];
  int8_t* bt = reinterpret_cast<int8_t*>(smem);                            // [NC][K]
  int* colsum = reinterpret_cast<int*>(smem + static_cast<size_t>(NC) * K);  // [NC]
  for (int idx = threadIdx.x; idx < NC * K; idx += blockDim.x) {
    const int n = idx / K;
    const int k = idx - n * K;
    bt[idx] = B[static_cast<size_t>(k) * NC + n];
  }
  __syncthreads();
  if (threadIdx.x < 32 * NC) {
    const int n = threadIdx.x >> 5;
    int s = 0;
    for (int k = dev::lane_idx(); k < K; k += 32) s += bt[n * K + k];
    s = warp_sum_i32(s);
    if (dev::lane_idx() == 0) colsum[n] = s;
  }
  __syncthreads();

  const int lane = static_cast<int>(dev::lane_idx());
  const int gwarp = static_cast<int>(blockIdx.x * (blockDim.x >> 5) + dev::warp_idx());
  const int nwarps = static_cast<int>(gridDim.x * (blockDim.x >> 5));
  const int NCH = K >> 4;  // 16-byte chunks per row

  for (int row0 = gwarp * kGemvRowsPerWarp; row0 < rows; row0 += nwarps * kGemvRowsPerWarp) {
    int acc[kGemvRowsPerWarp][NC];
    int asum[kGemvRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kGemvRowsPerWarp; ++r) {
      asum[r] = 0;
#pragma unroll
      for (int n = 0; n < NC; ++n) acc[r][n] = 0;
    }
    for (int c0 = 0; c0 < NCH; c0 += 32 * 4) {
      uint4 v[kGemvRowsPerWarp][4];
#pragma unroll
      for (int r = 0; r < kGemvRowsPerWarp; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = c0 + j * 32 + lane;
          const int m = row0 + r;
          v[r][j] = (m < rows && ch < NCH)
                        ? dev::ld_nc_v4(A + static_cast<size_t>(m) * K + static_cast<size_t>(ch) * 16)
                        : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
      for (int r = 0; r < kGemvRowsPerWarp; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = c0 + j * 32 + lane;
          if (ch >= NCH) continue;
          const int a0 = static_cast<int>(v[r][j].x), a1 = static_cast<int>(v[r][j].y);
          const int a2 = static_cast<int>(v[r][j].z), a3 = static_cast<int>(v[r][j].w);
          if (ep.zb != 0) {
            asum[r] = __dp4a(a0, 0x01010101, asum[r]);
            asum[r] = __dp4a(a1, 0x01010101, asum[r]);
            asum[r] = __dp4a(a2, 0x01010101, asum[r]);
            asum[r] = __dp4a(a3, 0x01010101, asum[r]);
          }
#pragma unroll
          for (int n = 0; n < NC; ++n) {
            const uint4 b = *reinterpret_cast<const uint4*>(bt + n * K + ch * 16);
            int d = acc[r][n];
            d = __dp4a(a0, static_cast<int>(b.x), d);
            d = __dp4a(a1, static_cast<int>(b.y), d);
            d = __dp4a(a2, static_cast<int>(b.z), d);
            d = __dp4a(a3, static_cast<int>(b.w), d);
            acc[r][n] = d;
          }
        }
    }
#pragma unroll
    for (int r = 0; r < kGemvRowsPerWarp; ++r) {
      const int m = row0 + r;
      const int sa = (ep.zb != 0) ? warp_sum_i32(asum[r]) : 0;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const int s = warp_sum_i32(acc[r][n]);
        if (lane == 0 && m < rows) {
          uint32_t a = static_cast<uint32_t>(s);
          a -= static_cast<uint32_t>(ep.za) * static_cast<uint32_t>(colsum[n]);
          a -= static_cast<uint32_t>(ep.zb) * static_cast<uint32_t>(sa);
          a += static_cast<uint32_t>(K) * static_cast<uint32_t>(ep.za) * static_cast<uint32_t>(ep.zb);
          const int32_t ai = static_cast<int32_t>(a);
          if (ep.mode == 3) {
            reinterpret_cast<int32_t*>(Cout)[static_cast<size_t>(m) * NC + n] = ai;
          } else {
            const float f = (ep.mode == 1)
                                ? static_cast<float>(ai) * ep.scale
                                : (static_cast<float>(ai) * ep.row_scale[m]) * ep.col_scale[n];
            reinterpret_cast<__half*>(Cout)[static_cast<size_t>(m) * NC + n] = __float2half_rn(f);
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// FP16: A fp16 [rows, K] streamed, B fp16 [K, NC] row-major, fp32 accumulate.
// C = alpha * A.B + beta * C.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr size_t gemv_f16_smem_bytes(int nc, int K) {
  return static_cast<size_t>(nc) * K * 2;
}

template <int NC>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_f16_kernel(const __half* __restrict__ A, const __half* __restrict__ B,
                    __half* __restrict__ C, int rows, int K, float alpha, float beta) {
  extern __shared__ __align__(16) uint8_t smem[];
  __half* bt = reinterpret_cast<__half*>(smem);  // [NC][K]
  for (int idx = threadIdx.x; idx < NC * K; idx += blockDim.x) {
    const int n = idx / K;
    const int k = idx - n * K;
    bt[idx] = B[static_cast<size_t>(k) * NC + n];
  }
  __syncthreads();

  const int lane = static_cast<int>(dev::lane_idx());
  const int gwarp = static_cast<int>(blockIdx.x * (blockDim.x >> 5) + dev::warp_idx());
  const int nwarps = static_cast<int>(gridDim.x * (blockDim.x >> 5));
  const int NCH = K >> 3;  // 16-byte chunks (8 halves)

  for (int row0 = gwarp * kGemvRowsPerWarp; row0 < rows; row0 += nwarps * kGemvRowsPerWarp) {
    float acc[kGemvRowsPerWarp][NC];
#pragma unroll
    for (int r = 0; r < kGemvRowsPerWarp; ++r)
#pragma unroll
      for (int n = 0; n < NC; ++n) acc[r][n] = 0.f;
    for (int c0 = 0; c0 < NCH; c0 += 32 * 4) {
      uint4 v[kGemvRowsPerWarp][4];
#pragma unroll
      for (int r = 0; r < kGemvRowsPerWarp; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = c0 + j * 32 + lane;
          const int m = row0 + r;
          v[r][j] = (m < rows && ch < NCH)
                        ? dev::ld_nc_v4(A + static_cast<size_t>(m) * K + static_cast<size_t>(ch) * 8)
                        : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
      for (int r = 0; r < kGemvRowsPerWarp; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = c0 + j * 32 + lane;
          if (ch >= NCH) continue;
          const __half2* ah = reinterpret_cast<const __half2*>(&v[r][j]);
          float2 a[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) a[u] = __half22float2(ah[u]);
#pragma unroll
          for (int n = 0; n < NC; ++n) {
            const uint4 b = *reinterpret_cast<const uint4*>(bt + n * K + ch * 8);
            const __half2* bh = reinterpret_cast<const __half2*>(&b);
            float s = acc[r][n];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 bf = __half22float2(bh[u]);
              s = fmaf(a[u].x, bf.x, s);
              s = fmaf(a[u].y, bf.y, s);
            }
            acc[r][n] = s;
          }
        }
    }
#pragma unroll
    for (int r = 0; r < kGemvRowsPerWarp; ++r) {
      const int m = row0 + r;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const float s = warp_sum_f32(acc[r][n]);
        if (lane == 0 && m < rows) {
          float out = alpha * s;
          __half* c = C + static_cast<size_t>(m) * NC + n;
          if (beta != 0.f) out += beta * __half2float(*c);
          *c = __float2half_rn(out);
        }
      }
    }
  }
}

}  // namespace kern
}  // namespace clove
