// quant_int4.cu -- packs fp16 weights into the INT4 layout clove_gemm_int4 reads.
//
// Layout (north_star / include/clove/kernels/gemm.cuh:67-87): codes [rows,K/2],
// element 2j in the high nibble of byte j (the nibble order of the reference's
// unpack_int4x2, src/kernels/gemm_int4.cu:27-34), unsigned codes 0..15; per
// 128-group fp16 scale and integer zero point [rows,K/128]. The reference has no
// quantizer (its weight loader is a stub), so the rounding rules are this build's
// specification, restated on the CPU in oracle/host_gemm.c
// (clove_oracle_quantize_int4) and matched bit for bit:
//   min, max over the group and 0 (the range contains 0, so all-positive and
//   constant groups keep their values)
//   scale = half((max - min) / 15)  (0 -> smallest subnormal, capped at 65504)
//   zero  = clamp(rint(-min / scale), 0, 15)
//   code  = clamp(rint(w / scale) + zero, 0, 15)
// in fp32 with IEEE division and ties-to-even rounding.
//
// One warp per (row, group): each lane holds four consecutive weights (one 8-byte
// load; the warp reads the group's 256 bytes contiguously), min / max by butterfly,
// two packed bytes per lane stored as one 16-bit word. HBM-bound: 2.5 bytes moved
// per weight.
#include <cuda_fp16.h>

#include <cstdint>

#include "../runtime/internal.h"

namespace clove {
namespace kern {

constexpr int kQuantThreads = 256;

__global__ void __launch_bounds__(kQuantThreads)
    quantize_int4_kernel(const __half* __restrict__ W, int rows, int K, uint8_t* __restrict__ codes,
                         __half* __restrict__ scales, __half* __restrict__ zeros) {
  const int ng = K >> 7;
  const long long task = (static_cast<long long>(blockIdx.x) * kQuantThreads + threadIdx.x) >> 5;
  const int lane = static_cast<int>(threadIdx.x & 31);
  if (task >= static_cast<long long>(rows) * ng) return;  // warp-uniform
  const int r = static_cast<int>(task / ng);
  const int g = static_cast<int>(task - static_cast<long long>(r) * ng);
  const __half* w = W + static_cast<size_t>(r) * K + static_cast<size_t>(g) * 128 + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(w);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  const float v[4] = {f01.x, f01.y, f23.x, f23.y};
  float mn = fminf(fminf(fminf(v[0], v[1]), fminf(v[2], v[3])), 0.0f);
  float mx = fmaxf(fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3])), 0.0f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  __half sh = __float2half_rn((mx - mn) / 15.0f);
  unsigned short bits = __half_as_ushort(sh);
  if ((bits & 0x7fffu) == 0) bits = 0x0001u;       // smallest positive subnormal
  if ((bits & 0x7fffu) > 0x7bffu) bits = 0x7bffu;  // 65504
  sh = __ushort_as_half(bits);
  const float sf = __half2float(sh);
  const float zf = fminf(fmaxf(rintf(-mn / sf), 0.0f), 15.0f);
  uint32_t q[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    q[e] = static_cast<uint32_t>(fminf(fmaxf(rintf(v[e] / sf) + zf, 0.0f), 15.0f));
  const uint32_t b0 = (q[0] << 4) | q[1];
  const uint32_t b1 = (q[2] << 4) | q[3];
  *reinterpret_cast<uint16_t*>(codes + static_cast<size_t>(r) * (K / 2) + static_cast<size_t>(g) * 64 +
                               lane * 2) = static_cast<uint16_t>(b0 | (b1 << 8));
  if (lane == 0) {
    scales[static_cast<size_t>(r) * ng + g] = sh;
    zeros[static_cast<size_t>(r) * ng + g] = __float2half_rn(static_cast<float>(static_cast<int>(zf)));
  }
}

}  // namespace kern

namespace rt {

int launch_quantize_int4(const void* W, int rows, int K, uint8_t* codes, void* scales, void* zeros,
                         cudaStream_t stream) {
  const long long warps = static_cast<long long>(rows) * (K / 128);
  const long long blocks = (warps * 32 + kern::kQuantThreads - 1) / kern::kQuantThreads;
  if (blocks > 0x7fffffffLL) return fail(CLOVE_ERR_UNSUPPORTED, "quantize_int4: too many groups");
  kern::quantize_int4_kernel<<<static_cast<unsigned>(blocks), kern::kQuantThreads, 0, stream>>>(
      static_cast<const __half*>(W), rows, K, codes, static_cast<__half*>(scales),
      static_cast<__half*>(zeros));
  return check_cuda(cudaGetLastError(), "quantize_int4 launch");
}

}  // namespace rt
}  // namespace clove
