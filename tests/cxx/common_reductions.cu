// The device helpers of include/clove/common.cuh (the reference's common.cuh
// interface: warp_reduce_sum/max, block_reduce_sum/max, half4/make_half4, CudaType)
// on seeded inputs. Prints one line per result with the float bits in hex, for the
// test to compare with the same reductions done on the CPU in the documented order.
#include <clove/common.cuh>

#include <cstdio>
#include <cstdint>
#include <cstring>
#include <type_traits>

static_assert(std::is_same<clove::CudaType<half>::type, half>::value, "CudaType<half>");
static_assert(clove::CudaType<float>::dtype == clove::DType::FP32, "CudaType<float>");
static_assert(clove::CudaType<int8_t>::dtype == clove::DType::INT8, "CudaType<int8_t>");
static_assert(sizeof(clove::half4) == 8 && sizeof(clove::half8) == 16, "half vectors");

constexpr int kBlock = 256;

// out[0..31]: warp sums of warp 0 lanes; out[32]: block sum (thread 0); out[33]:
// block max (thread 0); out[34]: a second block sum right after (back-to-back use);
// out[35]: block sum seen by thread 32 (warp 1: 0 by definition); out[36]:
// half4 round trip sum.
__global__ void probe(const float* x, float* out) {
  const int t = static_cast<int>(threadIdx.x);
  const float v = x[t];
  const float ws = clove::warp_reduce_sum(v);
  const float wm = clove::warp_reduce_max(v);
  if (t < 32) out[t] = ws;
  if (t == 0) out[40] = wm;
  const float bs = clove::block_reduce_sum<kBlock>(v);
  const float bm = clove::block_reduce_max<kBlock>(v);
  const float bs2 = clove::block_reduce_sum<kBlock>(2.0f * v);
  if (t == 0) {
    out[32] = bs;
    out[33] = bm;
    out[34] = bs2;
  }
  if (t == 32) out[35] = bs;
  if (t == 0) {
    const clove::half4 h = clove::make_half4(__float2half(1.5f), __float2half(-2.0f),
                                             __float2half(0.25f), __float2half(8.0f));
    out[36] = __half2float(h.x) + __half2float(h.y) + __half2float(h.z) + __half2float(h.w);
  }
}

int main() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    std::printf("no GPU\n");
    return 0;
  }
  float hx[kBlock];
  uint64_t s = 12345;
  for (int i = 0; i < kBlock; ++i) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    hx[i] = (static_cast<float>(s >> 40) / 16777216.0f - 0.5f) * 3.0f;
  }
  float *dx, *dout;
  cudaMalloc(&dx, sizeof(hx));
  cudaMalloc(&dout, 64 * sizeof(float));
  cudaMemcpy(dx, hx, sizeof(hx), cudaMemcpyHostToDevice);
  cudaMemset(dout, 0, 64 * sizeof(float));
  probe<<<1, kBlock>>>(dx, dout);
  float ho[64];
  const int rc = cudaMemcpy(ho, dout, sizeof(ho), cudaMemcpyDeviceToHost);
  for (int i = 0; i < kBlock; ++i) {
    uint32_t b;
    std::memcpy(&b, &hx[i], 4);
    std::printf("x %d %08x\n", i, b);
  }
  for (int i = 0; i < 41; ++i) {
    uint32_t b;
    std::memcpy(&b, &ho[i], 4);
    std::printf("out %d %08x\n", i, b);
  }
  std::printf("status %d\n", rc);
  cudaFree(dx);
  cudaFree(dout);
  return rc == 0 ? 0 : 1;
}
