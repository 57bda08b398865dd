// The drop-in C++ boundary: the call forms the reference runtime's linear layers
// use (src/runtime/inference.cu:139-194), plus the other entry points of
// clove/kernels/gemm.cuh, built against this library's headers and linked against
// its shared library. The CPU test suite compiles and links it (also together with
// the reference's other kernels); on a GPU it runs a transformer block's
// projections on seeded operands and, given an output directory, writes the
// operands and results of two of them -- a plain projection (beta = 0) and the
// in-place residual (beta = 1) -- as raw binary16 files for the test to check
// against the CPU oracle.
#include <clove/kernels/gemm.cuh>

#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

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

// Seeded values in [-scale, scale) as binary16 (64-bit LCG, top bits).
std::vector<half> seeded(size_t n, uint64_t seed, float scale) {
  std::vector<half> h(n);
  uint64_t s = seed * 6364136223846793005ull + 1442695040888963407ull;
  for (size_t i = 0; i < n; ++i) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    const float u = static_cast<float>(s >> 40) / 16777216.0f;  // [0, 1)
    h[i] = __float2half((2.0f * u - 1.0f) * scale);
  }
  return h;
}

half* to_device(const std::vector<half>& h) {
  half* d = nullptr;
  if (cudaMalloc(&d, h.size() * sizeof(half)) != cudaSuccess) std::exit(2);
  cudaMemcpy(d, h.data(), h.size() * sizeof(half), cudaMemcpyHostToDevice);
  return d;
}

bool dump(const std::string& dir, const char* name, const half* d, size_t n) {
  std::vector<half> h(n);
  if (cudaMemcpy(h.data(), d, n * sizeof(half), cudaMemcpyDeviceToHost) != cudaSuccess)
    return false;
  FILE* f = std::fopen((dir + "/" + name + ".f16").c_str(), "wb");
  if (f == nullptr) return false;
  const bool ok = std::fwrite(h.data(), sizeof(half), n, f) == n;
  std::fclose(f);
  return ok;
}
}  // namespace

int main(int argc, char** argv) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    std::printf("no GPU: link check only\n");
    return 0;
  }
  const int T = 128, H = 256, I = 512;
  const float wh = 1.0f / 16.0f;  // ~1/sqrt(H)
  half* X = to_device(seeded(static_cast<size_t>(T) * H, 1, 1.0f));
  half* Wq = to_device(seeded(static_cast<size_t>(H) * H, 2, wh));
  half* Wk = to_device(seeded(static_cast<size_t>(H) * H, 3, wh));
  half* Wv = to_device(seeded(static_cast<size_t>(H) * H, 4, wh));
  half* Wo = to_device(seeded(static_cast<size_t>(H) * H, 5, wh));
  half* Wg = to_device(seeded(static_cast<size_t>(H) * I, 6, wh));
  half* Wu = to_device(seeded(static_cast<size_t>(H) * I, 7, wh));
  half* Wd = to_device(seeded(static_cast<size_t>(I) * H, 8, 1.0f / 22.0f));
  half* attn = to_device(seeded(static_cast<size_t>(T) * H, 9, 1.0f));
  half* hidden = to_device(seeded(static_cast<size_t>(T) * H, 10, 1.0f));
  half *q, *k, *v, *mlp, *hidden0, *res;
  cudaMalloc(&q, sizeof(half) * T * H);
  cudaMalloc(&k, sizeof(half) * T * H);
  cudaMalloc(&v, sizeof(half) * T * H);
  cudaMalloc(&mlp, sizeof(half) * T * I);
  cudaMalloc(&hidden0, sizeof(half) * T * H);
  cudaMalloc(&res, sizeof(half) * T * H);
  cudaMemcpy(hidden0, hidden, sizeof(half) * T * H, cudaMemcpyDeviceToDevice);

  // The checked projections, on their own: q = X . Wq and res = attn . Wo + hidden0
  // computed in place in `res` (beta = 1, C read before it is overwritten).
  cudaMemcpy(res, hidden0, sizeof(half) * T * H, cudaMemcpyDeviceToDevice);
  clove::gemm_fp16(X, Wq, q, T, H, H);  // the default arguments
  clove::gemm_fp16(attn, Wo, res, T, H, H, 1.0f, 1.0f, 0);
  int rc = cudaDeviceSynchronize();
  bool ok = rc == 0;
  if (ok && argc > 1) {
    const std::string dir = argv[1];
    ok = dump(dir, "X", X, static_cast<size_t>(T) * H) &&
         dump(dir, "Wq", Wq, static_cast<size_t>(H) * H) &&
         dump(dir, "q", q, static_cast<size_t>(T) * H) &&
         dump(dir, "attn", attn, static_cast<size_t>(T) * H) &&
         dump(dir, "Wo", Wo, static_cast<size_t>(H) * H) &&
         dump(dir, "hidden0", hidden0, static_cast<size_t>(T) * H) &&
         dump(dir, "res", res, static_cast<size_t>(T) * H);
  }

  // The whole block, and the remaining entry points, for their status.
  block_forward(X, Wq, Wk, Wv, Wo, Wg, Wu, Wd, q, k, v, attn, hidden, mlp, T, H, I, 0);
  clove::gemm_int8(reinterpret_cast<const int8_t*>(X), reinterpret_cast<const int8_t*>(Wq), res,
                   T, 64, 256, 0.01f, 0, 0.02f, 0);
  clove::gemm_fp16_batched(X, Wq, res, 2, 64, 64, 64);
  rc = cudaDeviceSynchronize();
  std::printf("status %d dump %s\n", rc, ok ? "ok" : "failed");
  for (half* p : {X, Wq, Wk, Wv, Wo, Wg, Wu, Wd, attn, hidden, q, k, v, mlp, hidden0, res})
    cudaFree(p);
  return rc == 0 && ok ? 0 : 1;
}
