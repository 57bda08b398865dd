// capi.cpp -- the extern "C" entry points of include/clove/capi.h: argument
// validation, kernel-family dispatch, scratch management, error reporting.
//
// Reference behaviour kept: stateless, handle-free, asynchronous on the caller's
// stream, caller-owned device buffers (src/kernels/gemm_fp16.cu:277-305,
// gemm_int8.cu:119-137, gemm_int4.cu:195-216). Unlike the reference, failures
// are returned as status codes instead of exit().
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../kernels/params.h"
#include "internal.h"

namespace clove {
namespace rt {

namespace {
thread_local char g_last_error[512] = "no error";
std::atomic<int> g_ov_path{0}, g_ov_bn{0}, g_ov_split{0};
std::atomic<int> g_weight_prefetch{0};

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
DeviceInfo g_dev_cache[kMaxDevices];
bool g_dev_valid[kMaxDevices] = {};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
inline bool aligned2(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 1u) == 0; }
inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CLOVE_OK;
  return fail(CLOVE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int current_device(DeviceInfo* out) {
  int d = 0;
  int rc = check_cuda(cudaGetDevice(&d), "cudaGetDevice");
  if (rc) return rc;
  if (d < 0 || d >= kMaxDevices) return fail(CLOVE_ERR_DEVICE, "device ordinal %d", d);
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_dev_valid[d]) {
      *out = g_dev_cache[d];
      return CLOVE_OK;
    }
  }
  DeviceInfo info;
  info.device = d;
  rc = check_cuda(cudaDeviceGetAttribute(&info.num_sms, cudaDevAttrMultiProcessorCount, d),
                  "cudaDeviceGetAttribute(SMs)");
  if (rc) return rc;
  rc = check_cuda(cudaDeviceGetAttribute(&info.cc_major, cudaDevAttrComputeCapabilityMajor, d),
                  "cudaDeviceGetAttribute(cc)");
  if (rc) return rc;
  rc = check_cuda(cudaDeviceGetAttribute(&info.cc_minor, cudaDevAttrComputeCapabilityMinor, d),
                  "cudaDeviceGetAttribute(cc)");
  if (rc) return rc;
  if (info.cc_major != 10)
    return fail(CLOVE_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", d,
                info.cc_major, info.cc_minor);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  g_dev_cache[d] = info;
  g_dev_valid[d] = true;
  *out = info;
  return CLOVE_OK;
}

Override get_override() {
  return Override{g_ov_path.load(), g_ov_bn.load(), g_ov_split.load()};
}

bool weight_prefetch_enabled() { return g_weight_prefetch.load() != 0; }
bool ws_disabled() { return g_ov_path.load() == 2 && g_ov_bn.load() == 1; }
bool ws2_selected() { return g_ov_path.load() == 2 && g_ov_bn.load() == 2; }

// ---------------------------------------------------------------------------
// Tile-shape policy for the tensor-core kernels
// ---------------------------------------------------------------------------
// Per-tile time is roughly proportional to BN; narrower tiles pay extra for
// re-reading A. Choose the BN that minimises waves x BN x penalty; when even
// BN=64 leaves most SMs idle, split K over a cluster.
TcPlan plan_tc(int M, int N, int K, int elem, int num_sms) {
  const Override ov = get_override();
  const int bk = 128 / elem;
  const int kb_total = (K + bk - 1) / bk;
  const int tm = (M + 127) / 128;
  TcPlan best{256, 1, false};
  if (ov.bn != 0) {
    best.bn = ov.bn;
  } else {
    double best_cost = 1e30;
    const int cand[3] = {256, 128, 64};
    const double penalty[3] = {1.0, 1.15, 1.45};
    for (int i = 0; i < 3; ++i) {
      const int bn = cand[i];
      const long long tiles = static_cast<long long>(tm) * ((N + bn - 1) / bn);
      const long long waves = (tiles + num_sms - 1) / num_sms;
      const double cost = static_cast<double>(waves) * bn * penalty[i];
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best.bn = bn;
      }
    }
  }
  if (ov.split != 0) {
    best.split = ov.split;
  } else {
    const long long tiles64 = static_cast<long long>(tm) * ((N + 63) / 64);
    if (tiles64 * 2 <= num_sms && kb_total >= 4) {
      // Few output tiles: narrow tiles split over K inside a cluster.
      best.bn = (N <= 32 || tm * ((N + 63) / 64) * 4 <= num_sms) ? 32 : 64;
      if (ov.bn != 0) best.bn = ov.bn;
      const long long tiles = static_cast<long long>(tm) * ((N + best.bn - 1) / best.bn);
      long long s = num_sms / std::max<long long>(tiles, 1);
      s = std::min<long long>(s, 8);
      s = std::min<long long>(s, kb_total / 2);
      long long p2 = 1;  // cluster sizes 2, 4, 8 (a tile's rows split evenly)
      while (p2 * 2 <= s) p2 *= 2;
      best.split = static_cast<int>(p2);
      // One 128-row band (decode in the runtime's orientation): 128-column tiles
      // over 4-CTA clusters read twice the contiguous bytes of every B row (256
      // for fp16, 128 for int8) per CTA. fp16: that outweighs the larger cluster
      // exchange when few rows are live (only rows below M are exchanged) or K is
      // long -- 1 x 4096 x 4096 11.7 -> 10.4 us, 1 x 4096 x 11008 24.8 -> 19.0 us,
      // while with all 128 rows live at K = 4096 the 64-column tiles stay ahead
      // (12.6 against 13.3 us). int8: for long K only (1 x 4096 x 11008 14.1 ->
      // 12.6 us; at K = 4096 7.7 against 8.1 us even with one live row).
      const bool wide = elem == 2 ? (M <= 32 || kb_total >= 96) : kb_total >= 64;
      if (ov.bn == 0 && tm == 1 && best.bn == 64 && best.split == 2 && wide &&
          static_cast<long long>((N + 127) / 128) * 4 <= num_sms) {
        best.bn = 128;
        best.split = 4;
      }
    } else {
      best.split = 1;
    }
  }
  if (best.split > 1 && best.bn > 128) best.bn = 128;
  // CTA pairs (256 x 256 tiles) whenever the one-SM plan is 128 x 256 tiles and A
  // has at least 256 rows: a pair covers the same two 128 x 256 tiles on the same
  // two SMs, but each CTA loads only half of the B panel, so per SM a K block moves
  // 32 KB instead of 48 KB. Measured on B200 below one wave of pairs as well
  // (2048 x 2048 x 8192: 55.5 -> 50.9 us, 1792 x 2048 x 4096: 28.3 -> 26.8 us,
  // 2048^3: equal).
  if (ov.path == 4) {
    best.pair = true;
  } else if (ov.path == 0 && best.split == 1 && best.bn == 256 && N % 8 == 0 && M >= 256) {
    best.pair = true;
  }
  return best;
}

}  // namespace rt
}  // namespace clove

using namespace clove;
using namespace clove::rt;

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* clove_version(void) { return "clove-b200 0.1 (sm_100a, tcgen05)"; }

const char* clove_last_error_string(void) { return g_last_error; }

int clove_get_device_error(int* code) {
  if (code == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "code is NULL");
  int rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (rc) return rc;
  int v = 0;
  const int readers[5] = {read_clear_error_tc(), read_clear_error_gemv(), read_clear_error_simt(),
                          read_clear_error_int4(), read_clear_error_attn()};
  for (int r : readers) {
    if (r < 0) return fail(CLOVE_ERR_CUDA, "reading the device error word failed");
    if (v == 0 && r != 0) v = r;
  }
  // A kernel that gave up may have left stream-K tickets taken: clear them so the
  // next call starts from zero.
  if (v != 0) reset_stream_k_tickets();
  *code = v;
  return CLOVE_OK;
}

int clove_set_weight_prefetch(int enable) {
  g_weight_prefetch.store(enable ? 1 : 0);
  return CLOVE_OK;
}

int clove_set_dispatch_override(int path, int bn, int split) {
  g_ov_path.store(path);
  g_ov_bn.store(bn);
  g_ov_split.store(split);
  return CLOVE_OK;
}

// ---------------------------------------------------------------------------
// FP16
// ---------------------------------------------------------------------------
// peer != nullptr: the N-split replicated output (PeerOut); only the tensor-core
// tile kernels store it, so any other path returns CLOVE_ERR_UNSUPPORTED untouched.
static int gemm_fp16_impl(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                          float beta, cudaStream_t s, const char** chosen,
                          const PeerTargets* peer = nullptr) {
  if (M < 0 || N < 0 || K < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative size");
  if (M == 0 || N == 0) return CLOVE_OK;
  if (C == nullptr || (K > 0 && (A == nullptr || B == nullptr)))
    return fail(CLOVE_ERR_INVALID_ARG, "null matrix pointer");
  if (!aligned2(A) || !aligned2(B) || !aligned2(C))
    return fail(CLOVE_ERR_INVALID_ARG, "fp16 pointers must be 2-byte aligned");
  DeviceInfo dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  if (K == 0) {
    if (chosen) *chosen = "scale";
    return launch_scale_f16(C, static_cast<long long>(M) * N, beta, s);
  }
  const Override ov = get_override();
  const bool tc_ok = K % 8 == 0 && N % 8 == 0 && aligned16(A) && aligned16(B) && aligned16(C);
  const bool gemv_ok = N <= 8 && K % 8 == 0 && aligned16(A) && gemv_f16_smem(N, K) <= 200 * 1024;
  int path = ov.path;
  if ((path == 1 || path == 4) && !tc_ok) path = 0;
  if (path == 2 && !gemv_ok) path = 0;
  if (path == 0) path = (gemv_ok && N < 16) ? 2 : (tc_ok ? 1 : 3);
  if (peer != nullptr && path != 1 && path != 4) return CLOVE_ERR_UNSUPPORTED;
  if (path == 2) {
    if (chosen) *chosen = "gemv_f16";
    return launch_gemv_f16(A, B, C, M, N, K, alpha, beta, dev, s);
  }
  if (path == 3) {
    if (chosen) *chosen = "simt_f16";
    return launch_simt_f16(A, B, C, 1, M, N, K, alpha, beta, s);
  }
  const TcPlan plan = plan_tc(M, N, K, 2, dev.num_sms);
  if (chosen) *chosen = plan.pair ? "tc2_f16" : plan.split > 1 ? "tc_f16_split" : "tc_f16";
  kern::EpiParams ep{};
  ep.mode = kern::kEpiF16AlphaBeta;
  ep.alpha = alpha;
  ep.beta = beta;
  ep.c_in = static_cast<const __half*>(C);
  if (plan.pair) return launch_gemm_tc2(kTcF16, A, B, C, M, N, K, ep, dev, s, nullptr, peer);
  return launch_gemm_tc(kTcF16, plan.bn, plan.split, 2, A, B, C, M, N, K, ep, dev, s, 1, peer);
}

extern "C++" {  // internal C++ entry (nsplit.cpp), inside this file's extern "C" block
namespace clove {
namespace rt {
int gemm_fp16_replicated(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                         const PeerTargets& peer, cudaStream_t s) {
  return gemm_fp16_impl(A, B, C, M, N, K, alpha, 0.f, s, nullptr, &peer);
}
}  // namespace rt
}  // namespace clove
}

int clove_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                    float beta, void* stream) {
  return gemm_fp16_impl(A, B, C, M, N, K, alpha, beta, as_stream(stream), nullptr);
}

// Tile width for `batch` problems of M x N sharing one persistent launch: the
// plan_tc cost (waves x width x narrow-tile penalty) over all problems' tiles.
static int plan_bn_batched(int M, int N, int batch, int num_sms) {
  const Override ov = get_override();
  if (ov.bn == 64 || ov.bn == 128 || ov.bn == 256) return ov.bn;
  const long long tm = (M + 127) / 128;
  const int cand[3] = {256, 128, 64};
  const double penalty[3] = {1.0, 1.15, 1.45};
  int best = 256;
  double best_cost = 1e30;
  for (int i = 0; i < 3; ++i) {
    const long long tiles = tm * ((N + cand[i] - 1) / cand[i]) * batch;
    const long long waves = (tiles + num_sms - 1) / num_sms;
    const double cost = static_cast<double>(waves) * cand[i] * penalty[i];
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = cand[i];
    }
  }
  return best;
}

int clove_gemm_fp16_batched(const void* A, const void* B, void* C, int batch, int M, int N, int K,
                            float alpha, float beta, void* stream) {
  if (batch < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative batch");
  if (batch == 0 || M == 0 || N == 0) return CLOVE_OK;
  if (M < 0 || N < 0 || K < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative size");
  const size_t sa = static_cast<size_t>(M) * K * 2, sb = static_cast<size_t>(K) * N * 2,
               sc = static_cast<size_t>(M) * N * 2;
  if (batch > 1 && K > 0 && A != nullptr && B != nullptr && C != nullptr) {
    // Problems too small to fill the GPU on their own share one persistent launch
    // of the tile kernel (3D tensor maps, a batch plane per problem); larger ones
    // run back to back through the single-problem dispatch (CTA pairs etc.).
    DeviceInfo dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    const Override ov = get_override();
    const bool tc_ok = K % 8 == 0 && N % 8 == 0 && aligned16(A) && aligned16(B) && aligned16(C) &&
                       (ov.path == 0 || ov.path == 1) && (ov.split == 0 || ov.split == 1);
    const long long tiles1 = static_cast<long long>((M + 127) / 128) * ((N + 63) / 64);
    if (tc_ok && tiles1 < dev.num_sms) {
      kern::EpiParams ep{};
      ep.mode = kern::kEpiF16AlphaBeta;
      ep.alpha = alpha;
      ep.beta = beta;
      ep.c_in = static_cast<const __half*>(C);
      return launch_gemm_tc(kTcF16, plan_bn_batched(M, N, batch, dev.num_sms), 1, 2, A, B, C, M,
                            N, K, ep, dev, as_stream(stream), batch);
    }
  }
  for (int b = 0; b < batch; ++b) {
    const int rc = gemm_fp16_impl(static_cast<const char*>(A) + b * sa,
                                  static_cast<const char*>(B) + b * sb,
                                  static_cast<char*>(C) + b * sc, M, N, K, alpha, beta,
                                  as_stream(stream), nullptr);
    if (rc) return rc;
  }
  return CLOVE_OK;
}

// ---------------------------------------------------------------------------
// SwiGLU-fused projection (activations.cuh:37-46, declared but not defined in the
// reference): output = silu(input . W_gate) * (input . W_up).
// ---------------------------------------------------------------------------
static bool swiglu_fused_ok(const void* X, const void* Wg, const void* Wu, const void* out, int M,
                            int N, int K) {
  const Override ov = get_override();
  return (ov.path == 0 || ov.path == 4) && M >= 128 && K > 0 && K % 8 == 0 && N % 8 == 0 &&
         aligned16(X) && aligned16(Wg) && aligned16(Wu) && aligned16(out);
}

int clove_swiglu_fused(const void* input, const void* W_gate, const void* W_up, void* output,
                       int batch_seq, int hidden_dim, int intermediate_dim, void* stream) {
  const int M = batch_seq, K = hidden_dim, N = intermediate_dim;
  if (M < 0 || N < 0 || K < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative size");
  if (M == 0 || N == 0) return CLOVE_OK;
  if (output == nullptr || (K > 0 && (input == nullptr || W_gate == nullptr || W_up == nullptr)))
    return fail(CLOVE_ERR_INVALID_ARG, "null matrix pointer");
  DeviceInfo dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  if (swiglu_fused_ok(input, W_gate, W_up, output, M, N, K)) {
    kern::EpiParams ep{};
    ep.mode = kern::kEpiF16AlphaBeta;
    ep.alpha = 1.f;
    ep.beta = 0.f;
    return launch_gemm_tc2(kTcF16, input, W_gate, output, M, N, K, ep, dev, s, W_up);
  }
  // Unfused: both projections into stream-ordered scratch, then the elementwise op.
  const size_t n = static_cast<size_t>(M) * N;
  void* scratch = nullptr;
  rc = check_cuda(cudaMallocAsync(&scratch, 2 * n * sizeof(__half), s), "cudaMallocAsync(swiglu)");
  if (rc) return rc;
  __half* g = static_cast<__half*>(scratch);
  __half* u = g + n;
  rc = gemm_fp16_impl(input, W_gate, g, M, N, K, 1.f, 0.f, s, nullptr);
  if (!rc) rc = gemm_fp16_impl(input, W_up, u, M, N, K, 1.f, 0.f, s, nullptr);
  if (!rc) rc = launch_swiglu_f16(g, u, output, static_cast<long long>(n), s);
  const int rc2 = check_cuda(cudaFreeAsync(scratch, s), "cudaFreeAsync(swiglu)");
  return rc ? rc : rc2;
}

// ---------------------------------------------------------------------------
// INT8
// ---------------------------------------------------------------------------
extern "C++" {  // internal C++ entry (gemm_int8_noalloc.cu)
namespace clove {
namespace rt {
// Kernel family of an int8 call with fp16 C (see internal.h).
int int8_route(const int8_t* A, const int8_t* B, const void* C, int M, int N, int K,
               const char** family) {
  DeviceInfo dev;
  const int rc = current_device(&dev);
  if (rc) return rc;
  const Override ov = get_override();
  const bool tc_ok = K > 0 && K % 16 == 0 && N % 16 == 0 && aligned16(A) && aligned16(B) &&
                     aligned16(C);
  const bool gemv_ok = K > 0 && N <= 8 && K % 16 == 0 && aligned16(A) &&
                       gemv_int8_smem(N, K) <= 200 * 1024;
  int path = ov.path;
  if ((path == 1 || path == 4) && !tc_ok) path = 0;
  if (path == 2 && !gemv_ok) path = 0;
  if (path == 0) path = gemv_ok ? 2 : (tc_ok ? 1 : 3);
  if (path == 2) {
    *family = "gemv_int8";
  } else if (path == 3) {
    *family = "simt_int8";
  } else {
    const TcPlan plan = plan_tc(M, N, K, 1, dev.num_sms);
    *family = plan.pair ? "tc2_int8" : plan.split > 1 ? "tc_int8_split" : "tc_int8";
  }
  return CLOVE_OK;
}
}  // namespace rt
}  // namespace clove
}  // extern "C++"

// mode: 1 per-tensor, 2 row/col, 3 raw int32 accumulators.
static int gemm_int8_impl(const int8_t* A, const int8_t* B, void* C, int M, int N, int K, int mode,
                          float scale, int za, int zb, const float* rs, const float* cs,
                          cudaStream_t s, const char** chosen,
                          const PeerTargets* peer = nullptr) {
  if (M < 0 || N < 0 || K < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative size");
  if (M == 0 || N == 0) return CLOVE_OK;
  if (A == nullptr || B == nullptr || C == nullptr)
    return fail(CLOVE_ERR_INVALID_ARG, "null matrix pointer");
  if (mode == 2 && (rs == nullptr || cs == nullptr))
    return fail(CLOVE_ERR_INVALID_ARG, "null scale vector");
  const int out_bytes = mode == 3 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(C) & (out_bytes - 1)) != 0)
    return fail(CLOVE_ERR_INVALID_ARG, "misaligned C");
  DeviceInfo dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  const Override ov = get_override();
  const bool tc_ok = K > 0 && K % 16 == 0 && N % 16 == 0 && aligned16(A) && aligned16(B) &&
                     aligned16(C);
  const bool gemv_ok = K > 0 && N <= 8 && K % 16 == 0 && aligned16(A) &&
                       gemv_int8_smem(N, K) <= 200 * 1024;
  int path = ov.path;
  if ((path == 1 || path == 4) && !tc_ok) path = 0;
  if (path == 2 && !gemv_ok) path = 0;
  if (path == 0) path = gemv_ok ? 2 : (tc_ok ? 1 : 3);
  if (peer != nullptr && (path == 2 || path == 3 || out_bytes != 2)) return CLOVE_ERR_UNSUPPORTED;
  if (path == 2) {
    if (chosen) *chosen = "gemv_int8";
    kern::GemvI8Epi ep{mode, scale, rs, cs, za, zb};
    return launch_gemv_int8(A, B, C, M, N, K, ep, dev, s);
  }
  if (path == 3) {
    if (chosen) *chosen = "simt_int8";
    kern::SimtEpi ep{};
    ep.mode = mode;
    ep.scale = scale;
    ep.row_scale = rs;
    ep.col_scale = cs;
    ep.za = za;
    ep.zb = zb;
    return launch_simt_i8(A, B, C, M, N, K, ep, s);
  }
  const TcPlan plan = plan_tc(M, N, K, 1, dev.num_sms);
  if (chosen) *chosen = (plan.pair && out_bytes == 2) ? "tc2_int8" : plan.split > 1 ? "tc_int8_split" : "tc_int8";
  kern::EpiParams ep{};
  ep.mode = mode == 1 ? kern::kEpiI8Tensor : mode == 2 ? kern::kEpiI8RowCol : kern::kEpiI32Raw;
  ep.scale = scale;
  ep.row_scale = rs;
  ep.col_scale = cs;
  ep.za = za;
  ep.zb = zb;
  // Zero points: row sums of A (zb != 0) and column sums of B (za != 0) in
  // stream-ordered scratch.
  int32_t* sums = nullptr;
  if (za != 0 || zb != 0) {
    rc = check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&sums),
                                    sizeof(int32_t) * (static_cast<size_t>(M) + N), s),
                    "cudaMallocAsync(zero-point sums)");
    if (rc) return rc;
    if (zb != 0) rc = launch_int8_row_sums(A, sums, M, K, s);
    if (!rc && za != 0) rc = launch_int8_col_sums(B, sums + M, K, N, s);
    ep.row_sum = sums;
    ep.col_sum = sums + M;
  }
  if (!rc) {
    if (plan.pair && out_bytes == 2)
      rc = launch_gemm_tc2(kTcI8, A, B, C, M, N, K, ep, dev, s, nullptr, peer);
    else
      rc = launch_gemm_tc(kTcI8, plan.bn, plan.split, out_bytes, A, B, C, M, N, K, ep, dev, s, 1,
                          peer);
  }
  if (sums != nullptr) {
    const int rc2 = check_cuda(cudaFreeAsync(sums, s), "cudaFreeAsync(zero-point sums)");
    if (!rc) rc = rc2;
  }
  return rc;
}

int clove_gemm_int8(const int8_t* A_q, const int8_t* B_q, void* C, int M, int N, int K,
                    float A_scale, int8_t A_zero, float B_scale, int8_t B_zero, void* stream) {
  return gemm_int8_impl(A_q, B_q, C, M, N, K, 1, A_scale * B_scale, A_zero, B_zero, nullptr,
                        nullptr, as_stream(stream), nullptr);
}

int clove_gemm_int8_rowcol(const int8_t* A_q, const int8_t* B_q, void* C, int M, int N, int K,
                           const float* A_row_scale, const float* B_col_scale, void* stream) {
  return gemm_int8_impl(A_q, B_q, C, M, N, K, 2, 0.f, 0, 0, A_row_scale, B_col_scale,
                        as_stream(stream), nullptr);
}

int clove_debug_int8_acc(const int8_t* A_q, const int8_t* B_q, int32_t* acc, int M, int N, int K,
                         int8_t A_zero, int8_t B_zero, void* stream) {
  return gemm_int8_impl(A_q, B_q, acc, M, N, K, 3, 0.f, A_zero, B_zero, nullptr, nullptr,
                        as_stream(stream), nullptr);
}

// ---------------------------------------------------------------------------
// INT4
// ---------------------------------------------------------------------------
static int gemm_int4_impl(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                          const void* Bs, const void* Bz, void* C, int32_t* G, int M, int N, int K,
                          cudaStream_t s, const char** chosen, const PeerTargets* peer = nullptr) {
  if (M < 0 || N < 0 || K < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative size");
  if (M == 0 || N == 0) return CLOVE_OK;
  if (K % CLOVE_INT4_GROUP_SIZE != 0)
    return fail(CLOVE_ERR_UNSUPPORTED, "int4: K=%d is not a multiple of the group size 128", K);
  if (Aq == nullptr || As == nullptr || Az == nullptr || Bq == nullptr || Bs == nullptr ||
      Bz == nullptr || C == nullptr)
    return fail(CLOVE_ERR_INVALID_ARG, "null pointer");
  if (!aligned2(As) || !aligned2(Az) || !aligned2(Bs) || !aligned2(Bz) || !aligned2(C) ||
      (G != nullptr && !aligned4(G)))
    return fail(CLOVE_ERR_INVALID_ARG, "misaligned fp16 / int32 pointer");
  DeviceInfo dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  if (K == 0) return launch_scale_f16(C, static_cast<long long>(M) * N, 0.f, s);
  const Override ov = get_override();
  const int NG = K / 128;
  const bool gemv_n_ok = N <= 8 && aligned16(Aq) && aligned4(Bq) && gemv_int4_smem(N, K) <= 200 * 1024;
  const bool gemv_m_ok = M <= 8 && aligned16(Bq) && aligned4(Aq) && gemv_int4_smem(M, K) <= 200 * 1024;
  const bool tc_ok = gemm_int4_tc_eligible(Aq, As, Az, Bq, Bs, Bz, C, M, N, K);
  int path = ov.path;
  if (path == 1 && !tc_ok) path = 0;
  if (path == 2 && !(gemv_n_ok || gemv_m_ok)) path = 0;
  if (path == 0) path = (gemv_n_ok || gemv_m_ok) ? 2 : (tc_ok ? 1 : 3);
  if (peer != nullptr && (path != 1 || G != nullptr)) return CLOVE_ERR_UNSUPPORTED;
  if (path == 2) {
    if (gemv_n_ok && (N <= M || !gemv_m_ok)) {
      if (chosen) *chosen = "gemv_int4";
      return launch_gemv_int4(Aq, As, Az, Bq, Bs, Bz, C, G, M, N, K, N, 1,
                              static_cast<long long>(N) * NG, NG, dev, s);
    }
    if (chosen) *chosen = "gemv_int4_t";
    // Rows of B stream past the M (<= 8) vectors of A; C[m,n] at m*N + n.
    return launch_gemv_int4(Bq, Bs, Bz, Aq, As, Az, C, G, N, M, K, 1, N, NG,
                            static_cast<long long>(N) * NG, dev, s);
  }
  if (path == 1) {
    if (chosen) *chosen = "tc_int4";
    return launch_gemm_int4_tc(Aq, As, Az, Bq, Bs, Bz, C, G, M, N, K, dev, s, peer);
  }
  if (chosen) *chosen = "simt_int4";
  return launch_simt_i4(Aq, As, Az, Bq, Bs, Bz, C, G, M, N, K, s);
}

extern "C++" {  // internal C++ entry (nsplit.cpp), inside this file's extern "C" block
namespace clove {
namespace rt {
int gemm_int8_rowcol_replicated(const int8_t* A, const int8_t* B, void* C, int M, int N, int K,
                                const float* rs, const float* cs, const PeerTargets& peer,
                                cudaStream_t s) {
  return gemm_int8_impl(A, B, C, M, N, K, 2, 0.f, 0, 0, rs, cs, s, nullptr, &peer);
}
int gemm_int4_replicated(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                         const void* Bs, const void* Bz, void* C, int M, int N, int K,
                         const PeerTargets& peer, cudaStream_t s) {
  return gemm_int4_impl(Aq, As, Az, Bq, Bs, Bz, C, nullptr, M, N, K, s, nullptr, &peer);
}
}  // namespace rt
}  // namespace clove
}

int clove_gemm_int4(const uint8_t* A_q, const void* A_scale, const void* A_zero,
                    const uint8_t* B_q, const void* B_scale, const void* B_zero, void* C, int M,
                    int N, int K, void* stream) {
  return gemm_int4_impl(A_q, A_scale, A_zero, B_q, B_scale, B_zero, C, nullptr, M, N, K,
                        as_stream(stream), nullptr);
}

int clove_debug_int4_group_acc(const uint8_t* A_q, const void* A_scale, const void* A_zero,
                               const uint8_t* B_q, const void* B_scale, const void* B_zero,
                               void* C, int32_t* G, int M, int N, int K, void* stream) {
  if (G == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "G is NULL");
  return gemm_int4_impl(A_q, A_scale, A_zero, B_q, B_scale, B_zero, C, G, M, N, K,
                        as_stream(stream), nullptr);
}

int clove_quantize_int4(const void* W, int rows, int K, uint8_t* codes, void* scales, void* zeros,
                        void* stream) {
  if (rows < 0 || K < 0) return fail(CLOVE_ERR_INVALID_ARG, "negative size");
  if (K % CLOVE_INT4_GROUP_SIZE != 0)
    return fail(CLOVE_ERR_INVALID_ARG, "quantize_int4: K must be a multiple of 128");
  if (rows == 0 || K == 0) return CLOVE_OK;
  if (W == nullptr || codes == nullptr || scales == nullptr || zeros == nullptr)
    return fail(CLOVE_ERR_INVALID_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(W) & 7u) != 0 || (reinterpret_cast<uintptr_t>(codes) & 1u) != 0 ||
      !aligned2(scales) || !aligned2(zeros))
    return fail(CLOVE_ERR_INVALID_ARG, "quantize_int4: W 8-byte, codes/scales/zeros 2-byte aligned");
  DeviceInfo dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  return launch_quantize_int4(W, rows, K, codes, scales, zeros, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------
int clove_flash_attention(const void* Q, const void* K, const void* V, void* O, int batch,
                          int num_heads, int num_kv_heads, int seq_len, int head_dim, float scale,
                          int causal, int layout, void* stream) {
  if (Q == nullptr || K == nullptr || V == nullptr || O == nullptr)
    return fail(CLOVE_ERR_INVALID_ARG, "null tensor pointer");
  if (batch <= 0 || num_heads <= 0 || num_kv_heads <= 0 || seq_len <= 0)
    return fail(CLOVE_ERR_INVALID_ARG, "batch, heads and seq_len must be positive");
  if (num_heads % num_kv_heads != 0)
    return fail(CLOVE_ERR_INVALID_ARG, "num_heads (%d) is not a multiple of num_kv_heads (%d)",
                num_heads, num_kv_heads);
  if (layout != 0 && layout != 1) return fail(CLOVE_ERR_INVALID_ARG, "layout must be 0 or 1");
  if (!(scale > 0.f) || !std::isfinite(scale))
    return fail(CLOVE_ERR_INVALID_ARG, "scale must be positive and finite");
  if (head_dim != 128)
    return fail(CLOVE_ERR_UNSUPPORTED, "head_dim %d: only 128 is supported (as the reference)",
                head_dim);
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
    return fail(CLOVE_ERR_UNSUPPORTED, "attention needs 16-byte aligned tensors");
  DeviceInfo dev;
  const int rc = current_device(&dev);
  if (rc) return rc;
  return launch_attention(Q, K, V, O, batch, num_heads, num_kv_heads, seq_len, scale, causal != 0,
                          layout, dev, as_stream(stream));
}

int clove_debug_exp2_poly(const float* x, float* y, int n, void* stream) {
  if (x == nullptr || y == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "null pointer");
  if (n < 0 || n % 2 != 0) return fail(CLOVE_ERR_INVALID_ARG, "n must be even and non-negative");
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 7u) != 0)
    return fail(CLOVE_ERR_INVALID_ARG, "x and y must be 8-byte aligned");
  DeviceInfo dev;
  const int rc = current_device(&dev);
  if (rc) return rc;
  return launch_exp2_poly_probe(x, y, n, as_stream(stream));
}

int clove_debug_stream_read(const void* src, size_t nbytes, uint32_t* out, void* stream) {
  if (src == nullptr || out == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "null pointer");
  if (nbytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src) & 15u) != 0)
    return fail(CLOVE_ERR_INVALID_ARG, "stream_read needs 16-byte aligned, 16-byte multiple");
  DeviceInfo dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  return launch_stream_read(src, nbytes, out, dev, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Introspection
// ---------------------------------------------------------------------------
int clove_debug_stream_k_plan(int tiles, int pairs, int kb_total, int force, int* out) {
  if (out == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "null output");
  if (tiles < 0 || pairs < 1 || kb_total < 1 || force < 0 || force > 2)
    return fail(CLOVE_ERR_INVALID_ARG, "bad stream-K plan arguments");
  const SkPlan p = plan_stream_k(tiles, pairs, kb_total, force);
  out[0] = p.dp_tiles;
  out[1] = p.sk_tiles;
  out[2] = p.max_contrib;
  out[3] = p.pairs;
  return CLOVE_OK;
}

int clove_describe_dispatch(int dtype, int M, int N, int K, char* buf, size_t buflen) {
  if (buf == nullptr || buflen == 0) return fail(CLOVE_ERR_INVALID_ARG, "null buffer");
  DeviceInfo dev{0, 148, 10, 0};
  DeviceInfo real;
  if (current_device(&real) == CLOVE_OK) dev = real;
  const Override ov = get_override();
  const char* name = "?";
  int bn = 0, split = 0;
  if (M <= 0 || N <= 0) {
    name = "noop";
  } else if (dtype == 3) {
    // Projection shapes only (alignment is the caller's): fused unless M < 128 or
    // K, N are not multiples of 8.
    const Override ovs = get_override();
    const bool fused = (ovs.path == 0 || ovs.path == 4) && M >= 128 && K > 0 && K % 8 == 0 &&
                       N % 8 == 0;
    name = fused ? "tc2_swiglu" : "unfused_swiglu";
  } else if (dtype == 0) {
    const bool gemv = N <= 8 && K % 8 == 0 && gemv_f16_smem(N, K) <= 200 * 1024;
    const bool tc = K % 8 == 0 && N % 8 == 0 && K > 0;
    int path = ov.path ? ov.path : ((gemv && N < 16) ? 2 : (tc ? 1 : 3));
    name = path == 2 ? "gemv_f16" : path == 3 ? "simt_f16" : "tc_f16";
    if (path == 1 || path == 4) {
      const TcPlan p = plan_tc(M, N, K, 2, dev.num_sms);
      bn = p.bn;
      split = p.split;
      if (p.pair) name = "tc2_f16";
    }
  } else if (dtype == 1) {
    const bool gemv = N <= 8 && K % 16 == 0 && K > 0;
    const bool tc = K % 16 == 0 && N % 16 == 0 && K > 0;
    int path = ov.path ? ov.path : (gemv ? 2 : (tc ? 1 : 3));
    name = path == 2 ? "gemv_int8" : path == 3 ? "simt_int8" : "tc_int8";
    if (path == 1 || path == 4) {
      const TcPlan p = plan_tc(M, N, K, 1, dev.num_sms);
      bn = p.bn;
      split = p.split;
      if (p.pair) name = "tc2_int8";
    }
  } else {
    const bool gemv = (N <= 8 || M <= 8) && K % 128 == 0;
    const bool tc = K % 128 == 0 && N % 8 == 0;
    int path = ov.path ? ov.path : (gemv ? 2 : (tc ? 1 : 3));
    name = path == 2 ? (N <= 8 && (N <= M || M > 8) ? "gemv_int4" : "gemv_int4_t")
                     : path == 1 ? "tc_int4" : "simt_int4";
    if (path == 2 && ov.path == 0) {
      // Vectors on the N side, or (transposed) on the M side.
      const bool t = !(N <= 8 && (N <= M || M > 8));
      snprintf(buf, buflen, "%s (%s)", name,
               describe_gemv_int4(t ? N : M, t ? M : N, K, dev));
      return CLOVE_OK;
    }
  }
  snprintf(buf, buflen, "%s bn=%d split=%d", name, bn, split);
  return CLOVE_OK;
}

}  // extern "C"
