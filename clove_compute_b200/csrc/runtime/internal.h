// internal.h -- interfaces between the C-ABI layer (runtime/) and the kernel
// translation units (kernels/). Not installed; not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "clove/capi.h"

namespace clove {
namespace kern {
struct EpiParams;
struct PeerOut;
struct GemvI8Epi;
struct SimtEpi;
}  // namespace kern

namespace rt {

// Records a message for clove_last_error_string() (thread-local) and returns code.
int fail(int code, const char* fmt, ...);
// Maps a CUDA error to CLOVE_ERR_CUDA with a message; CLOVE_OK on cudaSuccess.
int check_cuda(cudaError_t e, const char* what);

struct DeviceInfo {
  int device;
  int num_sms;
  int cc_major, cc_minor;
};
// Current device's properties (cached per device). Fails unless cc 10.x.
int current_device(DeviceInfo* out);

// Dispatch override for tests (clove_set_dispatch_override).
struct Override {
  int path;   // 0 auto, 1 tensor core (one SM per tile), 2 gemv, 3 simt, 4 CTA-pair tiles
  int bn;     // 0 auto
  int split;  // 0 auto
};
Override get_override();

// clove_set_weight_prefetch: decode kernels may stream their weight operand before
// the previous kernel on the stream has finished.
bool weight_prefetch_enabled();
// Test hook: path 2 with bn == 1 forces the register GEMV instead of the
// warp-specialised one.
bool ws_disabled();
// Test hook: override (path 2, bn 2) picks the bulk-copy-ring INT4 decode kernel
// instead of the default direct-load one.
bool ws2_selected();

// Replicated output of an N-split fp16 GEMM (kern::PeerOut): the row-major
// [M, ldc] C of every rank, mapped into this process; this rank's columns start
// at col0. The tile launchers encode one TMA store map per rank from it. The
// receiver-ready handshake (kern::PeerOut) uses ready_slot[q] = slot `rank` of
// rank q's ready array, ready_in = this rank's ready array and epoch = this
// rank's count of completed replicated calls.
// mc: the multicast address of every rank's C (one NVLink multicast object bound
// to all of them), or null for per-rank stores through dst.
struct PeerTargets {
  int count;
  int ldc;
  int col0;
  int rank;
  void* mc;
  void* dst[8];
  unsigned long long* ready_slot[8];
  const unsigned long long* ready_in;
  const unsigned long long* epoch;
};

// Tile shape chosen for a tensor-core call (capi.cpp).
struct TcPlan {
  int bn;
  int split;
  bool pair;  // CTA-pair 256 x 256 kernel
};
TcPlan plan_tc(int M, int N, int K, int elem, int num_sms);
// Kernel family clove_gemm_int8 runs for this shape and these pointers (with the
// test override applied): "gemv_int8", "simt_int8", "tc2_int8" (CTA pairs),
// "tc_int8_split" or "tc_int8".
int int8_route(const int8_t* A, const int8_t* B, const void* C, int M, int N, int K,
               const char** family);

// ---- tensor-core tile kernels (kernels/gemm_tc_sm100.cu)
enum TcOp { kTcF16 = 0, kTcI8 = 1 };
// bn in {32,64,128,256}; split in [1,8] (split > 1 requires bn <= 64);
// out_bytes 2 (fp16 C) or 4 (int32 C, raw accumulators).
// batch > 1: `batch` densely packed problems ([batch,M,K] . [batch,K,N]) in one
// persistent launch (split must be 1).
int launch_gemm_tc(int op, int bn, int split, int out_bytes, const void* A, const void* B,
                   void* C, int M, int N, int K, const kern::EpiParams& ep,
                   const DeviceInfo& dev, cudaStream_t stream, int batch = 1,
                   const PeerTargets* peer = nullptr);
// Stream-K schedule of the CTA-pair kernel (kern::SkParams); pairs = CTA pairs to
// launch. force: 0 auto, 1 never, 2 whenever the tiles leave a partial wave.
struct SkPlan {
  int dp_tiles, sk_tiles, max_contrib, pairs;
};
SkPlan plan_stream_k(int tiles, int pairs, int kb_total, int force);
// CTA-pair kernel: 256 x 256 tiles on two SMs (fp16 C).
// B2 != nullptr: fp16 GLU, C = silu(A . B) * (A . B2) (256 x 128 output tiles).
// allow_stream_k = false keeps whole-K tiles, which need no workspace (the call
// then allocates nothing).
int launch_gemm_tc2(int op, const void* A, const void* B, void* C, int M, int N, int K,
                    const kern::EpiParams& ep, const DeviceInfo& dev, cudaStream_t stream,
                    const void* B2 = nullptr, const PeerTargets* peer = nullptr,
                    bool allow_stream_k = true);
// Clears every kept stream-K ticket array (after a kernel failure left tickets set).
void reset_stream_k_tickets();
// True when (op, bn, split, out_bytes) is an instantiated kernel.
bool gemm_tc_supported(int op, int bn, int split, int out_bytes);
int read_clear_error_tc();

// ---- GEMV kernels (kernels/gemv_sm100.cu)
const char* describe_gemv_int4(int rows, int nc, int K, const DeviceInfo& dev);
int launch_gemv_int4(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                     const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int rows, int nc,
                     int K, long long ldc_row, long long ldc_col, long long ldg_row,
                     long long ldg_col, const DeviceInfo& dev, cudaStream_t stream);
size_t gemv_int4_smem(int nc, int K);
int launch_gemv_int8(const int8_t* A, const int8_t* B, void* C, int rows, int nc, int K,
                     const kern::GemvI8Epi& ep, const DeviceInfo& dev, cudaStream_t stream);
size_t gemv_int8_smem(int nc, int K);
int launch_gemv_f16(const void* A, const void* B, void* C, int rows, int nc, int K, float alpha,
                    float beta, const DeviceInfo& dev, cudaStream_t stream);
size_t gemv_f16_smem(int nc, int K);
int read_clear_error_gemv();
// Bare read of nbytes (multiple of 16, 16-byte aligned) into nothing: the HBM floor
// of one launch of that size.
int launch_stream_read(const void* src, size_t nbytes, uint32_t* out, const DeviceInfo& dev,
                       cudaStream_t stream);

// out = silu(g) * u over n fp16 elements (kernels/fallback_simt.cu).
int launch_swiglu_f16(const void* g, const void* u, void* out, long long n, cudaStream_t stream);

// ---- attention (kernels/attention_sm100.cu)
// head_dim 128; layout 0: [batch, heads, seq, 128], 1: [batch, seq, heads, 128];
// K / V have kv_heads heads (heads % kv_heads == 0).
int launch_attention(const void* Q, const void* K, const void* V, void* O, int batch, int heads,
                     int kv_heads, int seq, float scale, bool causal, int layout,
                     const DeviceInfo& dev, cudaStream_t stream);
int read_clear_error_attn();
// y[i] = 2^x[i] through the attention kernel's FMA-pipe polynomial (test hook; n even).
int launch_exp2_poly_probe(const float* x, float* y, int n, cudaStream_t stream);

// ---- INT4 packing tool (kernels/quant_int4.cu)
int launch_quantize_int4(const void* W, int rows, int K, uint8_t* codes, void* scales, void* zeros,
                         cudaStream_t stream);

// ---- SIMT fallback + helpers (kernels/fallback_simt.cu)
int launch_simt_f16(const void* A, const void* B, void* C, int batch, int M, int N, int K,
                    float alpha, float beta, cudaStream_t stream);
int launch_simt_i8(const int8_t* A, const int8_t* B, void* C, int M, int N, int K,
                   const kern::SimtEpi& ep, cudaStream_t stream);
int launch_simt_i4(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                   const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int M, int N, int K,
                   cudaStream_t stream);
int launch_int8_row_sums(const int8_t* A, int32_t* out, int M, int K, cudaStream_t stream);
int launch_int8_col_sums(const int8_t* B, int32_t* out, int K, int N, cudaStream_t stream);
int launch_scale_f16(void* C, long long n, float beta, cudaStream_t stream);
int read_clear_error_simt();

// ---- INT4 tensor-core kernel (kernels/gemm_int4_sm100.cu)
// Gdbg (may be NULL): exact group accumulators G [M,N,K/128] for tests.
int launch_gemm_int4_tc(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                        const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int M, int N,
                        int K, const DeviceInfo& dev, cudaStream_t stream,
                        const PeerTargets* peer = nullptr);
// TMA store maps of a replicated output (gemm_tc_sm100.cu).
int encode_peer_maps(const PeerTargets& pt, int M, int N, uint32_t box_cols, int swizzle,
                     kern::PeerOut* out);
bool gemm_int4_tc_eligible(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                           const void* Bs, const void* Bz, const void* C, int M, int N, int K);
int read_clear_error_int4();

}  // namespace rt
}  // namespace clove
