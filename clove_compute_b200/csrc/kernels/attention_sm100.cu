// attention_sm100.cu -- host launcher of the tcgen05 attention kernel (attention_sm100.cuh).
#include <atomic>
#include <cmath>

#include "attention_sm100.cuh"
#include "../runtime/internal.h"
#include "../runtime/tensor_map.h"

namespace clove {
namespace rt {

CLOVE_DEFINE_ERROR_READER(read_clear_error_attn)

}  // namespace rt
}  // namespace clove

#ifdef CLOVE_TRACE
// Development builds only: the attention kernel's trace slots.
extern "C" int clove_trace_read_attn(unsigned long long* out, int n) {
  return static_cast<int>(
      cudaMemcpyFromSymbol(out, g_clove_trace, sizeof(unsigned long long) * (n < 256 ? n : 256)));
}
extern "C" int clove_trace_write_attn(const unsigned long long* in) {
  return static_cast<int>(cudaMemcpyToSymbol(g_clove_trace, in, sizeof(unsigned long long) * 256));
}
#endif

namespace clove {
namespace rt {

namespace {
std::atomic<uint64_t> g_attn_attr[2];

// Byte strides (seq, head, batch) of a [B,H,S,D] (layout 0) or [B,S,H,D] (layout 1)
// tensor with `heads` heads.
void attn_strides(int layout, int heads, int seq, uint64_t out[3]) {
  const uint64_t row = 128 * 2;  // head_dim 128, fp16
  if (layout == 0) {
    out[0] = row;
    out[1] = static_cast<uint64_t>(seq) * row;
    out[2] = static_cast<uint64_t>(heads) * seq * row;
  } else {
    out[0] = static_cast<uint64_t>(heads) * row;
    out[1] = row;
    out[2] = static_cast<uint64_t>(seq) * heads * row;
  }
}
}  // namespace

namespace {
// The softmax's polynomial exponential on an array, pair by pair (test hook).
__global__ void exp2_poly_probe_kernel(const float2* __restrict__ x, float2* __restrict__ y,
                                       int pairs) {
  const int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= pairs) return;
  const float2 v = x[i];
  float a, b;
  dev::f2_unpack(dev::f2_exp2_poly(dev::f2_pack(v.x, v.y)), a, b);
  y[i] = make_float2(a, b);
}
}  // namespace

int launch_exp2_poly_probe(const float* x, float* y, int n, cudaStream_t stream) {
  const int pairs = n / 2;
  if (pairs <= 0) return CLOVE_OK;
  exp2_poly_probe_kernel<<<(pairs + 255) / 256, 256, 0, stream>>>(
      reinterpret_cast<const float2*>(x), reinterpret_cast<float2*>(y), pairs);
  return check_cuda(cudaGetLastError(), "exp2_poly_probe launch");
}

int launch_attention(const void* Q, const void* K, const void* V, void* O, int batch, int heads,
                     int kv_heads, int seq, float scale, bool causal, int layout,
                     const DeviceInfo& dev, cudaStream_t stream) {
  using S = kern::AttnShape;
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint64_t qst[3], kvst[3];
  attn_strides(layout, heads, seq, qst);
  attn_strides(layout, kv_heads, seq, kvst);
  const uint64_t qdims[4] = {128, static_cast<uint64_t>(seq), static_cast<uint64_t>(heads),
                             static_cast<uint64_t>(batch)};
  const uint64_t kvdims[4] = {128, static_cast<uint64_t>(seq), static_cast<uint64_t>(kv_heads),
                              static_cast<uint64_t>(batch)};
  CUtensorMap tQ, tK, tV, tO;
  int rc;
  if ((rc = encode_tmap_4d(&tQ, F16, 2, Q, qdims, qst, 64, 128, 128))) return rc;
  if ((rc = encode_tmap_4d(&tK, F16, 2, K, kvdims, kvst, 64, 128, 128))) return rc;
  if ((rc = encode_tmap_4d(&tV, F16, 2, V, kvdims, kvst, 64, 128, 128))) return rc;
  if ((rc = encode_tmap_4d(&tO, F16, 2, O, qdims, qst, 64, 32, 128))) return rc;
  const void* fn = causal ? reinterpret_cast<const void*>(&kern::attention_fwd_kernel<true>)
                          : reinterpret_cast<const void*>(&kern::attention_fwd_kernel<false>);
  const uint64_t bit = 1ull << (dev.device & 63);
  std::atomic<uint64_t>& attr = g_attn_attr[causal ? 1 : 0];
  if ((attr.load(std::memory_order_acquire) & bit) == 0) {
    // The kernel moves registers between its warpgroups with setmaxnreg, planned for
    // a launch allocation of S::REGS_LAUNCH per thread: with fewer, an increase
    // would wait forever, so such a build is refused here rather than launched.
    cudaFuncAttributes fa{};
    rc = check_cuda(cudaFuncGetAttributes(&fa, fn), "cudaFuncGetAttributes(attention)");
    if (rc) return rc;
    if (fa.numRegs != S::REGS_LAUNCH)
      return fail(CLOVE_ERR_UNSUPPORTED,
                  "attention: built with %d registers per thread, its register plan needs %d",
                  fa.numRegs, S::REGS_LAUNCH);
    rc = check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::SMEM_BYTES),
                    "cudaFuncSetAttribute(attention smem)");
    if (rc) return rc;
    attr.fetch_or(bit, std::memory_order_acq_rel);
  }
  int kv_group = heads / kv_heads;
  float scale_log2 = scale * 1.4426950408889634f;  // log2(e)
  void* args[] = {&tQ, &tK, &tV, &tO, &seq, &heads, &kv_group, &scale_log2};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[0].val.programmaticStreamSerializationAllowed = 1;
  const int n_qt = (seq + S::BQ - 1) / S::BQ;
  const long long ctas = static_cast<long long>((n_qt + S::TILES - 1) / S::TILES) * heads * batch;
  if (ctas > 0x7fffffffLL) return fail(CLOVE_ERR_UNSUPPORTED, "attention: %lld CTAs exceed the grid limit", ctas);
  cfg.gridDim = dim3(static_cast<unsigned>(ctas), 1, 1);
  cfg.blockDim = dim3(S::THREADS, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(S::SMEM_BYTES);
  cfg.stream = stream;
  cfg.attrs = la;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelExC(&cfg, fn, args), "attention launch");
}

}  // namespace rt
}  // namespace clove
