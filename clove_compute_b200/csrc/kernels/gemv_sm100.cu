// gemv_sm100.cu -- host launchers for the N <= 8 GEMV kernels (gemv_sm100.cuh).
#include "gemv_sm100.cuh"
#include "../runtime/internal.h"

namespace clove {
namespace rt {

CLOVE_DEFINE_ERROR_READER(read_clear_error_gemv)

}  // namespace rt
}  // namespace clove

#ifdef CLOVE_TRACE
// Development builds only: trace slots of the decode kernels.
extern "C" int clove_trace_read_gemv(unsigned long long* out) {
  return static_cast<int>(cudaMemcpyFromSymbol(out, g_clove_trace, sizeof(unsigned long long) * 256));
}
extern "C" int clove_trace_write_gemv(const unsigned long long* in) {
  return static_cast<int>(cudaMemcpyToSymbol(g_clove_trace, in, sizeof(unsigned long long) * 256));
}
#endif

namespace clove {
namespace rt {

namespace {

// Enough CTAs to put every row block in flight at once, at most 8 CTAs per SM.
unsigned gemv_grid(int rows, const DeviceInfo& dev, int rows_per_warp = kern::kGemvRowsPerWarp) {
  const int warps_per_cta = kern::kGemvThreads / 32;
  const long long row_blocks = (rows + rows_per_warp - 1) / rows_per_warp;
  long long ctas = (row_blocks + warps_per_cta - 1) / warps_per_cta;
  const long long cap = static_cast<long long>(dev.num_sms) * 8;
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  return static_cast<unsigned>(ctas);
}

template <typename KernelT>
int prepare(KernelT kernel, size_t smem) {
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(
        reinterpret_cast<const void*>(kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(smem));
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(gemv smem)");
  }
  return CLOVE_OK;
}

// Launch with programmatic stream serialisation: the kernel may be scheduled while
// its predecessor on the stream drains; it orders every global access after
// griddepcontrol.wait, so results are those of a plain launch.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), unsigned grid, size_t smem, cudaStream_t stream,
               const char* what, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kern::kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, args...), what);
}

template <int NC, int PW>
int gemv_int4_ws2(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                  const void* Bs, const void* Bz, void* C, int rows, int K, long long ldc_row,
                  long long ldc_col, const DeviceInfo& dev, cudaStream_t stream) {
  int grid = dev.num_sms;
  if (rows < grid * 8) grid = (rows + 7) / 8;
  const int per_cta = (rows + grid - 1) / grid;
  const int chunks = (per_cta + kern::kWsChunkRows - 1) / kern::kWsChunkRows;
  const int chunk_bytes = kern::gemv_ws_chunk_bytes(K);
  // <= ~100 KB so that the next kernel's CTA fits beside this one (overlap under PDL).
  int slots = (100 * 1024) / (chunk_bytes + 16);
  if (slots > chunks) slots = chunks;
  if (slots < 1) slots = 1;
  const size_t part_bytes = static_cast<size_t>(per_cta) * kern::kWs2WindowGroups * NC * sizeof(float);
  const size_t smem = static_cast<size_t>(slots) * (chunk_bytes + 16) + part_bytes;
  auto kernel = kern::gemv_int4_ws2_kernel<NC, PW>;
  int rc = prepare(kernel, smem);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kern::kWs2Threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int early = weight_prefetch_enabled() ? 1 : 0;
  return check_cuda(
      cudaLaunchKernelEx(&cfg, kernel, Aq, static_cast<const __half*>(As),
                         static_cast<const __half*>(Az), Bq, static_cast<const __half*>(Bs),
                         static_cast<const __half*>(Bz), static_cast<__half*>(C), rows, K, ldc_row,
                         ldc_col, slots, early),
      "gemv_int4_ws2 launch");
}

template <int NC, int PW, int RMAX, int MINB, int RG, int WG>
int launch_int4_ldg(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                    const void* Bs, const void* Bz, void* C, int rows, int K, long long ldc_row,
                    long long ldc_col, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(RG * WG * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int early = weight_prefetch_enabled() ? 1 : 0;
  return check_cuda(
      cudaLaunchKernelEx(&cfg, kern::gemv_int4_ldg_kernel<NC, PW, RMAX, MINB, RG, WG>, Aq,
                         static_cast<const __half*>(As), static_cast<const __half*>(Az), Bq,
                         static_cast<const __half*>(Bs), static_cast<const __half*>(Bz),
                         static_cast<__half*>(C), rows, K, ldc_row, ldc_col, early),
      "gemv_int4_ldg launch");
}

template <int NC, int PW>
int gemv_int4_ldg(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                  const void* Bs, const void* Bz, void* C, int rows, int K, long long ldc_row,
                  long long ldc_col, const DeviceInfo& dev, cudaStream_t stream) {
  // One or two vectors and at least 2 x 148 x 8 rows: several CTAs per SM, one
  // window per lane, so that some CTAs' loads are in flight while others reduce,
  // and under programmatic launch the next call's CTAs start in the slots this
  // call's CTAs leave. Rows up to 4096 codes: four CTAs of 2 x 4 warps per SM
  // (<= 64 registers, 4 rows per warp and round); one vector with longer rows (up
  // to 12288 codes): two CTAs of 1 x 12 warps (8 rows per warp and round, <= 85
  // registers).
  if (NC == 2 && PW == 1 && rows >= 2 * dev.num_sms * 8)
    return launch_int4_ldg<2, 1, 4, 4, 2, 4>(Aq, As, Az, Bq, Bs, Bz, C, rows, K, ldc_row,
                                             ldc_col, 4 * dev.num_sms, stream);
  if (NC == 1 && rows >= 2 * dev.num_sms * 8) {
    if (PW == 1)
      return launch_int4_ldg<1, 1, 4, 4, 2, 4>(Aq, As, Az, Bq, Bs, Bz, C, rows, K, ldc_row,
                                               ldc_col, 4 * dev.num_sms, stream);
    return launch_int4_ldg<1, 1, 8, 2, 1, 12>(Aq, As, Az, Bq, Bs, Bz, C, rows, K, ldc_row,
                                              ldc_col, 2 * dev.num_sms, stream);
  }
  // Rows per warp and round: 8, or 4 when three windows per lane (K up to 12288)
  // would not leave the registers for 8.
  constexpr int RMAX = PW > 2 ? 4 : 8;
  int grid = dev.num_sms;
  if (rows < grid * 8) grid = (rows + 7) / 8;
  return launch_int4_ldg<NC, PW, RMAX, 1, 4, 4>(Aq, As, Az, Bq, Bs, Bz, C, rows, K, ldc_row,
                                                ldc_col, grid, stream);
}

template <int NC, int P>
int gemv_int4_reg(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                  const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int rows, int K,
                  long long ldc_row, long long ldc_col, long long ldg_row, long long ldg_col,
                  const DeviceInfo& dev, cudaStream_t stream) {
  constexpr int R = 2;
  const int early = weight_prefetch_enabled() ? 1 : 0;
  return launch_pdl(kern::gemv_int4_reg_kernel<NC, P, R>, gemv_grid(rows, dev, R), 0, stream,
                    "gemv_int4_reg launch", Aq, static_cast<const __half*>(As),
                    static_cast<const __half*>(Az), Bq, static_cast<const __half*>(Bs),
                    static_cast<const __half*>(Bz), static_cast<__half*>(C), Gdbg, rows, K,
                    ldc_row, ldc_col, ldg_row, ldg_col, early);
}

template <int NC>
int gemv_int4_nc(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                 const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int rows, int K,
                 long long ldc_row, long long ldc_col, long long ldg_row, long long ldg_col,
                 const DeviceInfo& dev, cudaStream_t stream) {
  const size_t smem = kern::gemv_int4_smem_bytes(NC, K);
  // One row per warp while every row still gets its own resident warp (the whole
  // matrix in flight at once); two rows per warp beyond that.
  const bool one = rows <= dev.num_sms * 32;
  int rc = one ? prepare(kern::gemv_int4_kernel<NC, 1>, smem)
               : prepare(kern::gemv_int4_kernel<NC, 2>, smem);
  if (rc) return rc;
  auto k = one ? kern::gemv_int4_kernel<NC, 1> : kern::gemv_int4_kernel<NC, 2>;
  k<<<gemv_grid(rows, dev, one ? 1 : 2), kern::kGemvThreads, smem, stream>>>(
      Aq, static_cast<const __half*>(As), static_cast<const __half*>(Az), Bq,
      static_cast<const __half*>(Bs), static_cast<const __half*>(Bz), static_cast<__half*>(C),
      Gdbg, rows, K, ldc_row, ldc_col, ldg_row, ldg_col);
  return check_cuda(cudaGetLastError(), "gemv_int4 launch");
}

template <int NC>
int gemv_int8_nc(const int8_t* A, const int8_t* B, void* C, int rows, int K,
                 const kern::GemvI8Epi& ep, const DeviceInfo& dev, cudaStream_t stream) {
  const size_t smem = kern::gemv_int8_smem_bytes(NC, K);
  int rc = prepare(kern::gemv_int8_kernel<NC>, smem);
  if (rc) return rc;
  kern::gemv_int8_kernel<NC><<<gemv_grid(rows, dev), kern::kGemvThreads, smem, stream>>>(
      A, B, C, rows, K, ep);
  return check_cuda(cudaGetLastError(), "gemv_int8 launch");
}

template <int NC>
int gemv_f16_nc(const void* A, const void* B, void* C, int rows, int K, float alpha, float beta,
                const DeviceInfo& dev, cudaStream_t stream) {
  const size_t smem = kern::gemv_f16_smem_bytes(NC, K);
  int rc = prepare(kern::gemv_f16_kernel<NC>, smem);
  if (rc) return rc;
  kern::gemv_f16_kernel<NC><<<gemv_grid(rows, dev), kern::kGemvThreads, smem, stream>>>(
      static_cast<const __half*>(A), static_cast<const __half*>(B), static_cast<__half*>(C), rows,
      K, alpha, beta);
  return check_cuda(cudaGetLastError(), "gemv_f16 launch");
}

}  // namespace

int launch_stream_read(const void* src, size_t nbytes, uint32_t* out, const DeviceInfo& dev,
                       cudaStream_t stream) {
  const size_t n16 = nbytes / 16;
  if (n16 == 0) return CLOVE_OK;
  kern::stream_read_kernel<<<static_cast<unsigned>(dev.num_sms * 2), kern::kStreamThreads, 0, stream>>>(
      static_cast<const uint4*>(src), n16, out);
  return check_cuda(cudaGetLastError(), "stream_read launch");
}

size_t gemv_int4_smem(int nc, int K) { return kern::gemv_int4_smem_bytes(nc, K); }
size_t gemv_int8_smem(int nc, int K) { return kern::gemv_int8_smem_bytes(nc, K); }
size_t gemv_f16_smem(int nc, int K) { return kern::gemv_f16_smem_bytes(nc, K); }

#define CLOVE_NC_SWITCH(nc, CALL) \
  switch (nc) {                   \
    case 1: return CALL(1);       \
    case 2: return CALL(2);       \
    case 3: return CALL(3);       \
    case 4: return CALL(4);       \
    case 5: return CALL(5);       \
    case 6: return CALL(6);       \
    case 7: return CALL(7);       \
    case 8: return CALL(8);       \
    default: break;               \
  }

// The variant launch_gemv_int4 takes for aligned operands and no debug output.
const char* describe_gemv_int4(int rows, int nc, int K, const DeviceInfo& dev) {
  const int P = (K + 1023) / 1024;
  // Direct-load instances: one vector with up to 12 windows, two with up to 4.
  if (K % 128 == 0 && ((nc == 1 && P <= 12) || (nc == 2 && P <= 4))) {
    if (rows >= 2 * dev.num_sms * 8)
      return P <= 4 ? "ldg 4 CTAs/SM of 2x4 warps" : "ldg 2 CTAs/SM of 1x12 warps";
    return "ldg 1 CTA/SM of 4x4 warps";
  }
  if (nc * P <= 8) return "register-B";
  return "shared-B";
}

int launch_gemv_int4(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                     const void* Bs, const void* Bz, void* C, int32_t* Gdbg, int rows, int nc,
                     int K, long long ldc_row, long long ldc_col, long long ldg_row,
                     long long ldg_col, const DeviceInfo& dev, cudaStream_t stream) {
  // Register-resident B when this lane's share of the vectors fits (nc * P <= 8,
  // P = 1024-element windows per row, the last one possibly partial) and the
  // 16-byte B loads are aligned.
  const int P = (K + 1023) / 1024;
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  // Direct 128-bit loads (gemv_int4_ldg_kernel): whole 128-code groups (16-byte
  // aligned rows of codes), up to 8 windows per vector (12 for one vector), no
  // debug output. The bulk-copy ring variant (gemv_int4_ws2_kernel, whole windows
  // only) stays reachable through the test override.
  if (Gdbg == nullptr && K % 128 == 0 && (nc * P <= 8 || (nc == 1 && P <= 12)) && a16(Aq) &&
      a16(As) && a16(Az) && a16(Bq) && !ws_disabled()) {
    const int PW = (P + kern::kWs2WindowGroups - 1) / kern::kWs2WindowGroups;
    if (ws2_selected() && K % 1024 == 0) {
#define WS2(n, pw)                                                                            \
  if (nc == n && PW == pw)                                                                     \
    return gemv_int4_ws2<n, pw>(Aq, As, Az, Bq, Bs, Bz, C, rows, K, ldc_row, ldc_col, dev, stream);
      WS2(1, 1) WS2(1, 2) WS2(2, 1)
#undef WS2
    }
#define LDG(n, pw)                                                                            \
  if (nc == n && PW == pw)                                                                     \
    return gemv_int4_ldg<n, pw>(Aq, As, Az, Bq, Bs, Bz, C, rows, K, ldc_row, ldc_col, dev, stream);
    LDG(1, 1) LDG(1, 2) LDG(1, 3) LDG(2, 1)
#undef LDG
  }
  if (nc * P <= 8 && (reinterpret_cast<uintptr_t>(Bq) & 15u) == 0) {
#define REG(n, p)                                                                          \
  if (nc == n && P == p)                                                                    \
    return gemv_int4_reg<n, p>(Aq, As, Az, Bq, Bs, Bz, C, Gdbg, rows, K, ldc_row, ldc_col, \
                               ldg_row, ldg_col, dev, stream);
    REG(1, 1) REG(1, 2) REG(1, 3) REG(1, 4) REG(1, 5) REG(1, 6) REG(1, 7) REG(1, 8)
    REG(2, 1) REG(2, 2) REG(2, 3) REG(2, 4)
#undef REG
  }
#define CALL(n)                                                                                  \
  gemv_int4_nc<n>(Aq, As, Az, Bq, Bs, Bz, C, Gdbg, rows, K, ldc_row, ldc_col, ldg_row, ldg_col, \
                  dev, stream)
  CLOVE_NC_SWITCH(nc, CALL)
#undef CALL
  return fail(CLOVE_ERR_UNSUPPORTED, "gemv_int4: %d vectors (max 8)", nc);
}

int launch_gemv_int8(const int8_t* A, const int8_t* B, void* C, int rows, int nc, int K,
                     const kern::GemvI8Epi& ep, const DeviceInfo& dev, cudaStream_t stream) {
#define CALL(n) gemv_int8_nc<n>(A, B, C, rows, K, ep, dev, stream)
  CLOVE_NC_SWITCH(nc, CALL)
#undef CALL
  return fail(CLOVE_ERR_UNSUPPORTED, "gemv_int8: %d columns (max 8)", nc);
}

int launch_gemv_f16(const void* A, const void* B, void* C, int rows, int nc, int K, float alpha,
                    float beta, const DeviceInfo& dev, cudaStream_t stream) {
#define CALL(n) gemv_f16_nc<n>(A, B, C, rows, K, alpha, beta, dev, stream)
  CLOVE_NC_SWITCH(nc, CALL)
#undef CALL
  return fail(CLOVE_ERR_UNSUPPORTED, "gemv_f16: %d columns (max 8)", nc);
}

}  // namespace rt
}  // namespace clove
