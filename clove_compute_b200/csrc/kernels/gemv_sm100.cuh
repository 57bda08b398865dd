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

template <int NC, int R>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_int4_kernel(const uint8_t* __restrict__ Aq, const __half* __restrict__ As,
                     const __half* __restrict__ Az, const uint8_t* __restrict__ Bq,
                     const __half* __restrict__ Bs, const __half* __restrict__ Bz,
                     __half* __restrict__ C, int32_t* __restrict__ Gdbg, int rows, int K,
                     long long ldc_row, long long ldc_col, long long ldg_row, long long ldg_col) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int NG = K >> 7;          // groups per row
  const int NCH = K >> 5;         // 16-byte chunks per row
  const int KB = K >> 1;          // bytes per row
  uint32_t* bp = reinterpret_cast<uint32_t*>(smem);                          // [NC][NCH*8]
  float* sb = reinterpret_cast<float*>(smem + static_cast<size_t>(NC) * K);  // [NC][NG]
  int* zs = reinterpret_cast<int*>(sb + NC * NG);                            // [NC][NG]

  const int lane = static_cast<int>(dev::lane_idx());
  const int gwarp = static_cast<int>(blockIdx.x * (blockDim.x >> 5) + dev::warp_idx());
  const int nwarps = static_cast<int>(gridDim.x * (blockDim.x >> 5));
  const int passes = (NCH + 31) >> 5;  // 512-byte windows per row

  // Loads of one 4-window slab (up to 2 KB of a row) for the R rows of a block.
  uint4 v[R][4];
  __half2 zsA[R][4];
  auto load_slab = [&](int row_blk, int p0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int m = row_blk + r;
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
  };

  // The first slab of this warp's first rows is requested before the B vectors are
  // touched, so its HBM latency overlaps the unpacking below.
  const int first_row = gwarp * R;
  load_slab(first_row, 0);

  // ---- unpack the B vectors (tiny: NC * K/2 bytes). Word order per 16-byte chunk:
  // word 2w = the 4 even-k codes (high nibbles) of A word w, 2w+1 the odd-k codes.
  // The 32 consecutive words a warp produces per iteration are exactly one 128-code
  // group (NC*NCH*8 and blockDim are multiples of 32), so the warp also reduces the
  // group's sum of (b - zB) for the zero-point term.
  for (int idx = threadIdx.x; idx < NC * NCH * 8; idx += blockDim.x) {
    const int n = idx / (NCH * 8);
    const int r = idx - n * NCH * 8;
    const int ch = r >> 3;
    const int w = (r >> 1) & 3;
    const int odd = r & 1;
    const int byte0 = ch * 16 + w * 4;
    const int g = ch >> 2;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(Bq + static_cast<size_t>(n) * KB + byte0);
    const int zb = __half2int_rn(Bz[static_cast<size_t>(n) * NG + g]);
    uint32_t packed = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t byte = (word >> (8 * t)) & 0xffu;
      const int code = odd ? static_cast<int>(byte & 0xfu) : static_cast<int>(byte >> 4);
      packed |= (static_cast<uint32_t>(code - zb) & 0xffu) << (8 * t);
    }
    bp[n * NCH * 8 + r] = packed;
    const int gsum = warp_sum_i32(__dp4a(static_cast<int>(packed), 0x01010101, 0));
    if (lane == 0) {
      zs[n * NG + g] = gsum;
      sb[n * NG + g] = __half2float(Bs[static_cast<size_t>(n) * NG + g]);
    }
  }
  __syncthreads();

  for (int row0 = first_row; row0 < rows; row0 += nwarps * R) {
    float acc[R][NC];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int n = 0; n < NC; ++n) acc[r][n] = 0.f;

    for (int p0 = 0; p0 < passes; p0 += 4) {
      if (row0 != first_row || p0 != 0) load_slab(row0, p0);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int m = row0 + r;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (p0 + j >= passes) continue;  // warp-uniform
          const int ch = (p0 + j) * 32 + lane;
          const bool valid = ch < NCH;
          const int chc = valid ? ch : 0;
          const uint32_t w[4] = {v[r][j].x, v[r][j].y, v[r][j].z, v[r][j].w};
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            hi[u] = (w[u] >> 4) & 0x0f0f0f0fu;
            lo[u] = w[u] & 0x0f0f0f0fu;
          }
#pragma unroll
          for (int n = 0; n < NC; ++n) {
            const uint4* b4 = reinterpret_cast<const uint4*>(bp + n * NCH * 8 + chc * 8);
            const uint4 b0 = b4[0];
            const uint4 b1 = b4[1];
            int d0 = __dp4a(static_cast<int>(hi[0]), static_cast<int>(b0.x), 0);
            int d1 = __dp4a(static_cast<int>(lo[0]), static_cast<int>(b0.y), 0);
            d0 = __dp4a(static_cast<int>(hi[1]), static_cast<int>(b0.z), d0);
            d1 = __dp4a(static_cast<int>(lo[1]), static_cast<int>(b0.w), d1);
            d0 = __dp4a(static_cast<int>(hi[2]), static_cast<int>(b1.x), d0);
            d1 = __dp4a(static_cast<int>(lo[2]), static_cast<int>(b1.y), d1);
            d0 = __dp4a(static_cast<int>(hi[3]), static_cast<int>(b1.z), d0);
            d1 = __dp4a(static_cast<int>(lo[3]), static_cast<int>(b1.w), d1);
            int d = valid ? d0 + d1 : 0;
            // The 4 lanes of a group (lane & ~3 .. +3) hold its 4 chunks.
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            if (valid && (lane & 3) == 0 && m < rows) {
              const int g = ch >> 2;
              const float2 zsa = __half22float2(zsA[r][j]);
              const int za = __half2int_rn(__low2half(zsA[r][j]));
              const int G = d - za * zs[n * NG + g];
              acc[r][n] += static_cast<float>(G) * (zsa.y * sb[n * NG + g]);
              if (Gdbg != nullptr) Gdbg[m * ldg_row + n * ldg_col + g] = G;
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int m = row0 + r;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const float s = warp_sum_f32(acc[r][n]);
        if (lane == 0 && m < rows) C[m * ldc_row + n * ldc_col] = __float2half_rn(s);
      }
    }
  }
}

// INT4, register-resident B (NC * P <= 8). Lane l of a warp always owns the
// 16-byte chunks l, l+32, ..., l+32(P-1) of a row, so the (b - zB) codes, the
// chunk sums of (b - zB) and the B scales for those chunks are built once per warp
// in registers and reused for every row the warp streams: no shared memory, no
// block barrier, no per-CTA preamble. Each lane forms its exact partial
// d - zA * sum(b - zB) for its 32 codes; the 4 lanes of a group add them into the
// group's exact G. R rows are streamed concurrently per warp.
template <int NC, int P, int R>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_int4_reg_kernel(const uint8_t* __restrict__ Aq, const __half* __restrict__ As,
                         const __half* __restrict__ Az, const uint8_t* __restrict__ Bq,
                         const __half* __restrict__ Bs, const __half* __restrict__ Bz,
                         __half* __restrict__ C, int32_t* __restrict__ Gdbg, int rows, int K,
                         long long ldc_row, long long ldc_col, long long ldg_row,
                         long long ldg_col, int weights_early) {
  dev::allow_dependent_launch();
  const int NG = K >> 7;
  const int NCH = K >> 5;
  const int KB = K >> 1;
  const int lane = static_cast<int>(dev::lane_idx());
  const int gwarp = static_cast<int>(blockIdx.x * (blockDim.x >> 5) + dev::warp_idx());
  const int nwarps = static_cast<int>(gridDim.x * (blockDim.x >> 5));

  if (!weights_early) dev::grid_dependency_wait();

  uint4 a[R][P];
  __half2 zsa[R][P];
  auto load_rows = [&](int row0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int m = row0 + r;
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int ch = p * 32 + lane;
        if (m < rows && ch < NCH) {
          a[r][p] = dev::ld_nc_v4(Aq + static_cast<size_t>(m) * KB + static_cast<size_t>(ch) * 16);
          const size_t gi = static_cast<size_t>(m) * NG + (ch >> 2);
          zsa[r][p] = __halves2half2(Az[gi], As[gi]);
        } else {
          a[r][p] = make_uint4(0u, 0u, 0u, 0u);
          zsa[r][p] = __halves2half2(__float2half(0.f), __float2half(0.f));
        }
      }
    }
  };
  int row0 = gwarp * R;
  if (row0 < rows) load_rows(row0);
  // With weights_early the first rows of A were requested before the previous
  // kernel finished; B, C and Gdbg are touched only after it has.
  if (weights_early) dev::grid_dependency_wait();

  // (b - zB) codes of this lane's chunks: word 2u = even-k codes (high nibbles) of
  // byte quad u, 2u+1 = odd-k codes; chunk sums of (b - zB); B group scales.
  uint32_t bw[NC][P][8];
  int bsum[NC][P];
  float bsc[NC][P];
#pragma unroll
  for (int n = 0; n < NC; ++n)
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int ch = p * 32 + lane;
      uint4 q = make_uint4(0u, 0u, 0u, 0u);
      int zb = 0;
      bsc[n][p] = 0.f;
      if (ch < NCH) {
        q = *reinterpret_cast<const uint4*>(Bq + static_cast<size_t>(n) * KB + static_cast<size_t>(ch) * 16);
        zb = __half2int_rn(Bz[static_cast<size_t>(n) * NG + (ch >> 2)]);
        bsc[n][p] = __half2float(Bs[static_cast<size_t>(n) * NG + (ch >> 2)]);
      }
      const uint32_t zq = static_cast<uint32_t>(zb & 0xff) * 0x01010101u;
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      int sum = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        bw[n][p][2 * u] = __vsub4((w[u] >> 4) & 0x0f0f0f0fu, zq);
        bw[n][p][2 * u + 1] = __vsub4(w[u] & 0x0f0f0f0fu, zq);
        sum = __dp4a(static_cast<int>(bw[n][p][2 * u]), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(bw[n][p][2 * u + 1]), 0x01010101, sum);
      }
      bsum[n][p] = ch < NCH ? sum : 0;
    }

  for (; row0 < rows; row0 += nwarps * R) {
    float acc[R][NC];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int n = 0; n < NC; ++n) acc[r][n] = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int m = row0 + r;
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int ch = p * 32 + lane;
        const uint32_t w[4] = {a[r][p].x, a[r][p].y, a[r][p].z, a[r][p].w};
        const int za = __half2int_rn(__low2half(zsa[r][p]));
        const float sa = __high2float(zsa[r][p]);
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          int d0 = 0, d1 = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            d0 = __dp4a(static_cast<int>((w[u] >> 4) & 0x0f0f0f0fu), static_cast<int>(bw[n][p][2 * u]), d0);
            d1 = __dp4a(static_cast<int>(w[u] & 0x0f0f0f0fu), static_cast<int>(bw[n][p][2 * u + 1]), d1);
          }
          int g = d0 + d1 - za * bsum[n][p];
          g += __shfl_xor_sync(0xffffffffu, g, 1);
          g += __shfl_xor_sync(0xffffffffu, g, 2);
          if ((lane & 3) == 0 && ch < NCH && m < rows) {
            acc[r][n] += static_cast<float>(g) * (sa * bsc[n][p]);
            if (Gdbg != nullptr) Gdbg[m * ldg_row + n * ldg_col + (ch >> 2)] = g;
          }
        }
      }
    }
    const int next = row0 + nwarps * R;
    if (next < rows) load_rows(next);  // next rows in flight during the reductions
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int m = row0 + r;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const float s = warp_sum_f32(acc[r][n]);
        if (lane == 0 && m < rows) C[m * ldc_row + n * ldc_col] = __float2half_rn(s);
      }
    }
  }
}

constexpr int kWsChunkRows = 8;  // rows moved per ring slot

// Shared bytes of one chunk: codes [8][K/2], then scales [8][K/128], zeros [8][K/128].
__host__ __device__ constexpr int gemv_ws_chunk_bytes(int K) {
  return kWsChunkRows * (K / 2 + 4 * (K / 128));
}

// INT4 decode, warp-specialised: one CTA per SM owns a contiguous block of rows.
// The producer warp (one thread) moves the block into a shared-memory ring in
// chunks of 8 rows -- three cp.async.bulk copies per chunk (codes, scales, zero
// points; a chunk's rows are contiguous in each of the three row-major arrays) --
// and issues every chunk that fits in the ring at once. With weights_early the
// copies are issued before griddepcontrol.wait, i.e. while the previous kernel on
// the stream drains (only valid when no in-flight kernel writes A). Consumer warp
// w = 4 * rg + wg reads rows rg and rg + 4 of every chunk and only the
// 1024-element windows p = wg, wg + 4, ... of each row, so a lane keeps just PW
// windows of (b - zB) codes in registers (56 registers: two CTAs of consecutive
// launches fit on one SM) and 16 warps hide shared-memory and shuffle latency. A lane forms the exact int32 partial d - zA * sum(b - zB) of its 32
// codes and adds float(partial) * sA * sB to the row's fp32 sum; one 5-shuffle
// butterfly reduces a warp's two rows, the four window partials of a row are
// added in fixed order (deterministic results) and stored once every chunk is done.
constexpr int kWs2RowGroups = 4;
constexpr int kWs2WindowGroups = 4;
constexpr int kWs2ConsumerWarps = kWs2RowGroups * kWs2WindowGroups;
constexpr int kWs2Threads = (kWs2ConsumerWarps + 1) * 32;
static_assert(kWsChunkRows == 2 * kWs2RowGroups, "two rows of a chunk per consumer warp");

template <int NC, int PW>
__global__ void __launch_bounds__(kWs2Threads, 2)
    gemv_int4_ws2_kernel(const uint8_t* __restrict__ Aq, const __half* __restrict__ As,
                         const __half* __restrict__ Az, const uint8_t* __restrict__ Bq,
                         const __half* __restrict__ Bs, const __half* __restrict__ Bz,
                         __half* __restrict__ C, int rows, int K, long long ldc_row,
                         long long ldc_col, int slots, int weights_early) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int NG = K >> 7;
  const int P = K >> 10;
  const int KB = K >> 1;
  const int chunk_bytes = gemv_ws_chunk_bytes(K);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(slots) * chunk_bytes);
  uint64_t* empty = full + slots;
  float* part = reinterpret_cast<float*>(empty + slots);  // [rows of this CTA][4][NC]
  __shared__ int abort_s;
  volatile int* abort_flag = &abort_s;

  const int warp = static_cast<int>(dev::warp_idx());
  const int lane = static_cast<int>(dev::lane_idx());
  const int per_cta = (rows + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per_cta;
  const int nrows = max(0, min(rows, r0 + per_cta) - r0);
  const int nchunks = (nrows + kWsChunkRows - 1) / kWsChunkRows;
#ifdef CLOVE_TRACE
  __shared__ int trace_k;
  CLOVE_TRACE_SEQ_BEGIN(trace_k);
#endif

  if (threadIdx.x == 0) {
    for (int i = 0; i < slots; ++i) {
      dev::mbar_init(&full[i], 1);
      dev::mbar_init(&empty[i], kWs2ConsumerWarps);
    }
    abort_s = 0;
    dev::fence_mbarrier_init();
  }
  __syncthreads();
  dev::allow_dependent_launch();
#ifdef CLOVE_TRACE
  if (threadIdx.x == 0) CLOVE_TRACE_SEQ_POINT(trace_k, 0);
#endif

  if (warp == kWs2ConsumerWarps) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      if (!weights_early) dev::grid_dependency_wait();
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % slots;
        const uint32_t use = static_cast<uint32_t>(c / slots);
        if (use > 0 && !dev::mbar_wait(&empty[s], (use & 1u) ^ 1u, abort_flag)) break;
        const int cr = min(kWsChunkRows, nrows - c * kWsChunkRows);
        const size_t m = static_cast<size_t>(r0 + c * kWsChunkRows);
        uint8_t* dst = smem + static_cast<size_t>(s) * chunk_bytes;
        dev::mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(cr * (KB + 4 * NG)));
        dev::bulk_load_1d(dst, Aq + m * KB, static_cast<uint32_t>(cr * KB), &full[s]);
        dev::bulk_load_1d(dst + kWsChunkRows * KB, As + m * NG, static_cast<uint32_t>(cr * 2 * NG),
                          &full[s]);
        dev::bulk_load_1d(dst + kWsChunkRows * (KB + 2 * NG), Az + m * NG,
                          static_cast<uint32_t>(cr * 2 * NG), &full[s]);
      }
#ifdef CLOVE_TRACE
      CLOVE_TRACE_SEQ_POINT(trace_k, 7);
#endif
      if (*abort_flag) {  // let copies still in flight land before the CTA exits
        volatile int no_abort = 0;
        for (int c = max(0, nchunks - slots); c < nchunks; ++c)
          dev::mbar_wait(&full[c % slots], static_cast<uint32_t>(c / slots) & 1u, &no_abort);
      }
    }
    __syncwarp();
    return;
  }

  // ------------------------------------------------------------------ consumers
  dev::grid_dependency_wait();  // B and C may belong to the previous kernel
#ifdef CLOVE_TRACE
  if (threadIdx.x == 0) CLOVE_TRACE_SEQ_POINT(trace_k, 2);
#endif
  const int rg = warp >> 2;
  const int wg = warp & 3;
  uint32_t bw[NC][PW][8];
  int bsum[NC][PW];
  float bsc[NC][PW];
#pragma unroll
  for (int n = 0; n < NC; ++n)
#pragma unroll
    for (int pw = 0; pw < PW; ++pw) {
      const int p = wg + kWs2WindowGroups * pw;
      const int ch = p * 32 + lane;
      uint4 q = make_uint4(0u, 0u, 0u, 0u);
      int zb = 0;
      bsc[n][pw] = 0.f;
      if (p < P) {
        q = *reinterpret_cast<const uint4*>(Bq + static_cast<size_t>(n) * KB + static_cast<size_t>(ch) * 16);
        zb = __half2int_rn(Bz[static_cast<size_t>(n) * NG + (ch >> 2)]);
        bsc[n][pw] = __half2float(Bs[static_cast<size_t>(n) * NG + (ch >> 2)]);
      }
      const uint32_t zq = static_cast<uint32_t>(zb & 0xff) * 0x01010101u;
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      int sum = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        bw[n][pw][2 * u] = __vsub4((w[u] >> 4) & 0x0f0f0f0fu, zq);
        bw[n][pw][2 * u + 1] = __vsub4(w[u] & 0x0f0f0f0fu, zq);
        sum = __dp4a(static_cast<int>(bw[n][pw][2 * u]), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(bw[n][pw][2 * u + 1]), 0x01010101, sum);
      }
      bsum[n][pw] = p < P ? sum : 0;
    }
#ifdef CLOVE_TRACE
  if (threadIdx.x == 0 && bsum[0][0] != 0x7fffffff) CLOVE_TRACE_SEQ_POINT(trace_k, 3);
#endif

  for (int c = 0; c < nchunks; ++c) {
    const int s = c % slots;
    const bool ok = dev::mbar_wait(&full[s], static_cast<uint32_t>(c / slots) & 1u, abort_flag);
    if (!__all_sync(0xffffffffu, ok)) break;
#ifdef CLOVE_TRACE
    if (threadIdx.x == 0 && c == 0) CLOVE_TRACE_SEQ_POINT(trace_k, 4);
#endif
    const uint8_t* base = smem + static_cast<size_t>(s) * chunk_bytes;
    float acc[2][NC];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rr = rg + kWs2RowGroups * h;
#pragma unroll
      for (int n = 0; n < NC; ++n) acc[h][n] = 0.f;
      if (c * kWsChunkRows + rr >= nrows) continue;  // warp-uniform: row not loaded
      const uint8_t* rowp = base + rr * KB;
      const __half* ras = reinterpret_cast<const __half*>(base + kWsChunkRows * KB) + rr * NG;
      const __half* raz = reinterpret_cast<const __half*>(base + kWsChunkRows * (KB + 2 * NG)) + rr * NG;
#pragma unroll
      for (int pw = 0; pw < PW; ++pw) {
        const int p = wg + kWs2WindowGroups * pw;
        if (p >= P) continue;  // warp-uniform
        const int ch = p * 32 + lane;
        const uint4 a = *reinterpret_cast<const uint4*>(rowp + ch * 16);
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
        const int za = __half2int_rn(raz[ch >> 2]);
        const float sa = __half2float(ras[ch >> 2]);
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          // High nibbles are used in place (16 x code as unsigned bytes); their
          // sum is a multiple of 16 and is shifted back exactly.
          int dh = 0, dl = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            dh = dev::dp4a_u8s8(w[u] & 0xf0f0f0f0u, bw[n][pw][2 * u], dh);
            dl = __dp4a(static_cast<int>(w[u] & 0x0f0f0f0fu), static_cast<int>(bw[n][pw][2 * u + 1]), dl);
          }
          const int d = dl + (dh >> 4) - za * bsum[n][pw];
          acc[h][n] = fmaf(static_cast<float>(d), sa * bsc[n][pw], acc[h][n]);
        }
      }
    }
    // Butterfly over the warp's two rows: lanes 0-15 end with row rg, 16-31 with rg + 4.
    const bool upper = (lane & 16) != 0;
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      const float send = upper ? acc[0][n] : acc[1][n];
      float keep = upper ? acc[1][n] : acc[0][n];
      keep += __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
      const int row_local = c * kWsChunkRows + rg + (upper ? kWs2RowGroups : 0);
      if ((lane & 15) == 0 && row_local < nrows) part[(row_local * kWs2WindowGroups + wg) * NC + n] = keep;
    }
    __syncwarp();
    if (lane == 0 && c + slots < nchunks) dev::mbar_arrive(&empty[s]);
  }
#ifdef CLOVE_TRACE
  if (threadIdx.x == 0) CLOVE_TRACE_SEQ_POINT(trace_k, 9);
#endif

  // Every consumer warp has written its partials: add the four windows of each row.
  asm volatile("bar.sync 1, %0;" ::"n"(kWs2ConsumerWarps * 32) : "memory");
#ifdef CLOVE_TRACE
  if (threadIdx.x == 0) CLOVE_TRACE_SEQ_POINT(trace_k, 11);
#endif
  if (*abort_flag) return;
  for (int i = static_cast<int>(threadIdx.x); i < nrows * NC; i += kWs2ConsumerWarps * 32) {
    const int r = i / NC;
    const int n = i - r * NC;
    const float* pr = part + r * kWs2WindowGroups * NC + n;
    const float t = ((pr[0] + pr[NC]) + pr[2 * NC]) + pr[3 * NC];
    C[static_cast<long long>(r0 + r) * ldc_row + n * ldc_col] = __float2half_rn(t);
  }
#ifdef CLOVE_TRACE
  if (threadIdx.x == 0) CLOVE_TRACE_SEQ_POINT(trace_k, 6);
#endif
}

// INT4 decode with direct 128-bit loads (no shared-memory ring). RG x WG warps:
// warp w = WG * rg + wg takes rows rg, rg + RG, ... of the CTA's block and the
// 1024-element windows wg, wg + WG, ... of each (4 x 4, the consumer decomposition
// of gemv_int4_ws2_kernel; 2 x 4 and 1 x 12 give every lane a single window of
// rows up to 4096 and 12288 codes) -- but every lane loads its own 16-byte chunks of up to RMAX rows
// with ld.global.nc straight into registers, all issued before any math, like a
// bare streaming read. With weights_early those loads are issued before
// griddepcontrol.wait. The RMAX row partials of a warp are reduced by one
// transposed butterfly (lane 4i ends with row i), the WG window partials of a row
// are added in fixed order through shared memory.
template <int NC, int PW, int RMAX, int MINB, int RG, int WG>
__global__ void __launch_bounds__(RG * WG * 32, MINB)
    gemv_int4_ldg_kernel(const uint8_t* __restrict__ Aq, const __half* __restrict__ As,
                         const __half* __restrict__ Az, const uint8_t* __restrict__ Bq,
                         const __half* __restrict__ Bs, const __half* __restrict__ Bz,
                         __half* __restrict__ C, int rows, int K, long long ldc_row,
                         long long ldc_col, int weights_early) {
  static_assert(RMAX == 8 || RMAX == 4, "the transposed butterfly reduces 8 or 4 row partials");
  constexpr int ROWS = RG * RMAX;  // rows of the block per round
  constexpr int THREADS = RG * WG * 32;
  __shared__ float part[ROWS][WG][NC];
  const int NG = K >> 7;
  const int P = (K + 1023) >> 10;  // 1024-code windows, the last one possibly partial
  const int KC = K >> 5;           // 16-byte chunks of a row (32 codes each)
  const int KB = K >> 1;
  const int warp = static_cast<int>(dev::warp_idx());
  const int lane = static_cast<int>(dev::lane_idx());
  const int rg = warp / WG;
  const int wg = warp - rg * WG;
  const int per_cta = (rows + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per_cta;
  const int nrows = max(0, min(rows, r0 + per_cta) - r0);

  dev::allow_dependent_launch();
  if (!weights_early) dev::grid_dependency_wait();

  uint4 a[RMAX][PW];
  __half2 zs[RMAX][PW];
  auto load_round = [&](int base) {
#pragma unroll
    for (int i = 0; i < RMAX; ++i) {
      const int rl = base + rg + RG * i;
#pragma unroll
      for (int pw = 0; pw < PW; ++pw) {
        const int p = wg + WG * pw;
        const int ch = p * 32 + lane;
        if (rl < nrows && p < P && ch < KC) {
          const size_t m = static_cast<size_t>(r0 + rl);
          a[i][pw] = dev::ld_nc_v4(Aq + m * KB + static_cast<size_t>(ch) * 16);
          const size_t gi = m * NG + (ch >> 2);
          zs[i][pw] = __halves2half2(Az[gi], As[gi]);
        } else {
          a[i][pw] = make_uint4(0u, 0u, 0u, 0u);
          zs[i][pw] = __halves2half2(__float2half(0.f), __float2half(0.f));
        }
      }
    }
  };
  load_round(0);
  if (weights_early) dev::grid_dependency_wait();  // B and C may belong to the previous kernel

  uint32_t bw[NC][PW][8];
  int bsum[NC][PW];
  float bsc[NC][PW];
#pragma unroll
  for (int n = 0; n < NC; ++n)
#pragma unroll
    for (int pw = 0; pw < PW; ++pw) {
      const int p = wg + WG * pw;
      const int ch = p * 32 + lane;
      uint4 q = make_uint4(0u, 0u, 0u, 0u);
      int zb = 0;
      bsc[n][pw] = 0.f;
      const bool valid = p < P && ch < KC;  // lanes past K (partial last window) add 0
      if (valid) {
        q = *reinterpret_cast<const uint4*>(Bq + static_cast<size_t>(n) * KB + static_cast<size_t>(ch) * 16);
        zb = __half2int_rn(Bz[static_cast<size_t>(n) * NG + (ch >> 2)]);
        bsc[n][pw] = __half2float(Bs[static_cast<size_t>(n) * NG + (ch >> 2)]);
      }
      const uint32_t zq = static_cast<uint32_t>(zb & 0xff) * 0x01010101u;
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      int sum = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        bw[n][pw][2 * u] = __vsub4((w[u] >> 4) & 0x0f0f0f0fu, zq);
        bw[n][pw][2 * u + 1] = __vsub4(w[u] & 0x0f0f0f0fu, zq);
        sum = __dp4a(static_cast<int>(bw[n][pw][2 * u]), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(bw[n][pw][2 * u + 1]), 0x01010101, sum);
      }
      bsum[n][pw] = valid ? sum : 0;
    }

  const bool b4 = (lane & 16) != 0;
  const bool b3 = (lane & 8) != 0;
  const bool b2 = (lane & 4) != 0;
  for (int base = 0; base < nrows; base += ROWS) {
    float v[RMAX][NC];
#pragma unroll
    for (int i = 0; i < RMAX; ++i) {
#pragma unroll
      for (int n = 0; n < NC; ++n) v[i][n] = 0.f;
#pragma unroll
      for (int pw = 0; pw < PW; ++pw) {
        const uint32_t w[4] = {a[i][pw].x, a[i][pw].y, a[i][pw].z, a[i][pw].w};
        const int za = __half2int_rn(__low2half(zs[i][pw]));
        const float sa = __high2float(zs[i][pw]);
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          // High nibbles used in place (16 x code, unsigned bytes), shifted back exactly.
          int dh = 0, dl = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            dh = dev::dp4a_u8s8(w[u] & 0xf0f0f0f0u, bw[n][pw][2 * u], dh);
            dl = __dp4a(static_cast<int>(w[u] & 0x0f0f0f0fu), static_cast<int>(bw[n][pw][2 * u + 1]), dl);
          }
          const int d = dl + (dh >> 4) - za * bsum[n][pw];
          v[i][n] = fmaf(static_cast<float>(d), sa * bsc[n][pw], v[i][n]);
        }
      }
    }
    // The registers of this round are consumed: the next round's rows in flight.
    if (base + ROWS < nrows) load_round(base + ROWS);
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      if constexpr (RMAX == 8) {
        float x[4], y[2];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float keep = b4 ? v[4 + q][n] : v[q][n];
          const float send = b4 ? v[q][n] : v[4 + q][n];
          x[q] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float keep = b3 ? x[2 + q] : x[q];
          const float send = b3 ? x[q] : x[2 + q];
          y[q] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        float z = (b2 ? y[1] : y[0]) + __shfl_xor_sync(0xffffffffu, b2 ? y[0] : y[1], 4);
        z += __shfl_xor_sync(0xffffffffu, z, 2);
        z += __shfl_xor_sync(0xffffffffu, z, 1);
        if ((lane & 3) == 0) part[rg + RG * (lane >> 2)][wg][n] = z;  // row lane/4
      } else {
        // Four row partials: after the 16- and 8-lane exchanges lane l holds row
        // l / 8 of its 8-lane group, summed over the group by three more steps.
        float x[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float keep = b4 ? v[2 + q][n] : v[q][n];
          const float send = b4 ? v[q][n] : v[2 + q][n];
          x[q] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
        float z = (b3 ? x[1] : x[0]) + __shfl_xor_sync(0xffffffffu, b3 ? x[0] : x[1], 8);
        z += __shfl_xor_sync(0xffffffffu, z, 4);
        z += __shfl_xor_sync(0xffffffffu, z, 2);
        z += __shfl_xor_sync(0xffffffffu, z, 1);
        if ((lane & 7) == 0) part[rg + RG * (lane >> 3)][wg][n] = z;  // row lane/8
      }
    }
    __syncthreads();
    for (int t = static_cast<int>(threadIdx.x); t < ROWS * NC; t += THREADS) {
      const int r = t / NC;
      const int n = t - r * NC;
      if (base + r < nrows) {
        float sum = part[r][0][n];
#pragma unroll
        for (int g = 1; g < WG; ++g) sum += part[r][g][n];  // fixed order
        C[static_cast<long long>(r0 + base + r) * ldc_row + n * ldc_col] = __float2half_rn(sum);
      }
    }
    __syncthreads();  // part is reused by the next round
  }
}

// Bare streaming read of n16 16-byte words (test hook, no GEMM): every thread
// keeps four 128-bit loads in flight and XOR-folds them. It measures what one
// kernel launch of this size can pull from HBM -- the floor under the decode
// GEMVs, which read the same number of bytes and also compute.
constexpr int kStreamThreads = 512;
__global__ void __launch_bounds__(kStreamThreads)
    stream_read_kernel(const uint4* __restrict__ src, size_t n16, uint32_t* __restrict__ out) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  uint32_t x = 0;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const size_t j = i + u * stride;
      v[u] = j < n16 ? dev::ld_nc_v4(reinterpret_cast<const uint8_t*>(src + j)) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) x ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
  // Keeps the loads live; the word is written only for one specific value.
  if (x == 0x9E3779B9u) out[0] = x;
}

__host__ __device__ constexpr size_t gemv_int8_smem_bytes(int nc, int K) {
  return static_cast<size_t>(nc) * K + 4 * 8;
}

template <int NC>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_int8_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ B,
                     void* __restrict__ Cout, int rows, int K, GemvI8Epi ep) {
  extern __shared__ __align__(128) uint8_t smem[];
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
  extern __shared__ __align__(128) uint8_t smem[];
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
