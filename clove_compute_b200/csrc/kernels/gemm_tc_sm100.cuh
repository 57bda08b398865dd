// gemm_tc_sm100.cuh -- tcgen05 GEMM for sm_100a: C[M,N] = epilogue(A[M,K] . B[K,N]).
//
// Replaces the reference's WMMA kernel (src/kernels/gemm_fp16.cu:30-215) and its
// SIMT int8 kernel (src/kernels/gemm_int8.cu:16-117). Layouts are the reference's:
// A row-major [M,K] (K-major operand), B row-major [K,N] (MN-major operand),
// C row-major [M,N] fp16.
//
// Structure (one CTA = 6 warps):
//   warp 0      TMA producer: A box [128 rows x 128 B] + B boxes [BK rows x swizzle width]
//               into a STAGES-deep ring of 128B/64B/32B-swizzled smem tiles.
//   warp 1      TMEM allocator + MMA issuer: 4 tcgen05.mma per stage (K = 32 bytes each),
//               tcgen05.commit frees the stage; accumulators double-buffered in TMEM.
//   warps 2-5   epilogue: tcgen05.ld (TMEM lane quarter = warp % 4), fp32/int32 math,
//               fp16 pack into swizzled smem, TMA store per 32-row slab.
// Persistent mode: grid <= #SMs, tiles strided over CTAs, grouped rasterisation.
// Split mode: a cluster of S CTAs shares one output tile, each CTA takes 1/S of the
// K blocks, partial accumulators are summed in a fixed order by CTA rank 0 over
// distributed shared memory (exact for int32, deterministic for fp32).
#pragma once

#include "params.h"
#include "sm100_ptx.cuh"

namespace clove {
namespace kern {

// Operand formats.
struct OpF16 {
  static constexpr int kElemBytes = 2;
  static constexpr bool kInt = false;
  // fp32 accumulator, f16 x f16, A K-major, B MN-major.
  static constexpr uint32_t idesc(int n) { return dev::make_idesc(1, 0, 0, 0, 1, n, 128); }
};
struct OpI8 {
  static constexpr int kElemBytes = 1;
  static constexpr bool kInt = true;
  // s32 accumulator, s8 x s8, A K-major, B MN-major.
  static constexpr uint32_t idesc(int n) { return dev::make_idesc(2, 1, 1, 0, 1, n, 128); }
};

constexpr int kSmemLimit = 232448;  // 227 KB opt-in per CTA on sm_100

template <class Op, int BN_, bool SPLIT_, int OUT_BYTES_>
struct TcShape {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr bool SPLIT = SPLIT_;
  static constexpr int OUT_BYTES = OUT_BYTES_;
  static constexpr int ELEM = Op::kElemBytes;
  static constexpr int BK = 128 / ELEM;      // K elements per 128-byte row
  static constexpr int UMMA_K = 32 / ELEM;   // K per tcgen05.mma
  static constexpr int KSTEPS = BK / UMMA_K;  // 4
  static constexpr int A_BYTES = BM * 128;
  static constexpr int BN_BYTES = BN * ELEM;
  static constexpr int B_SW = BN_BYTES >= 128 ? 128 : BN_BYTES;  // swizzle width of B
  static constexpr int B_ATOMS = BN_BYTES / B_SW;
  static constexpr int B_ATOM_ELEMS = B_SW / ELEM;
  static constexpr int B_BYTES = BK * BN_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int CHUNK = BN < (128 / OUT_BYTES) ? BN : (128 / OUT_BYTES);  // cols / store
  static constexpr int STG_ROW = CHUNK * OUT_BYTES;                             // bytes / row
  static constexpr int STG_BUF = 32 * STG_ROW;
  // C staging: 4 warps x 2 buffers x 4 KB (1 KB aligned); split-K tiles store rows directly.
  static constexpr int EPI_BYTES = SPLIT ? 0 : 4 * 2 * 4096;
  // Split-K receive buffer: (S-1) * BM/S <= 112 partial rows (S <= 8), padded rows.
  static constexpr int PART_ROW = BN * 4 + 16;
  static constexpr int PART_BYTES = SPLIT ? ((112 * PART_ROW + 1023) / 1024) * 1024 : 0;
  // Split-K: the tile's column factors (col_scale or col_sum), staged before the
  // accumulators are ready.
  static constexpr int COLV_BYTES = SPLIT ? BN * 4 : 0;
  static constexpr int ACC_BUFS = SPLIT ? 1 : 2;
  static constexpr int TMEM_COLS = (ACC_BUFS * BN) < 32 ? 32 : (ACC_BUFS * BN);
  static constexpr int BAR_BYTES = 256;
  static constexpr int STAGES_FIT =
      (kSmemLimit - 1024 - EPI_BYTES - PART_BYTES - COLV_BYTES - BAR_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int SMEM_BYTES =
      1024 + STAGES * STAGE_BYTES + EPI_BYTES + PART_BYTES + COLV_BYTES + BAR_BYTES;
  static constexpr int THREADS = 192;

  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N constraint for M=128");
  static_assert(BN_BYTES % B_SW == 0, "B tile must be whole swizzle atoms");
  static_assert(B_SW == 32 || B_SW == 64 || B_SW == 128, "B swizzle width");
  static_assert(STG_ROW == 32 || STG_ROW == 64 || STG_ROW == 128, "C staging row");
  static_assert(STG_BUF <= 4096, "staging buffer");
  static_assert(STAGES >= 2, "pipeline depth");
  static_assert(SMEM_BYTES <= kSmemLimit, "smem budget");
  static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0 && TMEM_COLS <= 512, "TMEM alloc size");
  static_assert(!SPLIT || BN <= 128, "split-K receive buffers hold at most 128 columns");
};

// Grouped rasterisation: bands of kGroupM M-tiles, N-tiles walked inside a band
// so that concurrently running CTAs share A rows and B columns in L2.
template <int kGroupM = 16>
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& m_blk,
                                            int& n_blk) {
  const int per_group = kGroupM * tiles_n;
  const int g = tile / per_group;
  const int first_m = g * kGroupM;
  const int gm = min(tiles_m - first_m, kGroupM);
  const int r = tile - g * per_group;
  m_blk = first_m + r % gm;
  n_blk = r / gm;
}

__device__ __forceinline__ uint32_t swz_chunk(uint32_t row, uint32_t chunk, uint32_t row_bytes) {
  // Swizzle<B,4,3> on the byte address of a row-major staging tile whose rows are
  // row_bytes wide (B = log2(row_bytes/16)): 16-byte chunk index ^= address bits 7+.
  const uint32_t mask = row_bytes / 16 - 1;
  return chunk ^ (((row * row_bytes) >> 7) & mask);
}

// Epilogue math of one CHUNK-column slice of this thread's row: fp16 (or raw
// int32) values packed into 16-byte packets. Column factors (col_scale / col_sum)
// come from global memory, or with COLV from `colv` (shared, indexed by j).
template <class Op, int OUT_BYTES, int CHUNK, bool COLV = false>
__device__ __forceinline__ void epi_pack(const uint32_t (&v)[CHUNK], const EpiParams& ep, int row,
                                         int ncol0, int M, int N, int K, float row_scale,
                                         int32_t row_corr,
                                         uint32_t (&pk)[CHUNK * OUT_BYTES / 16][4],
                                         const uint32_t* colv = nullptr, size_t c_off = 0) {
  constexpr int PKTS = CHUNK * OUT_BYTES / 16;
  if constexpr (OUT_BYTES == 2) {
    float f[CHUNK];
    if (ep.mode == kEpiF16AlphaBeta) {
#pragma unroll
      for (int j = 0; j < CHUNK; ++j) f[j] = ep.alpha * __uint_as_float(v[j]);
      if (ep.beta != 0.f && row < M) {
        const __half* crow = ep.c_in + c_off + static_cast<size_t>(row) * N;
#pragma unroll
        for (int j = 0; j < CHUNK; j += 8) {
          if (ncol0 + j < N) {  // N % 8 == 0 on this path
            const uint4 cv = *reinterpret_cast<const uint4*>(crow + ncol0 + j);
            const __half2* h = reinterpret_cast<const __half2*>(&cv);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 c2 = __half22float2(h[u]);
              f[j + 2 * u] += ep.beta * c2.x;
              f[j + 2 * u + 1] += ep.beta * c2.y;
            }
          }
        }
      }
    } else if (ep.mode == kEpiI8Tensor) {
#pragma unroll
      for (int j = 0; j < CHUNK; ++j) {
        uint32_t a = v[j] + static_cast<uint32_t>(row_corr);
        if (ep.za != 0) {
          const uint32_t cs =
              COLV ? colv[j] : static_cast<uint32_t>(ep.col_sum[min(ncol0 + j, N - 1)]);
          a += 0u - static_cast<uint32_t>(ep.za) * cs;
          a += static_cast<uint32_t>(K) * static_cast<uint32_t>(ep.za) *
               static_cast<uint32_t>(ep.zb);
        }
        f[j] = static_cast<float>(static_cast<int32_t>(a)) * ep.scale;
      }
    } else {  // kEpiI8RowCol
#pragma unroll
      for (int j = 0; j < CHUNK; ++j) {
        const float cs = COLV ? __uint_as_float(colv[j]) : ep.col_scale[min(ncol0 + j, N - 1)];
        f[j] = (static_cast<float>(static_cast<int32_t>(v[j])) * row_scale) * cs;
      }
    }
#pragma unroll
    for (int p = 0; p < PKTS; ++p)
#pragma unroll
      for (int u = 0; u < 4; ++u) pk[p][u] = dev::pack_half2(f[p * 8 + 2 * u], f[p * 8 + 2 * u + 1]);
  } else {  // int32 raw accumulators
#pragma unroll
    for (int j = 0; j < CHUNK; ++j) {
      uint32_t a = v[j] + static_cast<uint32_t>(row_corr);
      if (ep.za != 0) {
        const uint32_t cs =
            COLV ? colv[j] : static_cast<uint32_t>(ep.col_sum[min(ncol0 + j, N - 1)]);
        a += 0u - static_cast<uint32_t>(ep.za) * cs;
        a += static_cast<uint32_t>(K) * static_cast<uint32_t>(ep.za) *
             static_cast<uint32_t>(ep.zb);
      }
      pk[j / 4][j % 4] = a;
    }
  }
}

// Receiver-ready handshake of a replicated output (PeerOut), once per epilogue
// warp before its first store: the number of ranks to store to (all of them, or
// none after a timeout, which also raises the CTA's abort flag so every role
// unwinds). 0 without a replicated output.
__device__ __forceinline__ int peer_ready_warp(const PeerOut& po, uint32_t lane,
                                               volatile int* abort_flag) {
  if (po.count <= 0) return 0;
  int ok = 1;
  if (lane == 0) ok = dev::peer_ready_gate(po) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) return po.count;
  if (lane == 0) *abort_flag = 1;
  return 0;
}

// Epilogue of one CHUNK-column slice of a 32-row warp slab: epi_pack on this
// thread's row, swizzled staging, TMA store of the warp's slab.
template <class Op, int OUT_BYTES, int CHUNK>
__device__ __forceinline__ void store_chunk(const uint32_t (&v)[CHUNK], const EpiParams& ep,
                                            int row, int ncol0, int M, int N, int K,
                                            float row_scale, int32_t row_corr, uint32_t lane,
                                            uint8_t* stg_base, uint32_t& stg_count,
                                            const CUtensorMap* tmC, int store_row0,
                                            int peer_n, int plane = -1) {
  constexpr int STG_ROW = CHUNK * OUT_BYTES;
  constexpr int PKTS = STG_ROW / 16;
  uint32_t pk[PKTS][4];
  // Batch plane p reads its beta source from plane p of C.
  const size_t c_off = plane > 0 ? static_cast<size_t>(plane) * M * N : 0;
  epi_pack<Op, OUT_BYTES, CHUNK>(v, ep, row, ncol0, M, N, K, row_scale, row_corr, pk, nullptr,
                                 c_off);

  // Stage through swizzled smem and TMA-store this warp's 32-row slab.
  uint8_t* stg = stg_base + (stg_count & 1u) * 4096;
  if (lane == 0) dev::bulk_wait_group_read<1>();
  __syncwarp();
  const uint32_t stg_addr = dev::smem_u32(stg);
#pragma unroll
  for (int p = 0; p < PKTS; ++p) {
    const uint32_t off = lane * STG_ROW + swz_chunk(lane, p, STG_ROW) * 16;
    dev::st_shared_v4(stg_addr + off, pk[p][0], pk[p][1], pk[p][2], pk[p][3]);
  }
  dev::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (plane < 0)  // 2D map (CTA-pair kernel)
      dev::tma_store_2d(tmC, stg, ncol0, store_row0);
    else            // 3D [batch, M, N] map
      dev::tma_store_3d(tmC, stg, ncol0, store_row0, plane);
    if constexpr (OUT_BYTES == 2) {
      // Replicated output (never with batch planes): the same staged tile to every
      // rank's C. `ep` is the kernel's __grid_constant__ parameter here, so the
      // maps are addressed in parameter space. peer_n is ep.peer.count once the
      // warp has passed the receiver-ready handshake, 0 if that timed out.
      if (ep.peer.mc == 0) {
#pragma unroll 1
        for (int d = 0; d < peer_n; ++d)
          dev::tma_store_2d(&ep.peer.maps[d], stg, ep.peer.col0 + ncol0, store_row0);
      }
    }
    dev::bulk_commit_group();
  }
  if constexpr (OUT_BYTES == 2) {
    // Multicast replicated output: the whole warp sends the staged slab once.
    if (peer_n > 0 && ep.peer.mc != 0)
      dev::multicast_slab<STG_ROW>(ep.peer.mc, ep.peer.ldc, stg_addr, store_row0, M, ep.peer.col0,
                                   ncol0, N, lane, [](uint32_t r, uint32_t c) {
                                     return swz_chunk(r, c, STG_ROW);
                                   });
  }
  ++stg_count;
}

// Epilogue of one CHUNK-column slice of this thread's row, stored straight to C
// with 16-byte stores (split-K tiles, whose rows are finished by different CTAs).
template <class Op, int OUT_BYTES, int CHUNK>
__device__ __forceinline__ void store_row_direct(const uint32_t (&v)[CHUNK], const EpiParams& ep,
                                                 int row, int ncol0, int M, int N, int K,
                                                 float row_scale, int32_t row_corr,
                                                 const uint32_t* colv) {
  constexpr int PKTS = CHUNK * OUT_BYTES / 16;
  constexpr int COLS_PER_PKT = 16 / OUT_BYTES;
  uint32_t pk[PKTS][4];
  epi_pack<Op, OUT_BYTES, CHUNK, true>(v, ep, row, ncol0, M, N, K, row_scale, row_corr, pk, colv);
  if (row >= M) return;
  uint8_t* crow = static_cast<uint8_t*>(ep.c_out) +
                  (static_cast<size_t>(row) * N + ncol0) * OUT_BYTES;
#pragma unroll
  for (int p = 0; p < PKTS; ++p) {
    if (ncol0 + p * COLS_PER_PKT < N)  // N is a multiple of 8 on this path
      *reinterpret_cast<uint4*>(crow + p * 16) = make_uint4(pk[p][0], pk[p][1], pk[p][2], pk[p][3]);
  }
}

template <class Op, int BN, bool SPLIT, int OUT_BYTES>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, int M, int N, int K, int batch,
                   int a_rows, const __grid_constant__ EpiParams ep) {
  using S = TcShape<Op, BN, SPLIT, OUT_BYTES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = dev::align_smem_1024(smem_raw);
  uint8_t* stage_base = smem;
  uint8_t* epi_base = smem + S::STAGES * S::STAGE_BYTES;
  uint8_t* part_base = epi_base + S::EPI_BYTES;
  uint32_t* colv = reinterpret_cast<uint32_t*>(part_base + S::PART_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(part_base + S::PART_BYTES + S::COLV_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + S::STAGES;
  uint64_t* tfull = bars + 2 * S::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // split-K: peers' partial rows have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = dev::warp_idx();
  const uint32_t lane = dev::lane_idx();
  if (threadIdx.x == 0) {
    CLOVE_TRACE_POINT(0);
    CLOVE_TRACE_MIN(16);
    CLOVE_TRACE_MAX(17);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      dev::mbar_init(&full[s], 1);
      dev::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      dev::mbar_init(&tfull[b], 1);
      dev::mbar_init(&tempty[b], 4);
    }
    *abort_flag = 0;
    if constexpr (SPLIT) {
      // This CTA finishes rows [rank*BM/S, (rank+1)*BM/S) of the tile and receives
      // those rows' partials from the other S-1 CTAs of the cluster -- only the
      // rows below M, the only ones stored (decode tiles hold a few live rows).
      const int parts = static_cast<int>(gridDim.x);
      const int rs = S::BM / parts;
      const int tiles_n_ = (N + BN - 1) / BN;
      const int first = static_cast<int>(blockIdx.y) / tiles_n_ * S::BM +
                        static_cast<int>(blockIdx.x) * rs;
      const int live = min(max(M - first, 0), rs);
      dev::mbar_init(rbar, 1);
      dev::mbar_arrive_expect_tx(rbar, static_cast<uint32_t>((parts - 1) * live * BN * 4));
    }
    dev::fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&tmA);
    dev::prefetch_tmap(&tmB);
    dev::prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    dev::tmem_alloc(tmem_slot, S::TMEM_COLS);
    dev::tmem_relinquish_alloc_permit();
  }
  dev::tc_fence_before_sync();
  __syncthreads();
  dev::tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  if constexpr (SPLIT) dev::cluster_arrive();  // receive barriers initialised
  // Programmatic dependent launch: the set-up above overlaps the tail of the
  // previous kernel on the stream; no global memory is touched before it completes.
  dev::allow_dependent_launch();
  dev::grid_dependency_wait();
  if (threadIdx.x == 0) CLOVE_TRACE_POINT(1);

  // Tensor maps are 3D [batch, rows, cols]; tile t covers plane t / (tiles_m * tiles_n).
  const int tiles_m = (M + S::BM - 1) / S::BM;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_mn = tiles_m * tiles_n;
  const int num_tiles = tiles_mn * batch;
  const int kb_total = (K + S::BK - 1) / S::BK;
  int tile_first, tile_stride, kb_begin, kb_end;
  if constexpr (SPLIT) {
    const int rank = static_cast<int>(blockIdx.x);  // cluster spans gridDim.x
    const int parts = static_cast<int>(gridDim.x);
    tile_first = static_cast<int>(blockIdx.y);
    tile_stride = num_tiles;  // exactly one tile per cluster
    kb_begin = rank * kb_total / parts;
    kb_end = (rank + 1) * kb_total / parts;
  } else {
    tile_first = static_cast<int>(blockIdx.x);
    tile_stride = static_cast<int>(gridDim.x);
    kb_begin = 0;
    kb_end = kb_total;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t armed = 0;  // bit s: stage s has a load in flight (for error unwinding)
      uint32_t armed_parity = 0;
      for (int tile = tile_first; tile < num_tiles; tile += tile_stride) {
        int m_blk, n_blk;
        const int plane = tile / tiles_mn;
        if constexpr (SPLIT) {
          m_blk = tile / tiles_n;
          n_blk = tile % tiles_n;
        } else {
          tile_coords(tile - plane * tiles_mn, tiles_m, tiles_n, m_blk, n_blk);
        }
        bool ok = true;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!dev::mbar_wait<true>(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // A's box is a_rows tall (M rounded up to 8 when M < 128): rows past it in
          // the stage are stale and only feed accumulator rows that are never stored.
          dev::mbar_arrive_expect_tx(&full[stage], a_rows * 128 + S::B_BYTES);
          if (kb == kb_begin) CLOVE_TRACE_POINT(2);
          uint8_t* a_dst = stage_base + stage * S::STAGE_BYTES;
          uint8_t* b_dst = a_dst + S::A_BYTES;
          dev::tma_load_3d(a_dst, &tmA, &full[stage], kb * S::BK, m_blk * S::BM, plane);
#pragma unroll
          for (int a = 0; a < S::B_ATOMS; ++a) {
            dev::tma_load_3d(b_dst + a * (S::BK * S::B_SW), &tmB, &full[stage],
                             n_blk * BN + a * S::B_ATOM_ELEMS, kb * S::BK, plane);
          }
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      if (*abort_flag) {
        // Error unwinding: let every load still in flight land before the CTA exits.
        volatile int no_abort = 0;
        for (int s = 0; s < S::STAGES; ++s)
          if (armed & (1u << s)) dev::mbar_wait<true>(&full[s], (armed_parity >> s) & 1u, &no_abort);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = Op::idesc(BN);
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      for (int tile = tile_first; tile < num_tiles && ok; tile += tile_stride, ++it) {
        const uint32_t buf = static_cast<uint32_t>(it) & (S::ACC_BUFS - 1);
        const uint32_t use = static_cast<uint32_t>(it) / S::ACC_BUFS;
        if (!dev::mbar_wait<true>(&tempty[buf], (use & 1u) ^ 1u, abort_flag)) break;
        dev::tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!dev::mbar_wait<true>(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          if (kb == kb_begin) CLOVE_TRACE_POINT(3);
          dev::tc_fence_after_sync();
          const uint32_t a_addr = dev::smem_u32(stage_base + stage * S::STAGE_BYTES);
          const uint32_t b_addr = a_addr + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < S::KSTEPS; ++k) {
            const uint64_t adesc =
                dev::make_smem_desc(a_addr + k * 32, 0, 1024, dev::kLayoutSw128);
            const uint64_t bdesc = dev::make_smem_desc(
                b_addr + k * S::UMMA_K * S::B_SW, S::BK * S::B_SW, 8 * S::B_SW,
                dev::layout_for_swizzle_bytes(S::B_SW));
            const uint32_t acc = (kb > kb_begin || k > 0) ? 1u : 0u;
            if constexpr (Op::kInt)
              dev::mma_i8_ss(d_tmem, adesc, bdesc, kIdesc, acc);
            else
              dev::mma_f16_ss(d_tmem, adesc, bdesc, kIdesc, acc);
          }
          dev::mma_commit(&empty[stage]);
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        dev::mma_commit(&tfull[buf]);
        CLOVE_TRACE_POINT(4);
        CLOVE_TRACE_MAX(18);
        CLOVE_TRACE_MIN(22);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const uint32_t q = warp & 3u;  // TMEM lane quarter this warp may access
    const int row_in_tile = static_cast<int>(q * 32 + lane);
    uint8_t* stg_base = epi_base + (warp - 2) * (2 * 4096);
    uint32_t stg_count = 0;
    int it = 0;
    if constexpr (SPLIT) dev::cluster_wait();  // every peer's rbar is initialised
    // Replicated output: no remote store before every rank has reached this call.
    const int peer_n = peer_ready_warp(ep.peer, lane, abort_flag);
    for (int tile = tile_first; tile < num_tiles; tile += tile_stride, ++it) {
      int m_blk, n_blk;
      const int plane = tile / tiles_mn;
      if constexpr (SPLIT) {
        m_blk = tile / tiles_n;
        n_blk = tile % tiles_n;
      } else {
        tile_coords(tile - plane * tiles_mn, tiles_m, tiles_n, m_blk, n_blk);
      }
      const uint32_t buf = static_cast<uint32_t>(it) & (S::ACC_BUFS - 1);
      const uint32_t use = static_cast<uint32_t>(it) / S::ACC_BUFS;
      if constexpr (SPLIT) {
        // Stage the tile's column factors while the MMAs run (one tile per CTA in
        // split mode, and these warps never leave the tile early, so the named
        // barrier is always reached by all four).
        const bool rowcol = ep.mode == kEpiI8RowCol;
        if (rowcol || ((ep.mode == kEpiI8Tensor || ep.mode == kEpiI32Raw) && ep.za != 0)) {
          for (int j = static_cast<int>(threadIdx.x) - 64; j < BN; j += 128) {
            const int n = min(n_blk * BN + j, N - 1);
            colv[j] = rowcol ? __float_as_uint(ep.col_scale[n]) : static_cast<uint32_t>(ep.col_sum[n]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
      bool have_acc = kb_end > kb_begin;
      if (have_acc) {
        const bool got = __all_sync(0xffffffffu, dev::mbar_wait<true>(&tfull[buf], use & 1u, abort_flag));
        if (!got) {
          // Split mode must still pass the cluster barriers below (with zeros).
          if constexpr (!SPLIT) break;
          have_acc = false;
        }
      }
      dev::tc_fence_after_sync();
      if (warp == 2 && lane == 0) CLOVE_TRACE_POINT(5);
      const int m0 = m_blk * S::BM;
      const int n0 = n_blk * BN;
      const int row = m0 + row_in_tile;
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + buf * BN;

      // Per-row epilogue constants.
      float row_scale = 0.f;
      int32_t row_corr = 0;
      if (ep.mode == kEpiI8RowCol) row_scale = (row < M) ? ep.row_scale[row] : 0.f;
      if ((ep.mode == kEpiI8Tensor || ep.mode == kEpiI32Raw) && ep.zb != 0 && row < M)
        row_corr = static_cast<int32_t>(0u - static_cast<uint32_t>(ep.zb) *
                                                 static_cast<uint32_t>(ep.row_sum[row]));

      if constexpr (SPLIT) {
        // Reduce-scatter over the cluster: the rows of the tile are dealt out in S
        // equal slices (with S = 8 a warp's rows span two slices). Every CTA first
        // pushes its partials of the other slices into their owners' shared memory
        // (st.async, counted on the owner's rbar), then finishes its own slice:
        // own partial first, then the S-1 received ones by rank. TMEM loads are
        // warp-collective, so they sit in warp-uniform loops; only the pushes, the
        // wait on rbar and the stores depend on the lane's slice. No CTA waits
        // before it has pushed, so the exchange cannot deadlock.
        const int parts = static_cast<int>(gridDim.x);
        const int rank = static_cast<int>(dev::cluster_ctarank());
        const int rs = S::BM / parts;
        const int owner = row_in_tile / rs;
        const int srow = row_in_tile - owner * rs;
        const bool mine = owner == rank;
        const int slot = mine ? 0 : (rank < owner ? rank : rank - 1);
        const uint32_t dst = dev::map_shared_to_rank(
            dev::smem_u32(part_base + (slot * rs + srow) * S::PART_ROW), static_cast<uint32_t>(owner));
        const uint32_t rb = dev::map_shared_to_rank(dev::smem_u32(rbar), static_cast<uint32_t>(owner));
#pragma unroll
        for (int c = 0; c < BN; c += 16) {
          uint32_t v[16];
          __syncwarp();  // reconverge after the previous pushes
          if (have_acc) {
            dev::tmem_ld_x16(t_row + c, v);
            dev::tmem_ld_wait();
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = 0u;
          }
          if (!mine && row < M) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              dev::st_async_v4(dst + (c + j) * 4, v[j], v[j + 1], v[j + 2], v[j + 3], rb);
          }
        }
        bool got = true;
        if (mine) {
          got = dev::mbar_wait<true>(rbar, 0u, abort_flag);
          if (!got) {
            // Error path: give late pushes a second bounded window to land before
            // this CTA (and its shared memory) can exit.
            volatile int no_abort = 0;
            dev::mbar_wait<true>(rbar, 0u, &no_abort);
          }
        }
        if (mine && srow == 0) CLOVE_TRACE_MAX(19);
        __syncwarp();
        if (warp == 2 && lane == 0) CLOVE_TRACE_POINT(6);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += S::CHUNK) {
          uint32_t v[S::CHUNK];
          __syncwarp();  // reconverge after the previous slice's stores
#pragma unroll
          for (int j = 0; j < S::CHUNK; j += 16) {
            uint32_t t[16];
            if (have_acc) {
              dev::tmem_ld_x16(t_row + c0 + j, t);
              dev::tmem_ld_wait();
            } else {
#pragma unroll
              for (int u = 0; u < 16; ++u) t[u] = 0u;
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) v[j + u] = t[u];
          }
          if (!mine) continue;
          for (int p = 0; p < parts - 1 && got; ++p) {
            const uint8_t* src = part_base + (p * rs + srow) * S::PART_ROW + c0 * 4;
#pragma unroll
            for (int j = 0; j < S::CHUNK; j += 4) {
              const uint4 r = *reinterpret_cast<const uint4*>(src + j * 4);
              if constexpr (Op::kInt) {
                v[j + 0] += r.x;
                v[j + 1] += r.y;
                v[j + 2] += r.z;
                v[j + 3] += r.w;
              } else {
                v[j + 0] = __float_as_uint(__uint_as_float(v[j + 0]) + __uint_as_float(r.x));
                v[j + 1] = __float_as_uint(__uint_as_float(v[j + 1]) + __uint_as_float(r.y));
                v[j + 2] = __float_as_uint(__uint_as_float(v[j + 2]) + __uint_as_float(r.z));
                v[j + 3] = __float_as_uint(__uint_as_float(v[j + 3]) + __uint_as_float(r.w));
              }
            }
          }
          store_row_direct<Op, OUT_BYTES, S::CHUNK>(v, ep, row, n0 + c0, M, N, K, row_scale,
                                                    row_corr, colv + c0);
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += S::CHUNK) {
          uint32_t v[S::CHUNK];
#pragma unroll
          for (int j = 0; j < S::CHUNK; j += 16) {
            uint32_t t[16];
            dev::tmem_ld_x16(t_row + c0 + j, t);
            dev::tmem_ld_wait();
#pragma unroll
            for (int u = 0; u < 16; ++u) v[j + u] = t[u];
          }
          if (c0 + S::CHUNK >= BN) {
            // All of this accumulator buffer is in registers: hand it back to the MMA warp.
            dev::tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) dev::mbar_arrive(&tempty[buf]);
          }
          store_chunk<Op, OUT_BYTES, S::CHUNK>(v, ep, row, n0 + c0, M, N, K, row_scale, row_corr,
                                               lane, stg_base, stg_count, &tmC,
                                               m0 + static_cast<int>(q) * 32, peer_n, plane);
        }
      }
      if (warp == 2 && lane == 0) CLOVE_TRACE_POINT(7);
      if (*abort_flag) break;
    }
    // Before the CTA exits its TMA stores must have read their shared-memory source
    // (their global writes complete with the grid). A replicated output waits for the
    // writes themselves: the remote stores (lane 0's TMA stores, or every lane's
    // multicast stores) are ordered before the cross-rank signal that follows the
    // kernel on the stream.
    if (lane == 0) {
      if (ep.peer.count > 0)
        dev::bulk_wait_group<0>();
      else
        dev::bulk_wait_group_read<0>();
    }
    __syncwarp();
    if (ep.peer.count > 0) __threadfence_system();
    if (warp == 2 && lane == 0) CLOVE_TRACE_POINT(8);
    if (lane == 0) CLOVE_TRACE_MAX(20);
    __syncwarp();
  }

  if constexpr (SPLIT) {
    // Warps 0/1 complete the start-up phase here (the epilogue warps did before
    // pushing). No final cluster barrier: a CTA only exits after every push into
    // its shared memory has landed (its rbar completed), and nothing reads another
    // CTA's shared memory.
    if (warp < 2) dev::cluster_wait();
  }

  dev::tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after_sync();
    dev::tmem_dealloc(tmem_base, S::TMEM_COLS);
    if (lane == 0) CLOVE_TRACE_POINT(9);
    if (lane == 0) CLOVE_TRACE_MAX(21);
  }
}

}  // namespace kern
}  // namespace clove
