// gemm_tc2_sm100.cuh -- CTA-pair tcgen05 GEMM (cta_group::2), 256 x 256 tiles.
//
// Same operands, layouts and epilogues as gemm_tc_kernel (A row-major [M,K]
// K-major, B row-major [K,N] MN-major, C row-major fp16), for the large prefill
// shapes. A cluster of two CTAs on two SMs computes one 256 x 256 tile of C:
//   * each CTA TMA-loads its own 128 rows of A and its own 128 columns of B for a
//     K block (32 KB per stage instead of 48 KB for a 128 x 256 tile on one SM,
//     so the pair pulls a third less L2 data per FLOP and fits 6 stages); the
//     loads' transaction bytes complete on the leader CTA's full barrier;
//   * the leader's MMA thread issues tcgen05.mma.cta_group::2 (M = 256, N = 256):
//     the tensor cores of both SMs read A from their own CTA and B from both, and
//     each SM's TMEM receives its 128 rows x 256 fp32 accumulator columns;
//     tcgen05.commit multicasts stage-free and accumulator-ready arrivals to both
//     CTAs (a commit multicast, not a TMA multicast);
//   * each CTA's 4 epilogue warps drain their own TMEM (two 256-column buffers)
//     and arrive on the leader's accumulator-free barrier, remotely for the peer.
// No TMA load in this kernel uses .multicast::cluster.
#pragma once

#include "gemm_tc_sm100.cuh"

namespace clove {
namespace kern {

// Pair tiles are 256 rows tall: bands of 8 keep the band of A that concurrently
// running pairs share as tall as the one-SM kernel's 16 x 128 rows.
constexpr int kPairGroupM = 8;

template <class Op>
struct Tc2Shape {
  static constexpr int BM = 128;        // rows per CTA (256 per pair)
  static constexpr int BN = 256;        // accumulator columns (the pair's N tile)
  static constexpr int BNH = 128;       // columns of B loaded by each CTA
  static constexpr int ELEM = Op::kElemBytes;
  static constexpr int BK = 128 / ELEM;
  static constexpr int UMMA_K = 32 / ELEM;
  static constexpr int KSTEPS = BK / UMMA_K;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int BH_BYTES = BNH * ELEM;        // bytes of one B row (this CTA's half)
  static constexpr int B_SW = 128;
  static constexpr int B_ATOMS = BH_BYTES / B_SW;
  static constexpr int B_ATOM_ELEMS = B_SW / ELEM;
  static constexpr int B_BYTES = BK * BH_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int CHUNK = 64;                    // fp16 output columns per store
  static constexpr int EPI_BYTES = 4 * 2 * 4096;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int STAGES_FIT = (kSmemLimit - 1024 - EPI_BYTES - BAR_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static_assert(B_ATOMS >= 1 && BH_BYTES % B_SW == 0, "B half in whole 128-byte atoms");
  static_assert(STAGES >= 3 && SMEM_BYTES <= kSmemLimit, "smem budget");
  static_assert(TMEM_COLS <= 512, "TMEM");
};

// One piece of a pair's work: K blocks [kb0, kb1) of `tile`.
struct Tc2Work {
  int tile, kb0, kb1;
  int sk_idx;  // stream-K tile index (-1: a whole-K tile)
  int j, nc;   // this pair's contributor index within the tile, the tile's contributor count
};

// Work order of one pair (SkParams): its contiguous range of stream-K units (unit =
// one K block of one stream-K tile) first, then its round-robin whole-K tiles, so
// that the last contributor's sum over the partial slots (L2 round trips) overlaps
// the whole-K tiles' main loops instead of trailing the kernel. Producer, MMA
// issuer and epilogue each walk the same sequence.
struct Tc2Sched {
  int pair, pairs, dp_tiles, kb_total, next_dp;
  long long U, u, u_end;
  __device__ Tc2Sched(int pair_, int pairs_, const SkParams& sk, int kb_total_)
      : pair(pair_), pairs(pairs_), dp_tiles(sk.dp_tiles), kb_total(kb_total_), next_dp(pair_) {
    U = static_cast<long long>(sk.sk_tiles) * kb_total_;
    u = U * pair_ / pairs_;
    u_end = U * (pair_ + 1) / pairs_;
  }
  // The pair whose range [U p / P, U (p+1) / P) holds unit v.
  __device__ int owner(long long v) const {
    return static_cast<int>(((v + 1) * pairs + U - 1) / U) - 1;
  }
  __device__ bool next(Tc2Work& w) {
    if (u >= u_end) {
      if (next_dp >= dp_tiles) return false;
      w.tile = next_dp;
      w.kb0 = 0;
      w.kb1 = kb_total;
      w.sk_idx = -1;
      w.j = 0;
      w.nc = 1;
      next_dp += pairs;
      return true;
    }
    const int t = static_cast<int>(u / kb_total);
    const long long t0 = static_cast<long long>(t) * kb_total;
    w.kb0 = static_cast<int>(u - t0);
    w.kb1 = static_cast<int>(min(static_cast<long long>(kb_total), w.kb0 + (u_end - u)));
    const int first = owner(t0);
    w.tile = dp_tiles + t;
    w.sk_idx = t;
    w.j = pair - first;
    w.nc = owner(t0 + kb_total - 1) - first + 1;
    u += w.kb1 - w.kb0;
    return true;
  }
};

// GLU (fp16 only): C = silu(A . B) * (A . B2) with B = W_gate, B2 = W_up [K,N].
// The pair's 256 accumulator columns become 128 gate columns (B half loaded by the
// leader CTA) followed by the same 128 columns of up (loaded by the peer CTA), so
// one MMA stream computes both projections of a 256 x 128 output tile and the
// epilogue applies silu(gate) * up before the only store.
template <class Op, bool GLU = false>
__global__ void __launch_bounds__(192, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmC,
                    int M, int N, int K, const __grid_constant__ EpiParams ep, SkParams sk) {
  using S = Tc2Shape<Op>;
  static_assert(!GLU || !Op::kInt, "GLU epilogue is fp16");
  constexpr int TILE_N = GLU ? S::BNH : S::BN;  // output columns per pair tile
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = dev::align_smem_1024(smem_raw);
  uint8_t* stage_base = smem;
  uint8_t* epi_base = smem + S::STAGES * S::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_base + S::EPI_BYTES);
  uint64_t* full = bars;                    // leader's used (both CTAs' bytes)
  uint64_t* empty = bars + S::STAGES;       // both CTAs (commit multicast)
  uint64_t* tfull = bars + 2 * S::STAGES;   // both CTAs (commit multicast)
  uint64_t* tempty = tfull + 2;             // leader's used (4 local + 4 remote arrivals)
  uint64_t* skbar = tempty + 2;             // stream-K hand-offs among this CTA's epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(skbar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* sk_last = abort_flag + 1;   // this CTA holds a stream-K tile's last ticket

  const uint32_t warp = dev::warp_idx();
  const uint32_t lane = dev::lane_idx();
  const uint32_t rank = dev::cluster_ctarank();  // 0 = leader of the pair
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      dev::mbar_init(&full[s], 1);
      dev::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      dev::mbar_init(&tfull[b], 1);
      dev::mbar_init(&tempty[b], 8);
    }
    dev::mbar_init(&skbar[0], 4);
    dev::mbar_init(&skbar[1], 1);
    *abort_flag = 0;
    dev::fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&tmA);
    dev::prefetch_tmap(&tmB);
    dev::prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    dev::tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    dev::tmem_relinquish_alloc_permit_pair();
  }
  dev::tc_fence_before_sync();
  dev::cluster_sync_all();  // both CTAs' barriers initialised before any cross-CTA use
  dev::tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the set-up above overlaps the tail of the
  // previous kernel on the stream; no global memory is touched before it completes.
  dev::allow_dependent_launch();
  dev::grid_dependency_wait();

  const int tiles_m = (M + 2 * S::BM - 1) / (2 * S::BM);
  const int tiles_n = (N + TILE_N - 1) / TILE_N;
  const int kb_total = (K + S::BK - 1) / S::BK;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      Tc2Sched sched(pair, pairs, sk, kb_total);
      Tc2Work w;
      while (sched.next(w)) {
        int m_blk, n_blk;
        tile_coords<kPairGroupM>(w.tile, tiles_m, tiles_n, m_blk, n_blk);
        const int my_m = m_blk * 2 * S::BM + static_cast<int>(rank) * S::BM;
        const int my_n = GLU ? n_blk * S::BNH : n_blk * S::BN + static_cast<int>(rank) * S::BNH;
        const CUtensorMap* my_b = (GLU && rank == 1) ? &tmB2 : &tmB;
        bool ok = true;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!dev::mbar_wait<true>(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) dev::mbar_arrive_expect_tx(&full[stage], 2 * S::STAGE_BYTES);
          uint8_t* a_dst = stage_base + stage * S::STAGE_BYTES;
          uint8_t* b_dst = a_dst + S::A_BYTES;
          dev::tma_load_2d_pair(a_dst, &tmA, &full[stage], kb * S::BK, my_m);
#pragma unroll
          for (int a = 0; a < S::B_ATOMS; ++a)
            dev::tma_load_2d_pair(b_dst + a * (S::BK * S::B_SW), my_b, &full[stage],
                                  my_n + a * S::B_ATOM_ELEMS, kb * S::BK);
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      const uint32_t idesc = Op::kInt ? dev::make_idesc(2, 1, 1, 0, 1, S::BN, 2 * S::BM)
                                      : dev::make_idesc(1, 0, 0, 0, 1, S::BN, 2 * S::BM);
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      Tc2Sched sched(pair, pairs, sk, kb_total);
      Tc2Work w;
      for (; ok && sched.next(w); ++it) {
        const uint32_t buf = static_cast<uint32_t>(it) & 1u;
        const uint32_t use = static_cast<uint32_t>(it) >> 1;
        if (!dev::mbar_wait<true>(&tempty[buf], (use & 1u) ^ 1u, abort_flag)) break;
        dev::tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * S::BN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!dev::mbar_wait<true>(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          dev::tc_fence_after_sync();
          const uint32_t a_addr = dev::smem_u32(stage_base + stage * S::STAGE_BYTES);
          const uint32_t b_addr = a_addr + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < S::KSTEPS; ++k) {
            const uint64_t adesc = dev::make_smem_desc(a_addr + k * 32, 0, 1024, dev::kLayoutSw128);
            const uint64_t bdesc = dev::make_smem_desc(b_addr + k * S::UMMA_K * S::B_SW,
                                                       S::BK * S::B_SW, 8 * S::B_SW,
                                                       dev::kLayoutSw128);
            const uint32_t acc = (kb > w.kb0 || k > 0) ? 1u : 0u;
            if constexpr (Op::kInt)
              dev::mma_i8_ss_pair(d_tmem, adesc, bdesc, idesc, acc);
            else
              dev::mma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, acc);
          }
          dev::mma_commit_pair(&empty[stage], 0x3);  // frees the stage in both CTAs
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        dev::mma_commit_pair(&tfull[buf], 0x3);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const uint32_t q = warp & 3u;
    const int row_in_tile = static_cast<int>(q * 32 + lane);
    uint8_t* stg_base = epi_base + (warp - 2) * (2 * 4096);
    uint32_t stg_count = 0;
    uint32_t ph0 = 0, ph1 = 0;  // completed phases of skbar[0] / skbar[1]
    int it = 0;
    // Replicated output: no remote store before every rank has reached this call.
    const int peer_n = peer_ready_warp(ep.peer, lane, abort_flag);
    Tc2Sched sched(pair, pairs, sk, kb_total);
    Tc2Work w;
    for (; sched.next(w); ++it) {
      int m_blk, n_blk;
      tile_coords<kPairGroupM>(w.tile, tiles_m, tiles_n, m_blk, n_blk);
      const uint32_t buf = static_cast<uint32_t>(it) & 1u;
      const uint32_t use = static_cast<uint32_t>(it) >> 1;
      if (!__all_sync(0xffffffffu, dev::mbar_wait<true>(&tfull[buf], use & 1u, abort_flag))) break;
      dev::tc_fence_after_sync();
      const int m0 = m_blk * 2 * S::BM + static_cast<int>(rank) * S::BM;
      const int n0 = n_blk * TILE_N;
      const int row = m0 + row_in_tile;
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + buf * S::BN;

      float row_scale = 0.f;
      int32_t row_corr = 0;
      if (ep.mode == kEpiI8RowCol) row_scale = (row < M) ? ep.row_scale[row] : 0.f;
      if ((ep.mode == kEpiI8Tensor || ep.mode == kEpiI32Raw) && ep.zb != 0 && row < M)
        row_corr = static_cast<int32_t>(0u - static_cast<uint32_t>(ep.zb) *
                                                 static_cast<uint32_t>(ep.row_sum[row]));
      if constexpr (!GLU) {
        if (w.nc > 1) {
          // Stream-K piece: park the 32-bit partial accumulators in this piece's
          // slot, laid out [column quad][row] so that a warp's 16-byte stores
          // cover 512 contiguous bytes, then take a ticket; the last of the
          // tile's contributors sums every slot in contributor order and runs
          // the epilogue. The tile's first K piece (j = 0) usually finishes last
          // (it closes this pair's stream-K range; the other pieces open theirs):
          // if every other contributor has already parked its partial, it sums
          // them onto its own accumulator straight from TMEM and parks nothing,
          // in the same order, so both routes give the same bits.
          constexpr size_t kSlot = static_cast<size_t>(S::BN) * S::BM;  // words per CTA and piece
          const int tix = w.sk_idx * 2 + static_cast<int>(rank);
          const uint32_t* slot0 =
              sk.partials + (static_cast<size_t>(w.sk_idx) * sk.max_contrib * 2 + rank) * kSlot;
          bool ok = true;
          bool fast = false;
          if (w.j == 0) {
            if (warp == 2 && lane == 0) {
              int t;
              asm volatile("ld.acquire.gpu.global.b32 %0, [%1];"
                           : "=r"(t)
                           : "l"(sk.tickets + tix)
                           : "memory");
              *sk_last = t == w.nc - 1 ? 2 : 0;
              // Every other piece has taken its ticket and this one takes none: the
              // tile is done with its ticket, which goes back to zero for the next
              // launch (the ticket array is kept between calls, never memset).
              if (t == w.nc - 1) sk.tickets[tix] = 0;
              dev::mbar_arrive(&skbar[1]);
            }
            ok = __all_sync(0xffffffffu, dev::mbar_wait(&skbar[1], ph1 & 1u, abort_flag));
            ++ph1;
            if (!ok) break;
            fast = *sk_last == 2;
          }
          // Sums slots [j_from, nc) onto v (v already holds the earlier terms
          // when j_from > 0).
          auto add_slots = [&](uint32_t (&v)[S::CHUNK], int c0, int j_from) {
#pragma unroll 1
            for (int jj = j_from; jj < w.nc; ++jj) {
              const uint32_t* src =
                  slot0 + static_cast<size_t>(jj) * 2 * kSlot + ((c0 / 4) * S::BM + row_in_tile) * 4;
              uint4 x[S::CHUNK / 4];
#pragma unroll
              for (int qd = 0; qd < S::CHUNK / 4; ++qd)
                x[qd] = __ldcg(reinterpret_cast<const uint4*>(src + qd * S::BM * 4));
#pragma unroll
              for (int qd = 0; qd < S::CHUNK / 4; ++qd) {
                const uint32_t e[4] = {x[qd].x, x[qd].y, x[qd].z, x[qd].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  uint32_t& d = v[4 * qd + i];
                  if (jj == 0)
                    d = e[i];
                  else if constexpr (Op::kInt)
                    d += e[i];
                  else
                    d = __float_as_uint(__uint_as_float(d) + __uint_as_float(e[i]));
                }
              }
            }
          };
          if (fast) {
            __threadfence();
#pragma unroll 1
            for (int c0 = 0; c0 < S::BN; c0 += S::CHUNK) {
              uint32_t v[S::CHUNK];
#pragma unroll
              for (int j = 0; j < S::CHUNK; j += 16) {
                uint32_t t[16];
                dev::tmem_ld_x16(t_row + c0 + j, t);
                dev::tmem_ld_wait();
#pragma unroll
                for (int u = 0; u < 16; ++u) v[j + u] = t[u];
              }
              if (c0 + S::CHUNK >= S::BN) {
                dev::tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) {
                  if (leader)
                    dev::mbar_arrive(&tempty[buf]);
                  else
                    dev::mbar_arrive_remote(&tempty[buf], 0);
                }
              }
              add_slots(v, c0, 1);
              store_chunk<Op, 2, S::CHUNK>(v, ep, row, n0 + c0, M, N, K, row_scale, row_corr, lane,
                                           stg_base, stg_count, &tmC,
                                           m0 + static_cast<int>(q) * 32, peer_n);
            }
            if (*abort_flag) break;
            continue;
          }
          uint32_t* part = sk.partials +
                           ((static_cast<size_t>(w.sk_idx) * sk.max_contrib + w.j) * 2 + rank) * kSlot;
#pragma unroll 1
          for (int c0 = 0; c0 < S::BN; c0 += 32) {
            uint32_t t0[16], t1[16];
            dev::tmem_ld_x16(t_row + c0, t0);
            dev::tmem_ld_x16(t_row + c0 + 16, t1);
            dev::tmem_ld_wait();
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
              *reinterpret_cast<uint4*>(part + ((c0 / 4 + qd) * S::BM + row_in_tile) * 4) =
                  make_uint4(t0[4 * qd], t0[4 * qd + 1], t0[4 * qd + 2], t0[4 * qd + 3]);
              *reinterpret_cast<uint4*>(part + ((c0 / 4 + 4 + qd) * S::BM + row_in_tile) * 4) =
                  make_uint4(t1[4 * qd], t1[4 * qd + 1], t1[4 * qd + 2], t1[4 * qd + 3]);
            }
          }
          dev::tc_fence_before_sync();
          __threadfence();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              dev::mbar_arrive(&tempty[buf]);
            else
              dev::mbar_arrive_remote(&tempty[buf], 0);
            dev::mbar_arrive(&skbar[0]);
          }
          ok = dev::mbar_wait(&skbar[0], ph0 & 1u, abort_flag);
          ++ph0;
          if (warp == 2 && lane == 0 && ok) {
            __threadfence();
            const int old = atomicAdd(&sk.tickets[tix], 1);
            *sk_last = old == w.nc - 1 ? 1 : 0;
            if (old == w.nc - 1) sk.tickets[tix] = 0;  // last ticket: reset for the next launch
            dev::mbar_arrive(&skbar[1]);
          }
          ok = __all_sync(0xffffffffu, ok);
          ok = ok && dev::mbar_wait(&skbar[1], ph1 & 1u, abort_flag);
          ok = __all_sync(0xffffffffu, ok);
          ++ph1;
          if (!ok) break;
          if (*sk_last == 1) {
            __threadfence();
#pragma unroll 1
            for (int c0 = 0; c0 < S::BN; c0 += S::CHUNK) {
              uint32_t v[S::CHUNK];
              add_slots(v, c0, 0);
              store_chunk<Op, 2, S::CHUNK>(v, ep, row, n0 + c0, M, N, K, row_scale, row_corr, lane,
                                           stg_base, stg_count, &tmC,
                                           m0 + static_cast<int>(q) * 32, peer_n);
            }
          }
          if (*abort_flag) break;
          continue;
        }
      }
#pragma unroll 1
      for (int c0 = 0; c0 < TILE_N; c0 += S::CHUNK) {
        uint32_t v[S::CHUNK];
#pragma unroll
        for (int j = 0; j < S::CHUNK; j += 16) {
          uint32_t t[16];
          dev::tmem_ld_x16(t_row + c0 + j, t);
          if constexpr (GLU) {
            uint32_t tu[16];
            dev::tmem_ld_x16(t_row + S::BNH + c0 + j, tu);  // the same columns of up
            dev::tmem_ld_wait();
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const float g = __uint_as_float(t[u]);
              v[j + u] = __float_as_uint(g / (1.0f + expf(-g)) * __uint_as_float(tu[u]));
            }
          } else {
            dev::tmem_ld_wait();
#pragma unroll
            for (int u = 0; u < 16; ++u) v[j + u] = t[u];
          }
        }
        if (c0 + S::CHUNK >= TILE_N) {
          // Accumulator drained: release it to the leader's MMA thread.
          dev::tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              dev::mbar_arrive(&tempty[buf]);
            else
              dev::mbar_arrive_remote(&tempty[buf], 0);
          }
        }
        store_chunk<Op, 2, S::CHUNK>(v, ep, row, n0 + c0, M, N, K, row_scale, row_corr, lane,
                                     stg_base, stg_count, &tmC, m0 + static_cast<int>(q) * 32, peer_n);
      }
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
    __syncwarp();
  }

  // No CTA leaves while its pair may still touch its shared memory or TMEM.
  dev::tc_fence_before_sync();
  dev::cluster_sync_all();
  if (warp == 1) {
    dev::tc_fence_after_sync();
    dev::tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace kern
}  // namespace clove
