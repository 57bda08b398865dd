// attention_sm100.cuh -- attention forward on tcgen05 (sm_100a): S = Q.K^T and
// O = P.V on the tensor cores with fp32 TMEM accumulators, online softmax between.
//
// Replaces the reference's CUDA-core flash_attention_kernel
// (src/kernels/attention.cu:93-266; its GEMMs are the scalar loops at :185-204).
// Same arithmetic: S = scale * q.k, causal keys k > q masked, softmax over the
// keys with a running maximum, O = softmax(S) . V normalised by the row sum,
// fp16 in and out, fp32 accumulation. head_dim 128.
//
// One CTA computes two consecutive 128-query tiles of one (batch, head), which share
// every K and V tile; keys advance 128 at a time. 12 warps in three warpgroups
// (setmaxnreg: 56 registers for the control group, 224 for the softmax groups):
//   warp 0     TMA producer (one thread): both Q tiles once (two 64-column boxes
//              each, 128B swizzle), then K and V, each in a 2-stage ring, in the
//              order the tensor core frees their stages (K of block j+2 once both
//              S of block j are computed, V of block j+2 once both P.V of block j
//              are), so no load waits behind a buffer that frees later.
//   warp 1     TMEM allocator + MMA issuer (the warp runs the schedule, one elected
//              lane issues): per key block, S_t = Q_t.K^T for each tile into its fp32
//              TMEM buffer (8 x kind::f16 M=128 N=128 K=16, both operands K-major,
//              from shared memory), and O_t += P_t.V with P_t read from tensor memory
//              and V (MN-major) from shared memory, in the order PV_0(j), QK_0(j+1),
//              PV_1(j), QK_1(j+1): while one tile's softmax runs, the tensor core
//              works on the other tile. P.V starts on keys [0,64) as soon as the
//              softmax has written them.
//   warps 2-3  idle (fill the control warpgroup)
//   warps 4-11 softmax, one warpgroup per tile, one query row per thread (its TMEM
//              lane): the row of S into registers, mask, row maximum,
//              p = 2^(s*scale*log2e - m), row sum, P as fp16 pairs written back over
//              the first 64 columns of the tile's S buffer (the A operand of P.V), in
//              two halves of 64 keys, each handed to the MMA issuer on its own barrier.
//              The running maximum m is raised only when a block's maximum exceeds
//              it by more than 8 (in log2 units): then O (in TMEM) and the row sum
//              are rescaled by 2^(m_old - m_new) before the next P.V; otherwise the
//              stale m is kept, p stays <= 2^8 and nothing is rescaled. Numerator and
//              denominator always use the same m, so the result is the same softmax.
//              At the end: O / l to fp16, staged in shared memory, TMA-stored.
// Tensor-core ordering carries the TMEM hand-offs: the MMAs of one issuing thread
// run in issue order, and a tcgen05.commit arrives once all earlier ones complete.
// So when S_t(j) is complete, P_t(j-1).V has finished reading P_t(j-1) and adding
// into O_t (the softmax may overwrite S_t with P_t(j) and rescale O_t), and
// QK_t(j+1), issued after PV_t(j), overwrites P_t(j) only after it has been read.
// Layouts: Q, K, V, O are 4D tensor maps (head_dim, seq, heads, batch) with any
// strides, so [batch, heads, seq, head_dim] (the reference's flash_attention) and
// [batch, seq, heads, head_dim] (its runtime's q/k/v projections) both work; K and V
// may have fewer heads than Q (grouped-query attention: kv head = head / group).
// Rows past seq_len read as zero (their keys are masked) and are never stored.
#pragma once

#include "params.h"
#include "sm100_ptx.cuh"

namespace clove {
namespace kern {

struct AttnShape {
  static constexpr int D = 128;        // head_dim
  static constexpr int BQ = 128;       // queries per tile (TMEM lanes)
  static constexpr int TILES = 2;      // query tiles per CTA (ping-pong)
  static constexpr int BKV = 128;      // keys per block
  static constexpr int STAGES = 2;     // K ring and V ring depth
  static constexpr int HALF_TILE = 128 * 128;          // [128 rows x 64 cols] fp16, 128B swizzle
  static constexpr int TILE = 2 * HALF_TILE;           // [128 rows x 128 cols] fp16
  static constexpr int OFF_Q = 0;                      // Q of tile t at t * TILE
  static constexpr int OFF_K = OFF_Q + TILES * TILE;   // K stage s at OFF_K + s * TILE
  static constexpr int OFF_V = OFF_K + STAGES * TILE;  // V stage s at OFF_V + s * TILE
  static constexpr int OFF_BAR = OFF_V + STAGES * TILE;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = 1024 + OFF_BAR + BAR_BYTES;
  // 12 warps in warpgroups: warps 0-3 control (0 producer, 1 MMA, 2-3 idle), then
  // one softmax warpgroup per tile. Registers: launched at 168 per thread (the cap
  // for 384 threads), setmaxnreg then gives the control warpgroup 56 and the
  // softmax warpgroups 224 (a row of S, 128 fp32, plus the exponential's constants).
  static constexpr int SOFT0 = 4;
  static constexpr int THREADS = (SOFT0 + 4 * TILES) * 32;
  static constexpr int REGS_LAUNCH = 168;
  static constexpr int REGS_CTL = 56;
  static constexpr int REGS_SOFT = 224;
  static_assert(128 * REGS_CTL + (THREADS - 128) * REGS_SOFT <= THREADS * REGS_LAUNCH,
                "register split exceeds the launch allocation");
  // Warp w runs on sub-partition w % 4: one control and two softmax warps each.
  static_assert(32 * (REGS_CTL + TILES * REGS_SOFT) <= 16384, "per sub-partition registers");
  // S of tile t at columns t*128 (P_t over its first 64), O of tile t at 256 + t*128.
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_COL = 256;
  static_assert(SMEM_BYTES <= 232448, "smem budget");
};

// kind::f16, fp32 accumulate, M = 128, N = 128; S: both operands K-major;
// O: A (P, in tensor memory) K-major, B (V) MN-major.
constexpr uint32_t kAttnIdescS = dev::make_idesc(1, 0, 0, 0, 0, 128, 128);
constexpr uint32_t kAttnIdescO = dev::make_idesc(1, 0, 0, 0, 1, 128, 128);

// Key pairs (of every 16) whose exponentials run as the FMA-pipe polynomial
// (dev::f2_exp2_poly) rather than on the MUFU, spread evenly over the 16.
#ifndef CLOVE_ATTN_POLY
#define CLOVE_ATTN_POLY 4
#endif
constexpr int kAttnPolyPairs = CLOVE_ATTN_POLY;
static_assert(kAttnPolyPairs >= 0 && kAttnPolyPairs <= 16, "poly pairs per 16");
__device__ __forceinline__ constexpr bool attn_poly_pair(int u) {
  return (u * kAttnPolyPairs) / 16 != ((u + 1) * kAttnPolyPairs) / 16;
}

// K-major descriptor of a [128 rows x 128 fp16] operand held as two 64-column
// 128B-swizzled halves, for the 16-column K step k.
__device__ __forceinline__ uint64_t attn_kmajor_desc(uint32_t base, int k) {
  return dev::make_smem_desc(base + (k >> 2) * AttnShape::HALF_TILE + (k & 3) * 32, 0, 1024,
                             dev::kLayoutSw128);
}
// MN-major descriptor of V [128 keys x 128 head_dim] (two 64-column halves, each
// [128 keys x 128 B]) for the 16-key step k: N atoms 16 KB apart, 8-key groups 1 KB.
__device__ __forceinline__ uint64_t attn_v_desc(uint32_t base, int k) {
  return dev::make_smem_desc(base + k * 16 * 128, AttnShape::HALF_TILE, 1024, dev::kLayoutSw128);
}

// Key blocks query tile qt visits (0 when the tile lies past seq_len).
template <bool CAUSAL>
__device__ __forceinline__ int attn_blocks(int qt, int seq_len) {
  const int n_qt = (seq_len + AttnShape::BQ - 1) / AttnShape::BQ;
  if (qt >= n_qt) return 0;
  const int n_kb = (seq_len + AttnShape::BKV - 1) / AttnShape::BKV;
  return CAUSAL ? min(qt + 1, n_kb) : n_kb;
}

// Development timeline (-DCLOVE_TRACE builds only): clock64 of the first CTA at
// the point, into trace slot i.
#ifdef CLOVE_TRACE
#define ATTN_TRACE(i)                                                             \
  do {                                                                            \
    if (blockIdx.x == 0) g_clove_trace[(i)] = clock64();                          \
  } while (0)
#else
#define ATTN_TRACE(i) \
  do {                \
  } while (0)
#endif

template <bool CAUSAL>
__global__ void __launch_bounds__(AttnShape::THREADS, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV,
                         const __grid_constant__ CUtensorMap tmO, int seq_len, int heads,
                         int kv_group, float scale_log2) {
  using S = AttnShape;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = dev::align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* q_full = bars;            // [1]
  uint64_t* k_full = bars + 1;        // [STAGES]
  uint64_t* k_empty = bars + 3;       // [STAGES]
  uint64_t* v_full = bars + 5;        // [STAGES]
  uint64_t* v_empty = bars + 7;       // [STAGES]
  uint64_t* s_full = bars + 9;        // [TILES]
  uint64_t* p_full = bars + 11;       // [TILES][2]: keys [0,64) and [64,128) of P_t
  uint64_t* o_full = bars + 15;       // [TILES]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = dev::warp_idx();
  const uint32_t lane = dev::lane_idx();
  const int n_qt = (seq_len + S::BQ - 1) / S::BQ;
  const int n_pairs = (n_qt + 1) / 2;
  // One-dimensional grid, rank-major: CTA i takes tile pair rank i / (heads * batch)
  // of (batch, head) i % (heads * batch). Causal pairs are ranked by key blocks,
  // most first, so the block scheduler starts every head's heaviest pair before any
  // lighter one (longest job first) and the light pairs fill the last wave.
  const int n_bh = static_cast<int>(gridDim.x) / n_pairs;
  const int rk = static_cast<int>(blockIdx.x) / n_bh;
  const int bh = static_cast<int>(blockIdx.x) - rk * n_bh;
  const int pr = CAUSAL ? n_pairs - 1 - rk : rk;
  const int head = bh % heads;
  const int kv_head = head / kv_group;
  const int batch = bh / heads;
  // Tile t covers queries [q0 + 128 t, q0 + 128 t + 128).
  const int q0 = pr * S::TILES * S::BQ;
  const int nb0 = attn_blocks<CAUSAL>(2 * pr, seq_len);      // key blocks of tile 0
  const int nb1 = attn_blocks<CAUSAL>(2 * pr + 1, seq_len);  // and of tile 1 (0: absent)
  const int nb = max(nb0, nb1);
  const int n_tiles = nb1 > 0 ? 2 : 1;

  if (threadIdx.x == 0) {
    dev::mbar_init(q_full, 1);
    for (int st = 0; st < S::STAGES; ++st) {
      dev::mbar_init(&k_full[st], 1);
      dev::mbar_init(&k_empty[st], 1);
      dev::mbar_init(&v_full[st], 1);
      dev::mbar_init(&v_empty[st], 1);
    }
    for (int t = 0; t < S::TILES; ++t) {
      dev::mbar_init(&s_full[t], 1);
      dev::mbar_init(&p_full[2 * t], 4);
      dev::mbar_init(&p_full[2 * t + 1], 4);
      dev::mbar_init(&o_full[t], 1);
    }
    *abort_flag = 0;
    dev::fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&tmQ);
    dev::prefetch_tmap(&tmK);
    dev::prefetch_tmap(&tmV);
    dev::prefetch_tmap(&tmO);
  }
  if (warp == 1) {
    dev::tmem_alloc(tmem_slot, S::TMEM_COLS);
    dev::tmem_relinquish_alloc_permit();
  }
  dev::tc_fence_before_sync();
  __syncthreads();
  dev::tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the set-up above overlaps the previous kernel's
  // tail; no global memory is touched before it completes.
  dev::allow_dependent_launch();
  dev::grid_dependency_wait();
  if (threadIdx.x == 0) ATTN_TRACE(0);

  // Roles by warpgroup; each branch first reallocates its registers (one setmaxnreg
  // executed by all four warps of the group, ahead of the role's code).
  if (warp < S::SOFT0) {
    dev::setmaxnreg_dec<S::REGS_CTL>();
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      dev::mbar_arrive_expect_tx(q_full, n_tiles * S::TILE);
      for (int t = 0; t < n_tiles; ++t) {
        uint8_t* q_dst = smem + S::OFF_Q + t * S::TILE;
        dev::tma_load_4d(q_dst, &tmQ, q_full, 0, q0 + t * S::BQ, head, batch);
        dev::tma_load_4d(q_dst + S::HALF_TILE, &tmQ, q_full, 64, q0 + t * S::BQ, head, batch);
      }
      // Ring slot of block j: stage j & 1, used for the (j >> 1)-th time. Blocks 0
      // and 1 find their stages free; block j + 2 waits for block j's release.
      uint32_t armed = 0, par = 0;  // bit s: K stage s, bit 2 + s: V stage s
      auto load = [&](const CUtensorMap* tm, uint64_t* full, uint64_t* empty, int off, int j,
                      int bit) -> bool {
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
        if (!dev::mbar_wait<true>(&empty[st], ph ^ 1u, abort_flag)) return false;
        uint8_t* dst = smem + off + st * S::TILE;
        dev::mbar_arrive_expect_tx(&full[st], S::TILE);
        dev::tma_load_4d(dst, tm, &full[st], 0, j * S::BKV, kv_head, batch);
        dev::tma_load_4d(dst + S::HALF_TILE, tm, &full[st], 64, j * S::BKV, kv_head, batch);
        armed |= 1u << (bit + st);
        par = (par & ~(1u << (bit + st))) | (ph << (bit + st));
        return true;
      };
      bool go = true;
      for (int j = 0; j < nb && j < 2 && go; ++j) go = load(&tmK, k_full, k_empty, S::OFF_K, j, 0);
      for (int j = 0; j < nb && j < 2 && go; ++j) go = load(&tmV, v_full, v_empty, S::OFF_V, j, 2);
      for (int j = 2; j < nb && go; ++j) {
        go = load(&tmK, k_full, k_empty, S::OFF_K, j, 0);
        go = go && load(&tmV, v_full, v_empty, S::OFF_V, j, 2);
      }
      if (*abort_flag) {
        // Error unwinding: every load still in flight lands before the CTA exits.
        volatile int no_abort = 0;
        dev::mbar_wait<true>(q_full, 0u, &no_abort);
        for (int st = 0; st < S::STAGES; ++st) {
          if (armed & (1u << st)) dev::mbar_wait<true>(&k_full[st], (par >> st) & 1u, &no_abort);
          if (armed & (4u << st))
            dev::mbar_wait<true>(&v_full[st], (par >> (2 + st)) & 1u, &no_abort);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Software-pipelined over the key blocks: PV_0(j), QK_0(j+1), PV_1(j), QK_1(j+1),
    // so each tile's next S = Q.K^T is queued on the tensor core right behind its
    // P.V while the other tile's softmax still runs. The whole warp runs the loop
    // (waits, descriptor arithmetic stay warp-uniform) and one elected lane issues
    // every MMA and commit: at N = 128 each MMA is 64 tensor-core cycles, so the
    // issue path has to keep up.
    const bool leader = dev::elect_one();
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, dev::mbar_wait(bar, parity, abort_flag));
    };
    bool ok = wait_all(q_full, 0u);
    auto qk = [&](int t, int j) {
      if (!ok) return;
      const uint32_t q_addr = dev::smem_u32(smem + S::OFF_Q + t * S::TILE);
      const uint32_t k_addr = dev::smem_u32(smem + S::OFF_K + (j & 1) * S::TILE);
      const uint32_t s_tmem = tmem_base + static_cast<uint32_t>(t) * S::BKV;
      if (leader) {
        if (j < 16) ATTN_TRACE(192 + t * 16 + j);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          dev::mma_f16_ss(s_tmem, attn_kmajor_desc(q_addr, k), attn_kmajor_desc(k_addr, k),
                          kAttnIdescS, k > 0 ? 1u : 0u);
        dev::mma_commit(&s_full[t]);
      }
      __syncwarp();
    };
    // O_t += P_t.V over keys [0,64) as soon as the softmax has written them, then
    // over [64,128): the first half's MMAs overlap the second half's exponentials.
    auto pv = [&](int t, int j, int tnb) {
      const uint32_t v_addr = dev::smem_u32(smem + S::OFF_V + (j & 1) * S::TILE);
      const uint32_t p_tmem = tmem_base + static_cast<uint32_t>(t) * S::BKV;
      const uint32_t o_tmem = tmem_base + S::O_COL + static_cast<uint32_t>(t) * S::BKV;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        ok = ok && wait_all(&p_full[2 * t + h], static_cast<uint32_t>(j) & 1u);
        if (!ok) return;
        dev::tc_fence_after_sync();
        if (leader) {
          if (h == 0 && j < 16) ATTN_TRACE(160 + t * 16 + j);
#pragma unroll
          for (int k = 4 * h; k < 4 * h + 4; ++k)
            dev::mma_f16_ts(o_tmem, p_tmem + 8 * k, attn_v_desc(v_addr, k), kAttnIdescO,
                            (j > 0 || k > 0) ? 1u : 0u);
          if (h == 1 && j == tnb - 1) dev::mma_commit(&o_full[t]);

        }
        __syncwarp();
      }
    };
    auto k_ready = [&](int j) {
      ok = ok && wait_all(&k_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u);
      if (ok) dev::tc_fence_after_sync();
    };
    auto commit = [&](uint64_t* bar) {
      if (leader) dev::mma_commit(bar);
      __syncwarp();
    };
    if (nb > 0) {
      k_ready(0);
      if (nb0 > 0) qk(0, 0);
      if (nb1 > 0) qk(1, 0);
      if (ok) commit(&k_empty[0]);  // block 0's K: both S issued
    }
    for (int j = 0; j < nb && ok; ++j) {
      // V of block j and K of block j+1 landed long ago (two-stage rings); waiting
      // for them here keeps them off the path from a softmax to the next MMAs.
      ok = wait_all(&v_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u);
      const bool next = j + 1 < nb;
      if (next) k_ready(j + 1);
      if (j < nb0) pv(0, j, nb0);
      if (next && j + 1 < nb0) qk(0, j + 1);
      if (j < nb1) pv(1, j, nb1);
      if (!ok) break;
      commit(&v_empty[j & 1]);                              // block j's V: both P.V issued
      if (next && j + 1 < nb1) qk(1, j + 1);
      if (next && ok) commit(&k_empty[(j + 1) & 1]);        // block j+1's K: both S issued
    }
  }  // warps 2-3: idle
  } else {
    // ------------------------------------------------------------ softmax (2 warpgroups)
    dev::setmaxnreg_inc<S::REGS_SOFT>();
    const int t = static_cast<int>(warp - S::SOFT0) >> 2;  // this warpgroup's query tile
    const uint32_t quarter = warp & 3u;             // TMEM lane quarter of this warp
    const int row = static_cast<int>(quarter * 32 + lane);
    const int qt0 = q0 + t * S::BQ;                 // the tile's first query
    const int qi = qt0 + row;
    const int my_nb = t ? nb1 : nb0;
    const uint32_t t_lane = tmem_base + ((quarter * 32u) << 16);
    const uint32_t s_col = static_cast<uint32_t>(t) * S::BKV;
    const uint32_t o_col = S::O_COL + static_cast<uint32_t>(t) * S::BKV;
    float m = -__int_as_float(0x7f800000);  // running maximum (log2 units), may be stale
    float l = 0.f;                           // running sum of p under m
    bool ok = true;
    for (int j = 0; j < my_nb; ++j) {
      const uint32_t ph = static_cast<uint32_t>(j) & 1u;
      ok = __all_sync(0xffffffffu, dev::mbar_wait(&s_full[t], ph, abort_flag));
      if (!ok) break;
      if (row == 0 && j < 16) ATTN_TRACE(64 + t * 16 + j);
      dev::tc_fence_after_sync();
      float s[128];
#pragma unroll
      for (int c = 0; c < 128; c += 16) {
        uint32_t r[16];
        dev::tmem_ld_x16(t_lane + s_col + c, r);
#pragma unroll
        for (int u = 0; u < 16; ++u) s[c + u] = __uint_as_float(r[u]);
      }
      dev::tmem_ld_wait();

      const int k0 = j * S::BKV;
      // Keys past seq_len, and for causal attention keys after the query, are masked.
      const bool edge = (k0 + S::BKV > seq_len) || (CAUSAL && k0 + S::BKV - 1 > qt0);
      if (edge) {
        const int lim = CAUSAL ? min(seq_len - 1, qi) : seq_len - 1;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (k0 + i > lim) s[i] = -__int_as_float(0x7f800000);
      }
      // Row maximum as 8 independent chains of 3-input maxima, then a short tree.
      float mx8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx8[u] = fmaxf(s[2 * u], s[2 * u + 1]);
#pragma unroll
      for (int i = 16; i < 128; i += 16)
#pragma unroll
        for (int u = 0; u < 8; ++u) mx8[u] = dev::fmax3(mx8[u], s[i + 2 * u], s[i + 2 * u + 1]);
      float mx = dev::fmax3(dev::fmax3(mx8[0], mx8[1], mx8[2]), dev::fmax3(mx8[3], mx8[4], mx8[5]),
                            fmaxf(mx8[6], mx8[7]));
      mx *= scale_log2;
      const float m_new = fmaxf(m, mx);
      const bool raise = m_new > m + 8.0f;
      const bool any_raise = __any_sync(0xffffffffu, raise);
      float alpha = 1.f;
      if (raise) {
        alpha = dev::ex2_approx(m - m_new);
        m = m_new;
      }
      // O was last added to by P_t(j-1).V, which completed before S_t(j) did.
      if (any_raise && j > 0) {
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          uint32_t r[16];
          dev::tmem_ld_x16(t_lane + o_col + c, r);
          dev::tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 16; ++u) r[u] = __float_as_uint(__uint_as_float(r[u]) * alpha);
          dev::tmem_st_x16(t_lane + o_col + c, r);
        }
      }
      // p = 2^(s * scale * log2e - m) on key pairs (packed fp32 arithmetic), packed to
      // fp16 pairs (key 2c in the low half of column c of the tile's P), 32 keys per
      // tensor-memory store. kAttnPolyPairs of every 16 pairs take the FMA-pipe
      // exponential, the rest the MUFU's ex2, whose rate alone would bound the row.
      const uint64_t sc2 = dev::f2_pack(scale_log2, scale_log2);
      const uint64_t nm2 = dev::f2_pack(-m, -m);
      uint64_t sum2[2] = {0ull, 0ull};  // two packed partial sums (+0.0f pairs)
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        uint32_t r[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int i = 2 * (c + u);
          const uint64_t x = dev::f2_fma(dev::f2_pack(s[i], s[i + 1]), sc2, nm2);
          uint64_t pp;
          if (attn_poly_pair(u)) {
            pp = dev::f2_exp2_poly(x);
          } else {
            float x0, x1;
            dev::f2_unpack(x, x0, x1);
            pp = dev::f2_pack(dev::ex2_approx(x0), dev::ex2_approx(x1));
          }
          sum2[u & 1] = dev::f2_add(sum2[u & 1], pp);
          float p0, p1;
          dev::f2_unpack(pp, p0, p1);
          r[u] = dev::pack_half2(p0, p1);
        }
        dev::tmem_st_x16(t_lane + s_col + c, r);
        if (c == 16 || c == 48) {
          // Keys [0,64) (then [64,128)) of P written: hand them to P.V.
          dev::tmem_st_wait();
          dev::tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) dev::mbar_arrive(&p_full[2 * t + (c >> 5)]);
        }
      }
      float sa, sb, sc, sd;
      dev::f2_unpack(sum2[0], sa, sb);
      dev::f2_unpack(sum2[1], sc, sd);
      l = l * alpha + ((sa + sb) + (sc + sd));
      if (row == 0 && j < 16) ATTN_TRACE(96 + t * 16 + j);
    }
    if (ok && my_nb > 0) {
      ok = __all_sync(0xffffffffu, dev::mbar_wait<true>(&o_full[t], 0u, abort_flag));
      if (ok) {
        dev::tc_fence_after_sync();
        const float inv_l = 1.0f / l;
        // fp16 O rows staged in this tile's Q (free: its last S = Q.K^T completed
        // before its last P.V), two [32 rows x 64 cols] 128B-swizzled boxes per warp,
        // then TMA-stored.
        uint8_t* stg = smem + S::OFF_Q + t * S::TILE + quarter * 2 * 4096;
        const uint32_t stg_addr = dev::smem_u32(stg);
#pragma unroll
        for (int c = 0; c < 128; c += 16) {
          uint32_t r[16];
          dev::tmem_ld_x16(t_lane + o_col + c, r);
          dev::tmem_ld_wait();
          const uint32_t box = static_cast<uint32_t>(c >> 6) * 4096u;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t chunk = static_cast<uint32_t>(((c & 63) >> 3) + h);
            const uint32_t off = box + lane * 128u + ((chunk ^ (lane & 7u)) << 4);
            dev::st_shared_v4(
                stg_addr + off,
                dev::pack_half2(__uint_as_float(r[8 * h + 0]) * inv_l, __uint_as_float(r[8 * h + 1]) * inv_l),
                dev::pack_half2(__uint_as_float(r[8 * h + 2]) * inv_l, __uint_as_float(r[8 * h + 3]) * inv_l),
                dev::pack_half2(__uint_as_float(r[8 * h + 4]) * inv_l, __uint_as_float(r[8 * h + 5]) * inv_l),
                dev::pack_half2(__uint_as_float(r[8 * h + 6]) * inv_l, __uint_as_float(r[8 * h + 7]) * inv_l));
          }
        }
        dev::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int r0 = qt0 + static_cast<int>(quarter) * 32;
          dev::tma_store_4d(&tmO, stg, 0, r0, head, batch);
          dev::tma_store_4d(&tmO, stg + 4096, 64, r0, head, batch);
          dev::bulk_commit_group();
          dev::bulk_wait_group_read<0>();  // source read before exit; writes complete with the grid
        }
        __syncwarp();
      }
    }
  }

  dev::tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after_sync();
    dev::tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace kern
}  // namespace clove
