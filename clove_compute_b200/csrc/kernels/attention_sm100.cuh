// attention_sm100.cuh -- attention forward on tcgen05 (sm_100a): S = Q.K^T and
// O = P.V on the tensor cores with fp32 TMEM accumulators, online softmax between.
//
// Replaces the reference's CUDA-core flash_attention_kernel
// (src/kernels/attention.cu:93-266; its GEMMs are the scalar loops at :185-204).
// Same arithmetic: S = scale * q.k, causal keys k > q masked, softmax over the
// keys with a running maximum, O = softmax(S) . V normalised by the row sum,
// fp16 in and out, fp32 accumulation. head_dim 128.
//
// One CTA computes a 128-query tile of one (batch, head); keys advance 128 at a
// time. 6 warps:
//   warp 0     TMA producer: the Q tile once (two 64-column boxes, 128B swizzle),
//              then K and V tiles of each key block into a 2-stage ring (K and V
//              complete on separate barriers, so S = Q.K^T can start before V lands).
//   warp 1     TMEM allocator + MMA issuer (one thread): S_j = Q.K_j^T into one of
//              two fp32 TMEM buffers (8 x kind::f16 M=128 N=128 K=16, both operands
//              K-major), then O += P_{j-1}.V_{j-1} (P K-major from shared memory, V
//              MN-major), so the tensor core computes S_{j+1} while the softmax
//              warps work on S_j.
//   warps 2-5  softmax, one query row per thread (its TMEM lane): the row of S_j
//              into registers, mask, row maximum, p = 2^(s*scale*log2e - m), row sum,
//              P as fp16 into shared memory (the A operand of P.V, 128B swizzle).
//              The running maximum m is raised only when a block's maximum exceeds it
//              by more than 8 (in log2 units): then O (in TMEM) and the row sum are
//              rescaled by 2^(m_old - m_new) before the next P.V; otherwise the
//              stale m is kept, p stays <= 2^8 and nothing is rescaled. Numerator and
//              denominator always use the same m, so the result is the same softmax.
//              At the end: O / l to fp16, staged in shared memory, TMA-stored.
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
  static constexpr int BQ = 128;       // queries per CTA (TMEM lanes)
  static constexpr int BKV = 128;      // keys per block
  static constexpr int STAGES = 2;
  static constexpr int HALF_TILE = 128 * 128;          // [128 rows x 64 cols] fp16, 128B swizzle
  static constexpr int TILE = 2 * HALF_TILE;           // [128 rows x 128 cols] fp16
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + TILE;          // stage s: K at +0, V at +TILE
  static constexpr int OFF_P = OFF_KV + STAGES * 2 * TILE;
  static constexpr int OFF_BAR = OFF_P + TILE;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = 1024 + OFF_BAR + BAR_BYTES;
  static constexpr int TMEM_COLS = 512;                // S buffers at 0 and 128, O at 256
  static constexpr int O_COL = 256;
  static_assert(SMEM_BYTES <= 232448, "smem budget");
};

// kind::f16, fp32 accumulate, M = 128, N = 128; S: both operands K-major;
// O: A (P) K-major, B (V) MN-major.
constexpr uint32_t kAttnIdescS = dev::make_idesc(1, 0, 0, 0, 0, 128, 128);
constexpr uint32_t kAttnIdescO = dev::make_idesc(1, 0, 0, 0, 1, 128, 128);

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

template <bool CAUSAL>
__global__ void __launch_bounds__(192, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV,
                         const __grid_constant__ CUtensorMap tmO, int seq_len, int kv_group,
                         float scale_log2) {
  using S = AttnShape;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = dev::align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* q_full = bars;            // [1]
  uint64_t* k_full = bars + 1;        // [2]
  uint64_t* v_full = bars + 3;        // [2]
  uint64_t* kv_empty = bars + 5;      // [2]
  uint64_t* s_full = bars + 7;        // [2]
  uint64_t* s_empty = bars + 9;       // [2]
  uint64_t* p_full = bars + 11;       // [1]
  uint64_t* p_empty = bars + 12;      // [1]
  uint64_t* o_full = bars + 13;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = dev::warp_idx();
  const uint32_t lane = dev::lane_idx();
  const int n_qt = (seq_len + S::BQ - 1) / S::BQ;
  // Causal: the longest query tiles (most key blocks) start first.
  const int qt = CAUSAL ? n_qt - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
  const int head = static_cast<int>(blockIdx.y);
  const int kv_head = head / kv_group;
  const int batch = static_cast<int>(blockIdx.z);
  const int q0 = qt * S::BQ;
  const int n_kb_all = (seq_len + S::BKV - 1) / S::BKV;
  const int nb = CAUSAL ? min(qt + 1, n_kb_all) : n_kb_all;

  if (threadIdx.x == 0) {
    dev::mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(&k_full[s], 1);
      dev::mbar_init(&v_full[s], 1);
      dev::mbar_init(&kv_empty[s], 1);
      dev::mbar_init(&s_full[s], 1);
      dev::mbar_init(&s_empty[s], 4);
    }
    dev::mbar_init(p_full, 4);
    dev::mbar_init(p_empty, 1);
    dev::mbar_init(o_full, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint8_t* q_dst = smem + S::OFF_Q;
      dev::mbar_arrive_expect_tx(q_full, S::TILE);
      dev::tma_load_4d(q_dst, &tmQ, q_full, 0, q0, head, batch);
      dev::tma_load_4d(q_dst + S::HALF_TILE, &tmQ, q_full, 64, q0, head, batch);
      uint32_t armed = 0, armed_par = 0;
      for (int j = 0; j < nb; ++j) {
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
        if (!dev::mbar_wait<true>(&kv_empty[st], ph ^ 1u, abort_flag)) break;
        uint8_t* k_dst = smem + S::OFF_KV + st * 2 * S::TILE;
        uint8_t* v_dst = k_dst + S::TILE;
        const int k0 = j * S::BKV;
        dev::mbar_arrive_expect_tx(&k_full[st], S::TILE);
        dev::tma_load_4d(k_dst, &tmK, &k_full[st], 0, k0, kv_head, batch);
        dev::tma_load_4d(k_dst + S::HALF_TILE, &tmK, &k_full[st], 64, k0, kv_head, batch);
        dev::mbar_arrive_expect_tx(&v_full[st], S::TILE);
        dev::tma_load_4d(v_dst, &tmV, &v_full[st], 0, k0, kv_head, batch);
        dev::tma_load_4d(v_dst + S::HALF_TILE, &tmV, &v_full[st], 64, k0, kv_head, batch);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      if (*abort_flag) {
        // Error unwinding: every load still in flight lands before the CTA exits.
        volatile int no_abort = 0;
        dev::mbar_wait<true>(q_full, 0u, &no_abort);
        for (int st = 0; st < 2; ++st)
          if (armed & (1u << st)) {
            dev::mbar_wait<true>(&k_full[st], (armed_par >> st) & 1u, &no_abort);
            dev::mbar_wait<true>(&v_full[st], (armed_par >> st) & 1u, &no_abort);
          }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t q_addr = dev::smem_u32(smem + S::OFF_Q);
      const uint32_t p_addr = dev::smem_u32(smem + S::OFF_P);
      const uint32_t o_tmem = tmem_base + S::O_COL;
      // O += P_i . V_i once softmax i has written P_i (and rescaled O if needed).
      auto pv = [&](int i) -> bool {
        const int st = i & 1;
        if (!dev::mbar_wait(p_full, static_cast<uint32_t>(i) & 1u, abort_flag)) return false;
        if (!dev::mbar_wait(&v_full[st], static_cast<uint32_t>(i >> 1) & 1u, abort_flag))
          return false;
        dev::tc_fence_after_sync();
        const uint32_t v_addr = dev::smem_u32(smem + S::OFF_KV + st * 2 * S::TILE + S::TILE);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          dev::mma_f16_ss(o_tmem, attn_kmajor_desc(p_addr, k), attn_v_desc(v_addr, k),
                          kAttnIdescO, (i > 0 || k > 0) ? 1u : 0u);
        dev::mma_commit(&kv_empty[st]);
        dev::mma_commit(p_empty);
        return true;
      };
      bool ok = dev::mbar_wait(q_full, 0u, abort_flag);
      for (int j = 0; j < nb && ok; ++j) {
        const int st = j & 1;
        ok = dev::mbar_wait(&k_full[st], static_cast<uint32_t>(j >> 1) & 1u, abort_flag);
        ok = ok && dev::mbar_wait(&s_empty[st], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u,
                                  abort_flag);
        if (!ok) break;
        dev::tc_fence_after_sync();
        const uint32_t k_addr = dev::smem_u32(smem + S::OFF_KV + st * 2 * S::TILE);
        const uint32_t s_tmem = tmem_base + static_cast<uint32_t>(st) * S::BKV;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          dev::mma_f16_ss(s_tmem, attn_kmajor_desc(q_addr, k), attn_kmajor_desc(k_addr, k),
                          kAttnIdescS, k > 0 ? 1u : 0u);
        dev::mma_commit(&s_full[st]);
        if (j > 0) ok = pv(j - 1);
      }
      if (ok && nb > 0) ok = pv(nb - 1);
      if (ok) dev::mma_commit(o_full);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax (warps 2-5)
    const uint32_t quarter = warp & 3u;
    const int row = static_cast<int>(quarter * 32 + lane);
    const int qi = q0 + row;
    const uint32_t t_lane = tmem_base + ((quarter * 32u) << 16);
    float m = -__int_as_float(0x7f800000);  // running maximum (log2 units), may be stale
    float l = 0.f;                           // running sum of p under m
    bool ok = true;
    uint8_t* p_row = smem + S::OFF_P + row * 128;
    for (int j = 0; j < nb; ++j) {
      const int st = j & 1;
      ok = __all_sync(0xffffffffu,
                      dev::mbar_wait(&s_full[st], static_cast<uint32_t>(j >> 1) & 1u, abort_flag));
      if (!ok) break;
      dev::tc_fence_after_sync();
      float s[128];
#pragma unroll
      for (int c = 0; c < 128; c += 16) {
        uint32_t r[16];
        dev::tmem_ld_x16(t_lane + static_cast<uint32_t>(st) * S::BKV + c, r);
#pragma unroll
        for (int u = 0; u < 16; ++u) s[c + u] = __uint_as_float(r[u]);
      }
      dev::tmem_ld_wait();
      dev::tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(&s_empty[st]);

      const int k0 = j * S::BKV;
      // Keys past seq_len, and for causal attention keys after the query, are masked.
      const bool edge = (k0 + S::BKV > seq_len) || (CAUSAL && k0 + S::BKV - 1 > q0);
      if (edge) {
        const int lim = CAUSAL ? min(seq_len - 1, qi) : seq_len - 1;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (k0 + i > lim) s[i] = -__int_as_float(0x7f800000);
      }
      float mx = s[0];
#pragma unroll
      for (int i = 1; i < 128; ++i) mx = fmaxf(mx, s[i]);
      mx *= scale_log2;
      const float m_new = fmaxf(m, mx);
      const bool raise = m_new > m + 8.0f;
      const bool any_raise = __any_sync(0xffffffffu, raise);
      float alpha = 1.f;
      if (raise) {
        alpha = dev::ex2_approx(m - m_new);
        m = m_new;
      }
      // p = 2^(s * scale * log2e - m), packed to fp16 pairs.
      uint32_t pk[64];
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        const float p0 = dev::ex2_approx(fmaf(s[i], scale_log2, -m));
        const float p1 = dev::ex2_approx(fmaf(s[i + 1], scale_log2, -m));
        sum += p0 + p1;
        pk[i >> 1] = dev::pack_half2(p0, p1);
      }
      l = l * alpha + sum;
      // P's buffer and O are free once the previous P.V has completed.
      ok = __all_sync(0xffffffffu,
                      dev::mbar_wait(p_empty, (static_cast<uint32_t>(j) & 1u) ^ 1u, abort_flag));
      if (!ok) break;
      dev::tc_fence_after_sync();
      if (any_raise && j > 0) {
        const uint32_t o_lane = t_lane + S::O_COL;
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          uint32_t r[16];
          dev::tmem_ld_x16(o_lane + c, r);
          dev::tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 16; ++u) r[u] = __float_as_uint(__uint_as_float(r[u]) * alpha);
          dev::tmem_st_x16(o_lane + c, r);
        }
        dev::tmem_st_wait();
      }
      // P row into the 128B-swizzled A operand: keys [0,64) in the first half tile,
      // [64,128) in the second; 16-byte chunk c of a row at (c ^ row % 8).
      const uint32_t p_addr = dev::smem_u32(p_row);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t half = static_cast<uint32_t>(c >> 3) * S::HALF_TILE;
        const uint32_t off = half + ((static_cast<uint32_t>(c & 7) ^ (static_cast<uint32_t>(row) & 7u)) << 4);
        dev::st_shared_v4(p_addr + off, pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      dev::fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
      dev::tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(p_full);
    }
    if (ok && nb > 0) {
      ok = __all_sync(0xffffffffu, dev::mbar_wait<true>(o_full, 0u, abort_flag));
      if (ok) {
        dev::tc_fence_after_sync();
        const float inv_l = 1.0f / l;
        // fp16 O rows staged in the Q tile (free: every MMA has completed), two
        // [32 rows x 64 cols] 128B-swizzled boxes per warp, then TMA-stored.
        uint8_t* stg = smem + S::OFF_Q + quarter * 2 * 4096;
        const uint32_t stg_addr = dev::smem_u32(stg);
#pragma unroll
        for (int c = 0; c < 128; c += 16) {
          uint32_t r[16];
          dev::tmem_ld_x16(t_lane + S::O_COL + c, r);
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
          const int r0 = q0 + static_cast<int>(quarter) * 32;
          dev::tma_store_4d(&tmO, stg, 0, r0, head, batch);
          dev::tma_store_4d(&tmO, stg + 4096, 64, r0, head, batch);
          dev::bulk_commit_group();
          dev::bulk_wait_group<0>();
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
