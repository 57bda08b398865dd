// gemm_int4_sm100.cuh -- INT4 group-wise GEMM on tcgen05 kind::i8 (sm_100a).
//
// Replaces the reference's SIMT kernel (src/kernels/gemm_int4.cu:45-193) with the
// semantics its header documents (gemm.cuh:67-87): both operands K-packed,
// A_q [M,K/2], B_q [N,K/2] (element 2j in the high nibble of byte j), per-128-group
// fp16 scales and integer zero points [rows,K/128]; C[m,n] = sum_g sA sB G with
//   G[m,n,g] = sum_{k in g} (a - zA)(b - zB)   exact in int32.
//
// One CTA computes a 128 x 128 tile of C; K advances one group (128 codes,
// 64 packed bytes) at a time. 20 warps in four-warp groups (setmaxnreg gives the
// epilogue 136 registers, the transform 80, the control warps 40):
//   warp 0      TMA producer: packed A / B boxes [128 rows x 64 B] (64B swizzle)
//               into a 4-deep ring; every 8 groups, boxes [128 rows x 8 groups] of
//               A/B scales and zero points into a 2-slot ring (when K % 1024 == 0
//               and those arrays are 16-byte aligned; otherwise each transform
//               thread loads its own row's scale and zero point, one group ahead).
//   warp 1      TMEM allocator + MMA issuer: 4 x tcgen05.mma kind::i8 (K = 32) per
//               group into one of three int32 TMEM buffers (a fresh accumulator per
//               group), so every G leaves the tensor core exact; the A operand comes
//               from tensor memory, B from shared memory.
//   warps 2-3   idle (fill the control warpgroup)
//   warps 4-11  transform: warps 4-7 unpack row t of the A tile into TMEM lane t (a
//               32-column stage: the MMA's A operand, no shared-memory round trip),
//               warps 8-11 row t of the B tile into a 128B-swizzled u8 shared-memory
//               stage, holding the biased codes a'' = a - zA + 16 and b'' = b - zB + 16, both in
//               [1, 31], formed with plain adds (no per-byte carries). Within a
//               group both operands use the same K order (the high nibbles of a
//               4-byte word, then its low nibbles), which leaves the dot product
//               unchanged. Per row they also sum the codes: with R = sum(a - zA),
//               Cc = sum(b - zB),
//                 G = D - 16 R - 16 Cc - 32768,   D = sum a'' b''  (u8 x u8 MMA).
//               They publish, per group, the B scales (fp32), 16 Cc per column,
//               0x4B400000 - 16 R - 32768 per row and the A scales (fp32).
//   warps 12-19 epilogue: two warps per TMEM lane quarter, 64 columns each, read
//               16 columns at a time. One 3-input integer add turns D into the fp32
//               bit pattern of 12582912 + G (exact: |G| < 2^22), one subtraction
//               gives float(G); acc += float(G) * (sA * sB) with packed fp32x2
//               math, in registers, while the tensor core computes the next group;
//               finally fp16 through swizzled smem and a TMA store.
// Zero points must be integer codes in [0, 15].
#pragma once

#include "params.h"
#include "sm100_ptx.cuh"

namespace clove {
namespace kern {

struct I4Shape {
  static constexpr int BM = 128;
  static constexpr int BN = 128;
  static constexpr int GB = 64;                       // packed bytes per group per row
  static constexpr int PK_STAGES = 4;
  static constexpr int UN_STAGES = 4;
  static constexpr int ACC_BUFS = 3;                  // int32 TMEM accumulators
  static constexpr int SB_SLOTS = 4;
  static constexpr int PK_A = BM * GB;                // 8 KB
  static constexpr int PK_BYTES = (BM + BN) * GB;     // 16 KB
  static constexpr int UN_BYTES = BN * 128;           // 16 KB: unpacked B (A is in TMEM)
  static constexpr int META_BOX = 128 * 16;           // 128 rows x 8 groups x fp16
  static constexpr int META_BYTES = 4 * META_BOX;     // A scale, A zero, B scale, B zero
  static constexpr int META_SLOTS = 2;
  // Per slot (one group): B scales, 16 x column code sums, row terms, A scales.
  static constexpr int SBF_BYTES = SB_SLOTS * 4 * BN * 4;
  static constexpr int EPI_BYTES = 8 * 4096;          // 8 warps x 32 rows x 128 B
  // 20 warps in warpgroup-aligned roles: warp 0 producer, warp 1 MMA, warps 2-3
  // idle, warps 4-11 transform, warps 12-19 epilogue.
  static constexpr int XFORM0 = 4;
  static constexpr int EPI0 = 12;
  static constexpr int THREADS = 20 * 32;
  // Registers: launched at 96 per thread (the cap for 640 threads, 5 warps per
  // sub-partition); setmaxnreg then moves them to where they are needed -- the
  // producer / MMA warpgroup down to 40, the transform warpgroups to 80, the
  // epilogue warpgroups (64 fp32 accumulators plus 32 columns of TMEM loads in
  // flight per thread) up to 136.
  static constexpr int REGS_LAUNCH = 96;
  static constexpr int REGS_CTL = 40;
  static constexpr int REGS_XFORM = 80;
  static constexpr int REGS_EPI = 136;
  static_assert(128 * REGS_CTL + 256 * REGS_XFORM + 256 * REGS_EPI <= THREADS * REGS_LAUNCH,
                "register split exceeds the launch allocation");
  // Warp w runs on sub-partition w % 4, which therefore holds one warp of each
  // warpgroup: one control, two transform, two epilogue warps.
  static_assert(32 * (REGS_CTL + 2 * REGS_XFORM + 2 * REGS_EPI) <= 16384,
                "per sub-partition register file");
  // TMEM: accumulator b at columns b * BN; unpacked A stage u (128 lanes x 128 bytes)
  // at A_COL + 32 u.
  static constexpr int A_COL = ACC_BUFS * BN;
  static constexpr int TMEM_COLS = 512;
  static constexpr int OFF_UN = 0;                                      // 1024-aligned
  static constexpr int OFF_PK = OFF_UN + UN_STAGES * UN_BYTES;
  static constexpr int OFF_META = OFF_PK + PK_STAGES * PK_BYTES;
  // The output staging reuses the first unpacked stage: it is written only after
  // the last MMA has completed (its accumulator was drained).
  static constexpr int OFF_EPI = OFF_UN;
  static constexpr int OFF_SBF = OFF_META + META_SLOTS * META_BYTES;
  static constexpr int OFF_BAR = OFF_SBF + SBF_BYTES;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM_BYTES = 1024 + OFF_BAR + BAR_BYTES;
  static_assert(SMEM_BYTES <= 232448, "smem budget");
  static_assert(OFF_PK % 1024 == 0 && OFF_META % 1024 == 0 && OFF_EPI % 1024 == 0, "align");
  static_assert(EPI_BYTES <= UN_STAGES * UN_BYTES, "staging alias");
  static_assert(A_COL + UN_STAGES * 32 <= TMEM_COLS, "TMEM");
};

// kind::i8, s32 accumulator, u8 x u8, both operands K-major, M = N = 128.
constexpr uint32_t kI4Idesc = dev::make_idesc(2, 0, 0, 0, 0, I4Shape::BN, I4Shape::BM);
constexpr int32_t kF32Magic = 0x4B400000;  // bit pattern of 12582912.0f = 1.5 * 2^23

// Scales and zero points per row and group, read directly (the TMETA = false
// variant): Xs / Xz [rows, NG] binary16.
struct I4Meta {
  const __half* As;
  const __half* Az;
  const __half* Bs;
  const __half* Bz;
};

// DBG instantiation writes every exact group accumulator to Gdbg [M,N,K/128].
// TMETA: scales and zero points arrive by TMA in boxes of 8 groups (row pitch
// K/128 * 2 bytes a multiple of 16, i.e. K % 1024 == 0); otherwise each transform
// thread loads its row's scale and zero point of the next group itself (one group
// ahead), which serves any K % 128 == 0.
template <bool DBG, bool TMETA>
__global__ void __launch_bounds__(I4Shape::THREADS, 1)
    gemm_int4_tc_kernel(const __grid_constant__ CUtensorMap tmAq,
                        const __grid_constant__ CUtensorMap tmBq,
                        const __grid_constant__ CUtensorMap tmAs,
                        const __grid_constant__ CUtensorMap tmAz,
                        const __grid_constant__ CUtensorMap tmBs,
                        const __grid_constant__ CUtensorMap tmBz,
                        const __grid_constant__ CUtensorMap tmC, int M, int N, int K,
                        int32_t* __restrict__ Gdbg, const __grid_constant__ PeerOut peer,
                        I4Meta meta) {
  using S = I4Shape;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = dev::align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* pk_full = bars;                        // [4]
  uint64_t* pk_empty = bars + 4;                   // [4]
  uint64_t* un_full = bars + 8;                    // [4]
  uint64_t* un_empty = bars + 12;                  // [4]
  uint64_t* acc_full = bars + 16;                  // [4]
  uint64_t* acc_empty = bars + 20;                 // [4]
  uint64_t* meta_full = bars + 24;                 // [2]
  uint64_t* meta_empty = bars + 26;                // [2]
  uint64_t* sb_full = bars + 28;                   // [4]
  uint64_t* sb_empty = bars + 32;                  // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 36);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sbf = reinterpret_cast<float*>(smem + S::OFF_SBF);

  const uint32_t warp = dev::warp_idx();
  const uint32_t lane = dev::lane_idx();
  const int NG = K >> 7;
  const int m0 = static_cast<int>(blockIdx.y) * S::BM;
  const int n0 = static_cast<int>(blockIdx.x) * S::BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S::PK_STAGES; ++i) {
      dev::mbar_init(&pk_full[i], 1);
      dev::mbar_init(&pk_empty[i], 8);
    }
    for (int i = 0; i < S::UN_STAGES; ++i) {
      dev::mbar_init(&un_full[i], 8);
      dev::mbar_init(&un_empty[i], 1);
    }
    for (int i = 0; i < S::ACC_BUFS; ++i) {
      dev::mbar_init(&acc_full[i], 1);
      dev::mbar_init(&acc_empty[i], 8);
    }
    for (int i = 0; i < S::SB_SLOTS; ++i) {
      dev::mbar_init(&sb_full[i], 8);
      dev::mbar_init(&sb_empty[i], 8);
    }
    for (int i = 0; i < 2; ++i) {
      dev::mbar_init(&meta_full[i], 1);
      dev::mbar_init(&meta_empty[i], 8);  // the transform warps
    }
    *abort_flag = 0;
    dev::fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&tmAq);
    dev::prefetch_tmap(&tmBq);
    dev::prefetch_tmap(&tmAs);
    dev::prefetch_tmap(&tmAz);
    dev::prefetch_tmap(&tmBs);
    dev::prefetch_tmap(&tmBz);
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
  if (threadIdx.x == 0) CLOVE_TRACE_POINT(0);

  // Roles by warpgroup; each branch first reallocates its registers (one setmaxnreg
  // executed by all four warps of the group, ahead of the role's code).
  if (warp < S::XFORM0) {
    dev::setmaxnreg_dec<S::REGS_CTL>();
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;  // packed stages with a load in flight
      uint32_t meta_armed = 0, meta_par = 0;
      for (int g = 0; g < NG; ++g) {
        if (TMETA && (g & 7) == 0) {
          const int c = g >> 3;
          const int slot = c & 1;
          if (!dev::mbar_wait<true>(&meta_empty[slot], ((c >> 1) & 1) ^ 1u, abort_flag)) break;
          uint8_t* mt = smem + S::OFF_META + slot * S::META_BYTES;
          dev::mbar_arrive_expect_tx(&meta_full[slot], S::META_BYTES);
          dev::tma_load_2d(mt + 0 * S::META_BOX, &tmAs, &meta_full[slot], g, m0);
          dev::tma_load_2d(mt + 1 * S::META_BOX, &tmAz, &meta_full[slot], g, m0);
          dev::tma_load_2d(mt + 2 * S::META_BOX, &tmBs, &meta_full[slot], g, n0);
          dev::tma_load_2d(mt + 3 * S::META_BOX, &tmBz, &meta_full[slot], g, n0);
          meta_armed |= 1u << slot;
          meta_par = (meta_par & ~(1u << slot)) | (static_cast<uint32_t>((c >> 1) & 1) << slot);
        }
        const int s = g % S::PK_STAGES;
        const uint32_t use = static_cast<uint32_t>(g / S::PK_STAGES);
        if (!dev::mbar_wait<true>(&pk_empty[s], (use & 1u) ^ 1u, abort_flag)) break;
        uint8_t* pk = smem + S::OFF_PK + s * S::PK_BYTES;
        dev::mbar_arrive_expect_tx(&pk_full[s], S::PK_BYTES);
        dev::tma_load_2d(pk, &tmAq, &pk_full[s], g * S::GB, m0);
        dev::tma_load_2d(pk + S::PK_A, &tmBq, &pk_full[s], g * S::GB, n0);
        if (g < 32) CLOVE_TRACE_POINT(160 + g);
        armed |= 1u << s;
        armed_par = (armed_par & ~(1u << s)) | ((use & 1u) << s);
      }
      if (*abort_flag) {
        volatile int no_abort = 0;
        for (int s = 0; s < S::PK_STAGES; ++s)
          if (armed & (1u << s)) dev::mbar_wait(&pk_full[s], (armed_par >> s) & 1u, &no_abort);
        for (int s = 0; s < 2; ++s)
          if (meta_armed & (1u << s)) dev::mbar_wait(&meta_full[s], (meta_par >> s) & 1u, &no_abort);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      for (int g = 0; g < NG; ++g) {
        const int u = g % S::UN_STAGES;
        const int b = g % S::ACC_BUFS;
        if (!dev::mbar_wait(&un_full[u], static_cast<uint32_t>(g / S::UN_STAGES) & 1u, abort_flag))
          break;
        if (!dev::mbar_wait(&acc_empty[b], (static_cast<uint32_t>(g / S::ACC_BUFS) & 1u) ^ 1u,
                            abort_flag))
          break;
        dev::tc_fence_after_sync();
        if (g < 32) CLOVE_TRACE_POINT(96 + g);
        const uint32_t a_tm = tmem_base + S::A_COL + static_cast<uint32_t>(u) * 32;
        const uint32_t b_addr = dev::smem_u32(smem + S::OFF_UN + u * S::UN_BYTES);
        const uint32_t d = tmem_base + static_cast<uint32_t>(b) * S::BN;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t bd = dev::make_smem_desc(b_addr + k * 32, 0, 1024, dev::kLayoutSw128);
          dev::mma_i8_ts(d, a_tm + 8 * k, bd, kI4Idesc, k > 0 ? 1u : 0u);
        }
        dev::mma_commit(&un_empty[u]);
        dev::mma_commit(&acc_full[b]);
      }
    }
    __syncwarp();
  }  // warps 2-3: idle
  } else if (warp < S::EPI0) {
    // ------------------------------------------------------------ transform
    dev::setmaxnreg_dec<S::REGS_XFORM>();
    const int t = static_cast<int>(((warp - S::XFORM0) & 3) * 32 + lane);  // row of the A or B tile
    const int opw = static_cast<int>(warp - S::XFORM0) >> 2;                 // 0: A rows, 1: B rows
    // Direct scale / zero-point loads (TMETA = false): this thread's row, one group
    // ahead of its use; rows past the matrix read as scale 0, zero point 0.
    const int grow = (opw == 0 ? m0 : n0) + t;
    const bool row_in = grow < (opw == 0 ? M : N);
    const __half* row_s = (opw == 0 ? meta.As : meta.Bs) + static_cast<size_t>(grow) * NG;
    const __half* row_z = (opw == 0 ? meta.Az : meta.Bz) + static_cast<size_t>(grow) * NG;
    __half nxt_s = __float2half(0.f), nxt_z = __float2half(0.f);
    if (!TMETA && row_in) {
      nxt_s = row_s[0];
      nxt_z = row_z[0];
    }
#ifdef CLOVE_TRACE
    // Development timing of one transform thread (CTA 0, first A warp, lane 0), clock
    // cycles summed over groups 8-23: waits, unpack, proxy fence, hand-off.
    const bool xf_probe = blockIdx.x == 0 && blockIdx.y == 0 && warp == S::XFORM0 && lane == 0;
    long long xt0 = 0, xt1 = 0, xt2 = 0, xt3 = 0;
#endif
    for (int g = 0; g < NG; ++g) {
      const int c = g >> 3;
      const int mslot = c & 1;
      const int s = g % S::PK_STAGES;
      const int u = g % S::UN_STAGES;
      const int sbs = g % S::SB_SLOTS;
#ifdef CLOVE_TRACE
      if (xf_probe) xt0 = clock64();
#endif
      bool ok = true;
      if (TMETA && (g & 7) == 0)
        ok = dev::mbar_wait(&meta_full[mslot], static_cast<uint32_t>(c >> 1) & 1u, abort_flag);
      ok = ok && dev::mbar_wait(&pk_full[s], static_cast<uint32_t>(g / S::PK_STAGES) & 1u, abort_flag);
      ok = ok && dev::mbar_wait(&un_empty[u], (static_cast<uint32_t>(g / S::UN_STAGES) & 1u) ^ 1u, abort_flag);
      ok = ok && dev::mbar_wait(&sb_empty[sbs], (static_cast<uint32_t>(g / S::SB_SLOTS) & 1u) ^ 1u, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (warp == S::XFORM0 && lane == 0 && g < 32) CLOVE_TRACE_POINT(192 + g);
#ifdef CLOVE_TRACE
      if (xf_probe) xt1 = clock64();
#endif

      const int gi = g & 7;
      float rs;  // this row's scale for group g
      int rz;    // and its zero point
      if constexpr (TMETA) {
        const uint8_t* mt = smem + S::OFF_META + mslot * S::META_BYTES;
        const __half* meta_s = reinterpret_cast<const __half*>(mt + (opw == 0 ? 0 : 2) * S::META_BOX);
        const __half* meta_z = reinterpret_cast<const __half*>(mt + (opw == 0 ? 1 : 3) * S::META_BOX);
        rs = __half2float(meta_s[t * 8 + gi]);
        rz = __half2int_rn(meta_z[t * 8 + gi]);
      } else {
        rs = __half2float(nxt_s);
        rz = __half2int_rn(nxt_z);
        if (row_in && g + 1 < NG) {
          nxt_s = row_s[g + 1];
          nxt_z = row_z[g + 1];
        }
      }
      const int za = opw == 0 ? rz : 0;
      const int zb = opw == 1 ? rz : 0;
      float* slot = sbf + sbs * 4 * S::BN;  // [B scale][16 Cc][row term][A scale]
      if (opw == 1)
        slot[t] = rs;
      else
        slot[3 * S::BN + t] = rs;

      const uint8_t* pk = smem + S::OFF_PK + s * S::PK_BYTES;
      uint8_t* un = smem + S::OFF_UN + u * S::UN_BYTES;
#pragma unroll
      for (int op = 0; op < 2; ++op) {
        if (op != opw) continue;  // warp-uniform: this warp transforms one operand
        const uint8_t* src = pk + op * S::PK_A + t * 64;                 // 64B-swizzled packed row
        const int z = op == 0 ? za : zb;
        const uint32_t bias4 = static_cast<uint32_t>(16 - z) * 0x01010101u;
        uint32_t hs = 0, ls = 0;  // byte lanes: sums of 16 nibbles each (<= 240, no carries)
        uint32_t o[16];           // 64 unpacked codes: 16-byte chunks 4h .. 4h + 3 of the row
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 q = *reinterpret_cast<const uint4*>(src + ((j ^ ((t >> 1) & 3)) << 4));
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            const uint32_t hi = (w[x] >> 4) & 0x0f0f0f0fu;
            const uint32_t lo = w[x] & 0x0f0f0f0fu;
            hs += hi;
            ls += lo;
            o[(j & 1) * 8 + 2 * x] = hi + bias4;      // bytes code + 16 - z in [1, 31]: no carries
            o[(j & 1) * 8 + 2 * x + 1] = lo + bias4;
          }
          if (j & 1) {
            // Chunks c = 2j - 2 .. 2j + 1 (K bytes 16c ..) of the row.
            if (op == 0) {
              // A: TMEM lane t, columns 4c .. (four K-consecutive bytes per column).
              dev::tmem_st_x16(tmem_base + ((static_cast<uint32_t>(t & ~31)) << 16) + S::A_COL +
                                   static_cast<uint32_t>(u) * 32 + (j >> 1) * 16,
                               o);
            } else {
              // B: the 128B-swizzled K-major shared-memory operand.
              const uint32_t dst = dev::smem_u32(un + t * 128);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int c = 2 * (j - 1) + e;
                dev::st_shared_v4(dst + ((c ^ (t & 7)) << 4), o[4 * e], o[4 * e + 1], o[4 * e + 2],
                                  o[4 * e + 3]);
              }
            }
          }
        }
        const int codes = static_cast<int>(__dp4a(hs, 0x01010101u, __dp4a(ls, 0x01010101u, 0u)));
        const int r = codes - 128 * z;  // sum over the group of (code - z)
        if (op == 0)
          reinterpret_cast<int*>(slot)[2 * S::BN + t] = kF32Magic - 16 * r - 32768;
        else
          reinterpret_cast<int*>(slot)[S::BN + t] = 16 * r;
      }
#ifdef CLOVE_TRACE
      if (xf_probe) xt2 = clock64();
#endif
      if (opw == 0) {
        dev::tmem_st_wait();            // A stage written to TMEM
        dev::tc_fence_before_sync();
      } else {
        dev::fence_proxy_async_smem();  // generic-proxy writes -> tensor core reads
      }
#ifdef CLOVE_TRACE
      if (xf_probe) xt3 = clock64();
#endif
      __syncwarp();
      if (lane == 0) {
#ifdef CLOVE_TRACE
        if (xf_probe && g >= 8 && g < 24) {
          g_clove_trace[48] += static_cast<unsigned long long>(xt1 - xt0);  // waits
          g_clove_trace[49] += static_cast<unsigned long long>(xt2 - xt1);  // unpack
          g_clove_trace[50] += static_cast<unsigned long long>(xt3 - xt2);  // proxy fence
          g_clove_trace[51] += static_cast<unsigned long long>(clock64() - xt3);  // hand-off
        }
#endif
        if (warp == S::XFORM0 && g < 32) CLOVE_TRACE_POINT(64 + g);
        dev::mbar_arrive(&un_full[u]);
        dev::mbar_arrive(&sb_full[sbs]);
        dev::mbar_arrive(&pk_empty[s]);
        if (TMETA && (gi == 7 || g == NG - 1)) dev::mbar_arrive(&meta_empty[mslot]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    dev::setmaxnreg_inc<S::REGS_EPI>();
    const uint32_t q = warp & 3u;
    const int h = static_cast<int>(warp - S::EPI0) >> 2;  // column half of the tile
    const int row = static_cast<int>(q * 32 + lane);
    // Replicated output: announce that this rank reached the call (every earlier
    // kernel on its stream, the readers of its C included, has completed: this
    // kernel has no programmatic dependence); the remote stores wait below until
    // every rank has.
    unsigned long long ready_e = 0;
    if (peer.count > 0 && lane == 0) ready_e = dev::peer_ready_publish(peer);
    float2 acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = make_float2(0.f, 0.f);
    bool ok = true;
    for (int g = 0; g < NG && ok; ++g) {
      const int b = g % S::ACC_BUFS;
      const int sbs = g % S::SB_SLOTS;
      ok = dev::mbar_wait<true>(&acc_full[b], static_cast<uint32_t>(g / S::ACC_BUFS) & 1u, abort_flag);
      ok = ok && dev::mbar_wait(&sb_full[sbs], static_cast<uint32_t>(g / S::SB_SLOTS) & 1u, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (warp == S::EPI0 && lane == 0 && g < 32) CLOVE_TRACE_POINT(224 + g);
      dev::tc_fence_after_sync();
      const float* slot = sbf + sbs * 4 * S::BN;
      const float sa = slot[3 * S::BN + row];
      const float* sb = slot + h * 64;
      const int* colt = reinterpret_cast<const int*>(slot) + S::BN + h * 64;
      const int rowt = reinterpret_cast<const int*>(slot)[2 * S::BN + row];
      const float2 sa2 = make_float2(sa, sa);
      const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
      const uint32_t taddr = tmem_base + ((q * 32u) << 16) + static_cast<uint32_t>(b) * S::BN + h * 64;
#ifdef CLOVE_TRACE
      long long t_e0 = clock64();
#endif
#pragma unroll
      for (int qc = 0; qc < 2; ++qc) {  // 32 columns (two TMEM loads in flight) at a time
        uint32_t vv[32];
#ifdef CLOVE_TRACE
        long long t_ld0 = clock64();
#endif
        dev::tmem_ld_x16(taddr + qc * 32, *reinterpret_cast<uint32_t(*)[16]>(&vv[0]));
        dev::tmem_ld_x16(taddr + qc * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&vv[16]));
        dev::tmem_ld_wait();
#ifdef CLOVE_TRACE
        if (warp == S::EPI0 && lane == 0 && g == 12 && blockIdx.x == 0 && blockIdx.y == 0)
          g_clove_trace[40 + qc] = static_cast<unsigned long long>(clock64() - t_ld0 + (vv[0] & 0));
#endif
        if (qc == 1) {
          dev::tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) dev::mbar_arrive(&acc_empty[b]);
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const int col = qc * 32 + j;  // column within this warp's 64
          const float4 s4 = *reinterpret_cast<const float4*>(sb + col);
          const int4 c4 = *reinterpret_cast<const int4*>(colt + col);
          // fp32 bit patterns of 12582912 + G: one 3-input add each.
          const int f0 = static_cast<int>(vv[j + 0]) + rowt - c4.x;
          const int f1 = static_cast<int>(vv[j + 1]) + rowt - c4.y;
          const int f2 = static_cast<int>(vv[j + 2]) + rowt - c4.z;
          const int f3 = static_cast<int>(vv[j + 3]) + rowt - c4.w;
          const float2 g01 = __fadd2_rn(make_float2(__int_as_float(f0), __int_as_float(f1)), neg_magic);
          const float2 g23 = __fadd2_rn(make_float2(__int_as_float(f2), __int_as_float(f3)), neg_magic);
          const float2 s01 = __fmul2_rn(sa2, make_float2(s4.x, s4.y));
          const float2 s23 = __fmul2_rn(sa2, make_float2(s4.z, s4.w));
          const int a = col >> 1;
          acc[a] = __ffma2_rn(g01, s01, acc[a]);
          acc[a + 1] = __ffma2_rn(g23, s23, acc[a + 1]);
          if (DBG && m0 + row < M) {  // test hook: exact group accumulators
            const int nb = n0 + h * 64 + col;
            const int fs[4] = {f0, f1, f2, f3};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (nb + e < N)
                Gdbg[(static_cast<size_t>(m0 + row) * N + nb + e) * NG + g] = fs[e] - kF32Magic;
          }
        }
      }
#ifdef CLOVE_TRACE
      if (warp == S::EPI0 && lane == 0 && g == 12 && blockIdx.x == 0 && blockIdx.y == 0)
        g_clove_trace[44] = static_cast<unsigned long long>(clock64() - t_e0 + (acc[0].x == 1.5f));
#endif
      __syncwarp();
      if (lane == 0) {
        if (warp == S::EPI0 && g < 32) CLOVE_TRACE_POINT(128 + g);
        dev::mbar_arrive(&sb_empty[sbs]);
      }
    }
    if (ok) {
      // fp16 into a 128B-swizzled staging tile, one TMA store per warp.
      uint8_t* stg = smem + S::OFF_EPI + (warp - S::EPI0) * 4096;
      const uint32_t sa_ = dev::smem_u32(stg);
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const uint32_t o0 = dev::pack_half2(acc[p * 4 + 0].x, acc[p * 4 + 0].y);
        const uint32_t o1 = dev::pack_half2(acc[p * 4 + 1].x, acc[p * 4 + 1].y);
        const uint32_t o2 = dev::pack_half2(acc[p * 4 + 2].x, acc[p * 4 + 2].y);
        const uint32_t o3 = dev::pack_half2(acc[p * 4 + 3].x, acc[p * 4 + 3].y);
        dev::st_shared_v4(sa_ + lane * 128 + ((p ^ (lane & 7)) << 4), o0, o1, o2, o3);
      }
      dev::fence_proxy_async_smem();
      __syncwarp();
      int peer_n = 0;
      if (lane == 0) {
        dev::tma_store_2d(&tmC, stg, n0 + h * 64, m0 + static_cast<int>(q) * 32);
        // Replicated output of an N-split: the same staged slab to every rank's C,
        // once every rank is ready to receive it (none after a timeout).
        peer_n = peer.count > 0 && dev::peer_ready_wait(peer, ready_e) ? peer.count : 0;
        if (peer.mc == 0)
          for (int d = 0; d < peer_n; ++d)
            dev::tma_store_2d(&peer.maps[d], stg, peer.col0 + n0 + h * 64,
                              m0 + static_cast<int>(q) * 32);
        dev::bulk_commit_group();
        // Shared-memory source read before exit; the global writes themselves only
        // when a cross-rank signal follows (replicated output).
        if (peer.count > 0)
          dev::bulk_wait_group<0>();
        else
          dev::bulk_wait_group_read<0>();
      }
      peer_n = __shfl_sync(0xffffffffu, peer_n, 0);
      // Multicast replicated output: the whole warp sends the staged slab once.
      if (peer_n > 0 && peer.mc != 0)
        dev::multicast_slab<128>(peer.mc, peer.ldc, sa_, m0 + static_cast<int>(q) * 32, M,
                                 peer.col0, n0 + h * 64, N, lane,
                                 [](uint32_t r, uint32_t c) { return c ^ (r & 7u); });
      if (peer.count > 0) __threadfence_system();  // before the cross-rank signal
      __syncwarp();
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
