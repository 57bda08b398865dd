// sm100_ptx.cuh -- thin inline-PTX wrappers for the Blackwell (sm_100a) features the
// GEMM kernels use: mbarriers, TMA (cp.async.bulk.tensor), tcgen05 MMA / TMEM,
// cluster shared memory. Every wait on an mbarrier is bounded by a wall-clock
// limit; on expiry the caller gets `false`, records an error and unwinds.
//
// No TMA load in this library uses .multicast::cluster: the same kernels run in
// multi-GPU jobs, and every CTA loads its own tiles.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace clove {
namespace dev {

// Device-side error word, one per translation unit (internal linkage). 0 = no
// error. Written with atomicCAS so the first error wins; each kernel TU exports a
// host function that reads and clears its word for clove_get_device_error().
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrWaitTimeout = 1,   // an mbarrier wait ran past kWaitTimeoutNs
  kDevErrBadLaunch = 2,     // kernel launched with a shape it does not support
};

static __device__ int g_device_error = 0;

// 2 seconds: several orders of magnitude above any legitimate wait in these kernels.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// First 1024-byte aligned byte of the dynamic shared memory array. Indexing the
// array (rather than rounding its address as an integer) keeps the pointer in the
// shared state space, so plain C++ loads through it compile to shared-memory loads
// instead of generic ones.
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* smem_raw) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  return smem_raw + ((1024u - (a & 1023u)) & 1023u);
}

__device__ __forceinline__ uint32_t warp_idx() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lane_idx() { return threadIdx.x & 31; }

// One lane of the (fully active) warp returns true.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "elect.sync _|P1, %1;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// With SLEEP, a waiting thread may be suspended up to kTryWaitSuspendNs inside one
// try_wait (it resumes as soon as the phase completes), so warps that wait long
// (an epilogue waiting for a whole tile) do not compete for issue slots. Waits on
// short hand-offs use the plain form.
constexpr uint32_t kTryWaitSuspendNs = 1000000u;

template <bool SLEEP = false>
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (SLEEP) {
    asm volatile(
        "{\n\t.reg .pred P1;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kTryWaitSuspendNs)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred P1;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  }
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up (returns
// false) when *abort becomes non-zero or after kWaitTimeoutNs; on a timeout it
// records the error and raises *abort so that the CTA's other roles unwind too.
template <bool SLEEP = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait<SLEEP>(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait<SLEEP>(bar, parity)) return true;
    if ((i & (SLEEP ? 3u : 63u)) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        record_error(kDevErrWaitTimeout);
        *abort = 1;
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// TMA (tensor maps are __grid_constant__ kernel parameters)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2D tiled load global -> this CTA's shared memory, completion on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 3D tiled load (a box one plane deep of a batched tensor map), completion on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 1D bulk copy global -> this CTA's shared memory (no tensor map), completion on
// `bar`. Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// CTA-pair form: the executing CTA loads into its own shared memory, and the
// transaction bytes complete on the mbarrier at the same offset in the pair's
// leader CTA (the address's peer bit is cleared). No multicast.
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint64_t* bar,
                                                 int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar) & kPeerBitMask), "r"(c0), "r"(c1)
      : "memory");
}

// 2D tiled store shared -> global (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int32_t c0,
                                             int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}

// 4D tiled load (a box one deep in the two outer dimensions), completion on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* m, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, const void* src, int32_t c0,
                                             int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m, const void* src, int32_t c0,
                                             int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Makes generic-proxy writes to shared memory visible to the async proxy (TMA store).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_alloc_permit() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// CTA-pair TMEM allocation: issued by the same warp in both CTAs of the pair.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_alloc_permit_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// CTA-pair MMA (M = 256 across the pair), issued by the leader CTA only.
__device__ __forceinline__ void mma_f16_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_i8_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at this offset in every CTA of cta_mask when all
// prior tcgen05 ops of this thread complete (pair form).
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrive on the mbarrier at the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote)
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; 16-bit inputs, fp32 accumulate.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B with A read from tensor memory (a_tmem: lane 0, first column
// of the M x 16 fp16 slice, two K-consecutive elements per 32-bit column) and B from
// shared memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B; 8-bit integer inputs, int32 accumulate, A read from tensor
// memory (a_tmem: lane 0, first column of the M x 32 byte slice, four K-consecutive
// bytes per 32-bit column), B from shared memory.
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B; 8-bit integer inputs, int32 accumulate.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns: thread t of the warp gets lane
// (warp's quarter * 32 + t), columns [col, col+16).
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns: thread t of the warp writes lane
// (warp's quarter * 32 + t), columns [col, col+16).
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32"
      " [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ----------------------------------------------------------------------------
// Shared-memory matrix descriptors and instruction descriptors
// ----------------------------------------------------------------------------
// Layout-type field (bits 61-63) values.
enum SmemLayout : uint32_t {
  kLayoutNone = 0,
  kLayoutSw128 = 2,
  kLayoutSw64 = 4,
  kLayoutSw32 = 6,
};

__host__ __device__ constexpr uint32_t layout_for_swizzle_bytes(int bytes) {
  return bytes == 128 ? kLayoutSw128 : bytes == 64 ? kLayoutSw64 : bytes == 32 ? kLayoutSw32 : kLayoutNone;
}

// start address, leading-dimension byte offset, stride-dimension byte offset
// (all in bytes, encoded >>4), fixed version field 0b001 at bits 46-48,
// base offset 0 (operand tiles are 1024-byte aligned), layout type at 61-63.
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 / kind::i8 (dense):
//   bits 4-5 accumulator format (1 = f32, 2 = s32), 7-9 A format, 10-12 B format
//   (f16: 0 = f16, 1 = bf16; i8: 0 = u8, 1 = s8), 15 A major (0 = K), 16 B major
//   (1 = MN), 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t a_fmt, uint32_t b_fmt,
                                                  uint32_t a_mn_major, uint32_t b_mn_major,
                                                  uint32_t N, uint32_t M) {
  return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ----------------------------------------------------------------------------
// Clusters / distributed shared memory
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Full cluster barrier (every thread of every CTA in the cluster arrives).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// Split cluster barrier: arrive (release) early, wait (acquire) when needed. Every
// thread of every CTA in the cluster takes part in each phase.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 16-byte store into another CTA's shared memory (address from mapa); its bytes
// complete a transaction on that CTA's mbarrier `remote_bar` (also mapa'd).
__device__ __forceinline__ void st_async_v4(uint32_t remote_addr, uint32_t a, uint32_t b,
                                            uint32_t c, uint32_t d, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          remote_addr),
      "r"(a), "r"(b), "r"(c), "r"(d), "r"(remote_bar)
      : "memory");
}

__device__ __forceinline__ uint32_t map_shared_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}


// ----------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialisation attribute may start before its predecessor on the stream
// finishes; grid_dependency_wait() blocks until the predecessor has completed and
// its memory is visible, so every global access placed after it is ordered as
// with a plain launch. allow_dependent_launch() lets the next such kernel start.
// Both are no-ops for kernels launched without the attribute.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----------------------------------------------------------------------------
// Misc
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// dot product of four unsigned bytes of a with four signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_u8s8(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32: relative error about
// 2^-22, subnormal results flushed to zero; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs (the f32x2 arithmetic of sm_100): lane 0 in the low word.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for both lanes of a packed pair, on the FMA pipe instead of the MUFU
// (Cody-Waite style reduction, polynomial fitted here by the Remez exchange):
// x = j + f with j = round(x) (adding 1.5 * 2^23 leaves j in the low mantissa bits)
// and f = x - j in [-0.5, 0.5] (exact); 2^f from a degree-4 polynomial with minimax
// relative error 2.6e-6 on that interval (2.7e-6 evaluated in fp32); j added to the
// exponent field ((bits(x + 1.5 * 2^23) << 23) == j << 23 modulo 2^32). Inputs below
// -125 are clamped there (2^-125 = 2.4e-38: zero once rounded to fp16, and the
// exponent field stays normal); inputs must be <= 128.
__device__ __forceinline__ uint64_t f2_exp2_poly(uint64_t x) {
  float x0, x1;
  f2_unpack(x, x0, x1);
  const uint64_t xc = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = f2_add(xc, f2_pack(12582912.f, 12582912.f));
  const uint64_t j = f2_add(t, f2_pack(-12582912.f, -12582912.f));
  const uint64_t f = f2_fma(j, f2_pack(-1.f, -1.f), xc);
  uint64_t q = f2_fma(f, f2_pack(0.009570102207362652f, 0.009570102207362652f),
                      f2_pack(0.05591785907745361f, 0.05591785907745361f));
  q = f2_fma(q, f, f2_pack(0.240247443318367f, 0.240247443318367f));
  q = f2_fma(q, f, f2_pack(0.6931217908859253f, 0.6931217908859253f));
  q = f2_fma(q, f, f2_pack(0.9999992847442627f, 0.9999992847442627f));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  return f2_pack(__uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23)),
                 __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23)));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ----------------------------------------------------------------------------
// Register reallocation between warpgroups (setmaxnreg): every warp of a
// warpgroup executes the same one. The sum over the block of the new limits must
// not exceed what the block was launched with (threads x registers at launch), or
// an increase waits forever: callers check it with a static_assert and the host
// checks the launch register count.
// ----------------------------------------------------------------------------
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ----------------------------------------------------------------------------
// Cross-rank flags (system scope: the flag arrays of other ranks are IPC
// mappings reached over NVLink)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Spins until *flag >= target or timeout_ns has passed (then records a timeout
// and returns false).
__device__ __forceinline__ bool wait_flag_geq(const unsigned long long* flag,
                                              unsigned long long target, uint64_t timeout_ns) {
  if (ld_acquire_sys_u64(flag) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (ld_acquire_sys_u64(flag) >= target) return true;
    if (globaltimer_ns() - t0 > timeout_ns) {
      record_error(kDevErrWaitTimeout);
      return false;
    }
    __nanosleep(128);
  }
}

// Receiver-ready handshake of a replicated-output GEMM (kern::PeerOut), run by
// one thread of each epilogue warp before that warp's first store. The caller
// must have passed griddepcontrol.wait (or have been launched without
// programmatic dependence), so every earlier kernel on this rank's stream -- in
// particular whatever read this rank's replicated C after the previous call --
// has completed. Publishes "this rank reached call e" into every rank's ready
// array (all publishers of a call store the same e, so repeats are harmless), then
// waits until every rank has published e. False (error recorded) on a timeout.
template <class PeerOutT>
__device__ __forceinline__ unsigned long long peer_ready_publish(const PeerOutT& po) {
  const unsigned long long e = *reinterpret_cast<const volatile unsigned long long*>(po.epoch) + 1;
  for (int d = 0; d < po.count; ++d)
    if (d != po.rank) st_release_sys_u64(po.ready_slot[d], e);
  return e;
}
// 16 bytes to every device bound to the multicast object behind `mc` (an address
// of the multicast mapping, 16-byte aligned); plain data movement, bit-exact.
__device__ __forceinline__ void multimem_st_v4(unsigned long long mc, uint32_t a, uint32_t b,
                                               uint32_t c, uint32_t d) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// A warp's staged slab of rows [row0, row0 + 32) x bytes [0, row_bytes) of a
// row-major fp16 tile (16-byte chunks swizzled with `swz(row, chunk)`), written to
// the multicast C at (row0 + r, col0 + 8 chunk): consecutive lanes take consecutive
// chunks of a row, so each row leaves as one contiguous run. Rows >= rows and
// columns >= cols (the local tile's extent) are not stored.
template <int ROW_BYTES, class Swz>
__device__ __noinline__ void multicast_slab(unsigned long long mc, int ldc, uint32_t stg_addr,
                                               int row0, int rows, int col0, int ncol0, int cols,
                                               uint32_t lane, Swz swz) {
  constexpr int PKTS = ROW_BYTES / 16;
#pragma unroll
  for (int it = 0; it < PKTS; ++it) {
    const int i = it * 32 + static_cast<int>(lane);
    const int r = i / PKTS, c = i % PKTS;
    if (row0 + r < rows && ncol0 + 8 * c < cols) {
      uint32_t v0, v1, v2, v3;
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3)
                   : "r"(stg_addr + r * ROW_BYTES + swz(r, c) * 16));
      multimem_st_v4(mc + (static_cast<unsigned long long>(row0 + r) * ldc + col0 + ncol0 + 8 * c) * 2,
                     v0, v1, v2, v3);
    }
  }
}

template <class PeerOutT>
__device__ __forceinline__ bool peer_ready_wait(const PeerOutT& po, unsigned long long e) {
  bool ok = true;
  for (int d = 0; d < po.count && ok; ++d)
    if (d != po.rank) ok = wait_flag_geq(po.ready_in + d, e, kWaitTimeoutNs);
  return ok;
}
template <class PeerOutT>
__device__ __forceinline__ bool peer_ready_gate(const PeerOutT& po) {
  return peer_ready_wait(po, peer_ready_publish(po));
}

}  // namespace dev
}  // namespace clove

// Timeline tracing for kernel development: with -DCLOVE_TRACE, CLOVE_TRACE_POINT(i)
// stores %globaltimer into slot i of a per-TU device array when executed by the
// first CTA; without it the macro expands to nothing (the product build).
#ifdef CLOVE_TRACE
static __device__ unsigned long long g_clove_trace[256];
#define CLOVE_TRACE_POINT(i)                                                      \
  do {                                                                            \
    if (blockIdx.x == 0 && blockIdx.y == 0) g_clove_trace[(i)] = clove::dev::globaltimer_ns(); \
  } while (0)
// Earliest / latest time any CTA reaches a point (slots reset by the host).
#define CLOVE_TRACE_MIN(i) atomicMin(&g_clove_trace[(i)], clove::dev::globaltimer_ns())
#define CLOVE_TRACE_MAX(i) atomicMax(&g_clove_trace[(i)], clove::dev::globaltimer_ns())
// Start time of each launch, in launch order: slots 32..63, counter in slot 31.
#define CLOVE_TRACE_SEQ()                                                         \
  do {                                                                            \
    if (blockIdx.x == 0 && threadIdx.x == 0) {                                    \
      const unsigned long long k_ = atomicAdd(&g_clove_trace[31], 1ull);          \
      g_clove_trace[32 + (k_ & 31)] = clove::dev::globaltimer_ns();               \
    }                                                                             \
  } while (0)
// Per-launch timelines of the first CTA: launch k (in start order, counter in
// slot 63) writes point j to slot 64 + 16 * (k % 12) + j.
#define CLOVE_TRACE_SEQ_BEGIN(shared_k)                                           \
  do {                                                                            \
    if (threadIdx.x == 0)                                                         \
      shared_k = blockIdx.x == 0                                                  \
                     ? static_cast<int>(atomicAdd(&g_clove_trace[63], 1ull) % 12ull) \
                     : 0;                                                         \
  } while (0)
#define CLOVE_TRACE_SEQ_POINT(shared_k, j)                                        \
  do {                                                                            \
    if (blockIdx.x == 0) g_clove_trace[64 + 16 * (shared_k) + (j)] = clove::dev::globaltimer_ns(); \
  } while (0)
#else
#define CLOVE_TRACE_SEQ_BEGIN(shared_k) \
  do {                                  \
  } while (0)
#define CLOVE_TRACE_SEQ_POINT(shared_k, j) \
  do {                                     \
  } while (0)
#define CLOVE_TRACE_POINT(i) \
  do {                       \
  } while (0)
#define CLOVE_TRACE_MIN(i) \
  do {                     \
  } while (0)
#define CLOVE_TRACE_MAX(i) \
  do {                     \
  } while (0)
#define CLOVE_TRACE_SEQ() \
  do {                    \
  } while (0)
#endif

// Host side: read and clear this translation unit's device error word.
#define CLOVE_DEFINE_ERROR_READER(fn_name)                                        \
  int fn_name() {                                                                 \
    int v = 0;                                                                    \
    if (cudaMemcpyFromSymbol(&v, clove::dev::g_device_error, sizeof(int)) != cudaSuccess) \
      return -1;                                                                  \
    if (v != 0) {                                                                 \
      const int z = 0;                                                            \
      cudaMemcpyToSymbol(clove::dev::g_device_error, &z, sizeof(int));            \
    }                                                                             \
    return v;                                                                     \
  }
