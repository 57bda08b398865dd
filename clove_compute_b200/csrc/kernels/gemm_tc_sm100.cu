// gemm_tc_sm100.cu -- host launchers for the tcgen05 tile kernels (gemm_tc_sm100.cuh):
// TMA descriptor encoding, kernel instantiation table, persistent / cluster launch.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>
#include <vector>

#include "gemm_tc2_sm100.cuh"
#include "gemm_tc_sm100.cuh"
#include "../runtime/internal.h"
#include "../runtime/tensor_map.h"

namespace clove {
namespace rt {

CLOVE_DEFINE_ERROR_READER(read_clear_error_tc)

}  // namespace rt
}  // namespace clove

#ifdef CLOVE_TRACE
// Development builds only: copies the tile kernel's trace slots to the host.
extern "C" int clove_trace_read_tc(unsigned long long* out, int n) {
  return static_cast<int>(
      cudaMemcpyFromSymbol(out, g_clove_trace, sizeof(unsigned long long) * (n < 256 ? n : 256)));
}
extern "C" int clove_trace_write_tc(const unsigned long long* in) {
  return static_cast<int>(cudaMemcpyToSymbol(g_clove_trace, in, sizeof(unsigned long long) * 256));
}
#endif

namespace clove {
namespace rt {

namespace {

using kern::EpiParams;
using kern::OpF16;
using kern::OpI8;
using kern::TcShape;

typedef void (*TcKernelFn)(CUtensorMap, CUtensorMap, CUtensorMap, int, int, int, int, int,
                           EpiParams);

struct TcEntry {
  int op, bn, split, out_bytes;
  const void* fn;
  int smem_bytes;
  int bk, b_atom_elems, chunk, stg_row, b_sw;
};

template <class Op, int BN, bool SPLIT, int OUT>
TcEntry make_entry(int op) {
  using S = TcShape<Op, BN, SPLIT, OUT>;
  TcEntry e;
  e.op = op;
  e.bn = BN;
  e.split = SPLIT ? 2 : 1;  // "split" entries serve cluster sizes 2, 4 and 8
  e.out_bytes = OUT;
  e.fn = reinterpret_cast<const void*>(&kern::gemm_tc_kernel<Op, BN, SPLIT, OUT>);
  e.smem_bytes = S::SMEM_BYTES;
  e.bk = S::BK;
  e.b_atom_elems = S::B_ATOM_ELEMS;
  e.chunk = S::CHUNK;
  e.stg_row = S::STG_ROW;
  e.b_sw = S::B_SW;
  return e;
}

struct Table {
  static constexpr int kMax = 32;
  TcEntry e[kMax];
  std::atomic<uint64_t> attr_set[kMax];  // bit d: smem attribute set on device d
  int n = 0;
  template <class Op, int BN, bool SPLIT, int OUT>
  void add(int op) {
    attr_set[n].store(0);
    e[n++] = make_entry<Op, BN, SPLIT, OUT>(op);
  }
  Table() {
    add<OpF16, 64, false, 2>(kTcF16);
    add<OpF16, 128, false, 2>(kTcF16);
    add<OpF16, 256, false, 2>(kTcF16);
    add<OpF16, 32, true, 2>(kTcF16);
    add<OpF16, 64, true, 2>(kTcF16);
    add<OpF16, 128, true, 2>(kTcF16);
    add<OpI8, 64, false, 2>(kTcI8);
    add<OpI8, 128, false, 2>(kTcI8);
    add<OpI8, 256, false, 2>(kTcI8);
    add<OpI8, 32, true, 2>(kTcI8);
    add<OpI8, 64, true, 2>(kTcI8);
    add<OpI8, 128, true, 2>(kTcI8);
    add<OpI8, 64, false, 4>(kTcI8);
    add<OpI8, 128, false, 4>(kTcI8);
    add<OpI8, 256, false, 4>(kTcI8);
    add<OpI8, 32, true, 4>(kTcI8);
    add<OpI8, 64, true, 4>(kTcI8);
    add<OpI8, 128, true, 4>(kTcI8);
  }
};

Table& table() {
  static Table t;
  return t;
}

int find_entry(int op, int bn, int split, int out_bytes) {
  Table& t = table();
  const int want_split = split > 1 ? 2 : 1;
  for (int i = 0; i < t.n; ++i) {
    const TcEntry& e = t.e[i];
    if (e.op == op && e.bn == bn && e.split == want_split && e.out_bytes == out_bytes) return i;
  }
  return -1;
}

}  // namespace

bool gemm_tc_supported(int op, int bn, int split, int out_bytes) {
  // A split tile's 128 rows are dealt out evenly over the cluster.
  if (split != 1 && split != 2 && split != 4 && split != 8) return false;
  return find_entry(op, bn, split, out_bytes) >= 0;
}

int launch_gemm_tc(int op, int bn, int split, int out_bytes, const void* A, const void* B,
                   void* C, int M, int N, int K, const kern::EpiParams& ep,
                   const DeviceInfo& dev, cudaStream_t stream, int batch,
                   const PeerTargets* peer) {
  if (peer != nullptr && (batch > 1 || split > 1 || out_bytes != 2))
    return CLOVE_ERR_UNSUPPORTED;  // replicated output: plain fp16 tiles only
  if (batch < 1 || (batch > 1 && split > 1))
    return fail(CLOVE_ERR_UNSUPPORTED, "batched tiles need split 1 (batch %d split %d)", batch, split);
  const int ei = find_entry(op, bn, split, out_bytes);
  if (ei < 0)
    return fail(CLOVE_ERR_UNSUPPORTED, "no tensor-core kernel for op=%d bn=%d split=%d out=%d", op,
                bn, split, out_bytes);
  const TcEntry* e = &table().e[ei];
  std::atomic<uint64_t>& attr_set = table().attr_set[ei];
  const int elem = op == kTcF16 ? 2 : 1;
  const CUtensorMapDataType in_dt =
      op == kTcF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapDataType out_dt =
      out_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_INT32;

  CUtensorMap tmA, tmB, tmC;
  int rc;
  // All three as [batch, rows, cols] (batch 1 for a plain GEMM), densely packed.
  const uint64_t ub = static_cast<uint64_t>(batch);
  // A [M,K]: box 128 B of K x 128 rows, 128B swizzle.
  // A box: 128 rows, or M rounded up to 8 (a whole swizzle atom) when M < 128, so
  // that a decode-sized A does not stream 128 rows of zero fill per stage.
  int a_rows = M < 128 ? ((M + 7) / 8) * 8 : 128;
  rc = encode_tmap_3d(&tmA, in_dt, elem, A, K, M, ub, static_cast<uint64_t>(K) * elem,
                      static_cast<uint64_t>(M) * K * elem, e->bk, static_cast<uint32_t>(a_rows),
                      128);
  if (rc) return rc;
  // B [K,N]: box (swizzle width of N) x BK rows.
  rc = encode_tmap_3d(&tmB, in_dt, elem, B, N, K, ub, static_cast<uint64_t>(N) * elem,
                      static_cast<uint64_t>(K) * N * elem, e->b_atom_elems, e->bk, e->b_sw);
  if (rc) return rc;
  // C [M,N]: box CHUNK cols x 32 rows, swizzle = staging row bytes.
  rc = encode_tmap_3d(&tmC, out_dt, out_bytes, C, N, M, ub, static_cast<uint64_t>(N) * out_bytes,
                      static_cast<uint64_t>(M) * N * out_bytes, e->chunk, 32, e->stg_row);
  if (rc) return rc;

  const uint64_t bit = 1ull << (dev.device & 63);
  if ((attr_set.load(std::memory_order_acquire) & bit) == 0) {
    rc = check_cuda(cudaFuncSetAttribute(e->fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         e->smem_bytes),
                    "cudaFuncSetAttribute(max dynamic smem)");
    if (rc) return rc;
    attr_set.fetch_or(bit, std::memory_order_acq_rel);
  }

  const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  EpiParams epv = ep;
  epv.c_out = C;
  epv.peer.count = 0;
  if (peer != nullptr) {
    rc = encode_peer_maps(*peer, M, N, static_cast<uint32_t>(e->chunk), e->stg_row, &epv.peer);
    if (rc) return rc;
  }
  void* args[] = {&tmA, &tmB, &tmC, &M, &N, &K, &batch, &a_rows, &epv};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(e->smem_bytes);
  cfg.stream = stream;
  cfg.attrs = attr;
  if (split > 1) {
    cfg.gridDim = dim3(static_cast<unsigned>(split), static_cast<unsigned>(tiles), 1);
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(split);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  } else {
    const long long all = static_cast<long long>(tiles) * batch;
    const int grid = all < dev.num_sms ? static_cast<int>(all) : dev.num_sms;
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.numAttrs = 1;
  }
  return check_cuda(cudaLaunchKernelExC(&cfg, e->fn, args), "gemm_tc launch");
}

}  // namespace rt
}  // namespace clove

namespace clove {
namespace rt {

// One TMA store map per rank for the replicated output: rank d's C from column 0
// to this rank's last column (col0 + N), rows M, row pitch ldc; the box and swizzle
// of the kernel's own C store.
int encode_peer_maps(const PeerTargets& pt, int M, int N, uint32_t box_cols, int swizzle,
                     kern::PeerOut* out) {
  if (pt.count > kern::kMaxPeers) return fail(CLOVE_ERR_UNSUPPORTED, "too many ranks");
  if (pt.count > 1 && (pt.ready_in == nullptr || pt.epoch == nullptr))
    return fail(CLOVE_ERR_INVALID_ARG, "replicated output without its ready handshake");
  out->count = pt.count;
  out->col0 = pt.col0;
  out->rank = pt.rank;
  out->ldc = pt.ldc;
  out->mc = reinterpret_cast<unsigned long long>(pt.mc);
  out->ready_in = pt.ready_in;
  out->epoch = pt.epoch;
  if (pt.mc != nullptr && ((reinterpret_cast<uintptr_t>(pt.mc) & 15u) != 0 || pt.ldc % 8 != 0 ||
                           pt.col0 % 8 != 0 || N % 8 != 0))
    return fail(CLOVE_ERR_UNSUPPORTED, "multicast output needs 16-byte aligned rows and columns");
  for (int d = 0; d < kern::kMaxPeers; ++d)
    out->ready_slot[d] = d < pt.count ? pt.ready_slot[d] : nullptr;
  for (int d = 0; d < pt.count; ++d) {
    if (d != pt.rank && pt.ready_slot[d] == nullptr)
      return fail(CLOVE_ERR_INVALID_ARG, "replicated output without its ready handshake");
    if (pt.mc != nullptr) continue;  // one multicast store per tile instead of maps
    const int rc = encode_tmap_2d(&out->maps[d], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, pt.dst[d],
                                  static_cast<uint64_t>(pt.col0) + N, M,
                                  static_cast<uint64_t>(pt.ldc) * 2, box_cols, 32, swizzle);
    if (rc) return rc;
  }
  return CLOVE_OK;
}

namespace {
std::atomic<uint64_t> g_tc2_attr[3];
std::atomic<int> g_tc2_clusters[64][3];  // co-resident pairs per device and variant (0: unknown)

// Stream-ordered pool for the stream-K partials, one per device, that keeps its
// memory between calls (the default pool may return it to the driver at every
// synchronisation, and a 40 MB re-map per call would cost more than the schedule
// saves).
std::mutex g_sk_pool_mu;
cudaMemPool_t g_sk_pool[64];

// Stream-K tickets kept between calls, one zeroed array per (device, stream): a
// tile's last contributor resets its ticket, so the array is zero again when the
// kernel completes and no per-call memset is needed (a memset between two kernels
// would also end their programmatic overlap). One array per stream keeps calls on
// different streams apart. After a kernel failure the arrays are cleared
// (reset_stream_k_tickets, from clove_get_device_error).
struct TicketBuf {
  int device;
  cudaStream_t stream;
  int* ptr;
  size_t count;
};
std::mutex g_ticket_mu;
std::vector<TicketBuf> g_tickets;

// The ticket array for (device, stream) with at least `count` entries; nullptr when
// it would have to be created while the stream is being captured.
int stream_tickets(int device, cudaStream_t s, size_t count, bool capturing, int** out) {
  std::lock_guard<std::mutex> lock(g_ticket_mu);
  *out = nullptr;
  for (TicketBuf& t : g_tickets) {
    if (t.device != device || t.stream != s) continue;
    if (t.count >= count) {
      *out = t.ptr;
      return CLOVE_OK;
    }
    if (capturing) return CLOVE_OK;
    // Grow: the old array is released after the work already queued on the stream.
    int* np = nullptr;
    const size_t cap = std::max(count, 2 * t.count);
    int rc = check_cuda(cudaMalloc(&np, cap * sizeof(int)), "cudaMalloc(stream-K tickets)");
    if (!rc) rc = check_cuda(cudaMemsetAsync(np, 0, cap * sizeof(int), s), "cudaMemsetAsync(tickets)");
    if (rc) {
      if (np) cudaFree(np);
      return rc;
    }
    cudaFreeAsync(t.ptr, s);
    t.ptr = np;
    t.count = cap;
    *out = np;
    return CLOVE_OK;
  }
  if (capturing) return CLOVE_OK;
  int* np = nullptr;
  const size_t cap = std::max<size_t>(count, 1024);
  int rc = check_cuda(cudaMalloc(&np, cap * sizeof(int)), "cudaMalloc(stream-K tickets)");
  if (!rc) rc = check_cuda(cudaMemsetAsync(np, 0, cap * sizeof(int), s), "cudaMemsetAsync(tickets)");
  if (rc) {
    if (np) cudaFree(np);
    return rc;
  }
  g_tickets.push_back(TicketBuf{device, s, np, cap});
  *out = np;
  return CLOVE_OK;
}

int sk_pool(int device, cudaMemPool_t* out) {
  std::lock_guard<std::mutex> lock(g_sk_pool_mu);
  if (g_sk_pool[device & 63] == nullptr) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    cudaMemPool_t pool;
    int rc = check_cuda(cudaMemPoolCreate(&pool, &props), "cudaMemPoolCreate(stream-K)");
    if (rc) return rc;
    uint64_t keep = UINT64_MAX;
    rc = check_cuda(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep),
                    "cudaMemPoolSetAttribute(stream-K)");
    if (rc) return rc;
    g_sk_pool[device & 63] = pool;
  }
  *out = g_sk_pool[device & 63];
  return CLOVE_OK;
}

}  // namespace

// Stream-K plan of the CTA-pair kernel for `tiles` output tiles of kb_total K
// blocks on `pairs` co-resident pairs (SkParams). A partial last wave leaves
// (1 - tiles / (waves * pairs)) of the GPU idle for a whole tile; the last partial
// wave's tiles (plus one full wave when the partial wave is under half full, so
// that no tile is cut into more than three pieces) can instead be spread evenly
// over all pairs by K block. That costs a fixed ~10 us per launch (partial slots,
// the tickets' memset, which also ends the programmatic overlap with the previous
// kernel), and under the power cap the idle SMs of a partial wave let the busy
// ones clock higher, which recovers part of the loss anyway; measured on B200,
// the schedule only pays for long K ranges (>= 128 K blocks) with >= 10 % idle:
// FFN down 4096 x 2048 x 11008 146 -> 142 us, 3584 x 2048 x 11008 150 -> 133 us,
// while FFN up 11008 x 2048 x 4096 loses (130 -> 138 us). force: 1 = never, 2 =
// whenever the tile count is not a multiple of the pairs (and every pair gets a K
// block).
SkPlan plan_stream_k(int tiles, int pairs, int kb_total, int force) {
  SkPlan p{tiles, 0, 0, std::min(pairs, std::max(tiles, 1))};
  if (force == 1 || pairs <= 1 || tiles <= 0 || tiles % pairs == 0) return p;
  const long long waves = (tiles + pairs - 1) / pairs;
  const double idle = 1.0 - static_cast<double>(tiles) / static_cast<double>(waves * pairs);
  int sk = tiles % pairs;
  if (tiles > pairs && 2 * sk < pairs) sk += pairs;
  const long long units = static_cast<long long>(sk) * kb_total;
  // Automatic only with at least one full wave (then no piece is under half a
  // tile's K range); forced plans may cut a tile into many pieces (tests).
  if (force != 2 && (tiles < pairs || idle < 0.10 || kb_total < 128)) return p;
  if (units < pairs) return p;  // every pair needs at least one K block
  auto owner = [&](long long v) {
    return static_cast<int>(((v + 1) * pairs + units - 1) / units) - 1;
  };
  int mc = 1;
  for (int t = 0; t < sk; ++t) {
    const long long t0 = static_cast<long long>(t) * kb_total;
    mc = std::max(mc, owner(t0 + kb_total - 1) - owner(t0) + 1);
  }
  p.dp_tiles = tiles - sk;
  p.sk_tiles = sk;
  p.max_contrib = mc;
  p.pairs = pairs;
  return p;
}

// CTA-pair 256 x 256 tile kernel (fp16 C only).
int launch_gemm_tc2(int op, const void* A, const void* B, void* C, int M, int N, int K,
                    const kern::EpiParams& ep, const DeviceInfo& dev, cudaStream_t stream,
                    const void* B2, const PeerTargets* peer, bool allow_stream_k) {
  if (peer != nullptr && B2 != nullptr) return CLOVE_ERR_UNSUPPORTED;
  using SF = kern::Tc2Shape<kern::OpF16>;
  using SI = kern::Tc2Shape<kern::OpI8>;
  const bool f16 = op == kTcF16;
  const bool glu = B2 != nullptr;
  if (glu && !f16) return fail(CLOVE_ERR_UNSUPPORTED, "GLU epilogue is fp16 only");
  const void* fn =
      glu ? reinterpret_cast<const void*>(&kern::gemm_tc2_kernel<kern::OpF16, true>)
          : f16 ? reinterpret_cast<const void*>(&kern::gemm_tc2_kernel<kern::OpF16>)
                : reinterpret_cast<const void*>(&kern::gemm_tc2_kernel<kern::OpI8>);
  const int smem = f16 ? SF::SMEM_BYTES : SI::SMEM_BYTES;
  const int bk = f16 ? SF::BK : SI::BK;
  const int b_atom = f16 ? SF::B_ATOM_ELEMS : SI::B_ATOM_ELEMS;
  const int elem = f16 ? 2 : 1;
  const CUtensorMapDataType in_dt =
      f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap tmA, tmB, tmB2, tmC;
  int rc = encode_tmap_2d(&tmA, in_dt, elem, A, K, M, static_cast<uint64_t>(K) * elem, bk, 128, 128);
  if (rc) return rc;
  rc = encode_tmap_2d(&tmB, in_dt, elem, B, N, K, static_cast<uint64_t>(N) * elem, b_atom, bk, 128);
  if (rc) return rc;
  if (glu) {
    rc = encode_tmap_2d(&tmB2, in_dt, elem, B2, N, K, static_cast<uint64_t>(N) * elem, b_atom, bk,
                        128);
    if (rc) return rc;
  } else {
    tmB2 = tmB;
  }
  rc = encode_tmap_2d(&tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, C, N, M,
                      static_cast<uint64_t>(N) * 2, 64, 32, 128);
  if (rc) return rc;
  const uint64_t bit = 1ull << (dev.device & 63);
  std::atomic<uint64_t>& attr = g_tc2_attr[glu ? 2 : f16 ? 0 : 1];
  if ((attr.load(std::memory_order_acquire) & bit) == 0) {
    rc = check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                    "cudaFuncSetAttribute(tc2 smem)");
    if (rc) return rc;
    attr.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int tile_n = glu ? 128 : 256;
  const int tiles = ((M + 255) / 256) * ((N + tile_n - 1) / tile_n);
  kern::EpiParams epv = ep;
  epv.peer.count = 0;
  if (peer != nullptr) {
    rc = encode_peer_maps(*peer, M, N, 64, 128, &epv.peer);
    if (rc) return rc;
  }
  kern::SkParams skp = {};
  void* args[] = {&tmA, &tmB, &tmB2, &tmC, &M, &N, &K, &epv, &skp};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;

  // Pairs that can be resident at once (clusters must fit in one GPC).
  std::atomic<int>& known = g_tc2_clusters[dev.device & 63][glu ? 2 : f16 ? 0 : 1];
  int resident = known.load(std::memory_order_acquire);
  if (resident == 0) {
    cfg.gridDim = dim3(static_cast<unsigned>(dev.num_sms & ~1), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = dev.num_sms / 2;
    }
    resident = std::min(n, dev.num_sms / 2);
    known.store(resident, std::memory_order_release);
  }
  const int kb_total = (K + bk - 1) / bk;
  const Override ov = get_override();
  const SkPlan plan = plan_stream_k(tiles, resident, kb_total,
                                    (glu || !allow_stream_k) ? 1 : ov.path == 4 ? ov.split : 0);
  skp.dp_tiles = plan.dp_tiles;
  skp.sk_tiles = plan.sk_tiles;
  skp.max_contrib = plan.max_contrib;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * plan.pairs), 1, 1);

  void* ws = nullptr;
  if (plan.sk_tiles > 0) {
    const size_t n_tickets = static_cast<size_t>(plan.sk_tiles) * 2;
    const size_t ticket_bytes = (n_tickets * sizeof(int) + 255) & ~size_t(255);
    const size_t part_bytes = static_cast<size_t>(plan.sk_tiles) * plan.max_contrib * 2 *
                              (256 * 128) * sizeof(uint32_t);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    rc = check_cuda(cudaStreamIsCapturing(stream, &cap), "cudaStreamIsCapturing");
    if (rc) return rc;
    const bool capturing = cap != cudaStreamCaptureStatusNone;
    int* tickets = nullptr;
    rc = stream_tickets(dev.device, stream, n_tickets, capturing, &tickets);
    if (rc) return rc;
    // Partials (and, without a kept ticket array, the tickets) from stream-ordered
    // scratch: a private pool that keeps its memory, or a graph allocation node of
    // the graph's own pool under capture.
    const size_t scratch = part_bytes + (tickets ? 0 : ticket_bytes);
    if (!capturing) {
      cudaMemPool_t pool;
      rc = sk_pool(dev.device, &pool);
      if (rc) return rc;
      rc = check_cuda(cudaMallocFromPoolAsync(&ws, scratch, pool, stream),
                      "cudaMallocFromPoolAsync(stream-K)");
    } else {
      rc = check_cuda(cudaMallocAsync(&ws, scratch, stream), "cudaMallocAsync(stream-K)");
    }
    if (rc) return rc;
    if (tickets != nullptr) {
      skp.tickets = tickets;
      skp.partials = static_cast<uint32_t*>(ws);
    } else {
      skp.tickets = static_cast<int*>(ws);
      skp.partials = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + ticket_bytes);
      rc = check_cuda(cudaMemsetAsync(ws, 0, ticket_bytes, stream), "cudaMemsetAsync(stream-K)");
      if (rc) {
        cudaFreeAsync(ws, stream);
        return rc;
      }
    }
  }
  rc = check_cuda(cudaLaunchKernelExC(&cfg, fn, args), "gemm_tc2 launch");
  if (ws != nullptr) {
    const int rc2 = check_cuda(cudaFreeAsync(ws, stream), "cudaFreeAsync(stream-K)");
    if (rc == CLOVE_OK) rc = rc2;
  }
  return rc;
}

void reset_stream_k_tickets() {
  std::lock_guard<std::mutex> lock(g_ticket_mu);
  for (TicketBuf& t : g_tickets) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return;
    cudaSetDevice(t.device);
    cudaMemset(t.ptr, 0, t.count * sizeof(int));
    cudaDeviceSynchronize();
    cudaSetDevice(cur);
  }
}

}  // namespace rt
}  // namespace clove
