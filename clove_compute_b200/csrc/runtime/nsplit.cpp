// nsplit.cpp -- N-split of the GEMM over the GPUs of one node (one process per GPU).
//
// The reference has no multi-GPU code. The split is the natural one for this
// path: rank r owns a contiguous block of C's columns and the matching columns
// of B (rows of B_q for the K-packed INT4 layout); A is replicated. Each rank runs
// the single-GPU kernel on its shard with no communication. Only when the caller
// asks for a replicated C do the ranks exchange data: one ncclAllGather of the
// (padded) C shards into a stream-ordered staging buffer, then a re-layout kernel
// scatters the column blocks into row-major C [M,N].
//
// A replicated C registered with clove_nsplit_register_output (every rank's C
// mapped into every rank through CUDA IPC) skips the collective altogether: the
// fp16 GEMM's epilogue stores each finished tile into all ranks' C over NVLink
// while the remaining tiles compute, and a one-warp kernel then exchanges
// completion flags (system-scope release / acquire on IPC-mapped flag arrays).
//
// NCCL is opened with dlopen on first use so that loading this library never pins
// an NCCL build into the process (PyTorch ships its own; whichever libnccl.so.2 is
// already loaded is reused). The communicator is non-blocking: creation, every
// collective call and finalisation are polled with ncclCommGetAsyncError under a
// deadline, so a rank that never joins ends the others' call with
// CLOVE_ERR_TIMEOUT (communicator aborted) instead of a hang.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <string>
#include <vector>

#include "internal.h"
#include "../kernels/params.h"

namespace clove {
namespace kern {
struct PeerSync;
}  // namespace kern
namespace rt {
int launch_relayout_columns(const void* staging, void* C, int M, int N, int P, int Nmax,
                            int elem_bytes, cudaStream_t stream);
int launch_peer_signal_wait(int nranks, int rank, unsigned long long* epoch,
                            unsigned long long* const* flags, unsigned long long timeout_ns,
                            cudaStream_t stream);
int gemm_fp16_replicated(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                         const PeerTargets& peer, cudaStream_t s);
int gemm_int4_replicated(const uint8_t* Aq, const void* As, const void* Az, const uint8_t* Bq,
                         const void* Bs, const void* Bz, void* C, int M, int N, int K,
                         const PeerTargets& peer, cudaStream_t s);
int gemm_int8_rowcol_replicated(const int8_t* A, const int8_t* B, void* C, int M, int N, int K,
                                const float* rs, const float* cs, const PeerTargets& peer,
                                cudaStream_t s);
}  // namespace rt
}  // namespace clove

using namespace clove::rt;
using clove::kern::kMaxPeers;

namespace {
// Layout of each rank's IPC-shared flag array (unsigned long long words):
//   [0, kMaxPeers)            done[q]: rank q has finished storing call e into this
//                             rank's C (written by q's completion-signal kernel)
//   [kMaxPeers, 2 kMaxPeers)  ready[q]: rank q's stream has reached call e, so q's
//                             readers of its C from call e-1 have completed
//                             (written at the start of q's GEMM, kern::PeerOut)
//   [2 kMaxPeers]             this rank's count of completed replicated calls
constexpr int kFlagDone = 0;
constexpr int kFlagReady = kMaxPeers;
constexpr int kFlagEpoch = 2 * kMaxPeers;
constexpr size_t kFlagBytes = sizeof(unsigned long long) * (2 * kMaxPeers + 1);

// One IPC-shared buffer: this rank's pointer and every rank's, mapped here.
struct SharedBuf {
  void* local = nullptr;
  size_t bytes = 0;
  void* mc = nullptr;            // multicast address of every rank's buffer (else null)
  void* opened[kMaxPeers] = {};  // IPC mapping bases (to close), null for this rank
  void* ptr[kMaxPeers] = {};     // every rank's buffer as seen from this process
};
}  // namespace

// One IPC mapping of a peer allocation. Several shared buffers can live in one
// allocation (tensors of one caching-allocator segment), and a handle can be
// opened only once per process, so mappings are shared and counted.
struct IpcMapping {
  int rank;
  cudaIpcMemHandle_t handle;
  void* base;
  int refs;
};

struct clove_nsplit_ctx {
  ncclComm_t comm = nullptr;
  int rank;
  int nranks;
  int device;
  std::vector<SharedBuf> outputs;  // registered replicated outputs
  SharedBuf flags;                 // FlagLayout: done and ready slots + this rank's epoch
  void* flags_mem = nullptr;       // this rank's flag array (cudaMalloc)
  bool flags_ready = false;        // every rank's flag array is mapped here
  bool ipc_used = false;           // a registration was attempted (same on every rank)
  std::vector<IpcMapping> mappings;
};

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  std::string error;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

void load_nccl() {
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char* n : names) {
    g_nccl.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (g_nccl.handle) break;
  }
  if (!g_nccl.handle) {
    g_nccl.error = dlerror() ? dlerror() : "dlopen(libnccl.so.2) failed";
    return;
  }
#define CLOVE_SYM(field, name) \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(g_nccl.handle, name))
  CLOVE_SYM(GetUniqueId, "ncclGetUniqueId");
  CLOVE_SYM(CommInitRank, "ncclCommInitRank");
  CLOVE_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
  CLOVE_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  CLOVE_SYM(CommFinalize, "ncclCommFinalize");
  CLOVE_SYM(CommDestroy, "ncclCommDestroy");
  CLOVE_SYM(CommAbort, "ncclCommAbort");
  CLOVE_SYM(AllGather, "ncclAllGather");
  CLOVE_SYM(GetErrorString, "ncclGetErrorString");
#undef CLOVE_SYM
  if (!g_nccl.GetUniqueId || !g_nccl.CommInitRank || !g_nccl.CommDestroy || !g_nccl.AllGather ||
      !g_nccl.GetErrorString || !g_nccl.CommAbort || !g_nccl.CommInitRankConfig ||
      !g_nccl.CommGetAsyncError || !g_nccl.CommFinalize) {
    g_nccl.error = "libnccl is missing required symbols";
    g_nccl.handle = nullptr;
  }
}

int nccl_ready() {
  std::call_once(g_nccl_once, load_nccl);
  if (!g_nccl.handle) return fail(CLOVE_ERR_NCCL, "NCCL unavailable: %s", g_nccl.error.c_str());
  return CLOVE_OK;
}

int check_nccl(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return CLOVE_OK;
  return fail(CLOVE_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString(r));
}

// The communicator is non-blocking: a call may return ncclInProgress, and is done
// (initialised, or the collective enqueued) once ncclCommGetAsyncError reports
// anything else. Polls every 200 us up to the deadline; past it the communicator
// is aborted (so no rank is left waiting on it) and the call fails with
// CLOVE_ERR_TIMEOUT.
int settle_nccl(ncclComm_t comm, ncclResult_t r, const char* what, double deadline_s,
                bool* aborted = nullptr) {
  if (r != ncclInProgress) return check_nccl(r, what);
  const auto t0 = std::chrono::steady_clock::now();
  for (long polls = 0;; ++polls) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = g_nccl.CommGetAsyncError(comm, &st);
    if (q != ncclSuccess) return check_nccl(q, "ncclCommGetAsyncError");
    if (st != ncclInProgress) return check_nccl(st, what);
    const double el =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > deadline_s) {
      g_nccl.CommAbort(comm);
      if (aborted) *aborted = true;
      return fail(CLOVE_ERR_TIMEOUT, "%s: not done after %.0f s (a rank missing?); communicator aborted",
                  what, deadline_s);
    }
    // An enqueue finishes within microseconds: poll without sleeping for the first
    // millisecond (a fixed sleep here left the GPU idle between back-to-back calls),
    // then back off so that a long wait (communicator creation) does not spin a core.
    if (el < 1e-3)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(el < 0.1 ? 20 : 200));
  }
}

// Deadlines of the non-blocking communicator: creation waits for every rank to
// join; a collective call only has to be enqueued.
constexpr double kNcclInitDeadlineS = 120.0;
constexpr double kNcclCallDeadlineS = 30.0;

int shard_cols(int N, int P, int r) {
  return clove_nsplit_col_begin(N, P, r + 1) - clove_nsplit_col_begin(N, P, r);
}

// All-gathers the [M, N_r] shard of every rank into row-major C_full [M, N].
int gather_columns(clove_nsplit_ctx* ctx, const void* C_shard, void* C_full, int M, int N,
                   int elem_bytes, cudaStream_t s) {
  const int P = ctx->nranks;
  const int Nmax = (N + P - 1) / P;
  const int Nr = shard_cols(N, P, ctx->rank);
  const size_t slot = static_cast<size_t>(M) * Nmax * elem_bytes;
  void* staging = nullptr;
  int rc = check_cuda(cudaMallocAsync(&staging, slot * (P + 1), s), "cudaMallocAsync(staging)");
  if (rc) return rc;
  const void* send = C_shard;
  if (Nr != Nmax) {
    // Pad this rank's shard to the common slot width (zeros are never read back).
    char* pad = static_cast<char*>(staging) + slot * P;
    rc = check_cuda(cudaMemsetAsync(pad, 0, slot, s), "cudaMemsetAsync(pad)");
    if (!rc && Nr > 0)
      rc = check_cuda(cudaMemcpy2DAsync(pad, static_cast<size_t>(Nmax) * elem_bytes, C_shard,
                                        static_cast<size_t>(Nr) * elem_bytes,
                                        static_cast<size_t>(Nr) * elem_bytes, M,
                                        cudaMemcpyDeviceToDevice, s),
                      "cudaMemcpy2DAsync(pad)");
    send = pad;
  }
  if (!rc)
    rc = settle_nccl(ctx->comm, g_nccl.AllGather(send, staging, slot / 2, ncclHalf, ctx->comm, s),
                     "ncclAllGather", kNcclCallDeadlineS);
  if (!rc) rc = launch_relayout_columns(staging, C_full, M, N, P, Nmax, elem_bytes, s);
  const int rc2 = check_cuda(cudaFreeAsync(staging, s), "cudaFreeAsync(staging)");
  return rc ? rc : rc2;
}

// ---- CUDA IPC sharing of device buffers among the ranks ------------------------

typedef CUresult (*PfnMemGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);
PfnMemGetAddressRange g_get_range = nullptr;
std::once_flag g_range_once;

struct IpcRecord {
  cudaIpcMemHandle_t handle;
  unsigned long long offset;  // of the shared pointer inside its allocation
  unsigned long long bytes;
};

int open_mapping(clove_nsplit_ctx* ctx, int q, const cudaIpcMemHandle_t& h, void** base) {
  for (IpcMapping& m : ctx->mappings) {
    if (m.rank == q && memcmp(&m.handle, &h, sizeof(h)) == 0) {
      ++m.refs;
      *base = m.base;
      return CLOVE_OK;
    }
  }
  void* b = nullptr;
  const int rc = check_cuda(cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess),
                            "cudaIpcOpenMemHandle");
  if (rc) return rc;
  ctx->mappings.push_back(IpcMapping{q, h, b, 1});
  *base = b;
  return CLOVE_OK;
}

void close_shared(clove_nsplit_ctx* ctx, SharedBuf* sb) {
  for (int q = 0; q < kMaxPeers; ++q) {
    if (sb->opened[q] == nullptr) continue;
    for (size_t i = 0; i < ctx->mappings.size(); ++i) {
      IpcMapping& m = ctx->mappings[i];
      if (m.rank == q && m.base == sb->opened[q]) {
        if (--m.refs == 0) {
          cudaIpcCloseMemHandle(m.base);
          ctx->mappings.erase(ctx->mappings.begin() + static_cast<long>(i));
        }
        break;
      }
    }
  }
  *sb = SharedBuf();
}

// The IPC record of a device pointer (any offset inside a cudaMalloc allocation,
// such as a PyTorch tensor). Local only.
int make_record(void* local, size_t bytes, IpcRecord* rec) {
  std::call_once(g_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_get_range = reinterpret_cast<PfnMemGetAddressRange>(fn);
  });
  *rec = IpcRecord();
  CUdeviceptr base = 0;
  size_t range = 0;
  if (g_get_range == nullptr) return fail(CLOVE_ERR_CUDA, "cuMemGetAddressRange unavailable");
  if (g_get_range(&base, &range, reinterpret_cast<CUdeviceptr>(local)) != CUDA_SUCCESS)
    return fail(CLOVE_ERR_INVALID_ARG, "shared buffer is not device memory of this process");
  if (reinterpret_cast<CUdeviceptr>(local) - base + bytes > range)
    return fail(CLOVE_ERR_INVALID_ARG, "shared buffer runs past its allocation");
  const int rc = check_cuda(cudaIpcGetMemHandle(&rec->handle, reinterpret_cast<void*>(base)),
                            "cudaIpcGetMemHandle (buffer must come from cudaMalloc)");
  if (rc) return rc;
  rec->offset = reinterpret_cast<CUdeviceptr>(local) - base;
  rec->bytes = bytes;
  return CLOVE_OK;
}

// Collective: all-gathers `n` bytes from every rank into all[P * n] (host memory)
// through NCCL on a private stream.
int all_gather_host(clove_nsplit_ctx* ctx, const void* mine, size_t n, void* all) {
  const int P = ctx->nranks;
  cudaStream_t s = nullptr;
  int rc = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  if (rc) return rc;
  void* dbuf = nullptr;
  rc = check_cuda(cudaMalloc(&dbuf, n * (P + 1)), "cudaMalloc(all-gather)");
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(static_cast<char*>(dbuf) + n * P, mine, n,
                                    cudaMemcpyHostToDevice, s),
                    "cudaMemcpyAsync(all-gather in)");
  if (!rc)
    rc = settle_nccl(ctx->comm,
                     g_nccl.AllGather(static_cast<char*>(dbuf) + n * P, dbuf, n, ncclChar,
                                      ctx->comm, s),
                     "ncclAllGather(host records)", kNcclCallDeadlineS);
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(all, dbuf, n * P, cudaMemcpyDeviceToHost, s),
                    "cudaMemcpyAsync(all-gather out)");
  if (!rc) rc = check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(all-gather)");
  if (dbuf) cudaFree(dbuf);
  cudaStreamDestroy(s);
  return rc;
}

// Collective: true on every rank iff every rank passed ok. A failed exchange
// counts as not ok.
bool all_ok(clove_nsplit_ctx* ctx, bool ok) {
  int mine = ok ? 1 : 0;
  std::vector<int> all(ctx->nranks, 0);
  if (all_gather_host(ctx, &mine, sizeof(int), all.data()) != CLOVE_OK) return false;
  for (int v : all)
    if (v != 1) return false;
  return true;
}

// Maps every other rank's buffer of the all-gathered records into this process.
int open_shared(clove_nsplit_ctx* ctx, void* local, size_t bytes, const IpcRecord* all,
                SharedBuf* out) {
  SharedBuf sb;
  sb.local = local;
  sb.bytes = bytes;
  int rc = CLOVE_OK;
  for (int q = 0; q < ctx->nranks && !rc; ++q) {
    if (q == ctx->rank) {
      sb.ptr[q] = local;
      continue;
    }
    void* b = nullptr;
    rc = open_mapping(ctx, q, all[q].handle, &b);
    if (!rc) {
      sb.opened[q] = b;
      sb.ptr[q] = static_cast<char*>(b) + all[q].offset;
    }
  }
  if (rc) {
    close_shared(ctx, &sb);
    return rc;
  }
  *out = sb;
  return CLOVE_OK;
}

// Collective barrier on the communicator (one tiny all-gather, host-synchronous).
int host_barrier(clove_nsplit_ctx* ctx) {
  int mine = 0;
  std::vector<int> all(ctx->nranks);
  return all_gather_host(ctx, &mine, sizeof(int), all.data());
}

const SharedBuf* find_output(const clove_nsplit_ctx* ctx, const void* C_full) {
  for (const SharedBuf& b : ctx->outputs)
    if (b.local == C_full) return &b;
  return nullptr;
}

// The replicated-output targets of this rank: every rank's C and the ready
// handshake's flag words.
PeerTargets peer_targets(const clove_nsplit_ctx* ctx, const SharedBuf& out, int N) {
  PeerTargets peer = {};
  peer.count = ctx->nranks;
  peer.ldc = N;
  peer.col0 = clove_nsplit_col_begin(N, ctx->nranks, ctx->rank);
  peer.rank = ctx->rank;
  peer.mc = out.mc;
  unsigned long long* own = static_cast<unsigned long long*>(ctx->flags.local);
  peer.ready_in = own + kFlagReady;
  peer.epoch = own + kFlagEpoch;
  for (int q = 0; q < ctx->nranks; ++q) {
    peer.dst[q] = out.ptr[q];
    peer.ready_slot[q] = static_cast<unsigned long long*>(ctx->flags.ptr[q]) + kFlagReady + ctx->rank;
  }
  return peer;
}

// The completion signal that follows a replicated-output GEMM on the stream.
int signal_done(const clove_nsplit_ctx* ctx, cudaStream_t s) {
  unsigned long long* fl[kMaxPeers] = {};
  for (int q = 0; q < ctx->nranks; ++q)
    fl[q] = static_cast<unsigned long long*>(ctx->flags.ptr[q]) + kFlagDone;
  unsigned long long* epoch = static_cast<unsigned long long*>(ctx->flags.local) + kFlagEpoch;
  return launch_peer_signal_wait(ctx->nranks, ctx->rank, epoch, fl, 0, s);
}

// Replicated fp16 output without a collective (see the file comment). Returns
// CLOVE_ERR_UNSUPPORTED, with nothing launched, when the shapes or the kernel the
// dispatch picks cannot store into the replicated C directly; the caller then
// falls back to the all-gather.
//
// Every rank must take the same route (a rank on the all-gather would wait in NCCL
// for ranks that never join). The route therefore depends only on (M, N, K, P):
// equal shards whose width and offsets are multiples of 8 (N % 8P == 0); the tile
// plan for the shard [M, N/P] is the same on every rank; and operand alignment,
// which could differ between ranks, is an error here rather than a fallback.
int gemm_fp16_to_peers(clove_nsplit_ctx* ctx, const SharedBuf& out, const void* A,
                       const void* B_shard, void* C_shard, int M, int N, int K, float alpha,
                       cudaStream_t s) {
  const int P = ctx->nranks;
  if (P > kMaxPeers || N % (8 * P) != 0 || M <= 0 || K % 8 != 0 ||
      out.bytes < static_cast<size_t>(M) * N * 2)
    return CLOVE_ERR_UNSUPPORTED;
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(A) || !a16(B_shard) || !a16(C_shard))
    return fail(CLOVE_ERR_INVALID_ARG, "replicated output needs 16-byte aligned A, B_shard, C_shard");
  const PeerTargets peer = peer_targets(ctx, out, N);
  const int rc = gemm_fp16_replicated(A, B_shard, C_shard, M, N / P, K, alpha, peer, s);
  return rc ? rc : signal_done(ctx, s);
}

// INT4 (config 5's sharded weights): the same route through the INT4 tensor-core
// kernel's epilogue. Rank-independent conditions keep every rank on the tile
// kernel: equal shards (N % 8P == 0) wider than the decode GEMV's 8 columns, M > 8,
// K % 128 == 0, 16-byte aligned operands.
int gemm_int4_to_peers(clove_nsplit_ctx* ctx, const SharedBuf& out, const uint8_t* A_q,
                       const void* A_scale, const void* A_zero, const uint8_t* B_q,
                       const void* B_scale, const void* B_zero, void* C_shard, int M, int N,
                       int K, cudaStream_t s) {
  const int P = ctx->nranks;
  if (P > kMaxPeers || N % (8 * P) != 0 || N / P <= 8 || M <= 8 || K % 128 != 0 ||
      out.bytes < static_cast<size_t>(M) * N * 2)
    return CLOVE_ERR_UNSUPPORTED;
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(A_q) || !a16(A_scale) || !a16(A_zero) || !a16(B_q) || !a16(B_scale) ||
      !a16(B_zero) || !a16(C_shard))
    return fail(CLOVE_ERR_INVALID_ARG, "replicated output needs 16-byte aligned operands");
  const PeerTargets peer = peer_targets(ctx, out, N);
  const int rc = gemm_int4_replicated(A_q, A_scale, A_zero, B_q, B_scale, B_zero, C_shard, M,
                                      N / P, K, peer, s);
  return rc ? rc : signal_done(ctx, s);
}

// INT8 with per-row / per-column scales: the tile kernels' epilogue again. The
// tile kernels need N_r % 16 == 0 (N % 16P == 0), N_r > 8 keeps the GEMV away;
// a split-K plan (the same on every rank) declines and all ranks gather instead.
int gemm_int8_to_peers(clove_nsplit_ctx* ctx, const SharedBuf& out, const int8_t* A_q,
                       const int8_t* B_q, const float* rs, const float* cs, void* C_shard, int M,
                       int N, int K, cudaStream_t s) {
  const int P = ctx->nranks;
  if (P > kMaxPeers || N % (16 * P) != 0 || N / P <= 8 || K % 16 != 0 || M <= 0 ||
      out.bytes < static_cast<size_t>(M) * N * 2)
    return CLOVE_ERR_UNSUPPORTED;
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(A_q) || !a16(B_q) || !a16(C_shard))
    return fail(CLOVE_ERR_INVALID_ARG, "replicated output needs 16-byte aligned operands");
  const PeerTargets peer = peer_targets(ctx, out, N);
  const int rc = gemm_int8_rowcol_replicated(A_q, B_q, C_shard, M, N / P, K, rs, cs, peer, s);
  return rc ? rc : signal_done(ctx, s);
}

}  // namespace

extern "C" {

// Registration and its undoing are collective, and each takes the same collective
// steps on every rank whatever happens locally: local failures travel in the
// exchanged status instead of returning early (a rank that skipped a collective
// would leave the others waiting in NCCL), and a registration counts only if
// every rank mapped everything, so all ranks agree on which outputs take the
// epilogue route.
int clove_nsplit_register_output(clove_nsplit_ctx* ctx, void* C_full, size_t bytes) {
  if (ctx == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "ctx is NULL");
  ctx->ipc_used = true;
  const size_t fb = kFlagBytes;
  int lrc = CLOVE_OK;
  if (C_full == nullptr || bytes == 0)
    lrc = fail(CLOVE_ERR_INVALID_ARG, "bad register_output arguments");
  else if (ctx->nranks > kMaxPeers)
    lrc = fail(CLOVE_ERR_UNSUPPORTED, "replicated output supports up to %d ranks", kMaxPeers);
  else if ((reinterpret_cast<uintptr_t>(C_full) & 15u) != 0)
    lrc = fail(CLOVE_ERR_INVALID_ARG, "replicated C must be 16-byte aligned");
  else if (find_output(ctx, C_full) != nullptr)
    lrc = fail(CLOVE_ERR_INVALID_ARG, "buffer already registered");
  if (!lrc && ctx->flags_mem == nullptr) {
    // Done and ready slots, then this rank's epoch, zeroed before anyone signals.
    void* f = nullptr;
    lrc = check_cuda(cudaMalloc(&f, fb), "cudaMalloc(flags)");
    if (!lrc) lrc = check_cuda(cudaMemset(f, 0, fb), "cudaMemset(flags)");
    if (!lrc) lrc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(flags)");
    if (!lrc)
      ctx->flags_mem = f;
    else if (f)
      cudaFree(f);
  }
  struct Entry {
    IpcRecord flags, out;
    int status;
  } mine = {};
  if (!lrc) lrc = make_record(ctx->flags_mem, fb, &mine.flags);
  if (!lrc) lrc = make_record(C_full, bytes, &mine.out);
  mine.status = lrc == CLOVE_OK ? 1 : 0;
  std::vector<Entry> all(ctx->nranks);
  int rc = all_gather_host(ctx, &mine, sizeof(Entry), all.data());
  if (rc) return rc;
  bool ok = true;
  for (const Entry& e : all) ok = ok && e.status == 1 && e.out.bytes == bytes;
  if (!ok) return lrc ? lrc : fail(CLOVE_ERR_INVALID_ARG, "another rank could not register");
  SharedBuf flags, out;
  std::vector<IpcRecord> fr(ctx->nranks), orr(ctx->nranks);
  for (int q = 0; q < ctx->nranks; ++q) {
    fr[q] = all[q].flags;
    orr[q] = all[q].out;
  }
  int orc = CLOVE_OK;
  if (!ctx->flags_ready) orc = open_shared(ctx, ctx->flags_mem, fb, fr.data(), &flags);
  if (!orc) orc = open_shared(ctx, C_full, bytes, orr.data(), &out);
  if (!all_ok(ctx, orc == CLOVE_OK)) {
    if (flags.local != nullptr) close_shared(ctx, &flags);
    if (out.local != nullptr) close_shared(ctx, &out);
    return orc ? orc : fail(CLOVE_ERR_CUDA, "another rank could not map the shared buffers");
  }
  if (!ctx->flags_ready) {
    ctx->flags = flags;
    ctx->flags_ready = true;
  }
  ctx->outputs.push_back(out);
  return CLOVE_OK;
}

// The same collective for a C_full that the caller has bound, on every rank, to one
// NVLink multicast object (e.g. symmetric memory with a multicast mapping): mc is
// that object's address for this rank's C_full. No IPC mapping of C_full is made;
// the handshake flags are shared as for clove_nsplit_register_output.
int clove_nsplit_register_output_multicast(clove_nsplit_ctx* ctx, void* C_full, void* mc,
                                           size_t bytes) {
  if (ctx == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "ctx is NULL");
  ctx->ipc_used = true;
  const size_t fb = kFlagBytes;
  int lrc = CLOVE_OK;
  if (C_full == nullptr || mc == nullptr || bytes == 0)
    lrc = fail(CLOVE_ERR_INVALID_ARG, "bad register_output_multicast arguments");
  else if (ctx->nranks > kMaxPeers)
    lrc = fail(CLOVE_ERR_UNSUPPORTED, "replicated output supports up to %d ranks", kMaxPeers);
  else if (((reinterpret_cast<uintptr_t>(C_full) | reinterpret_cast<uintptr_t>(mc)) & 15u) != 0)
    lrc = fail(CLOVE_ERR_INVALID_ARG, "replicated C and its multicast address must be 16-byte aligned");
  else if (find_output(ctx, C_full) != nullptr)
    lrc = fail(CLOVE_ERR_INVALID_ARG, "buffer already registered");
  if (!lrc && ctx->flags_mem == nullptr) {
    void* f = nullptr;
    lrc = check_cuda(cudaMalloc(&f, fb), "cudaMalloc(flags)");
    if (!lrc) lrc = check_cuda(cudaMemset(f, 0, fb), "cudaMemset(flags)");
    if (!lrc) lrc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(flags)");
    if (!lrc)
      ctx->flags_mem = f;
    else if (f)
      cudaFree(f);
  }
  struct Entry {
    IpcRecord flags;
    unsigned long long bytes;
    int status;
  } mine = {};
  if (!lrc) lrc = make_record(ctx->flags_mem, fb, &mine.flags);
  mine.bytes = bytes;
  mine.status = lrc == CLOVE_OK ? 1 : 0;
  std::vector<Entry> all(ctx->nranks);
  int rc = all_gather_host(ctx, &mine, sizeof(Entry), all.data());
  if (rc) return rc;
  bool ok = true;
  for (const Entry& e : all) ok = ok && e.status == 1 && e.bytes == bytes;
  if (!ok) return lrc ? lrc : fail(CLOVE_ERR_INVALID_ARG, "another rank could not register");
  SharedBuf flags;
  std::vector<IpcRecord> fr(ctx->nranks);
  for (int q = 0; q < ctx->nranks; ++q) fr[q] = all[q].flags;
  int orc = CLOVE_OK;
  if (!ctx->flags_ready) orc = open_shared(ctx, ctx->flags_mem, fb, fr.data(), &flags);
  if (!all_ok(ctx, orc == CLOVE_OK)) {
    if (flags.local != nullptr) close_shared(ctx, &flags);
    return orc ? orc : fail(CLOVE_ERR_CUDA, "another rank could not map the shared buffers");
  }
  if (!ctx->flags_ready) {
    ctx->flags = flags;
    ctx->flags_ready = true;
  }
  SharedBuf out;
  out.local = C_full;
  out.bytes = bytes;
  out.mc = mc;
  for (int q = 0; q < ctx->nranks; ++q) out.ptr[q] = q == ctx->rank ? C_full : nullptr;
  ctx->outputs.push_back(out);
  return CLOVE_OK;
}

int clove_nsplit_unregister_output(clove_nsplit_ctx* ctx, void* C_full) {
  if (ctx == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "ctx is NULL");
  long idx = -1;
  for (size_t i = 0; i < ctx->outputs.size(); ++i)
    if (ctx->outputs[i].local == C_full) idx = static_cast<long>(i);
  if (!all_ok(ctx, idx >= 0))
    return idx < 0 ? fail(CLOVE_ERR_INVALID_ARG, "buffer is not registered")
                   : fail(CLOVE_ERR_INVALID_ARG, "buffer is not registered on another rank");
  int rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(unregister)");
  close_shared(ctx, &ctx->outputs[static_cast<size_t>(idx)]);
  ctx->outputs.erase(ctx->outputs.begin() + idx);
  // No rank frees its buffer while another still has it mapped.
  const int rc2 = host_barrier(ctx);
  return rc ? rc : rc2;
}

int clove_debug_peer_wait_timeout(unsigned long long* words, unsigned long long timeout_ns,
                                  void* stream) {
  if (words == nullptr || (reinterpret_cast<uintptr_t>(words) & 7u) != 0 || timeout_ns == 0 ||
      timeout_ns > 2000000000ull)
    return fail(CLOVE_ERR_INVALID_ARG, "bad peer-wait test arguments");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemsetAsync(words, 0, 8 * sizeof(unsigned long long), s),
                      "cudaMemsetAsync(peer-wait test)");
  if (rc) return rc;
  // Rank 0 of a two-rank group whose second rank never signals: words[0] is the
  // epoch, words[1..2] rank 0's flag array, words[3..4] the absent rank's.
  unsigned long long* fl[kMaxPeers] = {words + 1, words + 3};
  return launch_peer_signal_wait(2, 0, words, fl, timeout_ns, s);
}

int clove_nsplit_col_begin(int N, int nranks, int rank) {
  if (nranks <= 0) return 0;
  if (rank >= nranks) return N;
  const int base = N / nranks, extra = N % nranks;
  return rank * base + (rank < extra ? rank : extra);
}

int clove_nsplit_get_unique_id(uint8_t id_out[128]) {
  if (id_out == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "id_out is NULL");
  int rc = nccl_ready();
  if (rc) return rc;
  ncclUniqueId id;
  rc = check_nccl(g_nccl.GetUniqueId(&id), "ncclGetUniqueId");
  if (rc) return rc;
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
  memcpy(id_out, &id, sizeof(id));
  return CLOVE_OK;
}

int clove_nsplit_init(clove_nsplit_ctx** ctx, int nranks, int rank, const uint8_t id[128]) {
  if (ctx == nullptr || id == nullptr || nranks <= 0 || rank < 0 || rank >= nranks)
    return fail(CLOVE_ERR_INVALID_ARG, "bad nsplit_init arguments");
  int rc = nccl_ready();
  if (rc) return rc;
  clove_nsplit_ctx* c = new clove_nsplit_ctx();
  c->rank = rank;
  c->nranks = nranks;
  rc = check_cuda(cudaGetDevice(&c->device), "cudaGetDevice");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  // Non-blocking creation, polled under a deadline: a rank that never joins turns
  // into CLOVE_ERR_TIMEOUT on the others instead of a hang.
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  bool aborted = false;
  if (!rc)
    rc = settle_nccl(c->comm, g_nccl.CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg),
                     "ncclCommInitRankConfig", kNcclInitDeadlineS, &aborted);
  if (rc) {
    if (c->comm != nullptr && !aborted) g_nccl.CommAbort(c->comm);
    delete c;
    return rc;
  }
  *ctx = c;
  return CLOVE_OK;
}

int clove_nsplit_destroy(clove_nsplit_ctx* ctx) {
  if (ctx == nullptr) return CLOVE_OK;
  int rc = CLOVE_OK;
  if (ctx->ipc_used) {  // the same on every rank, so all take the barrier below
    rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(destroy)");
    for (SharedBuf& b : ctx->outputs) close_shared(ctx, &b);
    ctx->outputs.clear();
    if (ctx->flags_ready) close_shared(ctx, &ctx->flags);
    ctx->flags_ready = false;
    const int rc2 = host_barrier(ctx);  // peers unmapped our buffers before they are freed
    if (ctx->flags_mem) cudaFree(ctx->flags_mem);
    ctx->flags_mem = nullptr;
    if (!rc) rc = rc2;
  }
  if (g_nccl.handle && ctx->comm != nullptr) {
    // Finalize (non-blocking: polled under the deadline, aborted past it), then free.
    bool aborted = false;
    const int rc3 = settle_nccl(ctx->comm, g_nccl.CommFinalize(ctx->comm), "ncclCommFinalize",
                                kNcclInitDeadlineS, &aborted);
    if (!rc) rc = rc3;
    if (!aborted) {
      const int rc4 = check_nccl(g_nccl.CommDestroy(ctx->comm), "ncclCommDestroy");
      if (!rc) rc = rc4;
    }
  }
  delete ctx;
  return rc;
}

int clove_nsplit_rank(const clove_nsplit_ctx* ctx, int* rank, int* nranks) {
  if (ctx == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "ctx is NULL");
  if (rank) *rank = ctx->rank;
  if (nranks) *nranks = ctx->nranks;
  return CLOVE_OK;
}

int clove_nsplit_gemm_fp16(clove_nsplit_ctx* ctx, const void* A, const void* B_shard,
                           void* C_shard, void* C_full, int M, int N, int K, float alpha,
                           int replicate_C, void* stream) {
  if (ctx == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "ctx is NULL");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int Nr = shard_cols(N, ctx->nranks, ctx->rank);
  if (replicate_C && C_full != nullptr && K > 0) {
    if (const SharedBuf* out = find_output(ctx, C_full)) {
      const int rc = gemm_fp16_to_peers(ctx, *out, A, B_shard, C_shard, M, N, K, alpha, s);
      if (rc != CLOVE_ERR_UNSUPPORTED) return rc;
    }
  }
  int rc = Nr > 0 ? clove_gemm_fp16(A, B_shard, C_shard, M, Nr, K, alpha, 0.f, stream) : CLOVE_OK;
  if (rc || !replicate_C) return rc;
  if (C_full == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "C_full is NULL with replicate_C");
  return gather_columns(ctx, C_shard, C_full, M, N, 2, s);
}

int clove_nsplit_gemm_int4(clove_nsplit_ctx* ctx, const uint8_t* A_q, const void* A_scale,
                           const void* A_zero, const uint8_t* B_q_shard, const void* B_scale_shard,
                           const void* B_zero_shard, void* C_shard, void* C_full, int M, int N,
                           int K, int replicate_C, void* stream) {
  if (ctx == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "ctx is NULL");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int Nr = shard_cols(N, ctx->nranks, ctx->rank);
  if (replicate_C && C_full != nullptr && K > 0) {
    if (const SharedBuf* out = find_output(ctx, C_full)) {
      const int rc = gemm_int4_to_peers(ctx, *out, A_q, A_scale, A_zero, B_q_shard, B_scale_shard,
                                        B_zero_shard, C_shard, M, N, K, s);
      if (rc != CLOVE_ERR_UNSUPPORTED) return rc;
    }
  }
  int rc = Nr > 0 ? clove_gemm_int4(A_q, A_scale, A_zero, B_q_shard, B_scale_shard, B_zero_shard,
                                    C_shard, M, Nr, K, stream)
                  : CLOVE_OK;
  if (rc || !replicate_C) return rc;
  if (C_full == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "C_full is NULL with replicate_C");
  return gather_columns(ctx, C_shard, C_full, M, N, 2, s);
}

int clove_nsplit_gemm_int8_rowcol(clove_nsplit_ctx* ctx, const int8_t* A_q, const int8_t* B_q_shard,
                                  const float* A_row_scale, const float* B_col_scale_shard,
                                  void* C_shard, void* C_full, int M, int N, int K,
                                  int replicate_C, void* stream) {
  if (ctx == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "ctx is NULL");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int Nr = shard_cols(N, ctx->nranks, ctx->rank);
  if (replicate_C && C_full != nullptr && K > 0) {
    if (const SharedBuf* out = find_output(ctx, C_full)) {
      const int rc = gemm_int8_to_peers(ctx, *out, A_q, B_q_shard, A_row_scale,
                                        B_col_scale_shard, C_shard, M, N, K, s);
      if (rc != CLOVE_ERR_UNSUPPORTED) return rc;
    }
  }
  int rc = Nr > 0 ? clove_gemm_int8_rowcol(A_q, B_q_shard, C_shard, M, Nr, K, A_row_scale,
                                           B_col_scale_shard, stream)
                  : CLOVE_OK;
  if (rc || !replicate_C) return rc;
  if (C_full == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "C_full is NULL with replicate_C");
  return gather_columns(ctx, C_shard, C_full, M, N, 2, s);
}

}  // extern "C"
