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
// NCCL is opened with dlopen on first use so that loading this library never pins
// an NCCL build into the process (PyTorch ships its own; whichever libnccl.so.2 is
// already loaded is reused).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "internal.h"

namespace clove {
namespace rt {
int launch_relayout_columns(const void* staging, void* C, int M, int N, int P, int Nmax,
                            int elem_bytes, cudaStream_t stream);
}  // namespace rt
}  // namespace clove

using namespace clove::rt;

struct clove_nsplit_ctx {
  ncclComm_t comm;
  int rank;
  int nranks;
  int device;
};

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
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
  CLOVE_SYM(CommDestroy, "ncclCommDestroy");
  CLOVE_SYM(CommAbort, "ncclCommAbort");
  CLOVE_SYM(AllGather, "ncclAllGather");
  CLOVE_SYM(GetErrorString, "ncclGetErrorString");
#undef CLOVE_SYM
  if (!g_nccl.GetUniqueId || !g_nccl.CommInitRank || !g_nccl.CommDestroy || !g_nccl.AllGather ||
      !g_nccl.GetErrorString || !g_nccl.CommAbort) {
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
    rc = check_nccl(g_nccl.AllGather(send, staging, slot / 2, ncclHalf, ctx->comm, s),
                    "ncclAllGather");
  if (!rc) rc = launch_relayout_columns(staging, C_full, M, N, P, Nmax, elem_bytes, s);
  const int rc2 = check_cuda(cudaFreeAsync(staging, s), "cudaFreeAsync(staging)");
  return rc ? rc : rc2;
}

}  // namespace

extern "C" {

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
  if (!rc) rc = check_nccl(g_nccl.CommInitRank(&c->comm, nranks, uid, rank), "ncclCommInitRank");
  if (rc) {
    delete c;
    return rc;
  }
  *ctx = c;
  return CLOVE_OK;
}

int clove_nsplit_destroy(clove_nsplit_ctx* ctx) {
  if (ctx == nullptr) return CLOVE_OK;
  int rc = CLOVE_OK;
  if (g_nccl.handle) rc = check_nccl(g_nccl.CommDestroy(ctx->comm), "ncclCommDestroy");
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
  int rc = Nr > 0 ? clove_gemm_int8_rowcol(A_q, B_q_shard, C_shard, M, Nr, K, A_row_scale,
                                           B_col_scale_shard, stream)
                  : CLOVE_OK;
  if (rc || !replicate_C) return rc;
  if (C_full == nullptr) return fail(CLOVE_ERR_INVALID_ARG, "C_full is NULL with replicate_C");
  return gather_columns(ctx, C_shard, C_full, M, N, 2, s);
}

}  // extern "C"
