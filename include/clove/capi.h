/*
 * clove/capi.h -- C ABI of the B200 (sm_100a) GEMM hot path.
 *
 * Plain pointers and sizes only. Every matrix is row-major and every pointer is
 * a device pointer owned by the caller; fp16 data is IEEE binary16 passed as
 * `void*`. Calls are asynchronous on `stream` (a cudaStream_t, NULL = legacy
 * default stream) and never synchronise. Functions return CLOVE_OK or an error
 * code; clove_last_error_string() describes the last failure on the calling
 * thread. Nothing here calls exit().
 *
 * Entry points and the reference interfaces they replace (paths in the
 * clove_compute tree):
 *   clove_gemm_fp16        clove::gemm_fp16          include/clove/kernels/gemm.cuh:41-49,
 *                                                    src/kernels/gemm_fp16.cu:277-305
 *   clove_gemm_int8        clove::gemm_int8          gemm.cuh:57-65, gemm_int8.cu:119-137
 *   clove_gemm_int8_rowcol (extension: per-row / per-column scales of gemm.cuh:55's formula)
 *   clove_gemm_int4        clove::gemm_int4          gemm.cuh:77-87, gemm_int4.cu:195-216
 *   clove_gemm_fp16_batched clove::gemm_fp16_batched gemm.cuh:93-101, gemm_fp16.cu:366-383
 *   clove_flash_attention  clove::flash_attention    attention.cuh:44-56, attention.cu:93-310
 *   clove_debug_*          (test hooks: raw int32 accumulators for bit-exact checks)
 *   clove_nsplit_*         (extension: N-split over the GPUs of one node, NCCL all-gather)
 */
#ifndef CLOVE_CAPI_H
#define CLOVE_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define CLOVE_OK 0
#define CLOVE_ERR_INVALID_ARG 1   /* null pointer, negative size, bad layout    */
#define CLOVE_ERR_UNSUPPORTED 2   /* shape/alignment this build cannot run      */
#define CLOVE_ERR_CUDA 3          /* a CUDA runtime/driver call failed          */
#define CLOVE_ERR_NCCL 4          /* an NCCL call failed                        */
#define CLOVE_ERR_DEVICE 5        /* device is not an sm_100 GPU                */
#define CLOVE_ERR_TIMEOUT 6       /* a kernel's bounded wait expired            */

/* INT4 quantisation group along K (gemm.cuh:72). */
#define CLOVE_INT4_GROUP_SIZE 128

/* Library version string and build architecture. */
const char* clove_version(void);

/* Description of the last error raised on the calling host thread. */
const char* clove_last_error_string(void);

/* Reads and clears the device-side error word of the current device (a kernel
 * whose bounded wait expired sets it). Synchronises the device. *code = 0 when
 * no kernel reported an error, 1 when a bounded wait expired (mbarrier or
 * cross-rank flag), 2 when a kernel was launched with a shape it rejects. After an
 * error it also resets the library's kept stream-K state, so call it before
 * further GEMMs once a kernel may have failed. */
int clove_get_device_error(int* code);

/* ------------------------------------------------------------------------- */
/* FP16: C = alpha * A.B + beta * C.  A [M,K], B [K,N], C [M,N] binary16.       */
/* fp32 accumulation (the reference WMMA kernel accumulates in fp16).          */
/* beta == 0 never reads C; C may be the residual input when beta != 0.        */
/* ------------------------------------------------------------------------- */
int clove_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                    float beta, void* stream);

/* Batched: A [batch,M,K], B [batch,K,N], C [batch,M,N], densely packed. */
int clove_gemm_fp16_batched(const void* A, const void* B, void* C, int batch, int M, int N,
                            int K, float alpha, float beta, void* stream);

/* SwiGLU-fused projection, the reference's declared-only clove::swiglu_fused
 * (include/clove/kernels/activations.cuh:37-46): input [batch_seq, hidden],
 * W_gate / W_up [hidden, intermediate], output [batch_seq, intermediate] =
 * silu(input . W_gate) * (input . W_up), silu(x) = x / (1 + exp(-x)) in fp32 on
 * the fp32 accumulators. One CTA-pair kernel computes both projections of each
 * 256 x 128 output tile (batch_seq >= 128, hidden and intermediate multiples of 8,
 * 16-byte aligned pointers); other shapes run two GEMMs and an elementwise pass. */
int clove_swiglu_fused(const void* input, const void* W_gate, const void* W_up, void* output,
                       int batch_seq, int hidden_dim, int intermediate_dim, void* stream);

/* ------------------------------------------------------------------------- */
/* INT8 (reference signature): C = half( sum_k (A-A_zero)(B-B_zero) * A_scale*B_scale ) */
/* A_q [M,K] int8, B_q [K,N] int8, C [M,N] binary16; int32 accumulation.        */
/* ------------------------------------------------------------------------- */
int clove_gemm_int8(const int8_t* A_q, const int8_t* B_q, void* C, int M, int N, int K,
                    float A_scale, int8_t A_zero, float B_scale, int8_t B_zero, void* stream);

/* No-allocation variant of clove_gemm_int8 (same arguments and results). It has no
 * counterpart in the reference. For callers that cannot let a library allocate
 * device memory -- e.g. serving runtimes that reserve all of HBM for their own
 * pools, where a stray allocation can fail mid-serving: the zero-point row /
 * column sums that clove_gemm_int8 keeps in cudaMallocAsync scratch live here in
 * a fixed array compiled into the library (CLOVE_NOALLOC_MAX_SUMS int32 entries,
 * 256 KiB on every GPU that loads the library). Requires M + N <=
 * CLOVE_NOALLOC_MAX_SUMS on the tensor-core path, else CLOVE_ERR_UNSUPPORTED.
 * The first call on each device looks up the array's device address; make it
 * before any stream capture. Calls share the array: calls that overlap on the
 * GPU race. */
#define CLOVE_NOALLOC_MAX_SUMS 65536
int clove_gemm_int8_noalloc(const int8_t* A_q, const int8_t* B_q, void* C, int M, int N, int K,
                            float A_scale, int8_t A_zero, float B_scale, int8_t B_zero,
                            void* stream);

/* INT8 with per-row A scales [M] and per-column B scales [N] (fp32, device),
 * zero points 0: C[m,n] = half( float(acc) * A_row_scale[m] * B_col_scale[n] ). */
int clove_gemm_int8_rowcol(const int8_t* A_q, const int8_t* B_q, void* C, int M, int N, int K,
                           const float* A_row_scale, const float* B_col_scale, void* stream);

/* ------------------------------------------------------------------------- */
/* INT4, per-128-group scales and zero points on both operands, K-packed:       */
/*   A_q [M,K/2], B_q [N,K/2] bytes; element 2j of a row in the HIGH nibble of   */
/*   byte j, element 2j+1 in the low nibble; codes unsigned 0..15.              */
/*   A_scale, A_zero [M,K/128]; B_scale, B_zero [N,K/128] binary16. Zero points */
/*   hold integer codes (rounded to nearest).                                   */
/*   G[m,n,g] = sum_{k in g} (a-za)(b-zb)   exact int32                         */
/*   C[m,n]   = half( sum_g float(G) * sA[m,g] * sB[n,g] )  fp32 sum            */
/* K must be a multiple of 128.                                                 */
/* ------------------------------------------------------------------------- */
int clove_gemm_int4(const uint8_t* A_q, const void* A_scale, const void* A_zero,
                    const uint8_t* B_q, const void* B_scale, const void* B_zero, void* C, int M,
                    int N, int K, void* stream);

/* INT4 packing tool (no counterpart in the reference, whose weight loader is a
 * stub): W [rows,K] binary16 -> codes [rows,K/2], scales / zeros [rows,K/128] in
 * exactly the layout clove_gemm_int4 reads. Asymmetric min/max per 128-group over
 * a range that contains 0: scale = half((max-min)/15), zero = clamp(rint(-min/scale),0,15),
 * code = clamp(rint(w/scale)+zero,0,15). K % 128 == 0; W 8-byte aligned. */
int clove_quantize_int4(const void* W, int rows, int K, uint8_t* codes, void* scales, void* zeros,
                        void* stream);

/* ------------------------------------------------------------------------- */
/* Attention: O = softmax(scale * Q.K^T [causal mask]) . V on the tensor cores  */
/* (replaces clove::flash_attention, include/clove/kernels/attention.cuh:44-56, */
/* src/kernels/attention.cu:93-266 and 273-310, whose S = Q.K^T and P.V are     */
/* CUDA-core loops at attention.cu:185-204).                                    */
/* Q, O: num_heads heads; K, V: num_kv_heads heads (num_heads a multiple; head  */
/* h reads kv head h / (num_heads / num_kv_heads), grouped-query attention).   */
/* layout 0: [batch, heads, seq_len, head_dim] (the reference's flash_attention); */
/* layout 1: [batch, seq_len, heads, head_dim] (the runtime's q/k/v projection  */
/* outputs, the layout of its flash_attention_rope). head_dim must be 128 (as   */
/* the reference); causal masks keys after the query; fp16 in and out, fp32     */
/* accumulation and softmax. 16-byte aligned tensors; scale > 0.                */
/* ------------------------------------------------------------------------- */
int clove_flash_attention(const void* Q, const void* K, const void* V, void* O, int batch,
                          int num_heads, int num_kv_heads, int seq_len, int head_dim, float scale,
                          int causal, int layout, void* stream);

/* ------------------------------------------------------------------------- */
/* Test hooks: exact int32 accumulators through the same kernels.              */
/* ------------------------------------------------------------------------- */
/* acc[m,n] = sum_k (A-A_zero)(B-B_zero) (wrapping int32), acc [M,N]. */
int clove_debug_int8_acc(const int8_t* A_q, const int8_t* B_q, int32_t* acc, int M, int N,
                         int K, int8_t A_zero, int8_t B_zero, void* stream);
/* G[m,n,g] as above, G [M,N,K/128]; also writes C like clove_gemm_int4. */
int clove_debug_int4_group_acc(const uint8_t* A_q, const void* A_scale, const void* A_zero,
                               const uint8_t* B_q, const void* B_scale, const void* B_zero,
                               void* C, int32_t* G, int M, int N, int K, void* stream);

/* Bare streaming read of nbytes at src (16-byte aligned, a multiple of 16 bytes),
 * nothing computed; *out is written only for one specific XOR of the data. It times
 * what one launch of that size can pull from HBM: the floor under the decode GEMVs.
 * (Measurement hook; no counterpart in the reference.) */
int clove_debug_stream_read(const void* src, size_t nbytes, uint32_t* out, void* stream);

/* y[i] = 2^x[i] (n even, fp32 device arrays, 8-byte aligned) through the polynomial
 * exponential the attention softmax runs on the FMA pipe for part of its keys:
 * relative error <= 2.7e-6 for x in [-125, 128], inputs below -125 clamped to -125.
 * (Test hook; no counterpart in the reference.) */
int clove_debug_exp2_poly(const float* x, float* y, int n, void* stream);

/* Runs the N-split's cross-rank completion wait for rank 0 of a two-rank group
 * whose other rank never signals, with a wait limit of timeout_ns (at most 2 s;
 * the product uses 2 s): the wait runs out, the kernel records device error 1
 * for clove_get_device_error() and returns, and the context stays usable. words:
 * 8 device words (8-byte aligned) of scratch, zeroed here. Exercises the failure
 * path of a bounded cross-GPU wait on one GPU. (Test hook; no counterpart in the
 * reference, which has no multi-GPU code.) */
int clove_debug_peer_wait_timeout(unsigned long long* words, unsigned long long timeout_ns,
                                  void* stream);

/* Stream-K schedule the CTA-pair kernel uses for `tiles` 256 x 256 output tiles of
 * kb_total K blocks on `pairs` co-resident CTA pairs (force: 0 automatic, 1 never,
 * 2 whenever the tiles leave a partial wave). Writes {whole-K tiles, stream-K
 * tiles, partial slots per stream-K tile, pairs launched} to out[0..3]. Host only.
 * (Introspection hook; no counterpart in the reference.) */
int clove_debug_stream_k_plan(int tiles, int pairs, int kb_total, int force, int* out);

/* Forces a kernel family for subsequent calls from any thread (tests only).
 * path: 0 = automatic, 1 = tensor-core tiles on one SM, 2 = GEMV, 3 = SIMT
 * fallback, 4 = tensor-core 256 x 256 tiles on CTA pairs.
 * bn: tensor-core N tile (0 = automatic; 32/64/128/256). split: cluster split-K
 * factor (0 = automatic, 1 = none, 2..8); with path 4 it selects the stream-K
 * schedule instead (0 automatic, 1 never, 2 whenever the tiles leave a partial
 * wave). Returns CLOVE_OK. */
int clove_set_dispatch_override(int path, int bn, int split);

/* Decode kernels (N <= 8 or M <= 8) start streaming their large operand -- the
 * weight matrix -- before the previous kernel on the stream has finished, which
 * hides the launch and first-byte latency of back-to-back decode GEMMs (programmatic
 * dependent launch). Only valid when no kernel still running on the stream writes
 * that operand, as for model weights in a decode loop; the small operand and C are
 * always accessed after the previous kernel completes. Process-wide; default off. */
int clove_set_weight_prefetch(int enable);

/* Describes the kernel the automatic dispatch picks for a shape:
 * dtype 0 = fp16, 1 = int8, 2 = int4, 3 = swiglu_fused. Writes a short name into buf. */
int clove_describe_dispatch(int dtype, int M, int N, int K, char* buf, size_t buflen);

/* ------------------------------------------------------------------------- */
/* N-split over the GPUs of one node (one process per GPU).                    */
/* Each rank holds all of A and a column shard of B / C: rank r owns columns    */
/* [clove_nsplit_col_begin(N,P,r), clove_nsplit_col_begin(N,P,r+1)).            */
/* The sharded calls compute C_r = A . B_r on this rank's GPU with the          */
/* single-GPU kernels (no communication). With replicate_C = 1 they then        */
/* all-gather every rank's C_r over NCCL into the full row-major C [M,N] on     */
/* every rank, or, for an fp16 C_full registered with                           */
/* clove_nsplit_register_output, store it there from the GEMM epilogue.         */
/* The communicator is created by clove_nsplit_init.                            */
/* ------------------------------------------------------------------------- */
typedef struct clove_nsplit_ctx clove_nsplit_ctx;

/* Column split: ranks get ceil/floor shares, first (N % P) ranks one extra. */
int clove_nsplit_col_begin(int N, int nranks, int rank);

/* 128-byte opaque NCCL unique id, produced on one rank and shared out of band. */
int clove_nsplit_get_unique_id(uint8_t id_out[128]);
int clove_nsplit_init(clove_nsplit_ctx** ctx, int nranks, int rank, const uint8_t id[128]);
int clove_nsplit_destroy(clove_nsplit_ctx* ctx);
int clove_nsplit_rank(const clove_nsplit_ctx* ctx, int* rank, int* nranks);

/* Collective (every rank, same order, same byte count): maps this rank's
 * replicated-output buffer C_full (device memory from cudaMalloc, at any offset,
 * e.g. a PyTorch tensor; 16-byte aligned) into every other rank through CUDA IPC.
 * Afterwards clove_nsplit_gemm_fp16 / _int8_rowcol / _int4 with replicate_C = 1 and
 * this C_full store each finished tile straight into every rank's C_full over
 * NVLink (no all-gather, no staging) and end with a cross-rank completion signal.
 * The route depends only on (M, N, K, nranks): equal shards (N % 8P == 0; INT8
 * N % 16P == 0) that the tile kernels take (N/P > 8; INT4 also M > 8;
 * INT8 no cluster split-K); other shapes still take the NCCL
 * all-gather. Operands must then be 16-byte aligned. At most 8 ranks.
 * Ordering contract of this route, so that a C_full can be reused call after call:
 *   - every replicated call of one context goes on one stream per rank (or on
 *     streams ordered by events), in the same order on every rank;
 *   - when a call returns on the stream, every rank's tiles are in this rank's
 *     C_full: work queued on the stream afterwards may read it;
 *   - a call stores into other ranks' C_full only after each of them has reached
 *     that call on its own stream, i.e. after everything queued on their streams
 *     before it (the readers of the previous result) has completed. Readers on
 *     another stream must be joined into the call stream (an event) before the
 *     next call is queued.
 * No host barrier is needed between calls.
 * (Extension; no counterpart in the reference.) */
int clove_nsplit_register_output(clove_nsplit_ctx* ctx, void* C_full, size_t bytes);
/* Collective, as clove_nsplit_register_output, for a C_full that every rank has
 * bound to one NVLink multicast object (NVSwitch; e.g. CUDA symmetric memory with a
 * multicast mapping): mc is the multicast object's address in this process (the
 * mapping of C_full, 16-byte aligned). The replicated route then sends each finished
 * tile once, as multimem stores that the switch fabric delivers to every rank's
 * C_full, instead of one store per rank; same shapes, same ordering contract. The
 * caller keeps the binding alive until clove_nsplit_unregister_output returns on
 * every rank. (Extension; no counterpart in the reference.) */
int clove_nsplit_register_output_multicast(clove_nsplit_ctx* ctx, void* C_full, void* mc,
                                           size_t bytes);
/* Collective: unmaps C_full everywhere; returns once no rank maps it any more. */
int clove_nsplit_unregister_output(clove_nsplit_ctx* ctx, void* C_full);

/* B_shard [K, N_r] row-major; C_shard [M, N_r]; C_full [M,N] (only with
 * replicate_C, may be NULL otherwise). */
int clove_nsplit_gemm_fp16(clove_nsplit_ctx* ctx, const void* A, const void* B_shard,
                           void* C_shard, void* C_full, int M, int N, int K, float alpha,
                           int replicate_C, void* stream);
/* INT4: B_q_shard [N_r, K/2], B_scale/zero_shard [N_r, K/128]. */
int clove_nsplit_gemm_int4(clove_nsplit_ctx* ctx, const uint8_t* A_q, const void* A_scale,
                           const void* A_zero, const uint8_t* B_q_shard,
                           const void* B_scale_shard, const void* B_zero_shard, void* C_shard,
                           void* C_full, int M, int N, int K, int replicate_C, void* stream);
/* INT8 row/col: B_q_shard [K, N_r], B_col_scale_shard [N_r]. */
int clove_nsplit_gemm_int8_rowcol(clove_nsplit_ctx* ctx, const int8_t* A_q,
                                  const int8_t* B_q_shard, const float* A_row_scale,
                                  const float* B_col_scale_shard, void* C_shard, void* C_full,
                                  int M, int N, int K, int replicate_C, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CLOVE_CAPI_H */
