/*
 * host_gemm.h -- CPU oracle for the clove GEMM hot path (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the parity checker and the timed CPU baseline. It is never
 * linked into, loaded by or called from the product path (clove_compute_b200/).
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use it.
 *
 * It restates, in plain C with fp32 / int32 arithmetic, what the reference's
 * GEMM entry points compute (reference paths relative to the clove_compute tree):
 *
 *   fp16  C = alpha*A.B + beta*C, fp32 accumulate     src/kernels/gemm_fp16.cu:241-270
 *         (the naive kernel's math; the WMMA kernel :30-215 computes the same
 *          product but accumulates in fp16, so it is only checked within tolerance)
 *   int8  int32 sum (a-za)(b-zb), * A_scale*B_scale   src/kernels/gemm_int8.cu:87-114
 *   int4  per-128-group int32 G = sum (a-za)(b-zb),   include/clove/kernels/gemm.cuh:67-87
 *         C = sum_g sA*sB*G                           (documented intent; see
 *                                                     clove_oracle_gemm_int4_refcompat
 *                                                     for what gemm_int4.cu:45-193 does)
 *
 * Parity pinning: the reference ships no golden vectors or known-answer tests
 * for any of these paths (its only check is cuBLAS with fp16 accumulation,
 * tests/test_gemm.cu:64-93). The fp16 and int4-refcompat restatements are
 * pinned against the reference kernels themselves run on a B200 (fixtures in
 * tests/golden/). The int8 restatement is pinned only by known-answer tests
 * written here: its reference kernel reads shared memory out of bounds
 * (gemm_int8.cu:77,84) and is never run -- int8 parity is unpinned by the
 * reference.
 *
 * All entry points compute only output rows [row_begin, row_end) so that the
 * CPU baseline can time a bounded sample; nthreads <= 0 means "all cores".
 * Every output element is produced by one thread in a fixed k / group order,
 * so results do not depend on the thread count.
 */
#ifndef CLOVE_ORACLE_HOST_GEMM_H
#define CLOVE_ORACLE_HOST_GEMM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary32 (round to nearest even, like __float2half). */
float clove_oracle_h2f(uint16_t h);
uint16_t clove_oracle_f2h(float f);
void clove_oracle_h2f_array(const uint16_t* in, float* out, int64_t n);
void clove_oracle_f2h_array(const float* in, uint16_t* out, int64_t n);

/* Number of threads the oracle uses when nthreads <= 0. */
int clove_oracle_max_threads(void);

/* fp16: C[m,n] = half(alpha * sum_k A[m,k]*B[k,n] + beta * C[m,n]), fp32 math.
 * A [M,K], B [K,N], C [M,N], all row-major binary16. beta == 0 never reads C. */
void clove_oracle_gemm_fp16(const uint16_t* A, const uint16_t* B, uint16_t* C,
                            int M, int N, int K, float alpha, float beta,
                            int row_begin, int row_end, int nthreads);

/* int8: acc[m,n] = sum_k (A[m,k]-za)(B[k,n]-zb) in wrapping int32.
 * A [M,K], B [K,N] row-major int8. */
void clove_oracle_int8_acc(const int8_t* A, const int8_t* B, int32_t* acc,
                           int M, int N, int K, int za, int zb,
                           int row_begin, int row_end, int nthreads);

/* int8, per-tensor (the reference signature): C = half(float(acc) * (sA*sB)). */
void clove_oracle_gemm_int8(const int8_t* A, const int8_t* B, uint16_t* C,
                            int M, int N, int K, float sA, int za, float sB, int zb,
                            int row_begin, int row_end, int nthreads);

/* int8, per-row A / per-column B fp32 scales, zero points 0:
 * C = half(float(acc) * sA[m] * sB[n]). */
void clove_oracle_gemm_int8_rowcol(const int8_t* A, const int8_t* B, uint16_t* C,
                                   int M, int N, int K,
                                   const float* sA_row, const float* sB_col,
                                   int row_begin, int row_end, int nthreads);

/* int4 group accumulators, K-packed layout on both operands:
 *   Aq [M,K/2] bytes, element 2j in the high nibble of byte j, 2j+1 in the low;
 *   Az [M,K/128], Bq [N,K/2], Bz [N,K/128] binary16 zero points (rounded to the
 *   nearest integer);  G[m,n,g] = sum_{k in group g} (a-za)(b-zb), int32.
 * K must be a multiple of 128. */
void clove_oracle_int4_group_acc(const uint8_t* Aq, const uint16_t* Az,
                                 const uint8_t* Bq, const uint16_t* Bz,
                                 int32_t* G, int M, int N, int K,
                                 int row_begin, int row_end, int nthreads);

/* int4 GEMM: C[m,n] = half( sum_g float(G[m,n,g]) * (sA[m,g]*sB[n,g]) ), the
 * fp32 sum taken in increasing g. Scales As [M,K/128], Bs [N,K/128] binary16. */
void clove_oracle_gemm_int4(const uint8_t* Aq, const uint16_t* As, const uint16_t* Az,
                            const uint8_t* Bq, const uint16_t* Bs, const uint16_t* Bz,
                            uint16_t* C, int M, int N, int K,
                            int row_begin, int row_end, int nthreads);

/* What the reference int4 kernel computes (gemm_int4.cu:45-193): signed codes
 * (nibble-8), zero points ignored, B packed along N as [K,N/2] (high nibble =
 * even n), B scales [K/128,N], and the whole K-sum scaled by the scales of the
 * LAST 64-wide K tile's group only. Used to explain the reference kernel's
 * output, never as the product's semantics. */
void clove_oracle_gemm_int4_refcompat(const uint8_t* Aq, const uint16_t* As,
                                      const uint8_t* Bq_kn, const uint16_t* Bs_kn,
                                      uint16_t* C, int M, int N, int K,
                                      int row_begin, int row_end, int nthreads);

/* SwiGLU projection: out[m,n] = half(silu(g)*u), g = X.Wg, u = X.Wu (fp32, k
 * ascending), silu(x) = x/(1+expf(-x)) (reference activations.cu:9-11,76-121).
 * X [M,K], Wg/Wu [K,N], out [M,N] binary16; rows [row_begin,row_end) only. */
void clove_oracle_swiglu(const uint16_t* X, const uint16_t* Wg, const uint16_t* Wu, uint16_t* out,
                         int M, int N, int K, int row_begin, int row_end, int nthreads);

/* INT4 packing tool (this build's specification; the reference has none):
 * W [rows,K] binary16, K % 128 == 0 -> codes [rows,K/2] (element 2j in the high
 * nibble of byte j), scales / zeros [rows,K/128] binary16. Asymmetric min/max per
 * 128-group over a range that contains 0 (min <= 0 <= max):
 * scale = half((max-min)/15) (0 -> smallest subnormal, capped at 65504),
 * zero = clamp(rint(-min/scale),0,15), code = clamp(rint(w/scale)+zero,0,15). */
void clove_oracle_quantize_int4(const uint16_t* W, int rows, int K, uint8_t* codes,
                                uint16_t* scales, uint16_t* zeros);

/* Attention, the reference's flash_attention_kernel (src/kernels/attention.cu:93-266)
 * restated: per query row, keys in blocks of 64; S = scale * sum_d q_d k_d (fp32,
 * d ascending); causal keys after the query set to -FLT_MAX; online softmax with
 * expf (running max, rescale of the row sum and the fp32 output row by
 * expf(old_max - new_max)); O = half(acc / sum). head_dim D; K/V heads
 * kv_heads (head h reads kv head h / (heads / kv_heads)).
 * layout 0: [batch, heads, seq, D]; 1: [batch, seq, heads, D].
 * refcompat 1 reproduces the reference's non-causal handling of a ragged last
 * block: the keys padding seq up to a multiple of 64 are loaded as zeros and
 * NOT masked, so each adds expf(0 - max) to the row sum (a phantom key with
 * score 0 and value 0). refcompat 0 is ordinary attention over the seq keys. */
void clove_oracle_attention(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O,
                            int batch, int heads, int kv_heads, int seq, int D, float scale,
                            int causal, int layout, int refcompat, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
