/*
 * host_gemm.c -- CPU oracle for the clove GEMM hot path (TEST INFRASTRUCTURE ONLY).
 *
 * Plain C restatement of the reference arithmetic; see host_gemm.h for the
 * contract, the reference lines each function follows and the pinning status.
 * Built by oracle/Makefile into oracle/liboracle.so. Nothing in the product
 * package links or loads this file.
 */
#include "host_gemm.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* binary16 <-> binary32                                                      */
/* ------------------------------------------------------------------------- */

float clove_oracle_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t clove_oracle_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax < 0x38800000u) { /* below the smallest normal half: subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;                      /* 102..112 */
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;  /* 24-bit significand */
        uint32_t shift = 126u - e;                  /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    /* normal: rebias exponent, round 13 dropped bits to nearest even */
    uint32_t q = ((ax >> 13) - (112u << 10));
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

void clove_oracle_h2f_array(const uint16_t* in, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) out[i] = clove_oracle_h2f(in[i]);
}

void clove_oracle_f2h_array(const float* in, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) out[i] = clove_oracle_f2h(in[i]);
}

int clove_oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int resolve_threads(int nthreads) {
    int t = nthreads > 0 ? nthreads : clove_oracle_max_threads();
    return t < 1 ? 1 : t;
}

static void clamp_rows(int M, int* rb, int* re) {
    if (*rb < 0) *rb = 0;
    if (*re > M || *re < 0) *re = M;
}

/* Zero points arrive as binary16 holding integer codes; round to nearest
 * (ties to even), the same as __half2int_rn on the device. */
static int zero_point(uint16_t h) {
    return (int)nearbyintf(clove_oracle_h2f(h));
}

/* ------------------------------------------------------------------------- */
/* fp16 GEMM (fp32 accumulate)  -- src/kernels/gemm_fp16.cu:241-270          */
/* ------------------------------------------------------------------------- */

#define FP_MR 4   /* rows per micro-tile */
#define FP_NR 32  /* columns per micro-tile */

void clove_oracle_gemm_fp16(const uint16_t* A, const uint16_t* B, uint16_t* C,
                            int M, int N, int K, float alpha, float beta,
                            int row_begin, int row_end, int nthreads) {
    clamp_rows(M, &row_begin, &row_end);
    int rows = row_end - row_begin;
    if (rows <= 0 || N <= 0) return;
    int nt = resolve_threads(nthreads);

    /* Widen the operands once: B whole, A only for the rows computed. */
    float* Bf = (float*)malloc(sizeof(float) * (size_t)K * (size_t)N + 64);
    float* Af = (float*)malloc(sizeof(float) * (size_t)rows * (size_t)K + 64);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t i = 0; i < (int64_t)K * N; i++) Bf[i] = clove_oracle_h2f(B[i]);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t i = 0; i < (int64_t)rows * K; i++)
        Af[i] = clove_oracle_h2f(A[(int64_t)row_begin * K + i]);

    int mblocks = (rows + FP_MR - 1) / FP_MR;
    int nblocks = (N + FP_NR - 1) / FP_NR;
    /* n-panel outer so that one B panel [K, FP_NR] stays cache resident while
     * the row micro-tiles stream past it. */
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1) collapse(2)
    for (int nb = 0; nb < nblocks; nb++) {
        for (int mb = 0; mb < mblocks; mb++) {
            int n0 = nb * FP_NR;
            int m0 = mb * FP_MR;
            int nr = N - n0 < FP_NR ? N - n0 : FP_NR;
            int mr = rows - m0 < FP_MR ? rows - m0 : FP_MR;
            float acc[FP_MR][FP_NR];
            memset(acc, 0, sizeof(acc));
            if (nr == FP_NR && mr == FP_MR) {
                for (int k = 0; k < K; k++) {
                    const float* b = Bf + (int64_t)k * N + n0;
                    for (int i = 0; i < FP_MR; i++) {
                        float a = Af[(int64_t)(m0 + i) * K + k];
                        for (int j = 0; j < FP_NR; j++) acc[i][j] += a * b[j];
                    }
                }
            } else {
                for (int k = 0; k < K; k++) {
                    const float* b = Bf + (int64_t)k * N + n0;
                    for (int i = 0; i < mr; i++) {
                        float a = Af[(int64_t)(m0 + i) * K + k];
                        for (int j = 0; j < nr; j++) acc[i][j] += a * b[j];
                    }
                }
            }
            for (int i = 0; i < mr; i++) {
                int64_t row = (int64_t)(row_begin + m0 + i);
                for (int j = 0; j < nr; j++) {
                    float r = alpha * acc[i][j];
                    if (beta != 0.0f) r += beta * clove_oracle_h2f(C[row * N + n0 + j]);
                    C[row * N + n0 + j] = clove_oracle_f2h(r);
                }
            }
        }
    }
    free(Bf);
    free(Af);
}

/* ------------------------------------------------------------------------- */
/* int8 GEMM  -- src/kernels/gemm_int8.cu:87-114                             */
/* ------------------------------------------------------------------------- */

/* acc rows [row_begin,row_end) into acc_rows (row-major [rows, N]). The sum is
 * kept in uint32 so that overflow wraps exactly like the device's int32. */
static void int8_acc_rows(const int8_t* A, const int8_t* B, int32_t* acc_rows,
                          int N, int K, int za, int zb, int row_begin, int rows, int nt) {
    /* Widen (b - zb) once, transposed to [N, K] for a contiguous dot product. */
    int32_t* Bt = (int32_t*)malloc(sizeof(int32_t) * (size_t)N * (size_t)K + 64);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int n = 0; n < N; n++)
        for (int k = 0; k < K; k++) Bt[(int64_t)n * K + k] = (int32_t)B[(int64_t)k * N + n] - zb;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int r = 0; r < rows; r++) {
        const int8_t* a = A + (int64_t)(row_begin + r) * K;
        int32_t* arow = (int32_t*)malloc(sizeof(int32_t) * (size_t)K + 64);
        for (int k = 0; k < K; k++) arow[k] = (int32_t)a[k] - za;
        for (int n = 0; n < N; n++) {
            const int32_t* b = Bt + (int64_t)n * K;
            uint32_t s = 0;
            for (int k = 0; k < K; k++) s += (uint32_t)arow[k] * (uint32_t)b[k];
            acc_rows[(int64_t)r * N + n] = (int32_t)s;
        }
        free(arow);
    }
    free(Bt);
}

void clove_oracle_int8_acc(const int8_t* A, const int8_t* B, int32_t* acc,
                           int M, int N, int K, int za, int zb,
                           int row_begin, int row_end, int nthreads) {
    clamp_rows(M, &row_begin, &row_end);
    int rows = row_end - row_begin;
    if (rows <= 0 || N <= 0) return;
    int8_acc_rows(A, B, acc + (int64_t)row_begin * N, N, K, za, zb, row_begin, rows,
                  resolve_threads(nthreads));
}

void clove_oracle_gemm_int8(const int8_t* A, const int8_t* B, uint16_t* C,
                            int M, int N, int K, float sA, int za, float sB, int zb,
                            int row_begin, int row_end, int nthreads) {
    clamp_rows(M, &row_begin, &row_end);
    int rows = row_end - row_begin;
    if (rows <= 0 || N <= 0) return;
    int nt = resolve_threads(nthreads);
    int32_t* acc = (int32_t*)malloc(sizeof(int32_t) * (size_t)rows * (size_t)N + 64);
    int8_acc_rows(A, B, acc, N, K, za, zb, row_begin, rows, nt);
    float combined = sA * sB; /* gemm_int8.cu:40 */
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t i = 0; i < (int64_t)rows * N; i++)
        C[(int64_t)row_begin * N + i] = clove_oracle_f2h((float)acc[i] * combined);
    free(acc);
}

void clove_oracle_gemm_int8_rowcol(const int8_t* A, const int8_t* B, uint16_t* C,
                                   int M, int N, int K,
                                   const float* sA_row, const float* sB_col,
                                   int row_begin, int row_end, int nthreads) {
    clamp_rows(M, &row_begin, &row_end);
    int rows = row_end - row_begin;
    if (rows <= 0 || N <= 0) return;
    int nt = resolve_threads(nthreads);
    int32_t* acc = (int32_t*)malloc(sizeof(int32_t) * (size_t)rows * (size_t)N + 64);
    int8_acc_rows(A, B, acc, N, K, 0, 0, row_begin, rows, nt);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int r = 0; r < rows; r++) {
        int m = row_begin + r;
        for (int n = 0; n < N; n++)
            C[(int64_t)m * N + n] =
                clove_oracle_f2h(((float)acc[(int64_t)r * N + n] * sA_row[m]) * sB_col[n]);
    }
    free(acc);
}

/* ------------------------------------------------------------------------- */
/* int4 group GEMM  -- gemm.cuh:67-87 (layout), gemm_int4.cu:27-34 (nibbles) */
/* ------------------------------------------------------------------------- */

#define INT4_GROUP 128

/* code of element k of a K-packed row: byte k/2, high nibble for even k. */
static inline int nib(const uint8_t* row, int k) {
    uint8_t byte = row[k >> 1];
    return (k & 1) ? (byte & 0x0f) : (byte >> 4);
}

/* Unpack n rows of K codes minus their group zero point into int8 [n, K]. */
static void unpack_sub_zero(const uint8_t* q, const uint16_t* z, int8_t* out,
                            int row0, int nrows, int K, int nt) {
    int G = K / INT4_GROUP;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int r = 0; r < nrows; r++) {
        const uint8_t* row = q + (int64_t)(row0 + r) * (K / 2);
        for (int g = 0; g < G; g++) {
            int zp = zero_point(z[(int64_t)(row0 + r) * G + g]);
            for (int k = g * INT4_GROUP; k < (g + 1) * INT4_GROUP; k++)
                out[(int64_t)r * K + k] = (int8_t)(nib(row, k) - zp);
        }
    }
}

static inline int32_t dot_i8(const int8_t* a, const int8_t* b, int n) {
    int32_t s = 0;
    for (int k = 0; k < n; k++) s += (int32_t)a[k] * (int32_t)b[k];
    return s;
}

void clove_oracle_int4_group_acc(const uint8_t* Aq, const uint16_t* Az,
                                 const uint8_t* Bq, const uint16_t* Bz,
                                 int32_t* G, int M, int N, int K,
                                 int row_begin, int row_end, int nthreads) {
    clamp_rows(M, &row_begin, &row_end);
    int rows = row_end - row_begin;
    if (rows <= 0 || N <= 0 || K % INT4_GROUP != 0) return;
    int nt = resolve_threads(nthreads);
    int ng = K / INT4_GROUP;
    int8_t* a = (int8_t*)malloc((size_t)rows * (size_t)K + 64);
    int8_t* b = (int8_t*)malloc((size_t)N * (size_t)K + 64);
    unpack_sub_zero(Aq, Az, a, row_begin, rows, K, nt);
    unpack_sub_zero(Bq, Bz, b, 0, N, K, nt);
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int r = 0; r < rows; r++)
        for (int n = 0; n < N; n++)
            for (int g = 0; g < ng; g++)
                G[((int64_t)(row_begin + r) * N + n) * ng + g] =
                    dot_i8(a + (int64_t)r * K + g * INT4_GROUP,
                           b + (int64_t)n * K + g * INT4_GROUP, INT4_GROUP);
    free(a);
    free(b);
}

void clove_oracle_gemm_int4(const uint8_t* Aq, const uint16_t* As, const uint16_t* Az,
                            const uint8_t* Bq, const uint16_t* Bs, const uint16_t* Bz,
                            uint16_t* C, int M, int N, int K,
                            int row_begin, int row_end, int nthreads) {
    clamp_rows(M, &row_begin, &row_end);
    int rows = row_end - row_begin;
    if (rows <= 0 || N <= 0 || K % INT4_GROUP != 0) return;
    int nt = resolve_threads(nthreads);
    int ng = K / INT4_GROUP;
    int8_t* a = (int8_t*)malloc((size_t)rows * (size_t)K + 64);
    int8_t* b = (int8_t*)malloc((size_t)N * (size_t)K + 64);
    float* sb = (float*)malloc(sizeof(float) * (size_t)N * (size_t)ng + 64);
    unpack_sub_zero(Aq, Az, a, row_begin, rows, K, nt);
    unpack_sub_zero(Bq, Bz, b, 0, N, K, nt);
    for (int64_t i = 0; i < (int64_t)N * ng; i++) sb[i] = clove_oracle_h2f(Bs[i]);
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int r = 0; r < rows; r++) {
        int m = row_begin + r;
        for (int n = 0; n < N; n++) {
            float acc = 0.0f;
            for (int g = 0; g < ng; g++) {
                int32_t gsum = dot_i8(a + (int64_t)r * K + g * INT4_GROUP,
                                      b + (int64_t)n * K + g * INT4_GROUP, INT4_GROUP);
                float s = clove_oracle_h2f(As[(int64_t)m * ng + g]) * sb[(int64_t)n * ng + g];
                acc += (float)gsum * s;
            }
            C[(int64_t)m * N + n] = clove_oracle_f2h(acc);
        }
    }
    free(a);
    free(b);
    free(sb);
}

/* gemm_int4.cu:45-193 as written: 64-wide K tiles, codes-8, zeros ignored,
 * B [K,N/2] packed along N, B scales [K/128,N], final scale = last tile's group. */
void clove_oracle_gemm_int4_refcompat(const uint8_t* Aq, const uint16_t* As,
                                      const uint8_t* Bq_kn, const uint16_t* Bs_kn,
                                      uint16_t* C, int M, int N, int K,
                                      int row_begin, int row_end, int nthreads) {
    clamp_rows(M, &row_begin, &row_end);
    int rows = row_end - row_begin;
    if (rows <= 0 || N <= 0 || K <= 0) return;
    int nt = resolve_threads(nthreads);
    int ngroups = (K + INT4_GROUP - 1) / INT4_GROUP;          /* cdiv(K,128) */
    int last_tile_base = ((K + 63) / 64 - 1) * 64;            /* :212-216 */
    int last_group = last_tile_base / INT4_GROUP;
    int half_n = N / 2;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int r = 0; r < rows; r++) {
        int m = row_begin + r;
        float a_s = clove_oracle_h2f(As[(int64_t)m * ngroups + last_group]);
        for (int n = 0; n < N; n++) {
            float acc = 0.0f;
            int np = n >> 1;
            for (int k = 0; k < K; k++) {
                int a = 0, b = 0;
                if ((k >> 1) < K / 2) { /* :226 globalKPacked < K/2 */
                    uint8_t byte = Aq[(int64_t)m * (K / 2) + (k >> 1)];
                    a = ((k & 1) ? (byte & 0x0f) : (byte >> 4)) - 8;
                }
                if (np < half_n) { /* :246 globalNPacked < N/2 */
                    uint8_t byte = Bq_kn[(int64_t)k * half_n + np];
                    b = ((n & 1) ? (byte & 0x0f) : (byte >> 4)) - 8;
                }
                acc += (float)a * (float)b;
            }
            float b_s = clove_oracle_h2f(Bs_kn[(int64_t)last_group * N + n]);
            C[(int64_t)m * N + n] = clove_oracle_f2h(acc * a_s * b_s); /* :328 */
        }
    }
}

/* ------------------------------------------------------------------------- */
/* INT4 packing of fp16 weights into the layout clove_gemm_int4 consumes.     */
/* The reference has no quantizer (its safetensors loader is a stub,          */
/* src/runtime/model_loader.cpp:57-85); this is the specification of this     */
/* build's tool, restated on the CPU: asymmetric min/max per 128-group over  */
/* a range that contains 0 (min <= 0 <= max, so an all-positive or constant   */
/* group keeps its values), scale = half((max-min)/15) (0 -> smallest         */
/* subnormal, clamped to 65504),                                              */
/* zero = clamp(rint(-min/scale), 0, 15), code = clamp(rint(w/scale) + zero, */
/* 0, 15), fp32 arithmetic with IEEE division and ties-to-even rounding.      */
/* ------------------------------------------------------------------------- */
void clove_oracle_quantize_int4(const uint16_t* W, int rows, int K, uint8_t* codes,
                                uint16_t* scales, uint16_t* zeros) {
    if (rows <= 0 || K <= 0 || K % INT4_GROUP != 0) return;
    const int ng = K / INT4_GROUP;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        for (int g = 0; g < ng; g++) {
            const uint16_t* w = W + (int64_t)r * K + (int64_t)g * INT4_GROUP;
            float mn = 0.0f, mx = 0.0f; /* the range always contains 0 */
            for (int i = 0; i < INT4_GROUP; i++) {
                float v = clove_oracle_h2f(w[i]);
                mn = v < mn ? v : mn;
                mx = v > mx ? v : mx;
            }
            float s = (mx - mn) / 15.0f;
            uint16_t sh = clove_oracle_f2h(s);
            if ((sh & 0x7fff) == 0) sh = 0x0001;       /* smallest positive subnormal */
            if ((sh & 0x7fff) > 0x7bff) sh = 0x7bff;   /* 65504 */
            const float sf = clove_oracle_h2f(sh);
            float zf = rintf(-mn / sf);
            zf = zf < 0.0f ? 0.0f : (zf > 15.0f ? 15.0f : zf);
            const int z = (int)zf;
            scales[(int64_t)r * ng + g] = sh;
            zeros[(int64_t)r * ng + g] = clove_oracle_f2h((float)z);
            uint8_t* out = codes + (int64_t)r * (K / 2) + (int64_t)g * (INT4_GROUP / 2);
            for (int j = 0; j < INT4_GROUP / 2; j++) {
                int q[2];
                for (int e = 0; e < 2; e++) {
                    float t = rintf(clove_oracle_h2f(w[2 * j + e]) / sf) + (float)z;
                    t = t < 0.0f ? 0.0f : (t > 15.0f ? 15.0f : t);
                    q[e] = (int)t;
                }
                out[j] = (uint8_t)((q[0] << 4) | q[1]);
            }
        }
    }
}

/* ------------------------------------------------------------------------- */
/* SwiGLU projection: out = half(silu(g) * u), g = X.Wg, u = X.Wu in fp32       */
/* (k ascending), silu(x) = x / (1 + expf(-x)) as the reference's silu_f       */
/* (src/kernels/activations.cu:9-11) applied by its swiglu kernel (:76-121) -- */
/* here on the fp32 accumulators, which is what clove_swiglu_fused fuses       */
/* (the reference declares swiglu_fused, activations.cuh:37-46, and never      */
/* defines it).                                                               */
/* ------------------------------------------------------------------------- */
void clove_oracle_swiglu(const uint16_t* X, const uint16_t* Wg, const uint16_t* Wu, uint16_t* out,
                         int M, int N, int K, int row_begin, int row_end, int nthreads) {
    if (row_end > M) row_end = M;
    if (row_begin < 0) row_begin = 0;
    if (row_end <= row_begin || N <= 0) return;
    int nt = resolve_threads(nthreads);
    float* Wgf = (float*)malloc(sizeof(float) * (size_t)K * N + 1);
    float* Wuf = (float*)malloc(sizeof(float) * (size_t)K * N + 1);
    for (int64_t i = 0; i < (int64_t)K * N; i++) {
        Wgf[i] = clove_oracle_h2f(Wg[i]);
        Wuf[i] = clove_oracle_h2f(Wu[i]);
    }
#pragma omp parallel num_threads(nt)
    {
        float* g = (float*)malloc(sizeof(float) * (size_t)N);
        float* u = (float*)malloc(sizeof(float) * (size_t)N);
#pragma omp for schedule(dynamic, 1)
        for (int m = row_begin; m < row_end; m++) {
            for (int n = 0; n < N; n++) g[n] = u[n] = 0.0f;
            for (int k = 0; k < K; k++) {
                const float a = clove_oracle_h2f(X[(int64_t)m * K + k]);
                const float* bg = Wgf + (int64_t)k * N;
                const float* bu = Wuf + (int64_t)k * N;
                for (int n = 0; n < N; n++) {
                    g[n] += a * bg[n];
                    u[n] += a * bu[n];
                }
            }
            for (int n = 0; n < N; n++)
                out[(int64_t)m * N + n] = clove_oracle_f2h(g[n] / (1.0f + expf(-g[n])) * u[n]);
        }
        free(g);
        free(u);
    }
    free(Wgf);
    free(Wuf);
}

/* ------------------------------------------------------------------------- */
/* Attention (reference src/kernels/attention.cu:93-266)                      */
/* ------------------------------------------------------------------------- */
static inline int64_t attn_index(int layout, int heads, int seq, int D, int b, int h, int s) {
    if (layout == 0) return (((int64_t)b * heads + h) * seq + s) * D;
    return (((int64_t)b * seq + s) * heads + h) * D;
}

void clove_oracle_attention(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O,
                            int batch, int heads, int kv_heads, int seq, int D, float scale,
                            int causal, int layout, int refcompat, int nthreads) {
    const int group = heads / kv_heads;
    const int64_t rows = (int64_t)batch * heads * seq;
    const int BC = 64; /* key block of the reference kernel (FA_BC) */
#pragma omp parallel num_threads(resolve_threads(nthreads))
    {
        float* q = (float*)malloc(sizeof(float) * D);
        float* acc = (float*)malloc(sizeof(float) * D);
        float* sblk = (float*)malloc(sizeof(float) * BC);
#pragma omp for schedule(dynamic, 16)
        for (int64_t r = 0; r < rows; r++) {
            const int s_q = (int)(r % seq);
            const int h = (int)((r / seq) % heads);
            const int b = (int)(r / ((int64_t)seq * heads));
            const int hk = h / group;
            const uint16_t* qrow = Q + attn_index(layout, heads, seq, D, b, h, s_q);
            for (int d = 0; d < D; d++) q[d] = clove_oracle_h2f(qrow[d]);
            for (int d = 0; d < D; d++) acc[d] = 0.f;
            float row_max = -3.402823466e38f, row_sum = 0.f;
            /* Keys the reference visits: up to the end of the query's 64-row block
             * for causal attention (all later ones masked), all blocks otherwise. */
            const int q_start = s_q / 64 * 64;
            const int k_end = causal ? (seq < q_start + 64 ? seq : q_start + 64) : seq;
            for (int k0 = 0; k0 < k_end; k0 += BC) {
                float bmax = -3.402823466e38f;
                for (int j = 0; j < BC; j++) {
                    const int key = k0 + j;
                    float sc;
                    if (key < seq) {
                        const uint16_t* krow = K + attn_index(layout, kv_heads, seq, D, b, hk, key);
                        float sum = 0.f;
                        for (int d = 0; d < D; d++) sum += q[d] * clove_oracle_h2f(krow[d]);
                        sc = sum * scale;
                    } else {
                        sc = 0.f; /* zero-filled key row */
                    }
                    if (causal && s_q < key) sc = -3.402823466e38f;
                    else if (!causal && key >= seq && !refcompat) sc = -INFINITY; /* absent key */
                    sblk[j] = sc;
                    if (sc > bmax) bmax = sc;
                }
                const float new_max = fmaxf(row_max, bmax);
                const float scale_old = expf(row_max - new_max);
                row_sum *= scale_old;
                for (int d = 0; d < D; d++) acc[d] *= scale_old;
                float bsum = 0.f;
                for (int j = 0; j < BC; j++) {
                    const int key = k0 + j;
                    const float p = expf(sblk[j] - new_max);
                    bsum += p;
                    if (key < seq && p != 0.f) {
                        const uint16_t* vrow = V + attn_index(layout, kv_heads, seq, D, b, hk, key);
                        for (int d = 0; d < D; d++) acc[d] += p * clove_oracle_h2f(vrow[d]);
                    }
                }
                row_sum += bsum;
                row_max = new_max;
            }
            uint16_t* orow = O + attn_index(layout, heads, seq, D, b, h, s_q);
            const float inv = 1.0f / row_sum;
            for (int d = 0; d < D; d++) orow[d] = clove_oracle_f2h(acc[d] * inv);
        }
        free(q);
        free(acc);
        free(sblk);
    }
}
