"""CPU oracle for the clove GEMM hot path -- TEST INFRASTRUCTURE ONLY.

This package is the parity checker and the timed CPU baseline. Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs import it; the
product package ``clove_compute_b200`` never does.

The arithmetic lives in ``host_gemm.c`` (plain C, fp32/int32), a restatement
of the reference's GEMM math:

* fp16: ``src/kernels/gemm_fp16.cu:241-270`` (fp32 accumulate, alpha/beta)
* int8: ``src/kernels/gemm_int8.cu:87-114`` (int32 sum of (a-za)(b-zb) * sA*sB)
* int4: ``include/clove/kernels/gemm.cuh:67-87`` + nibble order of
  ``src/kernels/gemm_int4.cu:27-34`` (high nibble = even element), with
  per-128-group scales and zero points on both operands, K-packed ``[rows, K/2]``.
* ``gemm_int4_refcompat``: what ``gemm_int4.cu:45-193`` actually computes.

Pinning: fp16 and the int4 ref-compat restatement are pinned against outputs of
the reference kernels run on a B200 (``tests/golden/``); int8 has no reference
outputs or tests to pin against (parity unpinned by the reference; pinned by
known-answer tests only).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lock = threading.Lock()
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float

_SIGS = {
    "clove_oracle_max_threads": ([], _I),
    "clove_oracle_h2f_array": ([_P, _P, ctypes.c_int64], None),
    "clove_oracle_f2h_array": ([_P, _P, ctypes.c_int64], None),
    "clove_oracle_gemm_fp16": ([_P, _P, _P, _I, _I, _I, _F, _F, _I, _I, _I], None),
    "clove_oracle_int8_acc": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I], None),
    "clove_oracle_gemm_int8": ([_P, _P, _P, _I, _I, _I, _F, _I, _F, _I, _I, _I, _I], None),
    "clove_oracle_gemm_int8_rowcol": ([_P, _P, _P, _I, _I, _I, _P, _P, _I, _I, _I], None),
    "clove_oracle_int4_group_acc": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I], None),
    "clove_oracle_gemm_int4": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I], None),
    "clove_oracle_gemm_int4_refcompat": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I], None),
    "clove_oracle_quantize_int4": ([_P, _I, _I, _P, _P, _P], None),
    "clove_oracle_swiglu": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I], None),
    "clove_oracle_attention": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _I, _I, _I], None),
}


def build(force: bool = False) -> str:
    """Compile liboracle.so with oracle/Makefile (gcc, OpenMP)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            l = ctypes.CDLL(_LIB_PATH)
            for name, (args, res) in _SIGS.items():
                fn = getattr(l, name)
                fn.argtypes = args
                fn.restype = res
            _lib = l
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _rows(M, rows):
    if rows is None:
        return 0, M
    return int(rows[0]), int(rows[1])


def max_threads() -> int:
    return lib().clove_oracle_max_threads()


def h2f(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h).view(np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().clove_oracle_h2f_array(_ptr(h), _ptr(out), h.size)
    return out


def f2h(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    out = np.empty(f.shape, np.uint16)
    lib().clove_oracle_f2h_array(_ptr(f), _ptr(out), f.size)
    return out.view(np.float16)


def gemm_fp16(A, B, C=None, alpha=1.0, beta=0.0, rows=None, nthreads=0):
    """C = alpha*A@B + beta*C (fp32 accumulate, fp16 out). Returns C (fp16).

    ``rows=(r0, r1)`` computes only those output rows (others untouched)."""
    A = np.ascontiguousarray(A, np.float16)
    B = np.ascontiguousarray(B, np.float16)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    if C is None:
        C = np.zeros((M, N), np.float16)
    assert C.shape == (M, N) and C.dtype == np.float16 and C.flags["C_CONTIGUOUS"]
    r0, r1 = _rows(M, rows)
    lib().clove_oracle_gemm_fp16(_ptr(A), _ptr(B), _ptr(C), M, N, K, float(alpha), float(beta),
                                 r0, r1, nthreads)
    return C


def int8_acc(A, B, za=0, zb=0, rows=None, nthreads=0):
    """int32 acc[m,n] = sum_k (A[m,k]-za)(B[k,n]-zb), wrapping like int32."""
    A = np.ascontiguousarray(A, np.int8)
    B = np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    _, N = B.shape
    acc = np.zeros((M, N), np.int32)
    r0, r1 = _rows(M, rows)
    lib().clove_oracle_int8_acc(_ptr(A), _ptr(B), _ptr(acc), M, N, K, int(za), int(zb), r0, r1,
                                nthreads)
    return acc


def gemm_int8(A, B, A_scale, A_zero, B_scale, B_zero, rows=None, nthreads=0):
    """Reference per-tensor signature: C = half(float(acc) * (sA*sB))."""
    A = np.ascontiguousarray(A, np.int8)
    B = np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    _, N = B.shape
    C = np.zeros((M, N), np.float16)
    r0, r1 = _rows(M, rows)
    lib().clove_oracle_gemm_int8(_ptr(A), _ptr(B), _ptr(C), M, N, K, float(np.float32(A_scale)),
                                 int(A_zero), float(np.float32(B_scale)), int(B_zero), r0, r1,
                                 nthreads)
    return C


def gemm_int8_rowcol(A, B, sA_row, sB_col, rows=None, nthreads=0):
    """C = half(float(acc) * sA[m] * sB[n]) with zero points 0."""
    A = np.ascontiguousarray(A, np.int8)
    B = np.ascontiguousarray(B, np.int8)
    sA_row = np.ascontiguousarray(sA_row, np.float32)
    sB_col = np.ascontiguousarray(sB_col, np.float32)
    M, K = A.shape
    _, N = B.shape
    C = np.zeros((M, N), np.float16)
    r0, r1 = _rows(M, rows)
    lib().clove_oracle_gemm_int8_rowcol(_ptr(A), _ptr(B), _ptr(C), M, N, K, _ptr(sA_row),
                                        _ptr(sB_col), r0, r1, nthreads)
    return C


def _h(a):
    return np.ascontiguousarray(a, np.float16).view(np.uint16)


def int4_group_acc(Aq, Az, Bq, Bz, K, rows=None, nthreads=0):
    """int32 G[m,n,g] (north-star K-packed layout on both operands)."""
    Aq = np.ascontiguousarray(Aq, np.uint8)
    Bq = np.ascontiguousarray(Bq, np.uint8)
    M, N = Aq.shape[0], Bq.shape[0]
    G = np.zeros((M, N, K // 128), np.int32)
    r0, r1 = _rows(M, rows)
    Az_, Bz_ = _h(Az), _h(Bz)
    lib().clove_oracle_int4_group_acc(_ptr(Aq), _ptr(Az_), _ptr(Bq), _ptr(Bz_), _ptr(G), M, N, K,
                                      r0, r1, nthreads)
    return G


def gemm_int4(Aq, As, Az, Bq, Bs, Bz, K, rows=None, nthreads=0):
    """C[m,n] = half(sum_g float(G) * sA*sB), fp32 sum in increasing g."""
    Aq = np.ascontiguousarray(Aq, np.uint8)
    Bq = np.ascontiguousarray(Bq, np.uint8)
    M, N = Aq.shape[0], Bq.shape[0]
    C = np.zeros((M, N), np.float16)
    r0, r1 = _rows(M, rows)
    As_, Az_, Bs_, Bz_ = _h(As), _h(Az), _h(Bs), _h(Bz)
    lib().clove_oracle_gemm_int4(_ptr(Aq), _ptr(As_), _ptr(Az_), _ptr(Bq), _ptr(Bs_), _ptr(Bz_),
                                 _ptr(C.view(np.uint16)), M, N, K, r0, r1, nthreads)
    return C


def gemm_int4_refcompat(Aq, As, Bq_kn, Bs_kn, M, N, K, rows=None, nthreads=0):
    """What the reference gemm_int4 kernel computes (B packed along N)."""
    Aq = np.ascontiguousarray(Aq, np.uint8)
    Bq_kn = np.ascontiguousarray(Bq_kn, np.uint8)
    C = np.zeros((M, N), np.float16)
    r0, r1 = _rows(M, rows)
    As_, Bs_ = _h(As), _h(Bs_kn)
    lib().clove_oracle_gemm_int4_refcompat(_ptr(Aq), _ptr(As_), _ptr(Bq_kn), _ptr(Bs_),
                                           _ptr(C.view(np.uint16)), M, N, K, r0, r1, nthreads)
    return C


def rel_frobenius(x, ref) -> float:
    """||x - ref||_F / ||ref||_F in float64 (the north-star parity metric)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    return float(num / den) if den > 0 else float(num)


def quantize_int4(W):
    """(codes [rows,K/2] uint8, scales [rows,K/128] fp16, zeros [rows,K/128] fp16):
    this build's INT4 packing specification (min/max per 128-group) on the CPU."""
    W = np.ascontiguousarray(W, np.float16)
    rows, K = W.shape
    assert K % 128 == 0
    codes = np.zeros((rows, K // 2), np.uint8)
    scales = np.zeros((rows, K // 128), np.uint16)
    zeros = np.zeros((rows, K // 128), np.uint16)
    lib().clove_oracle_quantize_int4(_ptr(W.view(np.uint16)), rows, K, _ptr(codes), _ptr(scales),
                                     _ptr(zeros))
    return codes, scales.view(np.float16), zeros.view(np.float16)


def swiglu(X, Wg, Wu, rows=None, nthreads=0):
    """half(silu(X@Wg) * (X@Wu)) with fp32 accumulation (reference silu_f)."""
    X = np.ascontiguousarray(X, np.float16)
    Wg = np.ascontiguousarray(Wg, np.float16)
    Wu = np.ascontiguousarray(Wu, np.float16)
    M, K = X.shape
    assert Wg.shape == Wu.shape and Wg.shape[0] == K
    N = Wg.shape[1]
    out = np.zeros((M, N), np.float16)
    r0, r1 = _rows(M, rows)
    lib().clove_oracle_swiglu(_ptr(X.view(np.uint16)), _ptr(Wg.view(np.uint16)),
                              _ptr(Wu.view(np.uint16)), _ptr(out.view(np.uint16)), M, N, K, r0, r1,
                              nthreads)
    return out


def attention(Q, K, V, causal=True, scale=None, layout="bhsd", refcompat=False, nthreads=0):
    """O = softmax(scale * Q K^T [causal]) V in fp32, fp16 out: the reference's
    flash_attention_kernel (attention.cu:93-266) restated, 64-key blocks with its
    online softmax. layout "bhsd" [batch, heads, seq, D] or "bshd" [batch, seq,
    heads, D]; K/V may have fewer heads (head h reads kv head h // (H // Hkv)).
    refcompat=True keeps the reference's phantom zero-score keys that pad a ragged
    last block in non-causal attention."""
    Q = np.ascontiguousarray(Q, np.float16)
    K = np.ascontiguousarray(K, np.float16)
    V = np.ascontiguousarray(V, np.float16)
    if layout == "bhsd":
        B, H, S, D = Q.shape
        Hkv = K.shape[1]
    else:
        B, S, H, D = Q.shape
        Hkv = K.shape[2]
    assert K.shape == V.shape and H % Hkv == 0
    if scale is None:
        scale = 1.0 / D ** 0.5
    O = np.zeros_like(Q)
    lib().clove_oracle_attention(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), B, H, Hkv, S, D,
                                 float(scale), int(bool(causal)), 0 if layout == "bhsd" else 1,
                                 int(bool(refcompat)), nthreads)
    return O
