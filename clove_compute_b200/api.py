"""Tensor-level host API: the reference's GEMM functions over torch CUDA tensors.

Each function mirrors one entry point of the reference header
``include/clove/kernels/gemm.cuh`` (same names, argument order and meaning,
row-major layouts) and calls the matching ``clove_*`` C function. Shapes are
taken from the tensors; errors raise :class:`CloveError` instead of exiting.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib, INT4_GROUP_SIZE


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    if isinstance(stream, torch.cuda.Stream):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _need(t: torch.Tensor, name: str, dtype, ndim=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (row-major)")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")


def version() -> str:
    return lib().clove_version().decode()


def gemm_fp16(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor | None = None,
              alpha: float = 1.0, beta: float = 0.0, stream=None) -> torch.Tensor:
    """C = alpha * A @ B + beta * C; A [M,K], B [K,N], C [M,N] fp16 (gemm.cuh:41-49)."""
    _need(A, "A", torch.float16, 2)
    _need(B, "B", torch.float16, 2)
    M, K = A.shape
    K2, N = B.shape
    if K2 != K:
        raise ValueError(f"inner dimensions differ: A {tuple(A.shape)} B {tuple(B.shape)}")
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device=A.device)
        if beta != 0.0:
            raise ValueError("beta != 0 needs C")
    _need(C, "C", torch.float16, 2)
    if tuple(C.shape) != (M, N):
        raise ValueError(f"C must be {(M, N)}")
    check(lib().clove_gemm_fp16(_ptr(A), _ptr(B), _ptr(C), M, N, K, float(alpha), float(beta),
                                _stream(stream)))
    return C


def gemm_fp16_batched(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor | None = None,
                      alpha: float = 1.0, beta: float = 0.0, stream=None) -> torch.Tensor:
    """Per-batch C[b] = alpha * A[b] @ B[b] + beta * C[b] (gemm.cuh:93-101)."""
    _need(A, "A", torch.float16, 3)
    _need(B, "B", torch.float16, 3)
    batch, M, K = A.shape
    if B.shape[0] != batch or B.shape[1] != K:
        raise ValueError("A [b,M,K] and B [b,K,N] disagree")
    N = B.shape[2]
    if C is None:
        C = torch.empty((batch, M, N), dtype=torch.float16, device=A.device)
    _need(C, "C", torch.float16, 3)
    check(lib().clove_gemm_fp16_batched(_ptr(A), _ptr(B), _ptr(C), batch, M, N, K, float(alpha),
                                        float(beta), _stream(stream)))
    return C


def gemm_int8(A_q: torch.Tensor, B_q: torch.Tensor, A_scale: float, A_zero: int,
              B_scale: float, B_zero: int, C: torch.Tensor | None = None,
              stream=None) -> torch.Tensor:
    """C = (A_q - A_zero)*A_scale @ (B_q - B_zero)*B_scale; int8 [M,K] x [K,N] (gemm.cuh:55-65)."""
    _need(A_q, "A_q", torch.int8, 2)
    _need(B_q, "B_q", torch.int8, 2)
    M, K = A_q.shape
    K2, N = B_q.shape
    if K2 != K:
        raise ValueError("inner dimensions differ")
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device=A_q.device)
    _need(C, "C", torch.float16, 2)
    check(lib().clove_gemm_int8(_ptr(A_q), _ptr(B_q), _ptr(C), M, N, K, float(A_scale),
                                int(A_zero), float(B_scale), int(B_zero), _stream(stream)))
    return C


def gemm_int8_rowcol(A_q: torch.Tensor, B_q: torch.Tensor, A_row_scale: torch.Tensor,
                     B_col_scale: torch.Tensor, C: torch.Tensor | None = None,
                     stream=None) -> torch.Tensor:
    """C[m,n] = float(sum_k A_q B_q) * A_row_scale[m] * B_col_scale[n] (fp32 scales)."""
    _need(A_q, "A_q", torch.int8, 2)
    _need(B_q, "B_q", torch.int8, 2)
    M, K = A_q.shape
    K2, N = B_q.shape
    if K2 != K:
        raise ValueError("inner dimensions differ")
    _need(A_row_scale, "A_row_scale", torch.float32, 1)
    _need(B_col_scale, "B_col_scale", torch.float32, 1)
    if A_row_scale.numel() != M or B_col_scale.numel() != N:
        raise ValueError("scale vector length")
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device=A_q.device)
    _need(C, "C", torch.float16, 2)
    check(lib().clove_gemm_int8_rowcol(_ptr(A_q), _ptr(B_q), _ptr(C), M, N, K, _ptr(A_row_scale),
                                       _ptr(B_col_scale), _stream(stream)))
    return C


def _int4_shapes(A_q, A_scale, A_zero, B_q, B_scale, B_zero):
    _need(A_q, "A_q", torch.uint8, 2)
    _need(B_q, "B_q", torch.uint8, 2)
    M, KB = A_q.shape
    N, KB2 = B_q.shape
    if KB != KB2:
        raise ValueError("A_q [M,K/2] and B_q [N,K/2] disagree on K")
    K = 2 * KB
    G = K // INT4_GROUP_SIZE
    for t, name, rows in ((A_scale, "A_scale", M), (A_zero, "A_zero", M),
                          (B_scale, "B_scale", N), (B_zero, "B_zero", N)):
        _need(t, name, torch.float16, 2)
        if tuple(t.shape) != (rows, G):
            raise ValueError(f"{name} must be {(rows, G)}")
    return M, N, K


def gemm_int4(A_q: torch.Tensor, A_scale: torch.Tensor, A_zero: torch.Tensor,
              B_q: torch.Tensor, B_scale: torch.Tensor, B_zero: torch.Tensor,
              C: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Group-wise INT4 GEMM (gemm.cuh:77-87), K-packed on both operands:
    A_q [M,K/2], A_scale/A_zero [M,K/128]; B_q [N,K/2], B_scale/B_zero [N,K/128] -> C [M,N]."""
    M, N, K = _int4_shapes(A_q, A_scale, A_zero, B_q, B_scale, B_zero)
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device=A_q.device)
    _need(C, "C", torch.float16, 2)
    check(lib().clove_gemm_int4(_ptr(A_q), _ptr(A_scale), _ptr(A_zero), _ptr(B_q), _ptr(B_scale),
                                _ptr(B_zero), _ptr(C), M, N, K, _stream(stream)))
    return C


def debug_int8_acc(A_q: torch.Tensor, B_q: torch.Tensor, A_zero: int = 0, B_zero: int = 0,
                   stream=None) -> torch.Tensor:
    """Exact int32 accumulators sum_k (A-za)(B-zb) through the production kernels."""
    _need(A_q, "A_q", torch.int8, 2)
    _need(B_q, "B_q", torch.int8, 2)
    M, K = A_q.shape
    N = B_q.shape[1]
    acc = torch.empty((M, N), dtype=torch.int32, device=A_q.device)
    check(lib().clove_debug_int8_acc(_ptr(A_q), _ptr(B_q), _ptr(acc), M, N, K, int(A_zero),
                                     int(B_zero), _stream(stream)))
    return acc


def debug_int4_group_acc(A_q, A_scale, A_zero, B_q, B_scale, B_zero, stream=None):
    """(C, G): C as gemm_int4 and the exact int32 group accumulators G [M,N,K/128]."""
    M, N, K = _int4_shapes(A_q, A_scale, A_zero, B_q, B_scale, B_zero)
    C = torch.empty((M, N), dtype=torch.float16, device=A_q.device)
    G = torch.empty((M, N, K // INT4_GROUP_SIZE), dtype=torch.int32, device=A_q.device)
    check(lib().clove_debug_int4_group_acc(_ptr(A_q), _ptr(A_scale), _ptr(A_zero), _ptr(B_q),
                                           _ptr(B_scale), _ptr(B_zero), _ptr(C), _ptr(G), M, N, K,
                                           _stream(stream)))
    return C, G


def swiglu_fused(X: torch.Tensor, W_gate: torch.Tensor, W_up: torch.Tensor,
                 out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """out = silu(X @ W_gate) * (X @ W_up): X [T, H], W_gate / W_up [H, I] fp16
    (activations.cuh:37-46 of the reference, declared there but never defined)."""
    _need(X, "X", torch.float16, 2)
    _need(W_gate, "W_gate", torch.float16, 2)
    _need(W_up, "W_up", torch.float16, 2)
    T, H = X.shape
    if W_gate.shape[0] != H or W_up.shape != W_gate.shape:
        raise ValueError("X [T,H], W_gate and W_up [H,I] disagree")
    inter = W_gate.shape[1]
    if out is None:
        out = torch.empty((T, inter), dtype=torch.float16, device=X.device)
    _need(out, "out", torch.float16, 2)
    check(lib().clove_swiglu_fused(_ptr(X), _ptr(W_gate), _ptr(W_up), _ptr(out), T, H, inter,
                                   _stream(stream)))
    return out


def flash_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool = True,
                    scale: float | None = None, layout: str = "bhsd", O: torch.Tensor | None = None,
                    stream=None) -> torch.Tensor:
    """O = softmax(scale * Q K^T [causal]) V on the tensor cores (attention.cuh:44-56).

    layout "bhsd": Q, K, V [batch, heads, seq, 128] (the reference's flash_attention);
    "bshd": [batch, seq, heads, 128] (its runtime's projection outputs). K and V may
    have fewer heads than Q (grouped-query attention). scale defaults to 1/sqrt(128)."""
    for t, n in ((Q, "Q"), (K, "K"), (V, "V")):
        _need(t, n, torch.float16, 4)
    if layout not in ("bhsd", "bshd"):
        raise ValueError("layout must be 'bhsd' or 'bshd'")
    if layout == "bhsd":
        B, H, S, D = Q.shape
        Hkv = K.shape[1]
        kv_shape = (B, Hkv, S, D)
    else:
        B, S, H, D = Q.shape
        Hkv = K.shape[2]
        kv_shape = (B, S, Hkv, D)
    if tuple(K.shape) != kv_shape or tuple(V.shape) != kv_shape:
        raise ValueError(f"K and V must be {kv_shape}")
    if O is None:
        O = torch.empty_like(Q)
    _need(O, "O", torch.float16, 4)
    if scale is None:
        scale = 1.0 / D ** 0.5
    check(lib().clove_flash_attention(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), B, H, Hkv, S, D,
                                      float(scale), int(bool(causal)),
                                      0 if layout == "bhsd" else 1, _stream(stream)))
    return O


def quantize_int4(W: torch.Tensor, stream=None):
    """Pack fp16 weights W [rows, K] (K % 128 == 0) into the INT4 layout gemm_int4
    reads: (codes [rows, K/2] uint8, scales [rows, K/128] fp16, zeros [rows, K/128] fp16).
    Asymmetric min/max per 128-group; see include/clove/capi.h for the rounding rules."""
    _need(W, "W", torch.float16, 2)
    rows, K = W.shape
    if K % INT4_GROUP_SIZE:
        raise ValueError("K must be a multiple of 128")
    codes = torch.empty((rows, K // 2), dtype=torch.uint8, device=W.device)
    scales = torch.empty((rows, K // INT4_GROUP_SIZE), dtype=torch.float16, device=W.device)
    zeros = torch.empty((rows, K // INT4_GROUP_SIZE), dtype=torch.float16, device=W.device)
    check(lib().clove_quantize_int4(_ptr(W), rows, K, _ptr(codes), _ptr(scales), _ptr(zeros),
                                    _stream(stream)))
    return codes, scales, zeros


def debug_stream_read(src, out, stream=None) -> None:
    """Bare read of every byte of the contiguous CUDA tensor `src` (a multiple of 16
    bytes), nothing computed: the HBM floor of one launch of that size. `out` is an
    int32 CUDA tensor of at least one element (written only for one specific value)."""
    if not src.is_contiguous() or src.numel() * src.element_size() % 16:
        raise ValueError("src must be contiguous and a multiple of 16 bytes")
    check(lib().clove_debug_stream_read(_ptr(src), src.numel() * src.element_size(), _ptr(out),
                                        _stream(stream)))


def debug_exp2_poly(x: torch.Tensor, stream=None) -> torch.Tensor:
    """2^x through the attention softmax's FMA-pipe polynomial exponential (an even
    number of fp32 CUDA elements)."""
    _need(x, "x", torch.float32, 1)
    if x.numel() % 2:
        raise ValueError("x needs an even number of elements")
    y = torch.empty_like(x)
    check(lib().clove_debug_exp2_poly(_ptr(x), _ptr(y), x.numel(), _stream(stream)))
    return y


def debug_peer_wait_timeout(words: torch.Tensor, timeout_ns: int, stream=None) -> None:
    """Runs the N-split's cross-rank completion wait for a two-rank group whose
    other rank never signals (``words``: 8 int64 of device scratch); the bounded
    wait runs out after ``timeout_ns`` and records device error 1."""
    _need(words, "words", torch.int64, 1)
    if words.numel() < 8:
        raise ValueError("words needs 8 elements")
    check(lib().clove_debug_peer_wait_timeout(_ptr(words), int(timeout_ns), _stream(stream)))


def debug_stream_k_plan(tiles: int, pairs: int, kb_total: int, force: int = 0) -> dict:
    """The CTA-pair kernel's stream-K schedule for `tiles` output tiles of kb_total
    K blocks on `pairs` CTA pairs (host only; force 0 auto, 1 never, 2 always)."""
    out = (ctypes.c_int * 4)()
    check(lib().clove_debug_stream_k_plan(int(tiles), int(pairs), int(kb_total), int(force),
                                          ctypes.cast(out, ctypes.c_void_p)))
    return {"dp_tiles": out[0], "sk_tiles": out[1], "max_contrib": out[2], "pairs": out[3]}


def set_dispatch_override(path: int = 0, bn: int = 0, split: int = 0) -> None:
    """Force a kernel family (tests): path 0 auto, 1 tensor core, 2 GEMV, 3 SIMT."""
    check(lib().clove_set_dispatch_override(int(path), int(bn), int(split)))


def set_weight_prefetch(enable: bool) -> None:
    """Let decode kernels stream the weight operand before the previous kernel on the
    stream finishes (only when no in-flight kernel writes that operand)."""
    check(lib().clove_set_weight_prefetch(int(bool(enable))))


def describe_dispatch(dtype: str, M: int, N: int, K: int) -> str:
    code = {"fp16": 0, "int8": 1, "int4": 2, "swiglu": 3}[dtype]
    buf = ctypes.create_string_buffer(128)
    check(lib().clove_describe_dispatch(code, M, N, K, buf, len(buf)))
    return buf.value.decode()


def device_error() -> int:
    """Reads and clears the device-side error word (synchronises)."""
    v = ctypes.c_int(0)
    check(lib().clove_get_device_error(ctypes.byref(v)))
    return v.value
