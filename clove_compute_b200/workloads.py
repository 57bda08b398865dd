"""Seeded synthetic inputs for the benchmark configurations.

The reference has no datasets for this path; every configuration is synthetic.
Generator: ``numpy.random.default_rng(seed)`` (PCG64), values drawn in a fixed
stream order -- A, then B, then scales, then zero points -- with these
distributions:

* fp16: A, B iid N(0,1)/sqrt(K), rounded to binary16.
* int8: A, B uniform integers in [-127, 127]; per-row A and per-column B fp32
  scales uniform in [0.001, 0.01].
* int4: codes uniform in [0, 15], K-packed two per byte (even k in the high
  nibble); per-128-group fp16 scales uniform in [0.005, 0.02] and integer zero
  points uniform in [0, 15] (stored as fp16), for both operands.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

GROUP = 128


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """[rows, K] codes 0..15 -> [rows, K/2] bytes, element 2j in the high nibble."""
    codes = np.asarray(codes, np.uint8)
    return ((codes[:, 0::2] << 4) | (codes[:, 1::2] & 0x0F)).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    packed = np.asarray(packed, np.uint8)
    out = np.empty((packed.shape[0], packed.shape[1] * 2), np.uint8)
    out[:, 0::2] = packed >> 4
    out[:, 1::2] = packed & 0x0F
    return out


def fp16_operands(M: int, N: int, K: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    s = np.float32(1.0 / np.sqrt(K))
    A = (rng.standard_normal((M, K), dtype=np.float32) * s).astype(np.float16)
    B = (rng.standard_normal((K, N), dtype=np.float32) * s).astype(np.float16)
    return A, B


def int8_operands(M: int, N: int, K: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    B = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    sA = rng.uniform(0.001, 0.01, size=M).astype(np.float32)
    sB = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
    return A, B, sA, sB


@dataclass
class Int4Operands:
    A_q: np.ndarray      # [M, K/2] uint8
    A_scale: np.ndarray  # [M, K/128] fp16
    A_zero: np.ndarray   # [M, K/128] fp16 (integer codes)
    B_q: np.ndarray      # [N, K/2] uint8
    B_scale: np.ndarray  # [N, K/128] fp16
    B_zero: np.ndarray   # [N, K/128] fp16
    M: int
    N: int
    K: int


def int4_operands(M: int, N: int, K: int, seed: int = 0) -> Int4Operands:
    assert K % GROUP == 0, "K must be a multiple of 128"
    rng = np.random.default_rng(seed)
    G = K // GROUP
    a_codes = rng.integers(0, 16, size=(M, K), dtype=np.uint8)
    b_codes = rng.integers(0, 16, size=(N, K), dtype=np.uint8)
    sA = rng.uniform(0.005, 0.02, size=(M, G)).astype(np.float16)
    sB = rng.uniform(0.005, 0.02, size=(N, G)).astype(np.float16)
    zA = rng.integers(0, 16, size=(M, G)).astype(np.float16)
    zB = rng.integers(0, 16, size=(N, G)).astype(np.float16)
    return Int4Operands(pack_int4(a_codes), sA, zA, pack_int4(b_codes), sB, zB, M, N, K)


# The BASELINE configurations (M x N x K, row-major C[M,N] = A[M,K] . B[K,N]).
CONFIGS = {
    "fp16_1024": dict(dtype="fp16", M=1024, N=1024, K=1024),
    "int4_decode": dict(dtype="int4", M=4096, N=1, K=4096),
    "int8_batch32": dict(dtype="int8", M=4096, N=32, K=4096),
    "fp16_ffn_up": dict(dtype="fp16", M=11008, N=2048, K=4096),
    "fp16_ffn_down": dict(dtype="fp16", M=4096, N=2048, K=11008),
    "int4_8192": dict(dtype="int4", M=8192, N=8192, K=8192),
}
