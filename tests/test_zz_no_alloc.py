"""clove_gemm_int8_noalloc through the C ABI: the int8 GEMM for callers that
cannot let a library allocate device memory (their HBM is reserved up front by
their own pools). Its zero-point sums live in a fixed array inside the library
instead of cudaMallocAsync scratch; its results must equal clove_gemm_int8's.

Collected last (file name) so that a run stopping at the first failure has
already run every other test; it passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest
import torch

from clove_compute_b200 import workloads as wl
from tests.gpu_util import dev, host, rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-3  # same bound as the int8 parity tests


def _call_noalloc(lib, A, B, C, M, N, K, sa, za, sb, zb):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.clove_gemm_int8_noalloc(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                                       ctypes.c_void_p(C.data_ptr()), M, N, K, sa, za, sb, zb,
                                       stream)


def test_noalloc_matches_allocating_entry_point(clove_lib, cuda):
    lib = clove_lib.lib()
    # Consecutive calls with different shapes and zero points: stale contents of
    # the shared array from one call must not leak into the next.
    cases = [(512, 256, 1024, 3, -7, 1), (300, 272, 512, 0, 5, 2), (1024, 64, 4096, -5, 0, 3),
             (512, 256, 1024, 9, 4, 4)]
    for M, N, K, za, zb, seed in cases:
        A, B, _, _ = wl.int8_operands(M, N, K, seed=seed)
        Ad, Bd = dev(A), dev(B)
        C_ref = host(clove_lib.gemm_int8(Ad, Bd, 0.01, za, 0.02, zb))
        C_new = torch.empty((M, N), dtype=torch.float16, device="cuda")
        rc = _call_noalloc(lib, Ad, Bd, C_new, M, N, K, 0.01, za, 0.02, zb)
        assert rc == 0, lib.clove_last_error_string()
        got = host(C_new)
        assert rel_fro(got, C_ref) < TOL
        np.testing.assert_array_equal(got.view(np.uint16), C_ref.view(np.uint16))
    assert clove_lib.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_array(clove_lib, cuda):
    lib = clove_lib.lib()
    M, N, K = 65536, 16, 16
    A = torch.zeros((16, K), dtype=torch.int8, device="cuda")  # never read: rejected first
    B = torch.zeros((K, N), dtype=torch.int8, device="cuda")
    C = torch.zeros((16, N), dtype=torch.float16, device="cuda")
    rc = _call_noalloc(lib, A, B, C, M, N, K, 1.0, 1, 1.0, 1)
    assert rc == clove_lib.CLOVE_ERR_UNSUPPORTED
    assert b"static scratch" in lib.clove_last_error_string()
