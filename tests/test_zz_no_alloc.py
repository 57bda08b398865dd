"""clove_gemm_int8_noalloc through the C ABI: the int8 GEMM for callers that
cannot let a library allocate device memory (their HBM is reserved up front by
their own pools). Its zero-point sums live in a fixed array inside the library
instead of cudaMallocAsync scratch; its results must equal clove_gemm_int8's.

Collected last (file name) so that a run stopping at the first failure has
already run every other test; it passes alone in a fresh process too. It also
measures the promise itself: no device memory is allocated by the call."""
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


class _DefaultPool:
    """The device's default memory pool (where cudaMallocAsync scratch comes from),
    read through the driver API: its used-memory high-water mark can be reset and
    read back around a call."""

    def __init__(self):
        from cuda.bindings import driver as drv
        self.drv = drv
        self._ok(drv.cuInit(0))
        dev = self._ok(drv.cuDeviceGet(torch.cuda.current_device()))
        self.pool = self._ok(drv.cuDeviceGetDefaultMemPool(dev))
        self.attr = drv.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_HIGH

    def _ok(self, res):
        err, *rest = res if isinstance(res, tuple) else (res,)
        assert int(err) == 0, f"driver call failed: {err}"
        return rest[0] if rest else None

    def reset_high(self):
        self._ok(self.drv.cuMemPoolSetAttribute(self.pool, self.attr, self.drv.cuuint64_t(0)))

    def high(self) -> int:
        return int(self._ok(self.drv.cuMemPoolGetAttribute(self.pool, self.attr)))


def test_noalloc_allocates_nothing(clove_lib, cuda):
    """The entry point's promise, measured: around a zero-point call on the
    tensor-core path (one-SM tiles and CTA pairs), neither the default memory pool's
    used-memory high-water mark nor torch's allocator moves, while the allocating
    entry point on the same shape does raise the high-water mark."""
    lib = clove_lib.lib()
    pool = _DefaultPool()
    for M, N, K in [(512, 256, 1024), (2048, 2048, 1024)]:
        A, B, _, _ = wl.int8_operands(M, N, K, seed=M)
        Ad, Bd = dev(A), dev(B)
        C = torch.empty((M, N), dtype=torch.float16, device="cuda")
        assert _call_noalloc(lib, Ad, Bd, C, M, N, K, 0.01, 3, 0.02, -2) == 0  # first call: set-up
        torch.cuda.synchronize()
        torch_before = torch.cuda.memory_allocated()
        pool.reset_high()
        base = pool.high()
        for _ in range(2):
            rc = _call_noalloc(lib, Ad, Bd, C, M, N, K, 0.01, 3, 0.02, -2)
            assert rc == 0, lib.clove_last_error_string()
        torch.cuda.synchronize()
        assert pool.high() == base, (M, N, K, pool.high(), base)
        assert torch.cuda.memory_allocated() == torch_before
        # Control: the allocating entry point takes its sums from that pool.
        clove_lib.gemm_int8(Ad, Bd, 0.01, 3, 0.02, -2)
        torch.cuda.synchronize()
        assert pool.high() >= base + 4 * (M + N), (pool.high(), base)
    assert clove_lib.device_error() == 0


def test_noalloc_matches_allocating_entry_point(clove_lib, cuda):
    lib = clove_lib.lib()
    # Consecutive calls with different shapes and zero points: stale contents of
    # the shared array from one call must not leak into the next. (2048, 2048, 1024)
    # runs on CTA pairs, the others on one-SM tiles.
    cases = [(512, 256, 1024, 3, -7, 1), (300, 272, 512, 0, 5, 2), (1024, 64, 4096, -5, 0, 3),
             (2048, 2048, 1024, 6, -3, 5), (512, 256, 1024, 9, 4, 4)]
    assert clove_lib.describe_dispatch("int8", 2048, 2048, 1024).startswith("tc2_int8")
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
