"""INT8 parity on the GPU: int32 accumulators bit-exact against the oracle
(clove_debug_int8_acc runs the production kernels with a raw int32 epilogue),
fp16 C within tolerance (bit-exact in practice: same fp32 epilogue order)."""
import numpy as np
import pytest

from clove_compute_b200 import workloads as wl
from tests.gpu_util import dev, host, rel_fro

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _reset(clove_lib):
    yield
    clove_lib.set_dispatch_override(0, 0, 0)


def _acc(cc, oracle, M, N, K, za=0, zb=0, path=0, bn=0, split=0, seed=0):
    A, B, _, _ = wl.int8_operands(M, N, K, seed=seed)
    cc.set_dispatch_override(path, bn, split)
    got = host(cc.debug_int8_acc(dev(A), dev(B), za, zb))
    ref = oracle.int8_acc(A, B, za, zb)
    np.testing.assert_array_equal(got, ref)
    assert cc.device_error() == 0


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_tc_acc_exact(clove_lib, oracle_mod, cuda, bn):
    _acc(clove_lib, oracle_mod, 384, 512, 640, path=1, bn=bn, split=1, seed=bn)


@pytest.mark.parametrize("bn,split", [(32, 4), (64, 2), (32, 8)])
def test_tc_split_acc_exact(clove_lib, oracle_mod, cuda, bn, split):
    _acc(clove_lib, oracle_mod, 256, 64, 4096, path=1, bn=bn, split=split, seed=split)


@pytest.mark.parametrize("M", [1, 37, 100])
def test_tc_split_live_rows_exact(clove_lib, oracle_mod, cuda, M):
    """Split-K clusters exchange only the rows below M; int32 stays exact."""
    for bn, split in [(32, 4), (64, 8), (128, 2), (128, 4)]:
        _acc(clove_lib, oracle_mod, M, 256, 4096, za=3, zb=-5, path=1, bn=bn, split=split,
             seed=M + split)


def test_decode_long_k_plan_exact(clove_lib, oracle_mod, cuda):
    """One live row with K = 11008: 128-column tiles over 4-CTA clusters, exact."""
    assert clove_lib.describe_dispatch("int8", 1, 4096, 11008) == "tc_int8 bn=128 split=4"
    _acc(clove_lib, oracle_mod, 1, 4096, 11008, seed=11)


def test_tc_ragged_and_zero_points(clove_lib, oracle_mod, cuda):
    _acc(clove_lib, oracle_mod, 200, 48, 160, seed=1)
    _acc(clove_lib, oracle_mod, 300, 272, 512, za=3, zb=-7, seed=2)
    _acc(clove_lib, oracle_mod, 256, 32, 4096, za=-128, zb=127, seed=3)


@pytest.mark.parametrize("N", [1, 2, 5, 8])
def test_gemv_acc_exact(clove_lib, oracle_mod, cuda, N):
    _acc(clove_lib, oracle_mod, 1000, N, 4096, seed=N)
    _acc(clove_lib, oracle_mod, 77, N, 48, za=5, zb=-3, seed=N)


def test_simt_acc_exact(clove_lib, oracle_mod, cuda):
    _acc(clove_lib, oracle_mod, 70, 20, 100, za=2, zb=1)


def test_config3_batch32_rowcol(clove_lib, oracle_mod, cuda):
    """M=K=4096, N=32, per-row / per-column fp32 scales."""
    M, N, K = 4096, 32, 4096
    A, B, sA, sB = wl.int8_operands(M, N, K, seed=0)
    C = host(clove_lib.gemm_int8_rowcol(dev(A), dev(B), dev(sA), dev(sB)))
    ref = oracle_mod.gemm_int8_rowcol(A, B, sA, sB)
    assert rel_fro(C, ref) < 1e-3
    assert (C.view(np.uint16) != ref.view(np.uint16)).mean() < 1e-3
    acc = host(clove_lib.debug_int8_acc(dev(A), dev(B)))
    np.testing.assert_array_equal(acc, oracle_mod.int8_acc(A, B))


def test_per_tensor_reference_signature(clove_lib, oracle_mod, cuda):
    M, N, K = 512, 256, 1024
    A, B, _, _ = wl.int8_operands(M, N, K, seed=7)
    for (za, zb) in [(0, 0), (4, -9)]:
        C = host(clove_lib.gemm_int8(dev(A), dev(B), 0.01, za, 0.02, zb))
        ref = oracle_mod.gemm_int8(A, B, 0.01, za, 0.02, zb)
        assert rel_fro(C, ref) < 1e-3
    assert clove_lib.device_error() == 0


@pytest.mark.parametrize("sk", [0, 2])
@pytest.mark.parametrize("M,N,K", [(512, 512, 1024), (300, 272, 512), (768, 512, 4096)])
def test_tc_cta_pair_rowcol(clove_lib, oracle_mod, cuda, M, N, K, sk):
    """int8 on CTA pairs (kind::i8, cta_group::2): C bit-identical in practice; with
    the stream-K schedule forced (sk=2) the int32 partials of a tile's K pieces are
    summed exactly, so C stays bit-identical too."""
    A, B, sA, sB = wl.int8_operands(M, N, K, seed=M)
    clove_lib.set_dispatch_override(4, 0, sk)
    C = host(clove_lib.gemm_int8_rowcol(dev(A), dev(B), dev(sA), dev(sB)))
    ref = oracle_mod.gemm_int8_rowcol(A, B, sA, sB)
    assert rel_fro(C, ref) < 1e-3
    assert (C.view(np.uint16) != ref.view(np.uint16)).mean() < 1e-3
    C = host(clove_lib.gemm_int8(dev(A), dev(B), 0.01, 3, 0.02, -4))
    assert rel_fro(C, oracle_mod.gemm_int8(A, B, 0.01, 3, 0.02, -4)) < 1e-3
    assert clove_lib.device_error() == 0
