"""INT4 parity on the GPU: per-group int32 accumulators G bit-exact against the
oracle (clove_debug_int4_group_acc), C within the 1e-2 relative Frobenius
contract of the fp32 oracle (tight bound 2e-3)."""
import numpy as np
import pytest

from clove_compute_b200 import workloads as wl
from tests.gpu_util import dev, host, rel_fro

pytestmark = pytest.mark.gpu
TOL_TIGHT = 2e-3


@pytest.fixture(autouse=True)
def _reset(clove_lib):
    yield
    clove_lib.set_dispatch_override(0, 0, 0)


def _ops_dev(op):
    return (dev(op.A_q), dev(op.A_scale), dev(op.A_zero), dev(op.B_q), dev(op.B_scale),
            dev(op.B_zero))


def _check(cc, oracle, M, N, K, path=0, seed=0, check_g=True):
    op = wl.int4_operands(M, N, K, seed=seed)
    if path != 2:
        cc.set_dispatch_override(path, 0, 0)
    args = _ops_dev(op)
    C = host(cc.gemm_int4(*args))
    ref = oracle.gemm_int4(op.A_q, op.A_scale, op.A_zero, op.B_q, op.B_scale, op.B_zero, K)
    err = rel_fro(C, ref)
    assert err < 1e-2 and err < TOL_TIGHT, err
    if check_g:
        C2, G = cc.debug_int4_group_acc(*args)
        Gref = oracle.int4_group_acc(op.A_q, op.A_zero, op.B_q, op.B_zero, K)
        np.testing.assert_array_equal(host(G), Gref)
        assert rel_fro(host(C2), ref) < TOL_TIGHT
    assert cc.device_error() == 0


def test_config2_decode_gemv(clove_lib, oracle_mod, cuda):
    """weights A [4096, 4096] int4, activations B with N = 1."""
    _check(clove_lib, oracle_mod, 4096, 1, 4096)


@pytest.mark.parametrize("M", [5, 9000, 16384])
def test_decode_row_counts(clove_lib, oracle_mod, cuda, M):
    """Decode blocks of a few rows per CTA up to several 32-row rounds per CTA."""
    _check(clove_lib, oracle_mod, M, 1, 2048, seed=M, check_g=False)


@pytest.mark.parametrize("N", [2, 3, 4, 8])
def test_gemv_small_n(clove_lib, oracle_mod, cuda, N):
    _check(clove_lib, oracle_mod, 1000, N, 2048, seed=N)


@pytest.mark.parametrize("M,K", [(4096, 4096), (2368, 2048), (5000, 3200)])
def test_gemv_two_vectors_several_ctas(clove_lib, oracle_mod, cuda, M, K):
    """Two decode vectors from 2 x 148 x 8 rows on: four CTAs of 2 x 4 warps per SM."""
    assert clove_lib.describe_dispatch("int4", M, 2, K) == "gemv_int4 (ldg 4 CTAs/SM of 2x4 warps)"
    _check(clove_lib, oracle_mod, M, 2, K, seed=M + K)


@pytest.mark.parametrize("K", [128, 384, 8192, 12288])
def test_gemv_k_sizes(clove_lib, oracle_mod, cuda, K):
    _check(clove_lib, oracle_mod, 300, 1, K, seed=K)


@pytest.mark.parametrize("M,K", [(4096, 11008), (9000, 11008), (1000, 7040), (300, 3200),
                                 (2400, 8192), (2400, 12288), (2368, 3200), (2367, 4096)])
def test_gemv_partial_windows(clove_lib, oracle_mod, cuda, M, K):
    """K a multiple of 128 but not of 1024 (the Llama-7B down projection, K = 11008:
    11 windows of 1024 codes, the last one 768): the direct-load decode kernel masks
    the lanes past K. From 2 x 148 x 8 rows on, several CTAs per SM run with one
    window per lane: four of 2 x 4 warps up to 4096 codes, two of 1 x 12 warps
    beyond (8 windows of 12 used at K = 8192, all 12 at 12288; M = 9000: several
    rounds per CTA); below it one CTA of 4 x 4 warps per SM, with 3 windows per
    lane in 4-row rounds at M = 1000."""
    assert clove_lib.describe_dispatch("int4", M, 1, K).startswith("gemv_int4")
    _check(clove_lib, oracle_mod, M, 1, K, seed=M + K)


@pytest.mark.parametrize("M", [1, 3, 8])
def test_gemv_small_m_transposed(clove_lib, oracle_mod, cuda, M):
    _check(clove_lib, oracle_mod, M, 600, 1024, seed=M)


def test_large_shape(clove_lib, oracle_mod, cuda):
    _check(clove_lib, oracle_mod, 256, 192, 1024, seed=5)


@pytest.mark.parametrize("M,N,K", [(128, 128, 1024), (256, 384, 2048), (300, 136, 3072),
                                   (1000, 200, 1024)])
def test_tc_int4_exact_groups(clove_lib, oracle_mod, cuda, M, N, K):
    """tcgen05 kind::i8 path: every group accumulator bit-exact, C within tolerance."""
    assert clove_lib.describe_dispatch("int4", M, N, K).startswith("tc_int4")
    _check(clove_lib, oracle_mod, M, N, K, seed=M + N)


@pytest.mark.parametrize("M,N,K", [(128, 128, 384), (256, 136, 11008), (130, 256, 1152),
                                   (4096, 128, 11008)])
def test_tc_int4_any_group_count(clove_lib, oracle_mod, cuda, M, N, K):
    """K a multiple of 128 but not of 1024 (e.g. the Llama-7B down projection's
    K = 11008, 86 groups): the tensor-core kernel reads scales and zero points
    directly instead of in 8-group TMA boxes; every group accumulator bit-exact."""
    assert clove_lib.describe_dispatch("int4", M, N, K).startswith("tc_int4")
    _check(clove_lib, oracle_mod, M, N, K, seed=K + M, check_g=(M * N * K <= 256 * 256 * 11008))


def test_tc_int4_unaligned_metadata(clove_lib, oracle_mod, cuda):
    """Scales and zero points at 2-byte (not 16-byte) aligned addresses, K % 1024 == 0:
    the direct-load variant again, same exact G."""
    import torch
    M, N, K = 256, 256, 2048
    op = wl.int4_operands(M, N, K, seed=21)

    def off(a):  # the same values one fp16 element past a 16-byte boundary
        buf = torch.zeros(a.size + 8, dtype=torch.float16, device="cuda")
        v = buf[1:1 + a.size].view(a.shape)
        v.copy_(torch.from_numpy(np.ascontiguousarray(a)))
        return v

    args = (dev(op.A_q), off(op.A_scale), off(op.A_zero), dev(op.B_q), off(op.B_scale),
            off(op.B_zero))
    assert args[1].data_ptr() % 16 != 0
    C2, G = clove_lib.debug_int4_group_acc(*args)
    Gref = oracle_mod.int4_group_acc(op.A_q, op.A_zero, op.B_q, op.B_zero, K)
    np.testing.assert_array_equal(host(G), Gref)
    ref = oracle_mod.gemm_int4(op.A_q, op.A_scale, op.A_zero, op.B_q, op.B_scale, op.B_zero, K)
    assert rel_fro(host(clove_lib.gemm_int4(*args)), ref) < TOL_TIGHT
    assert clove_lib.device_error() == 0


def test_tc_int4_config5_rows(clove_lib, oracle_mod, cuda):
    """BASELINE config 5 shape (8192^3) on the tensor-core path, checked on a row sample
    against the oracle (the full oracle product takes minutes on the host)."""
    M = N = K = 8192
    op = wl.int4_operands(M, N, K, seed=0)
    C = host(clove_lib.gemm_int4(*_ops_dev(op)))
    rows = (0, 64)
    ref = oracle_mod.gemm_int4(op.A_q, op.A_scale, op.A_zero, op.B_q, op.B_scale, op.B_zero, K,
                               rows=rows)
    assert rel_fro(C[rows[0]:rows[1]], ref[rows[0]:rows[1]]) < TOL_TIGHT
    last = (M - 64, M)
    ref = oracle_mod.gemm_int4(op.A_q, op.A_scale, op.A_zero, op.B_q, op.B_scale, op.B_zero, K,
                               rows=last)
    assert rel_fro(C[last[0]:], ref[last[0]:]) < TOL_TIGHT
    assert np.isfinite(C.astype(np.float32)).all()


def test_simt_path(clove_lib, oracle_mod, cuda):
    _check(clove_lib, oracle_mod, 40, 24, 512, path=3, seed=6)


def test_k_not_multiple_of_group_rejected(clove_lib, cuda):
    import torch
    from clove_compute_b200 import CloveError
    M, N, K = 4, 4, 192
    z = lambda r: torch.zeros((r, 1), dtype=torch.float16, device="cuda")
    with pytest.raises((CloveError, ValueError)):
        clove_lib.gemm_int4(torch.zeros((M, K // 2), dtype=torch.uint8, device="cuda"), z(M), z(M),
                            torch.zeros((N, K // 2), dtype=torch.uint8, device="cuda"), z(N), z(N))


@pytest.mark.parametrize("prefetch", [False, True])
def test_decode_back_to_back_ordering(clove_lib, oracle_mod, cuda, prefetch):
    """Consecutive decode calls on one stream with programmatic dependent launch:
    each call must see the activation vector the preceding kernel just wrote, and
    each output must match the oracle (with and without weight prefetch)."""
    import torch
    M, K = 4096, 4096
    ops = [wl.int4_operands(M, 1, K, seed=s) for s in range(4)]
    Ad = [(dev(o.A_q), dev(o.A_scale), dev(o.A_zero)) for o in ops]
    Bsrc = [(dev(o.B_q), dev(o.B_scale), dev(o.B_zero)) for o in ops]
    Bq = torch.empty_like(Bsrc[0][0]); Bs = torch.empty_like(Bsrc[0][1]); Bz = torch.empty_like(Bsrc[0][2])
    outs = [torch.empty((M, 1), dtype=torch.float16, device="cuda") for _ in ops]
    clove_lib.set_weight_prefetch(prefetch)
    try:
        for rep in range(3):
            for i in range(len(ops)):
                Bq.copy_(Bsrc[i][0]); Bs.copy_(Bsrc[i][1]); Bz.copy_(Bsrc[i][2])
                clove_lib.gemm_int4(*Ad[i], Bq, Bs, Bz, outs[i])
        torch.cuda.synchronize()
    finally:
        clove_lib.set_weight_prefetch(False)
    for i, o in enumerate(ops):
        ref = oracle_mod.gemm_int4(o.A_q, o.A_scale, o.A_zero, o.B_q, o.B_scale, o.B_zero, K)
        assert rel_fro(host(outs[i]), ref) < TOL_TIGHT
    assert clove_lib.device_error() == 0


@pytest.mark.parametrize("N,K", [(1, 4096), (2, 4096), (1, 8192), (1, 1024)])
def test_bulk_copy_decode_path(clove_lib, oracle_mod, cuda, N, K):
    """The shared-memory ring variant of the decode GEMV (override path 2, bn 2)."""
    clove_lib.set_dispatch_override(2, 2, 0)
    _check(clove_lib, oracle_mod, 1000, N, K, path=2, seed=N + K, check_g=False)


def test_register_gemv_path(clove_lib, oracle_mod, cuda):
    """The register-resident GEMV (used when the bulk-copy kernel does not apply)."""
    clove_lib.set_dispatch_override(2, 1, 0)
    _check(clove_lib, oracle_mod, 4096, 1, 4096, path=2, seed=3, check_g=False)


@pytest.mark.gpu
def test_stream_read_hook(clove_lib, cuda):
    """The bare-read measurement hook runs on any 16-byte multiple and rejects others."""
    import torch
    buf = torch.ones(1 << 20, dtype=torch.uint8, device="cuda")
    sink = torch.zeros(4, dtype=torch.int32, device="cuda")
    clove_lib.debug_stream_read(buf, sink)
    torch.cuda.synchronize()
    assert int(sink[0]) == 0  # XOR of an even number of equal words is 0, not the sentinel
    with pytest.raises(ValueError):
        clove_lib.debug_stream_read(buf[:17], sink)


def test_tc_int4_extreme_codes_exact(clove_lib, oracle_mod, cuda):
    """Largest |G|: every code 15 against zero point 0 on one operand and code 0
    against zero point 15 on the other (each product -225, G = -28800), and the
    mirrored signs: the tensor-core group accumulators stay exact."""
    M = N = 128
    K = 1024
    for (ca, za, cb, zb) in [(15, 0, 0, 15), (15, 0, 15, 0), (0, 15, 0, 15)]:
        Aq = np.full((M, K // 2), ca * 17, np.uint8)
        Bq = np.full((N, K // 2), cb * 17, np.uint8)
        As = np.full((M, K // 128), 0.01, np.float16)
        Bs = np.full((N, K // 128), 0.02, np.float16)
        Az = np.full((M, K // 128), za, np.float16)
        Bz = np.full((N, K // 128), zb, np.float16)
        args = [dev(x) for x in (Aq, As, Az, Bq, Bs, Bz)]
        clove_lib.set_dispatch_override(1, 0, 0)
        C, G = clove_lib.debug_int4_group_acc(*args)
        Gref = oracle_mod.int4_group_acc(Aq, Az, Bq, Bz, K)
        np.testing.assert_array_equal(host(G), Gref)
        assert abs(int(Gref.flat[0])) == 28800
        ref = oracle_mod.gemm_int4(Aq, As, Az, Bq, Bs, Bz, K)
        assert rel_fro(host(C), ref) < TOL_TIGHT
    assert clove_lib.device_error() == 0
