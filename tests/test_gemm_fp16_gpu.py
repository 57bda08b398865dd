"""FP16 parity on the GPU: clove_gemm_fp16 (through the C ABI) vs the fp32 CPU oracle.

Contract (north star): C within 1e-2 relative Frobenius error of the
fp32-accumulating oracle. The kernels accumulate in fp32 too, so the observed
error is one fp16 rounding (~1e-4); the tests also hold them to 2e-3 to catch
partial-K or tiling bugs that a loose bound would miss."""
import numpy as np
import pytest
import torch

from clove_compute_b200 import workloads as wl
from tests.gpu_util import dev, host, rel_fro

pytestmark = pytest.mark.gpu
TOL_CONTRACT = 1e-2
TOL_TIGHT = 2e-3


@pytest.fixture(autouse=True)
def _reset(clove_lib):
    yield
    clove_lib.set_dispatch_override(0, 0, 0)


def _run(cc, oracle, M, N, K, path=0, bn=0, split=0, alpha=1.0, beta=0.0, seed=0):
    A, B = wl.fp16_operands(M, N, K, seed=seed)
    C0 = np.random.default_rng(seed + 1).uniform(-0.1, 0.1, (M, N)).astype(np.float16)
    cc.set_dispatch_override(path, bn, split)
    Cd = dev(C0.copy())
    cc.gemm_fp16(dev(A), dev(B), Cd, alpha=alpha, beta=beta)
    got = host(Cd)
    ref = oracle.gemm_fp16(A, B, C0.copy(), alpha=alpha, beta=beta)
    err = rel_fro(got, ref)
    assert err < TOL_CONTRACT
    assert err < TOL_TIGHT, f"rel Frobenius {err:.3e}"
    assert cc.device_error() == 0
    return err


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (128, 4096, 4096), (256, 256, 256),
                                   (64, 64, 64), (1000, 1000, 1000), (300, 136, 72)])
def test_tc_auto(clove_lib, oracle_mod, cuda, M, N, K):
    _run(clove_lib, oracle_mod, M, N, K)


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (384, 520, 200)])
def test_tc_tile_widths(clove_lib, oracle_mod, cuda, bn, M, N, K):
    _run(clove_lib, oracle_mod, M, N, K, path=1, bn=bn, split=1)


@pytest.mark.parametrize("bn,split", [(32, 2), (64, 2), (32, 4), (64, 8), (32, 8)])
def test_tc_cluster_split_k(clove_lib, oracle_mod, cuda, bn, split):
    _run(clove_lib, oracle_mod, 256, 96, 4096, path=1, bn=bn, split=split, seed=split)


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (1024, 1024, 2048), (384, 520, 200),
                                   (128, 256, 64), (640, 776, 1000)])
def test_tc_cta_pair(clove_lib, oracle_mod, cuda, M, N, K):
    """256 x 256 tiles on CTA pairs (tcgen05 cta_group::2), ragged M / N / K included
    (M = 128 and 384 leave one CTA of a pair entirely outside A)."""
    _run(clove_lib, oracle_mod, M, N, K, path=4, seed=M + K)


def test_tc_cta_pair_alpha_beta(clove_lib, oracle_mod, cuda):
    _run(clove_lib, oracle_mod, 768, 512, 256, path=4, alpha=0.5, beta=1.0, seed=2)


def test_ffn_shapes_choose_cta_pairs(clove_lib, cuda):
    assert clove_lib.describe_dispatch("fp16", 11008, 2048, 4096).startswith("tc2_f16")
    assert clove_lib.describe_dispatch("fp16", 4096, 2048, 11008).startswith("tc2_f16")


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (4, 1024, 1024), (16, 4096, 1024),
                                   (1, 4096, 11008), (37, 4096, 6144)])
def test_small_m_decode(clove_lib, oracle_mod, cuda, M, N, K):
    _run(clove_lib, oracle_mod, M, N, K)


def test_small_m_long_k_plan(clove_lib, cuda):
    """One 128-row band with few live rows or a long K takes 128-column tiles over
    4-CTA clusters; 64 live rows at K = 4096 keep 64-column tiles over pairs."""
    assert clove_lib.describe_dispatch("fp16", 1, 4096, 11008) == "tc_f16 bn=128 split=4"
    assert clove_lib.describe_dispatch("fp16", 1, 4096, 4096) == "tc_f16 bn=128 split=4"
    assert clove_lib.describe_dispatch("fp16", 64, 4096, 4096) == "tc_f16 bn=64 split=2"


@pytest.mark.parametrize("M", [1, 5, 31, 32, 33, 100])
def test_split_k_live_rows(clove_lib, oracle_mod, cuda, M):
    """Split-K clusters exchange only the rows below M: every cluster size and tile
    width with a partly live tile."""
    for bn, split in [(128, 4), (64, 2), (32, 8), (64, 8)]:
        _run(clove_lib, oracle_mod, M, 256, 4096, path=1, bn=bn, split=split, seed=M + bn)


def test_alpha_beta(clove_lib, oracle_mod, cuda):
    # tests/test_gemm.cu:221-243 runs this shape without a check; here it is checked.
    _run(clove_lib, oracle_mod, 128, 128, 128, alpha=0.5, beta=0.25)
    _run(clove_lib, oracle_mod, 1024, 512, 256, alpha=2.0, beta=1.0)


def test_beta_residual_in_place(clove_lib, oracle_mod, cuda):
    # The runtime adds the residual through beta=1 with C as input and output
    # (src/runtime/inference.cu:165-168).
    _run(clove_lib, oracle_mod, 512, 4096, 1024, alpha=1.0, beta=1.0, seed=9)


@pytest.mark.parametrize("N", [1, 2, 3, 4, 5, 8])
def test_gemv_small_n(clove_lib, oracle_mod, cuda, N):
    _run(clove_lib, oracle_mod, 4096, N, 4096, seed=N)
    _run(clove_lib, oracle_mod, 333, N, 520, path=2, seed=N, alpha=0.75, beta=0.5)


@pytest.mark.parametrize("M,N,K", [(7, 9, 11), (64, 30, 100), (130, 70, 33)])
def test_simt_fallback_ragged(clove_lib, oracle_mod, cuda, M, N, K):
    _run(clove_lib, oracle_mod, M, N, K, alpha=1.5, beta=-0.5)


def test_k_zero_scales_c(clove_lib, cuda):
    C0 = np.random.default_rng(0).uniform(-1, 1, (8, 8)).astype(np.float16)
    Cd = dev(C0.copy())
    a = torch.empty((8, 0), dtype=torch.float16, device="cuda")
    b = torch.empty((0, 8), dtype=torch.float16, device="cuda")
    clove_lib.gemm_fp16(a, b, Cd, alpha=1.0, beta=0.5)
    np.testing.assert_array_equal(host(Cd), (C0.astype(np.float32) * 0.5).astype(np.float16))


@pytest.mark.parametrize("batch,M,N,K", [
    (3, 128, 64, 96),      # one tile per problem: one batched launch
    (5, 200, 136, 128),    # ragged M and N: rows past M must not touch the next problem
    (64, 128, 128, 256),   # many problems share the persistent grid
    (2, 2048, 2048, 256),  # each problem fills the GPU: per-problem dispatch
])
def test_batched(clove_lib, oracle_mod, cuda, batch, M, N, K):
    rng = np.random.default_rng(4 + batch)
    A = (rng.standard_normal((batch, M, K)) / np.sqrt(K)).astype(np.float16)
    B = (rng.standard_normal((batch, K, N)) / np.sqrt(K)).astype(np.float16)
    C = host(clove_lib.gemm_fp16_batched(dev(A), dev(B)))
    for b in range(batch):
        assert rel_fro(C[b], oracle_mod.gemm_fp16(A[b], B[b])) < TOL_TIGHT, b


def test_batched_alpha_beta(clove_lib, oracle_mod, cuda):
    """beta reads each problem's own C plane in the single-launch batched path."""
    import torch
    batch, M, N, K = 4, 192, 72, 64
    rng = np.random.default_rng(11)
    A = (rng.standard_normal((batch, M, K)) / np.sqrt(K)).astype(np.float16)
    B = (rng.standard_normal((batch, K, N)) / np.sqrt(K)).astype(np.float16)
    C0 = rng.uniform(-1, 1, (batch, M, N)).astype(np.float16)
    Ad, Bd, Cd = dev(A), dev(B), dev(C0.copy())
    clove_lib.gemm_fp16_batched(Ad, Bd, Cd, alpha=0.5, beta=-2.0)
    torch.cuda.synchronize()
    C = host(Cd)
    for b in range(batch):
        ref = oracle_mod.gemm_fp16(A[b], B[b], C=C0[b].copy(), alpha=0.5, beta=-2.0)
        assert rel_fro(C[b], ref) < TOL_TIGHT, b


def test_no_writes_outside_c(clove_lib, oracle_mod, cuda):
    """Ragged tiles must not store past C: canaries around C stay intact."""
    M, N, K = 200, 136, 128
    A, B = wl.fp16_operands(M, N, K, seed=3)
    pad = 4096
    buf = torch.full((pad + M * N + pad,), 7.0, dtype=torch.float16, device="cuda")
    C = buf[pad:pad + M * N].view(M, N)
    clove_lib.gemm_fp16(dev(A), dev(B), C)
    h = host(buf)
    assert (h[:pad] == 7.0).all() and (h[pad + M * N:] == 7.0).all()
    assert rel_fro(h[pad:pad + M * N].reshape(M, N), oracle_mod.gemm_fp16(A, B)) < TOL_TIGHT


def test_dispatch_choices(clove_lib, cuda):
    assert clove_lib.describe_dispatch("fp16", 1024, 1024, 1024).startswith("tc_f16")
    assert clove_lib.describe_dispatch("fp16", 4096, 1, 4096).startswith("gemv_f16")


@pytest.mark.parametrize("M,N,K", [(512, 512, 4096), (768, 520, 1000), (640, 776, 2048),
                                   (256, 256, 8192), (1280, 1024, 64)])
def test_tc_cta_pair_stream_k_forced(clove_lib, oracle_mod, cuda, M, N, K):
    """Stream-K schedule forced on shapes with few tiles: each tile's K range is cut
    over many CTA pairs (up to ~19 partial slots), summed by the last contributor."""
    _run(clove_lib, oracle_mod, M, N, K, path=4, split=2, seed=K)


def test_tc_cta_pair_stream_k_alpha_beta(clove_lib, oracle_mod, cuda):
    _run(clove_lib, oracle_mod, 768, 512, 2048, path=4, split=2, alpha=0.5, beta=1.0, seed=3)


def _sampled_rows_check(cc, oracle, A, B, C, rows):
    ref = oracle.gemm_fp16(np.ascontiguousarray(A[rows]), B)
    assert rel_fro(C[rows], ref) < TOL_TIGHT


def test_ffn_down_stream_k(clove_lib, oracle_mod, cuda):
    """FFN down (4096 x 2048 x 11008): 128 pair tiles on 74 pairs, so the last 54
    tiles run as stream-K pieces. Rows from whole-K and stream-K tiles are checked
    against the oracle, and the result does not depend on which contributor
    finishes last (slots are summed in a fixed order)."""
    M, N, K = 4096, 2048, 11008
    rng = np.random.default_rng(21)
    A = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    B = rng.standard_normal((K, N)).astype(np.float16)
    Ad, Bd = dev(A), dev(B)
    C1 = clove_lib.gemm_fp16(Ad, Bd)
    C2 = clove_lib.gemm_fp16(Ad, Bd)
    torch.cuda.synchronize()
    h1, h2 = host(C1), host(C2)
    np.testing.assert_array_equal(h1, h2)
    rows = np.r_[0:8, 1020:1030, 2300:2310, 3580:3600, 4080:4096]
    _sampled_rows_check(clove_lib, oracle_mod, A, B, h1, rows)
    clove_lib.set_dispatch_override(4, 0, 1)  # same kernel, whole-K tiles only
    h3 = host(clove_lib.gemm_fp16(Ad, Bd))
    assert rel_fro(h1, h3) < 1e-3
    assert clove_lib.device_error() == 0


def test_stream_k_in_cuda_graph(clove_lib, cuda):
    """The stream-K workspace becomes an allocation node when captured; replays
    reproduce the eager result bit for bit."""
    M, N, K = 4096, 2048, 11008
    g = torch.Generator(device="cuda").manual_seed(5)
    A = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).half()
    B = torch.randn(K, N, device="cuda", generator=g).half()
    C = torch.empty(M, N, device="cuda", dtype=torch.float16)
    clove_lib.gemm_fp16(A, B, C)
    torch.cuda.synchronize()
    eager = C.clone()
    C.zero_()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            clove_lib.gemm_fp16(A, B, C, stream=s)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(C, eager)
    assert clove_lib.device_error() == 0
