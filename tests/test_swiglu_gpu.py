"""swiglu_fused (the reference's declared-only activations.cuh:37-46) on the GPU:
the fused CTA-pair kernel and the unfused fallback against the fp32 oracle."""
import numpy as np
import pytest

from tests.gpu_util import dev, host, rel_fro

pytestmark = pytest.mark.gpu
TOL_TIGHT = 2e-3


@pytest.fixture(autouse=True)
def _reset(clove_lib):
    yield
    clove_lib.set_dispatch_override(0, 0, 0)


def _operands(T, H, inter, seed):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((T, H)).astype(np.float16)
    Wg = (rng.standard_normal((H, inter)) / np.sqrt(H)).astype(np.float16)
    Wu = (rng.standard_normal((H, inter)) / np.sqrt(H)).astype(np.float16)
    return X, Wg, Wu


@pytest.mark.parametrize("T,H,inter,expect", [
    (256, 1024, 512, "tc2_swiglu"),
    (300, 200, 136, "tc2_swiglu"),     # ragged: partial pair tiles, K not a multiple of 64
    (1024, 512, 1536, "tc2_swiglu"),   # several waves of pair tiles
    (64, 512, 256, "unfused_swiglu"),  # too few tokens for the pair kernel
    (200, 100, 36, "unfused_swiglu"),  # hidden not a multiple of 8
])
def test_swiglu_fused(clove_lib, oracle_mod, cuda, T, H, inter, expect):
    assert clove_lib.describe_dispatch("swiglu", T, inter, H).startswith(expect)
    X, Wg, Wu = _operands(T, H, inter, seed=T + H + inter)
    out = host(clove_lib.swiglu_fused(dev(X), dev(Wg), dev(Wu)))
    ref = oracle_mod.swiglu(X, Wg, Wu)
    err = rel_fro(out, ref)
    assert err < 1e-2 and err < TOL_TIGHT, err
    assert clove_lib.device_error() == 0


def test_swiglu_fused_matches_unfused(clove_lib, cuda):
    """The fused epilogue and the two-GEMM path agree (fp16 intermediates are the
    only difference)."""
    X, Wg, Wu = _operands(512, 768, 384, seed=5)
    fused = host(clove_lib.swiglu_fused(dev(X), dev(Wg), dev(Wu)))
    clove_lib.set_dispatch_override(1, 0, 0)  # tile kernels only: the unfused route
    unfused = host(clove_lib.swiglu_fused(dev(X), dev(Wg), dev(Wu)))
    assert rel_fro(fused, unfused) < 2e-3
