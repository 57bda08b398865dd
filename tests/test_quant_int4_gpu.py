"""INT4 packing tool on the GPU: codes, scales and zero points bit-exact against the
CPU specification (oracle.quantize_int4), then packed operands through gemm_int4."""
import numpy as np
import pytest

from tests.gpu_util import dev, host, rel_fro

pytestmark = pytest.mark.gpu


def _weights(rows, K, seed, special=True):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((rows, K)) * rng.uniform(0.01, 3.0, (rows, 1))).astype(np.float16)
    if special and rows >= 8 and K >= 512:
        W[3, :128] = 0.25                     # constant positive group
        W[4, 128:256] = 0.0                   # all-zero group
        W[5, 256:384] = np.abs(W[5, 256:384])  # positive-only group
        W[6, :128] = -7.0                     # constant negative group
        W[7, 384:512] *= 2000                 # large magnitudes
    return W


@pytest.mark.parametrize("rows,K", [(1, 128), (37, 512), (300, 4096), (4096, 1024)])
def test_quantize_bit_exact(clove_lib, oracle_mod, cuda, rows, K):
    W = _weights(rows, K, seed=rows + K)
    codes, scales, zeros = clove_lib.quantize_int4(dev(W))
    rc, rs, rz = oracle_mod.quantize_int4(W)
    np.testing.assert_array_equal(host(codes), rc)
    np.testing.assert_array_equal(host(scales).view(np.uint16), rs.view(np.uint16))
    np.testing.assert_array_equal(host(zeros).view(np.uint16), rz.view(np.uint16))
    assert clove_lib.device_error() == 0


def test_quantize_rejects_ragged_k(clove_lib, cuda):
    import torch
    W = torch.zeros((4, 200), dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        clove_lib.quantize_int4(W)


def test_quantized_weights_through_gemm_int4(clove_lib, oracle_mod, cuda):
    """Weights and activations packed by the tool feed gemm_int4 directly: exact G
    against the oracle on the packed data, and C close to the fp32 product of the
    dequantized operands."""
    M, N, K = 256, 64, 1024
    Wa = _weights(M, K, seed=1, special=False)
    Wb = _weights(N, K, seed=2, special=False)
    A = clove_lib.quantize_int4(dev(Wa))
    B = clove_lib.quantize_int4(dev(Wb))
    C, G = clove_lib.debug_int4_group_acc(*A, *B)
    Aq, As, Az = (host(t) for t in A)
    Bq, Bs, Bz = (host(t) for t in B)
    np.testing.assert_array_equal(host(G), oracle_mod.int4_group_acc(Aq, Az, Bq, Bz, K))
    ref = oracle_mod.gemm_int4(Aq, As, Az, Bq, Bs, Bz, K)
    assert rel_fro(host(C), ref) < 2e-3

    def deq(q, s, z):
        v = np.empty((q.shape[0], K), np.float32)
        v[:, 0::2] = q >> 4
        v[:, 1::2] = q & 15
        return (v - np.repeat(z.astype(np.float32), 128, 1)) * np.repeat(s.astype(np.float32), 128, 1)

    exact = deq(Aq, As, Az) @ deq(Bq, Bs, Bz).T
    assert rel_fro(host(C), exact.astype(np.float16)) < 2e-3
