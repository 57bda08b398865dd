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


def test_checkpoint_tool_round_trip(clove_lib, oracle_mod, cuda, tmp_path):
    """quantize_checkpoint packs the 2-D float weights of a safetensors file on the
    GPU (fp16, bf16 and fp32 sources), leaves the rest untouched, and load_int4
    returns operands bit-exact with the CPU specification that gemm_int4 consumes."""
    import torch
    from clove_compute_b200 import quantize as q
    rng = np.random.default_rng(3)
    w16 = _weights(256, 1024, seed=1)
    w32 = rng.standard_normal((128, 512)).astype(np.float32)
    wbf = (rng.standard_normal((64, 256)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    bias = rng.standard_normal(256).astype(np.float32)
    odd = rng.standard_normal((8, 200)).astype(np.float16)
    src, dst = str(tmp_path / "in.safetensors"), str(tmp_path / "out.safetensors")
    q.write_safetensors(src, {
        "mlp.up.weight": q.Tensor.from_numpy(w16), "mlp.down.weight": q.Tensor.from_numpy(w32),
        "attn.q.weight": q.Tensor("BF16", wbf.shape, wbf.tobytes()),
        "mlp.up.bias": q.Tensor.from_numpy(bias), "odd.weight": q.Tensor.from_numpy(odd)},
        {"origin": "test"})
    packed = q.quantize_checkpoint(src, dst)
    assert sorted(packed) == ["attn.q.weight", "mlp.down.weight", "mlp.up.weight"]
    tensors, meta = q.read_safetensors(dst)
    assert meta["origin"] == "test" and meta["clove.int4"] == q.INT4_FORMAT
    np.testing.assert_array_equal(tensors["mlp.up.bias"].numpy(), bias)
    np.testing.assert_array_equal(tensors["odd.weight"].numpy(), odd)
    assert "mlp.up.weight" not in tensors
    sources = {"mlp.up.weight": w16, "mlp.down.weight": w32.astype(np.float16),
               "attn.q.weight": (wbf.astype(np.uint32) << 16).view(np.float32).astype(np.float16)}
    for name, W in sources.items():
        codes, scales, zeros = q.load_int4(dst, name)
        rc, rs, rz = oracle_mod.quantize_int4(W)
        np.testing.assert_array_equal(host(codes), rc)
        np.testing.assert_array_equal(host(scales).view(np.uint16), rs.view(np.uint16))
        np.testing.assert_array_equal(host(zeros).view(np.uint16), rz.view(np.uint16))
    # The packed weight as the A operand of gemm_int4 against quantised activations.
    codes, scales, zeros = q.load_int4(dst, "mlp.up.weight")
    X = rng.standard_normal((16, 1024)).astype(np.float16)
    xc, xs, xz = oracle_mod.quantize_int4(X)
    C = host(clove_lib.gemm_int4(codes, scales, zeros, dev(xc), dev(xs), dev(xz)))
    ref = oracle_mod.gemm_int4(host(codes), host(scales), host(zeros), xc, xs, xz, 1024)
    assert rel_fro(C[8:], ref[8:]) < 2e-3  # rows 3-7 hold the special groups (fp16 overflow)
    assert clove_lib.device_error() == 0
