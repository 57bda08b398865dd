"""Tensor-core attention (clove_flash_attention) against the CPU oracle's restatement
of the reference's flash_attention_kernel (src/kernels/attention.cu:93-266).

The kernel rounds P to fp16 before P.V (the oracle keeps it in fp32), so outputs are
compared by relative Frobenius error with the same 1e-2 bound as the fp16 GEMMs.
Shapes: one and several key blocks, ragged sequence lengths (masked padding keys,
clipped output rows), causal and full attention, both layouts, grouped-query heads,
a single query, and a long sequence whose running maximum rises several times."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _qkv(B, H, Hkv, S, seed, layout="bhsd", spread=1.0):
    rng = np.random.default_rng(seed)
    shp = (lambda h: (B, h, S, 128)) if layout == "bhsd" else (lambda h: (B, S, h, 128))
    Q = (rng.standard_normal(shp(H)) * spread).astype(np.float16)
    K = rng.standard_normal(shp(Hkv)).astype(np.float16)
    V = rng.standard_normal(shp(Hkv)).astype(np.float16)
    return Q, K, V


def _rel(x, r):
    x = x.astype(np.float64)
    r = r.astype(np.float64)
    return float(np.linalg.norm(x - r) / np.linalg.norm(r))


@pytest.mark.parametrize("B,H,Hkv,S,causal,layout", [
    (1, 2, 2, 128, True, "bhsd"),
    (1, 2, 2, 256, True, "bhsd"),
    (2, 3, 3, 384, False, "bhsd"),
    (1, 2, 2, 200, True, "bhsd"),      # ragged: padded keys masked, rows clipped
    (1, 2, 2, 200, False, "bhsd"),
    (1, 1, 1, 1, True, "bhsd"),        # a single query and key
    (1, 1, 1, 77, False, "bhsd"),
    (2, 8, 2, 300, True, "bshd"),      # runtime layout, grouped-query heads
    (1, 4, 1, 256, False, "bshd"),
])
def test_attention_matches_oracle(clove_lib, cuda, oracle_mod, B, H, Hkv, S, causal, layout):
    Q, K, V = _qkv(B, H, Hkv, S, seed=B * 100 + H * 10 + S, layout=layout)
    dev = lambda a: torch.from_numpy(a).cuda()
    O = clove_lib.flash_attention(dev(Q), dev(K), dev(V), causal=causal, layout=layout)
    torch.cuda.synchronize()
    ref = oracle_mod.attention(Q, K, V, causal=causal, layout=layout)
    got = O.cpu().numpy()
    assert np.isfinite(got).all()
    assert _rel(got, ref) < TOL
    assert clove_lib.device_error() == 0


def test_attention_long_sequence_rescales(clove_lib, cuda, oracle_mod):
    """2048 keys of growing magnitude: the running maximum is raised in later blocks,
    so O in TMEM and the row sums are rescaled mid-sequence."""
    B, H, S = 1, 2, 2048
    Q, K, V = _qkv(B, H, H, S, seed=5, spread=4.0)
    ramp = np.linspace(0.2, 3.0, S, dtype=np.float32)[None, None, :, None]
    K = (K.astype(np.float32) * ramp).astype(np.float16)
    dev = lambda a: torch.from_numpy(a).cuda()
    for causal in (True, False):
        O = clove_lib.flash_attention(dev(Q), dev(K), dev(V), causal=causal)
        torch.cuda.synchronize()
        ref = oracle_mod.attention(Q, K, V, causal=causal)
        assert _rel(O.cpu().numpy(), ref) < TOL, causal
    assert clove_lib.device_error() == 0


def test_attention_output_rows_outside_seq_untouched(clove_lib, cuda, oracle_mod):
    """A ragged last query tile stores only rows < seq_len: a [B, H, S, D] output
    viewed inside a larger buffer keeps its neighbours' bytes."""
    B, H, S = 1, 2, 130
    Q, K, V = _qkv(B, H, H, S, seed=9)
    dev = lambda a: torch.from_numpy(a).cuda()
    buf = torch.full((B * H * S * 128 + 4096,), 7.0, dtype=torch.float16, device="cuda")
    O = buf[:B * H * S * 128].view(B, H, S, 128)
    clove_lib.flash_attention(dev(Q), dev(K), dev(V), causal=True, O=O)
    torch.cuda.synchronize()
    assert torch.all(buf[B * H * S * 128:] == 7.0)
    assert _rel(O.cpu().numpy(), oracle_mod.attention(Q, K, V, causal=True)) < TOL


def test_attention_rejects_unsupported(clove_lib, cuda):
    x = torch.zeros((1, 1, 64, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(clove_lib.CloveError):
        clove_lib.flash_attention(x, x, x)  # head_dim 64: the reference supports 128 only
    q = torch.zeros((1, 3, 64, 128), dtype=torch.float16, device="cuda")
    kv = torch.zeros((1, 2, 64, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(clove_lib.CloveError):
        clove_lib.flash_attention(q, kv, kv)  # 3 heads over 2 kv heads


def _torch_ref(q, k, v, causal):
    """Plain PyTorch fp32 attention on the GPU (scale 1/sqrt(128))."""
    qf, kf, vf = q.float(), k.float(), v.float()
    s = torch.matmul(qf, kf.transpose(-1, -2)) / np.sqrt(128.0)
    if causal:
        n = s.shape[-1]
        s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool, device=s.device), 1),
                          float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), vf)


@pytest.mark.parametrize("B,H,S,causal", [(1, 32, 2048, True), (1, 32, 2048, False),
                                          (8, 32, 1024, True)])
def test_attention_benchmark_shapes(clove_lib, cuda, B, H, S, causal):
    """The benchmark's shapes: hundreds of CTAs over several waves, heaviest tile pairs
    first, every (batch, head) of the one-dimensional grid; against PyTorch fp32."""
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + S + causal)
    q, k, v = (torch.randn((B, H, S, 128), device="cuda", generator=g).half() for _ in range(3))
    O = clove_lib.flash_attention(q, k, v, causal=causal)
    ref = _torch_ref(q, k, v, causal)
    err = float((O.float() - ref).norm() / ref.norm())
    assert err < TOL, err
    assert clove_lib.device_error() == 0


def test_attention_back_to_back_calls(clove_lib, cuda):
    """Consecutive calls on one stream with different inputs (each kernel's set-up
    overlaps the previous kernel's tail): every output holds its own inputs' result."""
    g = torch.Generator(device="cuda").manual_seed(77)
    sets = [tuple(torch.randn((2, 8, 640, 128), device="cuda", generator=g).half()
                  for _ in range(3)) for _ in range(4)]
    outs = [torch.empty_like(s[0]) for s in sets]
    for rep in range(2):
        for (q, k, v), o in zip(sets, outs):
            clove_lib.flash_attention(q, k, v, causal=rep == 0, O=o)
    torch.cuda.synchronize()
    for (q, k, v), o in zip(sets, outs):
        ref = _torch_ref(q, k, v, False)
        err = float((o.float() - ref).norm() / ref.norm())
        assert err < TOL, err
    assert clove_lib.device_error() == 0


def test_exp2_polynomial_error_bound(clove_lib, cuda):
    """The softmax's FMA-pipe exponential (Remez-fitted degree-4 polynomial after a
    round-to-nearest range reduction) against float64 exp2: relative error within
    2.7e-6 over [-125, 8] (the arguments the softmax produces: s*scale*log2e - m <= 8),
    at integers, half-integers and random points; below -125 it returns 2^-125."""
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(-125.0, 8.0, 1 << 20), np.arange(-125, 9, dtype=np.float64),
                        np.arange(-124.5, 8.0, 1.0), [-1e-7, 1e-7, 0.0]]).astype(np.float32)
    if x.size % 2:
        x = np.append(x, np.float32(0.0))
    y = clove_lib.debug_exp2_poly(torch.from_numpy(x).cuda()).cpu().numpy().astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() <= 2.7e-6, (rel.max(), x[np.argmax(rel)])
    low = clove_lib.debug_exp2_poly(torch.tensor([-126.0, -1000.0], device="cuda")).cpu().numpy()
    assert np.all(np.abs(low / 2.0 ** -125 - 1.0) <= 2.7e-6)
    assert clove_lib.device_error() == 0
