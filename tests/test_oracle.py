"""CPU oracle checks: the C restatement against independent numpy models,
known-answer tests and (when present) golden vectors from the reference kernels.

The reference ships no golden vectors for this path, so the known answers are
constructed here from the documented arithmetic (gemm.cuh:37-87,
gemm_int8.cu:87-114, gemm_int4.cu:27-34)."""
import os

import numpy as np
import pytest

from clove_compute_b200 import workloads as wl

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# --------------------------------------------------------------------------- fp16 conversion
def test_h2f_all_halves(oracle_mod):
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = oracle_mod.h2f(h)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f2h_matches_numpy_rounding(oracle_mod):
    rng = np.random.default_rng(1)
    f = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 10,
        rng.standard_normal(50000).astype(np.float32) * 1e-5,   # subnormal range
        rng.standard_normal(50000).astype(np.float32) * 6e4,    # overflow range
        np.array([0.0, -0.0, 65504, 65519.99, 65520, -65520, 1e-8, 2.0**-24, 2.0**-25,
                  1.5 * 2.0**-24, np.inf, -np.inf], np.float32),
        # exact ties between two halves
        (np.arange(1, 2049, dtype=np.float32) + 0.5) * np.float32(2.0**-10),
    ])
    got = oracle_mod.f2h(f).view(np.uint16)
    ref = f.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, ref)


# --------------------------------------------------------------------------- fp16 GEMM
def _f16_ref(A, B, C0=None, alpha=1.0, beta=0.0):
    acc = A.astype(np.float64) @ B.astype(np.float64)
    out = alpha * acc
    if beta != 0.0:
        out = out + beta * C0.astype(np.float64)
    return out


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (7, 5, 3), (64, 64, 64), (33, 70, 129), (128, 256, 96)])
def test_gemm_fp16_vs_float64(oracle_mod, M, N, K):
    A, B = wl.fp16_operands(M, N, K, seed=M + N + K)
    C = oracle_mod.gemm_fp16(A, B)
    ref = _f16_ref(A, B)
    # fp32 accumulation + one fp16 rounding: within 1 fp16 ulp elementwise.
    assert np.allclose(C.astype(np.float64), ref, rtol=2 ** -10, atol=1e-6)
    assert oracle_mod.rel_frobenius(C, ref) < 1e-3


def test_gemm_fp16_alpha_beta(oracle_mod):
    M, N, K = 128, 128, 128  # tests/test_gemm.cu:221-243 shape, here with a real check
    A, B = wl.fp16_operands(M, N, K, seed=5)
    C0 = np.random.default_rng(6).uniform(-0.1, 0.1, (M, N)).astype(np.float16)
    C = oracle_mod.gemm_fp16(A, B, C0.copy(), alpha=0.5, beta=0.25)
    ref = _f16_ref(A, B, C0, 0.5, 0.25)
    assert np.allclose(C.astype(np.float64), ref, rtol=2 ** -10, atol=1e-5)


def test_gemm_fp16_rows_and_threads_independent(oracle_mod):
    A, B = wl.fp16_operands(97, 65, 200, seed=3)
    full = oracle_mod.gemm_fp16(A, B, nthreads=1)
    multi = oracle_mod.gemm_fp16(A, B, nthreads=0)
    assert np.array_equal(full.view(np.uint16), multi.view(np.uint16))
    part = np.zeros_like(full)
    oracle_mod.gemm_fp16(A, B, part, rows=(10, 50))
    assert np.array_equal(part[10:50].view(np.uint16), full[10:50].view(np.uint16))
    assert not part[:10].any() and not part[50:].any()


def test_gemm_fp16_known_answer_identity(oracle_mod):
    K = 64
    A = np.random.default_rng(0).standard_normal((32, K)).astype(np.float16)
    eye = np.eye(K, dtype=np.float16)
    assert np.array_equal(oracle_mod.gemm_fp16(A, eye).view(np.uint16), A.view(np.uint16))


# --------------------------------------------------------------------------- int8
@pytest.mark.parametrize("za,zb", [(0, 0), (3, -7), (-128, 127)])
def test_int8_acc_exact(oracle_mod, za, zb):
    M, N, K = 37, 29, 301
    A, B, _, _ = wl.int8_operands(M, N, K, seed=11)
    acc = oracle_mod.int8_acc(A, B, za, zb)
    ref = (A.astype(np.int64) - za) @ (B.astype(np.int64) - zb)
    assert np.array_equal(acc.astype(np.int64), ref)


def test_int8_acc_wraps_like_int32(oracle_mod):
    # (127 - (-128))^2 * K overflows int32 for K = 40000: the oracle wraps mod 2^32
    # exactly like the device's int32 accumulators (and the reference's).
    K = 40000
    A = np.full((1, K), 127, np.int8)
    B = np.full((K, 1), -128, np.int8)
    acc = oracle_mod.int8_acc(A, B, -128, 127)
    ref = ((255 * -255 * K) + 2 ** 31) % 2 ** 32 - 2 ** 31
    assert int(acc[0, 0]) == ref


def test_int8_per_tensor_and_rowcol(oracle_mod):
    M, N, K = 64, 48, 256
    A, B, sA, sB = wl.int8_operands(M, N, K, seed=2)
    acc = (A.astype(np.int64) - 2) @ (B.astype(np.int64) + 5)
    C = oracle_mod.gemm_int8(A, B, 0.01, 2, 0.02, -5)
    ref = (acc.astype(np.float32) * np.float32(np.float32(0.01) * np.float32(0.02))).astype(np.float16)
    assert np.array_equal(C.view(np.uint16), ref.view(np.uint16))
    acc0 = A.astype(np.int64) @ B.astype(np.int64)
    C2 = oracle_mod.gemm_int8_rowcol(A, B, sA, sB)
    ref2 = ((acc0.astype(np.float32) * sA[:, None]) * sB[None, :]).astype(np.float16)
    assert np.array_equal(C2.view(np.uint16), ref2.view(np.uint16))


# --------------------------------------------------------------------------- int4
def _int4_ref_G(op: wl.Int4Operands):
    a = wl.unpack_int4(op.A_q).astype(np.int64)
    b = wl.unpack_int4(op.B_q).astype(np.int64)
    za = np.rint(op.A_zero.astype(np.float32)).astype(np.int64)
    zb = np.rint(op.B_zero.astype(np.float32)).astype(np.int64)
    G = op.K // 128
    a = a.reshape(op.M, G, 128) - za[:, :, None]
    b = b.reshape(op.N, G, 128) - zb[:, :, None]
    return np.einsum("mgk,ngk->mng", a, b)


def _int4_ref_C(op: wl.Int4Operands, Gm):
    sA = op.A_scale.astype(np.float32)
    sB = op.B_scale.astype(np.float32)
    acc = np.zeros((op.M, op.N), np.float32)
    for g in range(op.K // 128):
        s = (sA[:, g][:, None] * sB[:, g][None, :]).astype(np.float32)
        acc = (acc + Gm[:, :, g].astype(np.float32) * s).astype(np.float32)
    return acc.astype(np.float16)


@pytest.mark.parametrize("M,N,K", [(1, 1, 128), (5, 3, 256), (40, 17, 512), (9, 64, 1024)])
def test_int4_group_acc_and_gemm(oracle_mod, M, N, K):
    op = wl.int4_operands(M, N, K, seed=M * N)
    G = oracle_mod.int4_group_acc(op.A_q, op.A_zero, op.B_q, op.B_zero, K)
    Gref = _int4_ref_G(op)
    assert np.array_equal(G.astype(np.int64), Gref)
    C = oracle_mod.gemm_int4(op.A_q, op.A_scale, op.A_zero, op.B_q, op.B_scale, op.B_zero, K)
    assert np.array_equal(C.view(np.uint16), _int4_ref_C(op, Gref).view(np.uint16))


def test_int4_known_answers(oracle_mod):
    K = 256
    ones = np.full((2, K // 2), 0xFF, np.uint8)  # every code = 15
    z0 = np.zeros((2, K // 128), np.float16)
    z15 = np.full((2, K // 128), 15, np.float16)
    G = oracle_mod.int4_group_acc(ones, z0, ones, z0, K)
    assert (G == 128 * 15 * 15).all()
    G = oracle_mod.int4_group_acc(ones, z15, ones, z0, K)
    assert (G == 0).all()
    # one-hot: only element k=5 of row 0 is 1 (odd k -> low nibble of byte 2)
    a = np.zeros((1, K // 2), np.uint8)
    a[0, 2] = 0x01
    b = np.zeros((1, K // 2), np.uint8)
    b[0, 2] = 0x07
    G = oracle_mod.int4_group_acc(a, np.zeros((1, 2), np.float16), b, np.zeros((1, 2), np.float16), K)
    assert G[0, 0, 0] == 7 and G[0, 0, 1] == 0
    # the same value placed at even k=4 (high nibble) pairs with b's high nibble only
    a[0, 2] = 0x10
    G = oracle_mod.int4_group_acc(a, np.zeros((1, 2), np.float16), b, np.zeros((1, 2), np.float16), K)
    assert G[0, 0, 0] == 0
    # scales: C = sum_g G*sA*sB
    sA = np.array([[0.5, 2.0]], np.float16)
    sB = np.array([[0.25, 1.0]], np.float16)
    a = np.full((1, K // 2), 0x11, np.uint8)  # all codes 1
    C = oracle_mod.gemm_int4(a, sA, np.zeros((1, 2), np.float16), a, sB,
                             np.zeros((1, 2), np.float16), K)
    assert float(C[0, 0]) == 128 * 0.5 * 0.25 + 128 * 2.0 * 1.0


def test_int4_zero_points_round_to_nearest(oracle_mod):
    K = 128
    a = np.full((1, 64), 0x88, np.uint8)  # codes 8
    zs = np.array([[7.4]], np.float16)    # rounds to 7
    G = oracle_mod.int4_group_acc(a, zs, a, np.zeros((1, 1), np.float16), K)
    assert G[0, 0, 0] == 128 * 1 * 8


def _refcompat_numpy(Aq, As, Bq_kn, Bs_kn, M, N, K):
    a = wl.unpack_int4(Aq).astype(np.float32) - 8
    # B packed along N: [K, N/2], high nibble = even n; odd N's last column reads 0
    b = np.zeros((K, N), np.float32)
    if N // 2 > 0:
        bb = wl.unpack_int4(Bq_kn).astype(np.float32) - 8
        b[:, : 2 * (N // 2)] = bb
    acc = np.zeros((M, N), np.float32)
    for k in range(K):  # sequential fp32 sum, exact for these integer magnitudes
        acc = (acc + np.outer(a[:, k], b[k, :])).astype(np.float32)
    last_group = (((K + 63) // 64 - 1) * 64) // 128
    ng = (K + 127) // 128
    a_s = As.reshape(M, ng)[:, last_group].astype(np.float32)
    b_s = Bs_kn.reshape(ng, N)[last_group, :].astype(np.float32)
    return ((acc * a_s[:, None]) * b_s[None, :]).astype(np.float16)


@pytest.mark.parametrize("M,N,K", [(8, 4, 256), (16, 6, 384), (4, 1, 128)])
def test_int4_refcompat_matches_numpy_model(oracle_mod, M, N, K):
    rng = np.random.default_rng(M + N)
    Aq = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    As = rng.uniform(0.005, 0.02, (M, K // 128)).astype(np.float16)
    Bq = rng.integers(0, 256, (K, max(N // 2, 1)), dtype=np.uint8)[:, : N // 2].copy()
    Bs = rng.uniform(0.005, 0.02, (K // 128, N)).astype(np.float16)
    C = oracle_mod.gemm_int4_refcompat(Aq, As, Bq, Bs, M, N, K)
    ref = _refcompat_numpy(Aq, As, Bq, Bs, M, N, K)
    assert np.array_equal(C.view(np.uint16), ref.view(np.uint16))


# --------------------------------------------------------------------------- golden vectors
def _golden_files(prefix):
    if not os.path.isdir(GOLDEN):
        return []
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith(prefix) and f.endswith(".npz"))


@pytest.mark.parametrize("fname", _golden_files("ref_fp16_") or ["<none>"])
def test_oracle_vs_reference_fp16_golden(oracle_mod, fname):
    """Outputs of the reference gemm_fp16 (WMMA / naive kernels, run on a B200)."""
    if fname == "<none>":
        pytest.skip("no reference fp16 golden vectors generated yet")
    d = np.load(os.path.join(GOLDEN, fname))
    A, B, C0, out = d["A"], d["B"], d["C0"], d["C_ref"]
    alpha, beta = float(d["alpha"]), float(d["beta"])
    C = oracle_mod.gemm_fp16(A, B, C0.copy(), alpha=alpha, beta=beta)
    # The reference's WMMA path accumulates in fp16 (gemm_fp16.cu:53); its naive
    # path accumulates in fp32 like the oracle.
    tol = float(d["tol"])
    assert oracle_mod.rel_frobenius(C, out) < tol
    if "naive" in fname:  # same arithmetic as the oracle: bit for bit
        assert np.array_equal(C.view(np.uint16), out.view(np.uint16))


@pytest.mark.parametrize("fname", _golden_files("ref_int4_") or ["<none>"])
def test_oracle_refcompat_vs_reference_int4_golden(oracle_mod, fname):
    """Outputs of the reference gemm_int4 kernel (run on a B200): bit-exact."""
    if fname == "<none>":
        pytest.skip("no reference int4 golden vectors generated yet")
    d = np.load(os.path.join(GOLDEN, fname))
    M, N, K = int(d["M"]), int(d["N"]), int(d["K"])
    C = oracle_mod.gemm_int4_refcompat(d["A_q"], d["A_scale"], d["B_q"], d["B_scale"], M, N, K)
    assert np.array_equal(C.view(np.uint16), d["C_ref"].view(np.uint16))


# ---------------------------------------------------------------------------
# INT4 packing tool: the C restatement against an independent numpy statement of
# the same specification, and known answers.
# ---------------------------------------------------------------------------
def _np_quantize_int4(W):
    rows, K = W.shape
    w = W.astype(np.float32).reshape(rows, K // 128, 128)
    mn = np.minimum(w.min(-1), np.float32(0))
    mx = np.maximum(w.max(-1), np.float32(0))
    s = ((mx - mn) / np.float32(15)).astype(np.float32)
    bits = s.astype(np.float16).view(np.uint16).copy()
    bits[(bits & 0x7FFF) == 0] = 1
    bits[(bits & 0x7FFF) > 0x7BFF] = 0x7BFF
    sh = bits.view(np.float16)
    sf = sh.astype(np.float32)
    z = np.clip(np.rint(-mn / sf), 0, 15).astype(np.float32) + np.float32(0)  # -0 -> +0
    q = np.clip(np.rint(w / sf[..., None]) + z[..., None], 0, 15).astype(np.uint8)
    codes = ((q[..., 0::2] << 4) | q[..., 1::2]).reshape(rows, K // 2)
    return codes, sh, z.astype(np.float16)


def test_quantize_int4_matches_numpy_statement(oracle_mod):
    rng = np.random.default_rng(21)
    W = (rng.standard_normal((37, 512)) * rng.uniform(0.01, 3.0, (37, 1))).astype(np.float16)
    W[3, :128] = 0.25          # constant positive group
    W[4, 128:256] = 0.0        # all-zero group
    W[5, 256:384] = np.abs(W[5, 256:384])  # positive-only group
    W[6, :128] = -7.0          # constant negative group
    W[7, 384:] *= 2000         # large magnitudes
    got = oracle_mod.quantize_int4(W)
    want = _np_quantize_int4(W)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(np.ascontiguousarray(g).view(np.uint8),
                                      np.ascontiguousarray(w).view(np.uint8))


def test_quantize_int4_known_answers(oracle_mod):
    W = np.full((1, 128), 0.5, np.float16)
    codes, s, z = oracle_mod.quantize_int4(W)
    assert codes.tolist() == [[0xFF] * 64] and float(z[0, 0]) == 0.0
    assert float(s[0, 0]) == float(np.float16(0.5 / 15))
    codes, s, z = oracle_mod.quantize_int4(np.zeros((1, 128), np.float16))
    assert not codes.any() and not z.astype(np.float32).any()
    # ramp -1 .. 1 over one group: scale 2/15, zero rint(7.5) = 8 (ties to even)
    W = np.linspace(-1, 1, 128, dtype=np.float32).astype(np.float16)[None]
    codes, s, z = oracle_mod.quantize_int4(W)
    assert float(z[0, 0]) == 8.0
    assert codes[0, 0] >> 4 == 0 and codes[0, -1] & 15 == 15


def test_quantize_int4_round_trip_error(oracle_mod):
    rng = np.random.default_rng(22)
    W = rng.standard_normal((16, 1024)).astype(np.float16)
    codes, s, z = oracle_mod.quantize_int4(W)
    q = np.empty((16, 1024), np.float32)
    q[:, 0::2] = codes >> 4
    q[:, 1::2] = codes & 15
    sf = np.repeat(s.astype(np.float32), 128, axis=1)
    zf = np.repeat(z.astype(np.float32), 128, axis=1)
    err = np.abs((q - zf) * sf - W.astype(np.float32))
    # Half a step, except where the fp16-rounded scale pulls an extreme value one
    # code past 15 (clamped): at most one step.
    assert np.all(err <= sf * (1 + 1e-3))
    assert np.mean(err <= 0.5 * sf * (1 + 1e-3) + 1e-6) > 0.99


def test_swiglu_matches_float64(oracle_mod):
    rng = np.random.default_rng(31)
    X = rng.standard_normal((9, 256)).astype(np.float16)
    Wg = (rng.standard_normal((256, 40)) / 16).astype(np.float16)
    Wu = (rng.standard_normal((256, 40)) / 16).astype(np.float16)
    out = oracle_mod.swiglu(X, Wg, Wu).astype(np.float64)
    g = X.astype(np.float64) @ Wg.astype(np.float64)
    u = X.astype(np.float64) @ Wu.astype(np.float64)
    ref = g / (1 + np.exp(-g)) * u
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-3
    part = oracle_mod.swiglu(X, Wg, Wu, rows=(2, 5))
    np.testing.assert_array_equal(part[2:5], oracle_mod.swiglu(X, Wg, Wu)[2:5])
    assert not part[:2].any() and not part[5:].any()


# ---------------------------------------------------------------------------
# Attention: the C restatement of the reference's flash_attention_kernel against a
# float64 numpy statement of attention, and (when present) the reference kernel's
# own outputs recorded on a B200.
# ---------------------------------------------------------------------------
def _np_attention(Q, K, V, causal, scale, layout="bhsd", phantom=0):
    if layout == "bshd":
        Q, K, V = (x.transpose(0, 2, 1, 3) for x in (Q, K, V))
    q, k, v = (x.astype(np.float64) for x in (Q, K, V))
    H, Hkv, S = q.shape[1], k.shape[1], q.shape[2]
    k = np.repeat(k, H // Hkv, axis=1)
    v = np.repeat(v, H // Hkv, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    if causal:
        s[..., np.triu(np.ones((S, S), bool), 1)] = -np.inf
    mx = s.max(-1, keepdims=True)
    p = np.exp(s - mx)
    den = p.sum(-1, keepdims=True) + phantom * np.exp(-mx)  # phantom keys: score 0, value 0
    o = np.einsum("bhqk,bhkd->bhqd", p, v) / den
    return o.transpose(0, 2, 1, 3) if layout == "bshd" else o


@pytest.mark.parametrize("B,H,Hkv,S,causal,layout", [
    (1, 2, 2, 64, True, "bhsd"), (1, 1, 1, 150, True, "bhsd"), (2, 2, 2, 128, False, "bhsd"),
    (1, 4, 2, 90, True, "bshd"), (1, 3, 1, 70, False, "bshd")])
def test_attention_vs_float64(oracle_mod, B, H, Hkv, S, causal, layout):
    rng = np.random.default_rng(S + H)
    shp = (lambda h: (B, h, S, 128)) if layout == "bhsd" else (lambda h: (B, S, h, 128))
    Q = rng.standard_normal(shp(H)).astype(np.float16)
    K = rng.standard_normal(shp(Hkv)).astype(np.float16)
    V = rng.standard_normal(shp(Hkv)).astype(np.float16)
    scale = 1 / np.sqrt(128)
    O = oracle_mod.attention(Q, K, V, causal=causal, scale=scale, layout=layout)
    ref = _np_attention(Q, K, V, causal, scale, layout)
    assert oracle_mod.rel_frobenius(O, ref) < 1e-3


def test_attention_refcompat_phantom_keys(oracle_mod):
    """Non-causal with a ragged last key block: the reference counts the zero keys that
    pad seq to a multiple of 64 in the row sum (score 0, value 0)."""
    rng = np.random.default_rng(3)
    S = 100
    Q, K, V = (rng.standard_normal((1, 1, S, 128)).astype(np.float16) for _ in range(3))
    scale = 1 / np.sqrt(128)
    O = oracle_mod.attention(Q, K, V, causal=False, scale=scale, refcompat=True)
    assert oracle_mod.rel_frobenius(O, _np_attention(Q, K, V, False, scale, phantom=28)) < 1e-3
    # Causal attention masks the padding: refcompat changes nothing there.
    a = oracle_mod.attention(Q, K, V, causal=True, scale=scale, refcompat=True)
    b = oracle_mod.attention(Q, K, V, causal=True, scale=scale)
    assert np.array_equal(a, b)


def test_attention_known_answers(oracle_mod):
    """Identical keys give uniform weights (O = mean of the visible values); one
    dominant key gives O = its value."""
    S = 64
    Q = np.ones((1, 1, S, 128), np.float16)
    K = np.ones((1, 1, S, 128), np.float16)
    V = np.tile(np.arange(S, dtype=np.float16)[:, None], (1, 128))[None, None]
    O = oracle_mod.attention(Q, K, V, causal=True, scale=0.01)
    want = np.array([np.arange(q + 1).mean() for q in range(S)], np.float64)
    assert np.allclose(O[0, 0, :, 0].astype(np.float64), want, rtol=2e-3)
    K2 = np.zeros_like(K)
    K2[0, 0, 17] = 4.0
    O2 = oracle_mod.attention(Q, K2, V, causal=False, scale=1.0)
    assert np.allclose(O2[0, 0, :, 5].astype(np.float64), 17.0, rtol=1e-3)


@pytest.mark.parametrize("fname", _golden_files("ref_attn_") or ["<none>"])
def test_oracle_vs_reference_attention_golden(oracle_mod, fname):
    """Outputs of the reference flash_attention kernel (run on a B200). The oracle
    follows its steps (64-key blocks, expf online softmax); the GPU's expf and
    summation order differ from the host's in the last bits only."""
    if fname == "<none>":
        pytest.skip("no reference attention golden vectors generated yet")
    d = np.load(os.path.join(GOLDEN, fname))
    causal = bool(d["causal"])
    O = oracle_mod.attention(d["Q"], d["K"], d["V"], causal=causal, scale=float(d["scale"]),
                             refcompat=True)
    ref = d["O_ref"]
    assert oracle_mod.rel_frobenius(O, ref) < 2e-3
    diff = np.abs(O.astype(np.float32) - ref.astype(np.float32))
    assert diff.max() <= 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))
