"""Records golden vectors from the reference's own GEMM kernels (run on a B200).

The reference ships no golden vectors or known-answer tests for this path, so
these fixtures pin the CPU oracle against the reference itself:

* ``ref_fp16_*.npz``: inputs and the output of the reference clove::gemm_fp16
  (src/kernels/gemm_fp16.cu:277-305; WMMA kernel for M,N >= 128, naive kernel
  otherwise). The WMMA kernel accumulates in fp16, so the oracle must match it
  within the recorded ``tol`` (relative Frobenius), the naive one within 1e-3.
* ``ref_int4_*.npz``: inputs and the output of the reference clove::gemm_int4
  (gemm_int4.cu:195-216); the oracle's ref-compat restatement must match it
  bit for bit, which pins the nibble order, the packing and the scale indexing.
* ``ref_attn_*.npz``: inputs and the output of the reference clove::flash_attention
  (attention.cu:93-310, head_dim 128, [batch, heads, seq, 128]) through
  oracle/ref_attn_shim.cu, which only lifts the kernel's 48 KB shared-memory launch
  limit that the reference never raises. Pins the oracle's attention restatement
  (scale, causal mask, online softmax, and the phantom keys of a ragged non-causal
  last block).

Run on a GPU box from the repo root after ``make -C oracle ref``:
    python tests/golden/make_golden.py [OUT_DIR] [--only gemm|attn]
It only writes OUT_DIR/*.npz (default tests/golden/). Shapes keep every reference kernel inside
the bounds it handles (M, N multiples of 16 for the WMMA store).
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from clove_compute_b200 import workloads as wl  # noqa: E402

REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libclove_ref.so")
REF_ATTN_LIB = os.path.join(ROOT, "oracle", "_ref", "libclove_ref_attn.so")

# (name, batch, heads, seq, causal): shapes the reference kernel handles (head_dim
# 128; a ragged seq only causal, or non-causal to record its phantom keys).
ATTN_CASES = [("causal_1x2x256", 1, 2, 256, True), ("causal_1x2x200", 1, 2, 200, True),
              ("full_2x1x128", 2, 1, 128, False), ("full_ragged_1x1x100", 1, 1, 100, False)]


def attention_cases(out_dir: str):
    lib = ctypes.CDLL(REF_ATTN_LIB)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.clove_ref_flash_attention.argtypes = [P, P, P, P, I, I, I, I, F, I, P]
    for name, B, H, S, causal in ATTN_CASES:
        rng = np.random.default_rng(B * 1000 + H * 100 + S)
        Q, K, V = (rng.standard_normal((B, H, S, 128)).astype(np.float16) for _ in range(3))
        Qd, Kd, Vd = (torch.from_numpy(x).cuda() for x in (Q, K, V))
        Od = torch.zeros_like(Qd)
        scale = 1.0 / np.sqrt(128.0)
        rc = lib.clove_ref_flash_attention(*[ctypes.c_void_p(t.data_ptr()) for t in (Qd, Kd, Vd, Od)],
                                           B, H, S, 128, scale, int(causal), None)
        torch.cuda.synchronize()
        assert rc == 0, rc
        np.savez(os.path.join(out_dir, f"ref_attn_{name}.npz"), Q=Q, K=K, V=V,
                 O_ref=Od.cpu().numpy(), scale=scale, causal=causal)


def main(out_dir: str = HERE, only: str = ""):
    os.makedirs(out_dir, exist_ok=True)
    if only == "attn":
        attention_cases(out_dir)
        print("golden vectors written to", out_dir)
        return
    lib = ctypes.CDLL(REF_LIB)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.clove_ref_gemm_fp16.argtypes = [P, P, P, I, I, I, F, F, P]
    lib.clove_ref_gemm_int4.argtypes = [P, P, P, P, P, P, P, I, I, I, P]
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    p = lambda t: ctypes.c_void_p(t.data_ptr())

    fp16_cases = [  # (name, M, N, K, alpha, beta, tol)
        ("naive_64", 64, 64, 64, 1.0, 0.0, 1e-3),
        ("naive_decode_1x256x256", 1, 256, 256, 1.0, 0.0, 1e-3),
        ("wmma_128x128x256", 128, 128, 256, 1.0, 0.0, 1e-2),
        ("wmma_alpha_beta_128", 128, 128, 128, 0.5, 0.25, 1e-2),
    ]
    for name, M, N, K, alpha, beta, tol in fp16_cases:
        A, B = wl.fp16_operands(M, N, K, seed=M + N + K)
        C0 = np.random.default_rng(7).uniform(-0.1, 0.1, (M, N)).astype(np.float16)
        # Keep every device tensor referenced until the kernel has run: a temporary
        # freed inside the argument list is handed out again by torch's caching
        # allocator to the next operand.
        Ad, Bd, Cd = d(A), d(B), d(C0.copy())
        rc = lib.clove_ref_gemm_fp16(p(Ad), p(Bd), p(Cd), M, N, K, alpha, beta, None)
        torch.cuda.synchronize()
        assert rc == 0, rc
        np.savez(os.path.join(out_dir, f"ref_fp16_{name}.npz"), A=A, B=B, C0=C0,
                 C_ref=Cd.cpu().numpy(), alpha=alpha, beta=beta, tol=tol)

    int4_cases = [(64, 64, 256), (128, 8, 512), (64, 3, 256), (32, 2, 4096)]
    for M, N, K in int4_cases:
        rng = np.random.default_rng(M * 1000 + N)
        Aq = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
        As = rng.uniform(0.005, 0.02, (M, K // 128)).astype(np.float16)
        Az = np.zeros((M, K // 128), np.float16)  # read by nobody (gemm_int4.cu:48)
        Bq = rng.integers(0, 256, (K, N // 2), dtype=np.uint8)
        Bs = rng.uniform(0.005, 0.02, (K // 128, N)).astype(np.float16)
        Bz = np.zeros((K // 128, N), np.float16)
        C = torch.zeros((M, N), dtype=torch.float16, device="cuda")
        Bq_d = d(Bq) if Bq.size else torch.zeros(1, dtype=torch.uint8, device="cuda")
        ops = [d(Aq), d(As), d(Az), Bq_d, d(Bs), d(Bz), C]
        rc = lib.clove_ref_gemm_int4(*[p(t) for t in ops], M, N, K, None)
        torch.cuda.synchronize()
        assert rc == 0, rc
        np.savez(os.path.join(out_dir, f"ref_int4_{M}x{N}x{K}.npz"), A_q=Aq, A_scale=As, B_q=Bq,
                 B_scale=Bs, C_ref=C.cpu().numpy(), M=M, N=N, K=K)
    if only != "gemm":
        attention_cases(out_dir)
    print("golden vectors written to", out_dir)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--only")]
    only = next((a.split("=", 1)[1] for a in sys.argv[1:] if a.startswith("--only=")), "")
    main(args[0] if args else HERE, only)
