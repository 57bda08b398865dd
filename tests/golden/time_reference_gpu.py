"""Times the reference's own GEMM kernels on a B200, as a reported baseline.

The reference kernels (clove::gemm_fp16 -> WMMA kernel for M,N >= 128, naive
kernel otherwise, src/kernels/gemm_fp16.cu:277-305; clove::gemm_int4,
src/kernels/gemm_int4.cu:195-216) are built unmodified from the reference tree by
``make -C oracle ref`` into oracle/_ref/libclove_ref.so. The reference int8 kernel
is not run: it reads shared memory out of bounds (gemm_int8.cu:77,84).

Every shape below keeps the reference kernels inside the bounds they handle: M and
N multiples of 128 for the WMMA kernel's unmasked 16x16 stores; the int4 kernel
guards all of its loads and stores. The int4 kernel computes different math from
the documented layout (zero points ignored, last group's scales) and takes B as
[K,N/2], so decode is timed at N=2; these are timings, not parity cases.

Run on a GPU box from the repo root:
    python tests/golden/time_reference_gpu.py OUT.json
Timing: CUDA events around back-to-back launches after warm-up, median of 5.
"""
from __future__ import annotations

import ctypes
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libclove_ref.so")


def _time(fn, iters: int) -> float:
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) / iters)
    ts.sort()
    return ts[2]  # ms


def main(out_path: str) -> None:
    lib = ctypes.CDLL(REF_LIB)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.clove_ref_gemm_fp16.argtypes = [P, P, P, I, I, I, F, F, P]
    lib.clove_ref_gemm_int4.argtypes = [P, P, P, P, P, P, P, I, I, I, P]
    g = torch.Generator(device="cuda").manual_seed(0)
    rows = []

    fp16_cases = [  # name, M, N, K, iters
        ("fp16 decode 1x4096x4096 (naive kernel)", 1, 4096, 4096, 20),
        ("fp16 1024^3 (config 1)", 1024, 1024, 1024, 20),
        ("fp16 4096^3", 4096, 4096, 4096, 5),
        ("fp16 FFN up 11008x2048x4096 (config 4)", 11008, 2048, 4096, 3),
        ("fp16 FFN down 4096x2048x11008 (config 4)", 4096, 2048, 11008, 3),
        ("fp16 8192^3", 8192, 8192, 8192, 2),
    ]
    for name, M, N, K, iters in fp16_cases:
        A = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g) / K ** 0.5
        B = torch.randn(K, N, device="cuda", dtype=torch.float16, generator=g) / K ** 0.5
        C = torch.empty(M, N, device="cuda", dtype=torch.float16)
        stream = torch.cuda.current_stream().cuda_stream

        def run():
            rc = lib.clove_ref_gemm_fp16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K,
                                         1.0, 0.0, stream)
            assert rc == 0, rc

        ms = _time(run, iters)
        rows.append({"kernel": "reference gemm_fp16", "case": name, "M": M, "N": N, "K": K,
                     "ms": round(ms, 4), "TFLOPS": round(2.0 * M * N * K / ms / 1e9, 2)})
        print(rows[-1], flush=True)
        del A, B, C

    int4_cases = [  # name, M, N, K, iters
        ("int4 decode 4096x2x4096 (config 2 at N=2)", 4096, 2, 4096, 20),
        ("int4 8192^3 (config 5)", 8192, 8192, 8192, 2),
    ]
    for name, M, N, K, iters in int4_cases:
        Aq = torch.randint(0, 256, (M, K // 2), device="cuda", dtype=torch.uint8, generator=g)
        As = torch.full((M, K // 128), 0.01, device="cuda", dtype=torch.float16)
        Az = torch.full((M, K // 128), 8.0, device="cuda", dtype=torch.float16)
        Bq = torch.randint(0, 256, (K, N // 2), device="cuda", dtype=torch.uint8, generator=g)
        Bs = torch.full((K // 128, N), 0.01, device="cuda", dtype=torch.float16)
        Bz = torch.full((K // 128, N), 8.0, device="cuda", dtype=torch.float16)
        C = torch.empty(M, N, device="cuda", dtype=torch.float16)
        stream = torch.cuda.current_stream().cuda_stream

        def run():
            rc = lib.clove_ref_gemm_int4(Aq.data_ptr(), As.data_ptr(), Az.data_ptr(), Bq.data_ptr(),
                                         Bs.data_ptr(), Bz.data_ptr(), C.data_ptr(), M, N, K, stream)
            assert rc == 0, rc

        ms = _time(run, iters)
        nbytes = M * K // 2 + 2 * 2 * M * K // 128 + K * N // 2 + 2 * 2 * N * K // 128 + 2 * M * N
        rows.append({"kernel": "reference gemm_int4", "case": name, "M": M, "N": N, "K": K,
                     "ms": round(ms, 4), "TOPS": round(2.0 * M * N * K / ms / 1e9, 3),
                     "GBps": round(nbytes / ms / 1e6, 1)})
        print(rows[-1], flush=True)
        del Aq, As, Az, Bq, Bs, Bz, C

    with open(out_path, "w") as f:
        json.dump({"device": torch.cuda.get_device_name(0), "rows": rows}, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "ref_gpu.json")
