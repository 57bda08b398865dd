"""The drop-in C++ boundary on the GPU.

* tests/cxx/runtime_linear_layers.cu: the reference runtime's linear-layer call
  forms through include/clove/kernels/gemm.cuh, built against the library and run.
  Every call returns without a CUDA error, and a seeded projection (beta = 0) and
  the in-place residual (beta = 1) match the CPU oracle.
* tests/cxx/common_reductions.cu: the reference-compatible device helpers of
  include/clove/common.cuh, bit for bit against the same reductions in the
  documented order on the CPU."""
import os
import shutil
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _nvcc():
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else shutil.which("nvcc")
    if nvcc is None:
        pytest.skip("nvcc not available")
    return nvcc


def test_cxx_runtime_call_sites_run(clove_lib, cuda, oracle_mod, tmp_path):
    lib_dir = os.path.dirname(clove_lib.library_path())
    exe = str(tmp_path / "runtime_linear_layers")
    r = subprocess.run([_nvcc(), "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                        "-I" + os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "cxx", "runtime_linear_layers.cu"), "-o", exe,
                        "-L" + lib_dir, "-lclove_b200", "-Xlinker", "-rpath=" + lib_dir],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    run = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "status 0 dump ok" in run.stdout

    T, H = 128, 256
    ld = lambda n, shape: np.fromfile(str(tmp_path / (n + ".f16")), np.float16).reshape(shape)
    X, Wq, q = ld("X", (T, H)), ld("Wq", (H, H)), ld("q", (T, H))
    attn, Wo = ld("attn", (T, H)), ld("Wo", (H, H))
    hidden0, res = ld("hidden0", (T, H)), ld("res", (T, H))
    rel = lambda x, y: float(np.linalg.norm(x.astype(np.float64) - y.astype(np.float64)) /
                             np.linalg.norm(y.astype(np.float64)))
    assert rel(q, oracle_mod.gemm_fp16(X, Wq)) < 1e-2
    ref = oracle_mod.gemm_fp16(attn, Wo, C=hidden0.copy(), alpha=1.0, beta=1.0)
    assert rel(res, ref) < 1e-2
    # the residual really was added (beta = 1 read C before overwriting it)
    assert rel(res, oracle_mod.gemm_fp16(attn, Wo)) > 0.1


def _butterfly_sum(v):
    """warp_reduce_sum of clove/common.cuh in float32: lanes fold at XOR distances
    16, 8, 4, 2, 1."""
    v = np.asarray(v, np.float32).copy()
    lanes = np.arange(32)
    for d in (16, 8, 4, 2, 1):
        v = (v + v[lanes ^ d]).astype(np.float32)
    return v


def test_common_header_reductions(cuda, tmp_path):
    exe = str(tmp_path / "common_reductions")
    r = subprocess.run([_nvcc(), "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                        "-I" + os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "cxx", "common_reductions.cu"), "-o", exe],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and "status 0" in run.stdout, run.stdout[-500:] + run.stderr
    x = np.zeros(256, np.uint32)
    out = np.zeros(41, np.uint32)
    for line in run.stdout.splitlines():
        f = line.split()
        if f[0] == "x":
            x[int(f[1])] = int(f[2], 16)
        elif f[0] == "out":
            out[int(f[1])] = int(f[2], 16)
    x = x.view(np.float32)
    got = out.view(np.float32)
    # warp 0's lanes
    np.testing.assert_array_equal(got[:32], _butterfly_sum(x[:32]))
    assert got[40] == np.max(x[:32])
    # block: per-warp totals (lane 0 of each warp), folded by warp 0 with zero padding
    warp_tot = np.array([_butterfly_sum(x[w * 32:(w + 1) * 32])[0] for w in range(8)], np.float32)
    pad = np.zeros(32, np.float32)
    pad[:8] = warp_tot
    assert got[32] == _butterfly_sum(pad)[0]
    assert got[33] == np.max(x)
    x2 = (2.0 * x).astype(np.float32)
    warp_tot2 = np.array([_butterfly_sum(x2[w * 32:(w + 1) * 32])[0] for w in range(8)], np.float32)
    pad[:8] = warp_tot2
    assert got[34] == _butterfly_sum(pad)[0]  # back-to-back reductions in one kernel
    assert got[35] == 0.0                      # the result lives in warp 0
    assert got[36] == 7.75                     # half4 via make_half4
