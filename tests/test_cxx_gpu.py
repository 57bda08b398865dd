"""The drop-in C++ boundary on the GPU: tests/cxx/runtime_linear_layers.cu (the
reference runtime's linear-layer call forms through include/clove/kernels/gemm.cuh)
built against the library and run; every call must return without a CUDA error."""
import os
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cxx_runtime_call_sites_run(clove_lib, cuda, tmp_path):
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else shutil.which("nvcc")
    if nvcc is None:
        pytest.skip("nvcc not available")
    lib_dir = os.path.dirname(clove_lib.library_path())
    exe = str(tmp_path / "runtime_linear_layers")
    r = subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                        "-I" + os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "cxx", "runtime_linear_layers.cu"), "-o", exe,
                        "-L" + lib_dir, "-lclove_b200", "-Xlinker", "-rpath=" + lib_dir],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "status 0" in run.stdout
