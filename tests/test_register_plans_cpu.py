"""Register and spill plans that the kernels' speed rests on, checked on the CPU from
ptxas's report (nvcc cross-compiles for sm_100a without a GPU):

* the INT4 decode GEMVs that run several CTAs per SM: four CTAs of 256 threads need at
  most 64 registers per thread, two of 384 at most 85, and none may spill;
* the attention kernel, whose setmaxnreg split assumes exactly 168 registers at launch
  (the host refuses any other count at run time), spills nothing;
* the INT4 tensor-core kernel, planned for 96 registers at launch the same way.
"""
import concurrent.futures as cf
import os
import re
import subprocess

import pytest

from clove_compute_b200 import build as B

KERNELS = os.path.join(B.CSRC, "kernels")


def _ptxas(src, tmp):
    obj = os.path.join(tmp, os.path.basename(src) + ".o")
    cmd = [B._nvcc()] + B.COMMON + B.ARCH + ["-Xptxas", "-v", "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stderr


def _report(log):
    """{mangled entry name: [registers, (spill store bytes, spill load bytes)]}."""
    out, cur = {}, None
    for line in log.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            cur = m.group(1)
            out[cur] = [None, None]
            continue
        if cur is None:
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and out[cur][1] is None:
            out[cur][1] = (int(m.group(1)), int(m.group(2)))
        m = re.search(r"Used (\d+) registers", line)
        if m and out[cur][0] is None:
            out[cur][0] = int(m.group(1))
    return out


@pytest.fixture(scope="module")
def reports(tmp_path_factory):
    tmp = str(tmp_path_factory.mktemp("ptxas"))
    srcs = [os.path.join(KERNELS, f) for f in
            ("gemv_sm100.cu", "attention_sm100.cu", "gemm_int4_sm100.cu")]
    with cf.ThreadPoolExecutor(len(srcs)) as ex:
        logs = list(ex.map(lambda s: _ptxas(s, tmp), srcs))
    rep = {}
    for log in logs:
        rep.update(_report(log))
    return rep


def _entries(rep, pattern):
    hits = {k: v for k, v in rep.items() if re.search(pattern, k)}
    assert hits, f"no kernel matches {pattern}"
    return hits


# gemv_int4_ldg_kernel<NC, PW, RMAX, MINB, RG, WG>
@pytest.mark.parametrize("pattern,max_regs", [
    (r"gemv_int4_ldg_kernelILi1ELi1ELi4ELi4ELi2ELi4E", 64),   # 4 CTAs x 256 threads
    (r"gemv_int4_ldg_kernelILi2ELi1ELi4ELi4ELi2ELi4E", 64),   # 4 CTAs x 256 threads
    (r"gemv_int4_ldg_kernelILi1ELi1ELi8ELi2ELi1ELi12E", 85),  # 2 CTAs x 384 threads
])
def test_decode_gemv_several_ctas_per_sm(reports, pattern, max_regs):
    for name, (regs, spill) in _entries(reports, pattern).items():
        assert regs is not None and regs <= max_regs, (name, regs)
        assert spill == (0, 0), (name, spill)


def test_attention_register_plan(reports):
    hits = _entries(reports, r"attention_fwd_kernel")
    assert len(hits) == 2  # causal and full
    for name, (regs, spill) in hits.items():
        assert regs == 168, (name, regs)
        assert spill == (0, 0), (name, spill)


def test_int4_tensor_core_register_plan(reports):
    for name, (regs, spill) in _entries(reports, r"gemm_int4_tc_kernel").items():
        assert regs == 96, (name, regs)
        assert spill == (0, 0), (name, spill)
