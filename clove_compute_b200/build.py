"""Builds the in-tree shared library ``clove_compute_b200/libclove_b200.so``.

Every CUDA source is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``); nvcc cross-compiles without a GPU. Objects
go to ``clove_compute_b200/_build/`` and are rebuilt when a source or any
header under ``csrc/`` or ``include/`` is newer. Run ``python -m
clove_compute_b200.build`` (``-v`` prints ptxas register / spill reports).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libclove_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [
    "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*", "*.cu")) +
                  glob.glob(os.path.join(CSRC, "*", "*.cpp")))


def _headers():
    return (glob.glob(os.path.join(CSRC, "*", "*.cuh")) + glob.glob(os.path.join(CSRC, "*", "*.h")) +
            glob.glob(os.path.join(ROOT, "include", "clove", "**", "*.h*"), recursive=True))


def _obj(src: str) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(src: str, verbose: bool) -> str:
    obj = _obj(src)
    cmd = [_nvcc()] + COMMON + ARCH + ["-c", src, "-o", obj]
    if verbose and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if verbose else ""


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    newest_hdr = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    todo = []
    for s in srcs:
        o = _obj(s)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), newest_hdr):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for s, log in zip(todo, ex.map(lambda x: _compile(x, verbose), todo)):
                if log:
                    print(f"== {os.path.relpath(s, ROOT)}\n{log}", file=sys.stderr)
    objs = [_obj(s) for s in srcs]
    if todo or force or not os.path.exists(LIB) or \
            os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [_nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
