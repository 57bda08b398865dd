"""CPU checks of the product library: it loads, exports every entry point that
include/clove/capi.h declares, and its pure host logic behaves (no GPU needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    txt = open(os.path.join(ROOT, "include", "clove", "capi.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(clove_[a-z0-9_]+)\s*\(", txt)))


def test_header_declares_expected_entry_points():
    names = _declared_functions()
    for n in ["clove_gemm_fp16", "clove_gemm_int8", "clove_gemm_int4", "clove_gemm_fp16_batched",
              "clove_gemm_int8_rowcol", "clove_debug_int4_group_acc", "clove_last_error_string"]:
        assert n in names


def test_library_exports_every_declared_symbol(clove_lib):
    lib = ctypes.CDLL(clove_lib.library_path())
    missing = [n for n in _declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header(clove_lib):
    from clove_compute_b200._lib import SIGNATURES
    assert set(_declared_functions()) <= set(SIGNATURES)


def test_version_and_error_string(clove_lib):
    lib = clove_lib.lib()
    assert b"sm_100a" in lib.clove_version()
    assert isinstance(lib.clove_last_error_string(), bytes)


@pytest.mark.parametrize("N,P", [(2048, 8), (11008, 8), (7, 8), (0, 4), (13, 3), (1, 2)])
def test_nsplit_column_partition(clove_lib, N, P):
    bounds = [clove_lib.col_begin(N, P, r) for r in range(P + 1)]
    assert bounds[0] == 0 and bounds[-1] == N
    widths = [b - a for a, b in zip(bounds, bounds[1:])]
    assert all(w >= 0 for w in widths)
    assert max(widths) - min(widths) <= 1
    assert widths == sorted(widths, reverse=True)  # extra columns go to the first ranks


def test_dispatch_description_without_gpu(clove_lib):
    d = clove_lib.describe_dispatch("fp16", 11008, 2048, 4096)
    assert d.startswith("tc2_f16")  # CTA-pair 256x256 tiles for the FFN shape
    assert clove_lib.describe_dispatch("int4", 4096, 1, 4096).startswith("gemv_int4")
    # INT4 prefill at the FFN down projection's K = 11008 stays on the tensor cores.
    assert clove_lib.describe_dispatch("int4", 4096, 2048, 11008).startswith("tc_int4")
    assert clove_lib.describe_dispatch("int8", 4096, 32, 4096).startswith("tc_int8")
    assert "split" in clove_lib.describe_dispatch("int8", 4096, 32, 4096)


@pytest.mark.parametrize("M,N,K,want", [
    (4096, 1, 4096, "ldg 4 CTAs/SM of 2x4 warps"),      # config 2
    (12288, 1, 4096, "ldg 4 CTAs/SM of 2x4 warps"),     # Q/K/V in one call
    (4096, 1, 11008, "ldg 2 CTAs/SM of 1x12 warps"),    # down projection, 11 windows
    (4096, 2, 4096, "ldg 4 CTAs/SM of 2x4 warps"),      # two vectors
    (2367, 1, 4096, "ldg 1 CTA/SM of 4x4 warps"),       # below 2 x 148 x 8 rows
    (4096, 2, 8192, "shared-B"),                        # 16 windows of B
    (4096, 4, 2048, "register-B"),                      # 3-8 vectors, <= 8 windows in all
    (1, 4096, 4096, "ldg 4 CTAs/SM of 2x4 warps"),      # transposed: rows of B stream
])
def test_int4_decode_variant_without_gpu(clove_lib, M, N, K, want):
    """The decode GEMV variant follows from the shape alone (148 SMs assumed here)."""
    d = clove_lib.describe_dispatch("int4", M, N, K)
    assert d.startswith("gemv_int4") and d.endswith(f"({want})"), d


def test_small_m_fp16_plan_without_gpu(clove_lib):
    # One 128-row band: 128-column tiles on 4-CTA clusters for up to 32 live rows
    # or K of at least 96 blocks of 64; otherwise 64-column tiles on 2-CTA clusters.
    assert clove_lib.describe_dispatch("fp16", 1, 4096, 4096) == "tc_f16 bn=128 split=4"
    assert clove_lib.describe_dispatch("fp16", 32, 4096, 4096) == "tc_f16 bn=128 split=4"
    assert clove_lib.describe_dispatch("fp16", 64, 4096, 4096) == "tc_f16 bn=64 split=2"
    assert clove_lib.describe_dispatch("fp16", 64, 4096, 6080) == "tc_f16 bn=64 split=2"
    assert clove_lib.describe_dispatch("fp16", 64, 4096, 6144) == "tc_f16 bn=128 split=4"
    assert clove_lib.describe_dispatch("fp16", 128, 4096, 11008) == "tc_f16 bn=128 split=4"
    # int8 (128 codes per K block): long K only.
    assert clove_lib.describe_dispatch("int8", 1, 4096, 4096) == "tc_int8 bn=64 split=2"
    assert clove_lib.describe_dispatch("int8", 1, 4096, 8064) == "tc_int8 bn=64 split=2"
    assert clove_lib.describe_dispatch("int8", 1, 4096, 8192) == "tc_int8 bn=128 split=4"
    assert clove_lib.describe_dispatch("int8", 1, 4096, 11008) == "tc_int8 bn=128 split=4"


def test_swiglu_dispatch_without_gpu(clove_lib):
    assert clove_lib.describe_dispatch("swiglu", 2048, 11008, 4096).startswith("tc2_swiglu")
    assert clove_lib.describe_dispatch("swiglu", 64, 11008, 4096).startswith("unfused")
    assert clove_lib.describe_dispatch("swiglu", 2048, 11008, 4100).startswith("unfused")


def test_split_k_clusters_are_powers_of_two(clove_lib):
    # A split tile's 128 rows are dealt out evenly over the cluster: 2, 4 or 8 CTAs.
    for M, N, K in [(4096, 32, 4096), (256, 96, 4096), (128, 64, 8192), (384, 64, 4096)]:
        d = clove_lib.describe_dispatch("int8", M, N, K)
        split = int(d.split("split=")[1].split()[0])
        assert split in (1, 2, 4, 8), d


def test_host_argument_checks_need_no_gpu(clove_lib):
    """Argument errors are reported before any device work."""
    lib = clove_lib.lib()
    # K not a multiple of the 128-element group
    assert lib.clove_quantize_int4(None, 4, 200, None, None, None, None) == clove_lib.CLOVE_ERR_INVALID_ARG
    assert lib.clove_quantize_int4(None, -1, 128, None, None, None, None) == clove_lib.CLOVE_ERR_INVALID_ARG
    assert lib.clove_swiglu_fused(None, None, None, None, -1, 8, 8, None) == clove_lib.CLOVE_ERR_INVALID_ARG
    assert lib.clove_gemm_fp16_batched(None, None, None, -2, 8, 8, 8, 1.0, 0.0, None) == \
        clove_lib.CLOVE_ERR_INVALID_ARG
    # empty problems are no-ops
    assert lib.clove_swiglu_fused(None, None, None, None, 0, 8, 8, None) == clove_lib.CLOVE_OK
    assert lib.clove_quantize_int4(None, 0, 128, None, None, None, None) == clove_lib.CLOVE_OK


def _stream_k_pieces(plan, kb):
    """Restates the CTA-pair kernel's per-pair work order (Tc2Sched in
    csrc/kernels/gemm_tc2_sm100.cuh): each pair's contiguous range of stream-K
    units, then its round-robin whole-K tiles. Yields (pair, tile, kb0, kb1, sk_idx,
    j, nc)."""
    P, dp, sk = plan["pairs"], plan["dp_tiles"], plan["sk_tiles"]
    U = sk * kb
    owner = lambda v: ((v + 1) * P + U - 1) // U - 1
    for p in range(P):
        u, ue = U * p // P, U * (p + 1) // P
        while u < ue:
            t = u // kb
            kb0 = u - t * kb
            kb1 = min(kb, kb0 + ue - u)
            first = owner(t * kb)
            yield p, dp + t, kb0, kb1, t, p - first, owner(t * kb + kb - 1) - first + 1
            u += kb1 - kb0
        for t in range(p, dp, P):
            yield p, t, 0, kb, -1, 0, 1


@pytest.mark.parametrize("tiles,pairs,kb,force", [
    (344, 74, 64, 2),    # FFN up: 4.65 waves
    (128, 74, 172, 0),   # FFN down: 1.73 waves
    (256, 74, 64, 2),    # 4096^3: a partial wave under half full -> one full wave joins it
    (80, 74, 64, 2), (1024, 74, 128, 0), (296, 74, 64, 2), (112, 74, 172, 0),
    (5, 74, 64, 2), (7, 3, 5, 2), (10, 4, 3, 2), (1, 74, 200, 2), (3, 2, 1, 2)])
def test_stream_k_schedule_covers_each_k_block_once(clove_lib, tiles, pairs, kb, force):
    plan = clove_lib.debug_stream_k_plan(tiles, pairs, kb, force)
    assert plan["dp_tiles"] + plan["sk_tiles"] == tiles
    pieces = list(_stream_k_pieces(plan, kb))
    by_tile = {}
    for p, t, kb0, kb1, ski, j, nc in pieces:
        assert 0 <= kb0 < kb1 <= kb
        by_tile.setdefault(t, []).append((kb0, kb1, ski, j, nc, p))
    assert sorted(by_tile) == list(range(tiles))
    load = [0] * plan["pairs"]
    for t, ps in by_tile.items():
        ps.sort()
        assert ps[0][0] == 0 and ps[-1][1] == kb
        assert all(a[1] == b[0] for a, b in zip(ps, ps[1:]))  # contiguous, no overlap
        nc = len(ps)
        assert all(x[4] == nc for x in ps)
        assert sorted(x[3] for x in ps) == list(range(nc))     # one partial slot each
        assert [x[5] for x in ps] == sorted(x[5] for x in ps)  # consecutive pairs
        if nc > 1:
            assert nc <= plan["max_contrib"]
        for kb0, kb1, ski, j, _, p in ps:
            if ski >= 0:
                load[p] += kb1 - kb0
    if plan["sk_tiles"]:
        assert max(load) - min(load) <= 1  # stream-K ranges differ by at most one K block


def test_stream_k_plans_for_the_ffn_shapes(clove_lib):
    up = clove_lib.debug_stream_k_plan(43 * 8, 74, 64)       # 11008 x 2048, K = 4096
    down = clove_lib.debug_stream_k_plan(16 * 8, 74, 172)    # 4096 x 2048, K = 11008
    assert up["sk_tiles"] == 0  # 7 % idle over 64 K blocks: not worth the fixed cost
    assert down["sk_tiles"] == 128 % 74 and down["max_contrib"] <= 3
    assert clove_lib.debug_stream_k_plan(43 * 8, 74, 64, 2)["sk_tiles"] == 344 % 74
    # A last wave of 1024 / 74 = 13.8 waves idles 1 %: plain persistent tiles.
    assert clove_lib.debug_stream_k_plan(1024, 74, 128)["sk_tiles"] == 0
    assert clove_lib.debug_stream_k_plan(100, 74, 64, 1)["sk_tiles"] == 0
    assert clove_lib.debug_stream_k_plan(5, 74, 64)["pairs"] == 5


def test_cxx_runtime_call_sites_compile_and_link(clove_lib, tmp_path):
    """The reference runtime's linear-layer calls (inference.cu:139-194) compile
    against include/clove/kernels/gemm.cuh and link against the library, as a C++
    integration would (nvcc cross-compiles; the binary is not run here)."""
    import shutil
    import subprocess
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else shutil.which("nvcc")
    if nvcc is None:
        pytest.skip("nvcc not available")
    lib_dir = os.path.dirname(clove_lib.library_path())
    exe = str(tmp_path / "runtime_linear_layers")
    cmd = [nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I" + os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "cxx", "runtime_linear_layers.cu"),
           "-o", exe, "-L" + lib_dir, "-lclove_b200", "-Xlinker", "-rpath=" + lib_dir]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    assert os.path.exists(exe)


def test_reference_kernels_build_against_dropin_headers(clove_lib, tmp_path):
    """The integration recipe: this repository's include/ ahead of the reference's.
    The reference's other kernels (layernorm, softmax, activations, rope, attention,
    which use CudaType, half4/half8 and the warp / block reductions of clove/common.cuh)
    still compile against it and link, together with the runtime's linear-layer call
    sites, against the library. Needs the reference source tree (CLOVE_REF_DIR, by
    default a `reference` directory beside this repository); skipped without it."""
    import shutil
    import subprocess
    from conftest import reference_dir
    ref = reference_dir()
    if ref is None:
        pytest.skip("reference source tree not present")
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else shutil.which("nvcc")
    if nvcc is None:
        pytest.skip("nvcc not available")
    lib_dir = os.path.dirname(clove_lib.library_path())
    kernels = [os.path.join(ref, "src", "kernels", f + ".cu")
               for f in ("layernorm", "softmax", "activations", "rope", "attention")]
    exe = str(tmp_path / "block_with_reference_kernels")
    # The reference's own build flags plus the two forced includes its headers
    # need with GCC 13 (<cstdint>, <cassert>). One object per source, compiled in
    # parallel, then one link.
    flags = ["-std=c++17", "-O3", "--use_fast_math", "--expt-relaxed-constexpr",
             "-include", "cstdint", "-include", "cassert",
             "-gencode", "arch=compute_100a,code=sm_100a",
             "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(ref, "include")]
    srcs = [os.path.join(ROOT, "tests", "cxx", "runtime_linear_layers.cu"), *kernels]
    objs = [str(tmp_path / (os.path.basename(f) + ".o")) for f in srcs]

    def compile_one(i):
        # attention.cu's kernels take minutes in the device optimiser (cicc): they are
        # compiled unoptimised (-Xcicc -O0), which still runs the front end these
        # headers affect, and keeps this CPU test to seconds.
        extra = ["-Xcicc", "-O0"] if srcs[i].endswith("attention.cu") else []
        return subprocess.run([nvcc, *flags, *extra, "-c", srcs[i], "-o", objs[i]],
                              capture_output=True, text=True)

    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        results = list(ex.map(compile_one, range(len(srcs))))
    for f, r in zip(srcs, results):
        assert r.returncode == 0, f + ": " + r.stderr[-3000:]
    r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", exe,
                        "-L" + lib_dir, "-lclove_b200", "-Xlinker", "-rpath=" + lib_dir],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    assert os.path.exists(exe)


def test_common_header_compiles_in_host_only_code(tmp_path):
    """clove/common.cuh keeps its device helpers behind __CUDACC__, so a host-only
    translation unit (the reference's model_loader.cpp includes it) compiles with g++."""
    import shutil
    import subprocess
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    src = tmp_path / "host_only.cpp"
    src.write_text("#include <clove/common.cuh>\n"
                   "int main() { return clove::cdiv(7, 2) == 4 && "
                   "clove::dtype_size(clove::DType::FP16) == 2 ? 0 : 1; }\n")
    r = subprocess.run([gxx, "-std=c++17", "-I" + os.path.join(ROOT, "include"),
                        "-I/usr/local/cuda/include", str(src), "-o", str(tmp_path / "h")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    assert subprocess.run([str(tmp_path / "h")]).returncode == 0
