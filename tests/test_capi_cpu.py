"""The C-ABI library (no GPU needed): it loads, exports every entry point that
include/mxk.h declares and every C++ function of include/kmeans.cuh, and the
Python binding declares a signature for each."""
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mxk.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(mxk_[a-z0-9_]+)\s*\(", text)))


def _exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_loads_and_exports_header(mxk):
    lib = mxk.load()
    assert lib.mxk_version() >= 100
    exported = _exported(mxk.LIB_PATH)
    missing = [f for f in _declared() if f not in exported]
    assert not missing, f"declared in mxk.h but not exported: {missing}"


def test_binding_covers_header(mxk):
    missing = [f for f in _declared() if f not in mxk.SIGNATURES]
    assert not missing, f"no ctypes signature for {missing}"


def test_cpp_dropin_symbols(mxk):
    out = subprocess.run(["nm", "-DC", "--defined-only", mxk.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    for sig in ["kmeans_mixed(int, int, int, float const*, float*, int*, KMeansOptions const&)",
                "compute_l2_norm(int, int, float const*, float*)",
                "update_centroids(int, int, int, float const*, int const*, float const*, float*, int*)",
                "centroid_shift(int, float const*, float const*, float*)",
                "assign_clusters(int, int, float const*, float const*, float const*, int const*, int*, float*)",
                "precompute_point_bounds(int, int, float const*, float const*, float*)",
                "assign_precisions(int, int, float const*, float const*, float, float, int*)",
                "quantize_rows(int, int, int, float const*, int const*, void*, Scale*, float*)",
                "gemm_fp32(int, int, int, float const*, float const*, float*)",
                "gemm_mx(int, int, int, int, void const*, Scale const*, MXFP8 const*, Scale const*, float*)",
                # additive multi-GPU entry (include/kmeans_multi.cuh)
                "kmeans_mixed_multi(long, int, int, float const*, float*, int*, KMeansOptions const&, int)"]:
        assert sig in out, f"C++ drop-in symbol missing: {sig}"


def test_multi_gpu_entry_validates_before_cuda(mxk):
    import numpy as np
    lib = mxk.load()
    it = mxk.ctypes.c_int(0)
    opts = mxk.Options(max_iterations=1, tolerance=0.0)
    st = lib.mxk_kmeans_mixed_multi(4, 128, 4, None, None, None, mxk.ctypes.byref(opts), 1, mxk.ctypes.byref(it))
    assert st == mxk.ERR_INVALID and b"null pointer" in lib.mxk_last_error()
    x = np.zeros((8, 128), np.float32)
    c = np.zeros((4, 128), np.float32)
    lab = np.zeros(8, np.int32)
    with pytest.raises(ValueError, match="num_gpus >= 1"):
        mxk.kmeans_mixed_multi(x, c, lab, opts, 0)


def test_errors_are_reported_without_a_gpu(mxk):
    # argument validation happens before any CUDA call
    lib = mxk.load()
    st = lib.mxk_quantize_rows(5, 4, 32, None, None, None, None, None, None)
    assert st == mxk.ERR_INVALID
    assert b"Precision must be 4, 6, or 8" in lib.mxk_last_error()
    with pytest.raises(ValueError):
        mxk.check(st)


def test_build_flags_target_sm100a():
    mk = open(os.path.join(ROOT, "mx-kmeans_b200", "Makefile")).read()
    assert "ARCH    := -gencode arch=compute_100a,code=sm_100a" in mk


def test_forced_mxfp8_flag_matches_select_precision(tmp_path):
    """The Lloyd driver skips the precision policy's inputs while
    kSelectPrecisionIsForcedMxfp8 holds; the header's select_precision must then
    return MXFP8 for every input, including NaN and infinite ones."""
    import subprocess
    src = tmp_path / "p.cpp"
    src.write_text(r'''
#include <cmath>
#include <cstdio>
#include <initializer_list>
#include <limits>
#include "precision.hpp"
int main() {
    static_assert(kSelectPrecisionIsForcedMxfp8, "flag");
    const float inf = std::numeric_limits<float>::infinity(), nan = std::nanf("");
    const float v[] = {0.0f, -0.0f, 1e-30f, 0.5f, 1.0f, 64.0f, 1e6f, 3e38f, inf, -inf, nan, -1.0f};
    int bad = 0;
    for (float p4 : v) for (float p6 : v) for (float lc : v) for (float ec : v) for (float gap : v)
        for (int d : {1, 96, 128, 4096}) bad += select_precision(p4, p6, lc, ec, d, gap) != 8;
    std::printf("%d\n", bad);
    return bad != 0;
}
''')
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = tmp_path / "p"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(root, "include"), str(src), "-o", str(exe)],
                   check=True, timeout=120)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "0"


def test_missing_library_fails_loudly(mxk, tmp_path):
    """No fallback: without the built library the binding raises instead of
    computing anything another way."""
    with pytest.raises(FileNotFoundError, match="is not built"):
        mxk.load(str(tmp_path / "libmxkmeans.so"))


def test_product_never_reaches_the_oracle():
    """The oracle is test infrastructure: nothing in the library, its headers,
    the CLI or the binding names, imports or links it."""
    hits = []
    for base in (os.path.join(ROOT, "mx-kmeans_b200"), os.path.join(ROOT, "include")):
        for dirpath, _, files in os.walk(base):
            if "_build" in dirpath:
                continue
            for f in files:
                if f.endswith((".cu", ".cuh", ".cpp", ".hpp", ".h", ".py", "Makefile")):
                    text = open(os.path.join(dirpath, f), errors="replace").read()
                    if re.search(r"\boracle\b|liboracle|_ref/", text):
                        hits.append(os.path.join(dirpath, f))
    assert not hits, f"product files reference the oracle: {hits}"


def test_precision_policy_hook_values(mxk):
    """mxk_set_precision_policy accepts 0 (the reference's rule) and 1 (the
    candidate) and rejects anything else; it needs no GPU."""
    mxk.set_precision_policy(1)
    mxk.set_precision_policy(0)
    with pytest.raises(ValueError):
        mxk.set_precision_policy(2)
