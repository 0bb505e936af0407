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
                "gemm_mx(int, int, int, int, void const*, Scale const*, MXFP8 const*, Scale const*, float*)"]:
        assert sig in out, f"C++ drop-in symbol missing: {sig}"


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
