"""Host side of the CLI (mxk_host_* in include/mxk.h) against the reference's
own include/host_utils.hpp (compiled into oracle/_ref/libref_host.so) and the
committed golden selections: K-Means++ and farthest-first initialisation pick
the same rows; the CSV reader accepts and rejects the same files
(tests/host_checks.cpp:41-68)."""
import ctypes
import os

import numpy as np
import pytest

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_vectors.npz")


def test_init_matches_golden(mxk):
    g = np.load(GOLDEN)
    pts = g["init_points"]
    assert np.array_equal(mxk.host_init_kmeanspp(pts, 16, 7), g["init_kmeanspp_seed7"])
    assert np.array_equal(mxk.host_init_farthest(pts, 16), g["init_farthest"])


def test_init_reference_known_answers(mxk):
    # tests/host_checks.cpp:41-50
    pts = np.array([[0, 0], [2, 2], [8, 8], [10, 10]], np.float32)
    assert mxk.host_init_farthest(pts, 4).ravel().tolist() == [0, 0, 10, 10, 2, 2, 8, 8]
    c = mxk.host_init_kmeanspp(pts, 4, 42)
    assert np.array_equal(c, mxk.host_init_kmeanspp(pts, 4, 42))
    assert sorted(c[:, 0].tolist()) == [0, 2, 8, 10]
    dup = np.full((4, 2), 3, np.float32)
    assert np.all(mxk.host_init_kmeanspp(dup, 4, 1) == 3)


@pytest.fixture(scope="module")
def ref_host(orc):
    lib = orc.ref_lib("libref_host.so")
    if lib is None:
        if not os.path.isdir("/root/reference"):
            pytest.skip("oracle/_ref not built and the reference checkout is absent")
        orc.build_ref()
        lib = orc.ref_lib("libref_host.so")
    return lib


@pytest.mark.parametrize("seed,n,d,k", [(1, 1000, 64, 32), (9, 3000, 128, 64), (123, 257, 7, 12)])
def test_init_matches_reference_code(mxk, ref_host, seed, n, d, k):
    g = np.random.default_rng(seed)
    pts = (g.standard_normal((n, d)) * g.uniform(0.1, 10)).astype(np.float32)
    pts[5] = pts[9]  # duplicate rows
    exp = np.empty((k, d), np.float32)
    ref_host.ref_init_kmeanspp(ctypes.c_void_p(pts.ctypes.data), n, d, k, ctypes.c_uint32(seed),
                               ctypes.c_void_p(exp.ctypes.data))
    assert np.array_equal(mxk.host_init_kmeanspp(pts, k, seed), exp)
    ref_host.ref_init_farthest(ctypes.c_void_p(pts.ctypes.data), n, d, k, ctypes.c_void_p(exp.ctypes.data))
    assert np.array_equal(mxk.host_init_farthest(pts, k), exp)


CSV_CASES = [
    ("x,y,label\r\n1,2,a\r\n3,4,b", 2, True),
    ("x,y,label\r\n1,2,a\r\n3,4,b", 1, False),
    ("x,y,label\r\n1,2,a\r\n3,4,b", 3, False),
    ("x,y\n1,2\n3,4\n", 2, True),
    ("x,y\n1,nan\n", 1, False),
    ("x,y\n1,2,3\n", 1, False),
    ("x,y\n1,2oops\n", 1, False),
    ("x,y\n1,inf\n", 1, False),
    ("x,y\n\n1, 2 \n\n", 1, True),
    ("x,y,\n1,2,\n", 1, True),
    ("", 1, False),
    ("x\n1\n", 1, False),
]


@pytest.mark.parametrize("text,n,ok", CSV_CASES)
def test_csv_reader_matches_reference(mxk, ref_host, tmp_path, text, n, ok):
    p = tmp_path / "pts.csv"
    p.write_text(text)
    ref_out = np.zeros((n, 128), np.float32)
    ref_rc = ref_host.ref_read_points(str(p).encode(), n, 2, 128, ctypes.c_void_p(ref_out.ctypes.data))
    assert (ref_rc == 0) == ok
    if ok:
        got = mxk.host_read_points(p, n, 2, 128)
        assert np.array_equal(got, ref_out)
        assert got[0, 2] == 0 and got[-1, 127] == 0
    else:
        with pytest.raises(ValueError):
            mxk.host_read_points(p, n, 2, 128)
