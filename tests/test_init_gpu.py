"""GPU centroid initialisation (mxk_init_farthest / mxk_init_kmeanspp) against the
reference's own host code (include/host_utils.hpp:80-141, built into
oracle/_ref/libref_host.so from the reference sources): the chosen rows must be
identical, bit for bit."""
import ctypes

import numpy as np
import pytest

from conftest import blobs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref(orc):
    lib = orc.ref_lib("libref_host.so")
    if lib is None:
        pytest.fail("oracle/_ref/libref_host.so is missing (build it with `make -C oracle ref`)")
    lib.ref_init_kmeanspp.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint32,
                                      ctypes.c_void_p]
    lib.ref_init_farthest.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return lib


def _ref_init(ref, x, k, seed=None):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros((k, x.shape[1]), np.float32)
    if seed is None:
        ref.ref_init_farthest(x.ctypes.data, x.shape[0], x.shape[1], k, out.ctypes.data)
    else:
        ref.ref_init_kmeanspp(x.ctypes.data, x.shape[0], x.shape[1], k, seed, out.ctypes.data)
    return out


def _gpu_init(torch, mxk, x, k, seed=None):
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    ct = torch.full((k, x.shape[1]), np.nan, dtype=torch.float32, device="cuda")
    if seed is None:
        mxk.init_farthest(xt, ct)
    else:
        mxk.init_kmeanspp(xt, ct, seed)
    torch.cuda.synchronize()
    return ct.cpu().numpy()


def _datasets():
    g = np.random.default_rng(5)
    yield "blobs", blobs(6000, 96, 40, seed=11)
    yield "integer", np.rint(blobs(3000, 128, 25, seed=12, spread=6.0, sigma=1.5))
    few = g.normal(size=(5, 128)).astype(np.float32)
    yield "duplicates", few[g.integers(0, 5, size=64)]  # only 5 distinct rows
    yield "tiny", g.normal(size=(9, 4)).astype(np.float32)


@pytest.mark.parametrize("name,x", list(_datasets()))
def test_farthest_matches_reference(torch_cuda, mxk, ref, name, x):
    k = min(len(x), 48)
    np.testing.assert_array_equal(_gpu_init(torch_cuda, mxk, x, k), _ref_init(ref, x, k))


@pytest.mark.parametrize("name,x", list(_datasets()))
@pytest.mark.parametrize("seed", [1, 42])
def test_kmeanspp_matches_reference(torch_cuda, mxk, ref, name, x, seed):
    # k above the number of distinct rows reaches the reference's "first point
    # not yet chosen" branch (every remaining distance is zero)
    k = min(len(x), 48)
    np.testing.assert_array_equal(_gpu_init(torch_cuda, mxk, x, k, seed), _ref_init(ref, x, k, seed))


def test_kmeanspp_nonfinite_distances_take_the_exact_path(torch_cuda, mxk, ref):
    # a NaN row keeps an infinite distance, so the running sum is infinite: the
    # GPU cannot bound it and the host replays the reference's loop
    x = blobs(500, 64, 8, seed=13)
    x[17, 5] = np.nan
    k = 12
    np.testing.assert_array_equal(_gpu_init(torch_cuda, mxk, x, k, 7), _ref_init(ref, x, k, 7))


def test_kmeanspp_large_n(torch_cuda, mxk, ref):
    # 2^17 points: every draw goes through the bounded parallel search
    x = blobs(131072, 96, 64, seed=14)
    k = 24
    np.testing.assert_array_equal(_gpu_init(torch_cuda, mxk, x, k, 3), _ref_init(ref, x, k, 3))


def test_init_rejects_bad_shapes(torch_cuda, mxk):
    torch = torch_cuda
    x = torch.zeros((10, 128), device="cuda")
    with pytest.raises(mxk.MxkInvalidArgument):
        mxk.init_farthest(x, torch.zeros((11, 128), device="cuda"))  # k > n
    with pytest.raises(mxk.MxkInvalidArgument):
        mxk.init_kmeanspp(torch.zeros((10, 6), device="cuda"), torch.zeros((2, 6), device="cuda"), 1)  # d % 4
