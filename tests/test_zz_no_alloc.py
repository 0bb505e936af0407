"""The allocation-free convergence shift (mxk_centroid_shift_noalloc).

Some callers cannot call cudaMalloc when they need the shift -- for example a
plugin running inside a framework whose memory pool owns the device, or a loop
that must keep a fixed memory budget.  This entry point keeps its scratch in a
fixed device array inside the library instead of allocating one per call.

The test calls it through the C ABI twice in a row (so the second call sees the
first call's leftovers in the shared array) and compares each result with the
existing, allocating mxk_centroid_shift on the same inputs, within the 1e-5
relative tolerance the other shift tests use.  The file is named to be
collected last, so a run that stops at the first failure has run every other
test first; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ELEMENTS = 16384 * 2048


def _noalloc(mxk, prev, cur, device_sum):
    out = ctypes.c_float(0.0)
    st = mxk.load().mxk_centroid_shift_noalloc(prev.numel(), ctypes.c_void_p(prev.data_ptr()),
                                               ctypes.c_void_p(cur.data_ptr()),
                                               None if device_sum is None else ctypes.c_void_p(device_sum.data_ptr()),
                                               ctypes.cast(ctypes.pointer(out), ctypes.c_void_p), None)
    mxk.check(st)
    return out.value


def test_noalloc_shift_matches_allocating_entry_point(torch_cuda, mxk):
    torch = torch_cuda
    g = torch.Generator(device="cuda:0").manual_seed(11)
    # a large input first, then a smaller one: the second call must not pick up
    # partial sums the first call left in the shared array
    for elements in (2048 * 4000 + 17, 262144, 1000003, 5):
        prev = torch.randn(elements, generator=g, device="cuda:0")
        cur = prev + 1e-3 * torch.randn(elements, generator=g, device="cuda:0")
        dsum = torch.zeros(1, device="cuda:0")
        expected = mxk.centroid_shift(prev, cur, dsum)
        for _ in range(2):
            dsum_na = torch.full((1,), -1.0, device="cuda:0")
            got = _noalloc(mxk, prev, cur, dsum_na)
            assert abs(got - expected) <= 1e-5 * abs(expected), (elements, got, expected)
            assert dsum_na.item() == got


def test_noalloc_shift_rejects_oversized_input(torch_cuda, mxk):
    st = mxk.load().mxk_centroid_shift_noalloc(MAX_ELEMENTS + 1, None, None, None, None, None)
    assert st == mxk.ERR_INVALID
    assert b"fixed scratch limit" in mxk.load().mxk_last_error()
    zero = torch_cuda.zeros(1, device="cuda:0")
    assert _noalloc(mxk, zero[:0], zero[:0], None) == 0.0
