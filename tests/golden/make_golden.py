"""Generate the golden fixtures under tests/golden/.

Run in a container that has the reference checkout and the vendored CUTLASS
headers (to build oracle/_ref): every vector written here is produced by the C
oracle AND checked against the reference's own conversion library (CUTLASS
4.5.0 host types + CUDA cuda_fp6, oracle/_ref/libcutlass_pin.so) and, for the
initialisations, against the reference's include/host_utils.hpp compiled into
oracle/_ref/libref_host.so.  The fixtures then travel to machines without the
reference, where tests/test_oracle_cpu.py re-derives them from the oracle.

    python tests/golden/make_golden.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
import oracle  # noqa: E402
from conftest import reference_fixture_a, reference_fixture_b  # noqa: E402


def pin_encode(lib, fmt, x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.size, np.uint8)
    lib.pin_encode(ctypes.c_int(fmt), ctypes.c_int64(x.size), ctypes.c_void_p(x.ctypes.data),
                   ctypes.c_void_p(out.ctypes.data))
    return out.reshape(x.shape)


def main():
    oracle.build_ref()
    pin = oracle.ref_lib("libcutlass_pin.so")
    ref = oracle.ref_lib("libref_host.so")
    assert pin is not None and ref is not None, "oracle/_ref must be built (needs the reference checkout)"

    # 1. quantization of the reference's GPU-test fixture (tests/cuda_checks.cu:37-55)
    a, b = reference_fixture_a(), reference_fixture_b()
    pid = np.arange(a.shape[0] - 1, -1, -1, dtype=np.int32)
    out = {"pid": pid}
    for bits in (4, 6, 8):
        v, s, e = oracle.quantize_rows(bits, a, pid, errors=True)
        # cross-check every element against the reference's conversion library
        fmt = {8: oracle.E4M3, 6: oracle.E2M3, 4: oracle.E2M1}[bits]
        src = a[pid]
        scale_ref = pin_encode(pin, oracle.UE8M0, np.where(
            np.abs(src).reshape(len(pid), -1, 32).max(axis=2) > 0,
            np.abs(src).reshape(len(pid), -1, 32).max(axis=2) / np.float32({8: 448.0, 6: 7.5, 4: 6.0}[bits]),
            np.float32(1.0)).astype(np.float32))
        assert np.array_equal(scale_ref, s), "scales differ from CUTLASS float_ue8m0_t"
        sval = oracle.decode(oracle.UE8M0, s).repeat(32, axis=1)
        codes_ref = pin_encode(pin, fmt, (src / sval).astype(np.float32))
        codes = oracle.decode(fmt, codes_ref)  # value check through decode
        deq = oracle.dequantize_rows(bits, v, s, a.shape[1])
        assert np.array_equal(deq, (codes * sval).astype(np.float32)), "values differ from CUTLASS conversion"
        out[f"q{bits}_values"], out[f"q{bits}_scales"], out[f"q{bits}_errors"] = v, s, e
    vb, sb, _ = oracle.quantize_rows(8, b)
    out["qb_values"], out["qb_scales"] = vb, sb

    # 2. K-Means++ and farthest-first selections of the reference's host code
    g = np.random.default_rng(42)
    pts = (g.standard_normal((200, 32)) * 3).astype(np.float32)
    kpp = np.empty((16, 32), np.float32)
    ref.ref_init_kmeanspp(ctypes.c_void_p(pts.ctypes.data), 200, 32, 16, ctypes.c_uint32(7),
                          ctypes.c_void_p(kpp.ctypes.data))
    far = np.empty((16, 32), np.float32)
    ref.ref_init_farthest(ctypes.c_void_p(pts.ctypes.data), 200, 32, 16, ctypes.c_void_p(far.ctypes.data))
    out["init_points"], out["init_kmeanspp_seed7"], out["init_farthest"] = pts, kpp, far

    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_vectors.npz"))


if __name__ == "__main__":
    main()
