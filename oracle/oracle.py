"""numpy/ctypes front end of the C oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the CPU
baseline leg of bench.py as the checker.  The product never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

E4M3, E2M3, E2M1, E3M2, UE8M0 = range(5)

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        sig = {
            "orc_encode_batch": [_I, _I64, _P, _P],
            "orc_decode_batch": [_I, _I64, _P, _P],
            "orc_l2_norm": [_I64, _I, _P, _P],
            "orc_quantize_rows": [_I, _I64, _I, _P, _P, _P, _P, _P],
            "orc_point_bounds": [_I64, _I, _P, _P, _P],
            "orc_assign_precisions": [_I64, _I, _P, _P, _F, _F, _P],
            "orc_dequantize_rows": [_I, _I64, _I, _P, _P, _P],
            "orc_gemm_mx": [_I, _I64, _I64, _I, _P, _P, _P, _P, _P, _P],
            "orc_gemm_f32": [_I64, _I64, _I, _P, _P, _P],
            "orc_assign_clusters": [_I64, _I, _P, _P, _P, _P, _P, _P],
            "orc_top2": [_I64, _I, _P, _P, _P, _P, _P, _P],
            "orc_update_centroids": [_I64, _I, _I, _P, _P, _P, _P, _P],
            "orc_kmeans_mixed": [_I64, _I, _I, _P, _P, _P, _I, _I, _F, _I],
            "orc_kmeans_mixed_ex": [_I64, _I, _I, _P, _P, _P, _I, _I, _F, _I, _I, _P],
            "orc_lloyd_step": [_I64, _I, _I, _P, _P, _P, _P, _P, _I],
            "orc_lloyd_fp32": [_I64, _I, _I, _P, _P, _P, _I, _F, _I],
        }
        for name, args in sig.items():
            getattr(L, name).argtypes = args
        L.orc_precision_candidate.argtypes = [_F, _F, _F, _I, _F]
        L.orc_select_precision.argtypes = [_F, _F, _F, _F, _I, _F]
        L.orc_centroid_shift.argtypes = [_I64, _P, _P]
        L.orc_centroid_shift.restype = _F
        L.orc_inertia.argtypes = [_I64, _I, _P, _P, _P]
        L.orc_inertia.restype = ctypes.c_double
        L.orc_lloyd_step.restype = _F
        L.orc_hardware_threads.restype = _I
        _lib = L
    return _lib


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def encode(fmt, x):
    x = _c(x, np.float32)
    out = np.empty(x.size, np.uint8)
    lib().orc_encode_batch(fmt, x.size, _p(x), _p(out))
    return out.reshape(x.shape)


def decode(fmt, codes):
    c = _c(codes, np.uint8)
    out = np.empty(c.size, np.float32)
    lib().orc_decode_batch(fmt, c.size, _p(c), _p(out))
    return out.reshape(c.shape)


def l2_norm(x):
    x = _c(x, np.float32)
    out = np.empty(x.shape[0], np.float32)
    lib().orc_l2_norm(x.shape[0], x.shape[1], _p(x), _p(out))
    return out


def quantize_rows(bits, points, pid=None, errors=False):
    """-> (packed bytes [rows, d*bits/8], scales [rows, d/32], max sq errors or None)"""
    points = _c(points, np.float32)
    d = points.shape[1]
    rows = points.shape[0] if pid is None else len(pid)
    pid_a = None if pid is None else _c(pid, np.int32)
    values = np.zeros((rows, d * bits // 8), np.uint8)
    scales = np.zeros((rows, d // 32), np.uint8)
    err = np.zeros(rows, np.float32) if errors else None
    st = lib().orc_quantize_rows(bits, rows, d, _p(points), _p(pid_a), _p(values), _p(scales), _p(err))
    if st != 0:
        raise ValueError("orc_quantize_rows rejected its arguments")
    return values, scales, err


def dequantize_rows(bits, values, scales, d):
    values = _c(values, np.uint8)
    scales = _c(scales, np.uint8)
    rows = scales.shape[0]
    out = np.empty((rows, d), np.float32)
    lib().orc_dequantize_rows(bits, rows, d, _p(values), _p(scales), _p(out))
    return out


def gemm_mx(bits, a, a_scales, b, b_scales, k):
    """double products of reconstructed values and their absolute-sum magnitude"""
    a = _c(a, np.uint8); a_scales = _c(a_scales, np.uint8)
    b = _c(b, np.uint8); b_scales = _c(b_scales, np.uint8)
    m, n = a_scales.shape[0], b_scales.shape[0]
    out = np.empty((m, n), np.float64)
    mag = np.empty((m, n), np.float64)
    lib().orc_gemm_mx(bits, m, n, k, _p(a), _p(a_scales), _p(b), _p(b_scales), _p(out), _p(mag))
    return out, mag


def gemm_f32(a, b):
    a = _c(a, np.float32); b = _c(b, np.float32)
    out = np.empty((a.shape[0], b.shape[0]), np.float64)
    lib().orc_gemm_f32(a.shape[0], b.shape[0], a.shape[1], _p(a), _p(b), _p(out))
    return out


def assign_clusters(point_norms, centroid_norms, dots, pid=None, n_points=None):
    dots = _c(dots, np.float32)
    rows, k = dots.shape
    pn = _c(point_norms, np.float32); cn = _c(centroid_norms, np.float32)
    n_points = n_points if n_points is not None else (rows if pid is None else pn.shape[0])
    labels = np.zeros(n_points, np.int32)
    gaps = np.zeros(n_points, np.float32)
    pid_a = None if pid is None else _c(pid, np.int32)
    lib().orc_assign_clusters(rows, k, _p(pn), _p(cn), _p(dots), _p(pid_a), _p(labels), _p(gaps))
    return labels, gaps


def top2(point_norms, centroid_norms, dots):
    dots = _c(dots, np.float32)
    rows, k = dots.shape
    pn = _c(point_norms, np.float32); cn = _c(centroid_norms, np.float32)
    nearest = np.zeros(rows, np.int32)
    first = np.zeros(rows, np.float32)
    second = np.zeros(rows, np.float32)
    lib().orc_top2(rows, k, _p(pn), _p(cn), _p(dots), _p(nearest), _p(first), _p(second))
    return nearest, first, second


def point_bounds(points, norms):
    points = _c(points, np.float32); norms = _c(norms, np.float32)
    n, d = points.shape
    upper = np.zeros(((n + 31) // 32) * 96, np.float32)
    lib().orc_point_bounds(n, d, _p(points), _p(norms), _p(upper))
    return upper


def assign_precisions(n, d, upper, gaps, lc, ec):
    upper = _c(upper, np.float32); gaps = _c(gaps, np.float32)
    out = np.zeros(n, np.int32)
    lib().orc_assign_precisions(n, d, _p(upper), _p(gaps), lc, ec, _p(out))
    return out


def precision_candidate(p4, p6, lc, d, gap):
    return lib().orc_precision_candidate(p4, p6, lc, d, gap)


def select_precision(p4, p6, lc, ec, d, gap):
    return lib().orc_select_precision(p4, p6, lc, ec, d, gap)


def update_centroids(points, labels, old_centroids):
    points = _c(points, np.float32); labels = _c(labels, np.int32); old = _c(old_centroids, np.float32)
    k, d = old.shape
    cent = np.zeros_like(old)
    counts = np.zeros(k, np.int32)
    lib().orc_update_centroids(points.shape[0], d, k, _p(points), _p(labels), _p(old), _p(cent), _p(counts))
    return cent, counts


def centroid_shift(prev, cur):
    prev = _c(prev, np.float32); cur = _c(cur, np.float32)
    return lib().orc_centroid_shift(prev.size, _p(prev), _p(cur))


def inertia(points, centroids, labels):
    points = _c(points, np.float32); centroids = _c(centroids, np.float32); labels = _c(labels, np.int32)
    return lib().orc_inertia(points.shape[0], points.shape[1], _p(points), _p(centroids), _p(labels))


def kmeans_mixed(points, centroids, max_iterations=300, fp32_iterations=0, tolerance=1e-4, threads=0,
                 policy=0, group_sizes=False):
    """-> (iterations, centroids, labels[, group sizes [max_iterations, 3]]);
    iterations < 0 on a non-finite shift.  policy 1 lets precision_candidate's
    choice stand (the library's mxk_set_precision_policy(1))."""
    points = _c(points, np.float32)
    cent = _c(centroids, np.float32).copy()
    labels = np.zeros(points.shape[0], np.int32)
    groups = np.zeros((max_iterations, 3), np.int32) if group_sizes else None
    it = lib().orc_kmeans_mixed_ex(points.shape[0], points.shape[1], cent.shape[0], _p(points), _p(cent),
                                   _p(labels), max_iterations, fp32_iterations, tolerance, threads, policy,
                                   _p(groups))
    return (it, cent, labels, groups) if group_sizes else (it, cent, labels)


def lloyd_step(points, point_norms, centroids, threads=0, want_dots=False):
    """One MX Lloyd step; -> (shift, new centroids, labels, dots or None)"""
    points = _c(points, np.float32); pn = _c(point_norms, np.float32)
    cent = _c(centroids, np.float32).copy()
    n, d = points.shape
    k = cent.shape[0]
    labels = np.zeros(n, np.int32)
    dots = np.zeros((n, k), np.float32) if want_dots else None
    shift = lib().orc_lloyd_step(n, d, k, _p(points), _p(pn), _p(cent), _p(labels), _p(dots), threads)
    return shift, cent, labels, dots


def lloyd_fp32(points, centroids, max_iterations, tolerance, threads=0):
    points = _c(points, np.float32)
    cent = _c(centroids, np.float32).copy()
    labels = np.zeros(points.shape[0], np.int32)
    it = lib().orc_lloyd_fp32(points.shape[0], points.shape[1], cent.shape[0], _p(points), _p(cent), _p(labels),
                              max_iterations, tolerance, threads)
    return it, cent, labels


def hardware_threads():
    return lib().orc_hardware_threads()


# ----------------------------------------------------------------------------- oracle/_ref pins

def ref_lib(name):
    """ctypes handle of a library built into oracle/_ref (None if absent)."""
    p = os.path.join(REF_DIR, name)
    return ctypes.CDLL(p) if os.path.exists(p) else None


def build_ref():
    """Build oracle/_ref from the reference sources (needs the reference checkout)."""
    subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)
