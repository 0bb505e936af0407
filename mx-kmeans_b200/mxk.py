"""ctypes binding of libmxkmeans.so, the B200 MX-KMeans library (C ABI: include/mxk.h).

The low-level functions take device pointers (ints) exactly as the C ABI does;
the helpers take torch CUDA tensors and pass their data pointers (torch is only
used for device memory and streams here).  Loading fails loudly if the shared
library has not been built -- there is no fallback implementation.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmxkmeans.so")

OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_NONFINITE, ERR_TIMEOUT, ERR_COMM = range(7)


class MxkError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"mxk status {status}: {message}")
        self.status = status
        self.message = message


class MxkInvalidArgument(MxkError, ValueError):
    pass


class Options(ctypes.Structure):
    """mxk_options; defaults of the reference's KMeansOptions (include/kmeans.cuh:11-16)."""

    _fields_ = [("max_iterations", ctypes.c_int), ("fp32_iterations", ctypes.c_int),
                ("tolerance", ctypes.c_float), ("verbose", ctypes.c_int)]

    def __init__(self, max_iterations=300, fp32_iterations=0, tolerance=1e-4, verbose=False):
        super().__init__(max_iterations, fp32_iterations, tolerance, int(bool(verbose)))


class Trace(ctypes.Structure):
    """mxk_trace: device buffers the next Lloyd call fills per iteration."""

    _fields_ = [("centroids", ctypes.c_void_p), ("labels", ctypes.c_void_p), ("group_sizes", ctypes.c_void_p),
                ("max_iterations", ctypes.c_int)]


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 48), ("launches", ctypes.c_uint64), ("total_ms", ctypes.c_double)]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

SIGNATURES = {
    "mxk_version": ([], _I),
    "mxk_last_error": ([], ctypes.c_char_p),
    "mxk_launch_count": ([], ctypes.c_uint64),
    "mxk_compute_l2_norm": ([_I64, _I, _P, _P, _P], _I),
    "mxk_quantize_rows": ([_I, _I64, _I, _P, _P, _P, _P, _P, _P], _I),
    "mxk_precompute_point_bounds": ([_I64, _I, _P, _P, _P, _P], _I),
    "mxk_assign_precisions": ([_I64, _I, _P, _P, _F, _F, _P, _P], _I),
    "mxk_check_mxfp8_scale_codec": ([_P, _P], _I),
    "mxk_check_wait_timeout": ([ctypes.c_longlong, _P, _P], _I),
    "mxk_release_workspace": ([], _I),
    "mxk_gemm_tiles_multiplied": ([ctypes.POINTER(ctypes.c_ulonglong), _I], _I),
    "mxk_gemm_rows_processed": ([ctypes.POINTER(ctypes.c_ulonglong), _I], _I),
    "mxk_init_farthest": ([_I64, _I, _I, _P, _P, _P], _I),
    "mxk_init_kmeanspp": ([_I64, _I, _I, _P, _P, ctypes.c_uint32, _P], _I),
    "mxk_gemm_mx": ([_I, _I64, _I64, _I, _P, _P, _P, _P, _P, _P], _I),
    "mxk_gemm_fp32": ([_I64, _I64, _I, _P, _P, _P, _P], _I),
    "mxk_assign_clusters": ([_I64, _I, _P, _P, _P, _P, _P, _P, _P], _I),
    "mxk_update_centroids": ([_I64, _I, _I, _P, _P, _P, _P, _P, _P], _I),
    "mxk_centroid_shift": ([_I64, _P, _P, _P, _P, _P], _I),
    "mxk_centroid_shift_noalloc": ([_I64, _P, _P, _P, _P, _P], _I),
    "mxk_assign_mx_fused": ([_I, _I64, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "mxk_assign_f32_fused": ([_I64, _I, _I, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "mxk_kmeans_mixed": ([_I64, _I, _I, _P, _P, _P, ctypes.POINTER(Options), ctypes.POINTER(_I), _P], _I),
    "mxk_kmeans_mixed_cached": ([_I64, _I, _I, _P, _P, _P, ctypes.POINTER(Options), ctypes.POINTER(_I), _P], _I),
    "mxk_set_precision_policy": ([_I], _I),
    "mxk_trace_next_call": ([ctypes.POINTER(Trace)], _I),
    "mxk_comm_unique_id": ([ctypes.c_char_p], _I),
    "mxk_comm_init": ([ctypes.POINTER(_P), _I, _I, ctypes.c_char_p], _I),
    "mxk_comm_destroy": ([_P], _I),
    "mxk_inject_rank_failure": ([_I, _I], _I),
    "mxk_kmeans_mixed_sharded": ([_P, _I64, _I, _I, _P, _P, _P, ctypes.POINTER(Options), ctypes.POINTER(_I), _P], _I),
    "mxk_kmeans_mixed_multi": ([_I64, _I, _I, _P, _P, _P, ctypes.POINTER(Options), _I, ctypes.POINTER(_I)], _I),
    "mxk_host_init_kmeanspp": ([_P, _I64, _I, _I, ctypes.c_uint32, _P], _I),
    "mxk_host_init_farthest": ([_P, _I64, _I, _I, _P], _I),
    "mxk_host_read_points": ([ctypes.c_char_p, _I64, _I, _I, _P], _I),
    "mxk_host_read_points_ex": ([ctypes.c_char_p, _I64, _I, _I, _I, _I64, _P], _I),
    "mxk_host_read_points_f32": ([ctypes.c_char_p, _I64, _I, _I, _P], _I),
    "mxk_host_write_labels": ([ctypes.c_char_p, _P, _I64], _I),
    "mxk_profile_enable": ([_I], _I),
    "mxk_profile_read": ([ctypes.POINTER(KernelStat), _I, ctypes.POINTER(_I)], _I),
}

_lib = None


def load(path=None):
    """Load libmxkmeans.so (once) and declare every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise FileNotFoundError(f"{p} is not built; run `make -C mx-kmeans_b200` or __graft_entry__.build()")
    lib = ctypes.CDLL(p)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


def check(status):
    if status != OK:
        msg = load().mxk_last_error().decode(errors="replace")
        if status == ERR_INVALID:
            raise MxkInvalidArgument(status, msg)
        raise MxkError(status, msg)


# ----------------------------------------------------------------------------- torch helpers

def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def quantize_rows(bits, points, values, scales, pid=None, max_errors=None, rows=None, stream=None):
    rows = points.shape[0] if rows is None and pid is None else (rows if rows is not None else pid.shape[0])
    check(load().mxk_quantize_rows(bits, rows, points.shape[1], _ptr(points), _ptr(pid), _ptr(values),
                                   _ptr(scales), _ptr(max_errors), _stream(stream)))


def compute_l2_norm(points, norms, stream=None):
    check(load().mxk_compute_l2_norm(points.shape[0], points.shape[1], _ptr(points), _ptr(norms), _stream(stream)))


def precompute_point_bounds(points, norms, upper, stream=None):
    check(load().mxk_precompute_point_bounds(points.shape[0], points.shape[1], _ptr(points), _ptr(norms),
                                             _ptr(upper), _stream(stream)))


def assign_precisions(n, d, upper, gaps, lc, ec, precision, stream=None):
    check(load().mxk_assign_precisions(n, d, _ptr(upper), _ptr(gaps), lc, ec, _ptr(precision), _stream(stream)))


def init_farthest(points, centroids, stream=None):
    """Farthest-first initial centroids (the reference's init_centroids_farthest)
    from device points [n, d] into device centroids [k, d]."""
    n, d = points.shape
    check(load().mxk_init_farthest(n, d, centroids.shape[0], _ptr(points), _ptr(centroids), _stream(stream)))


def init_kmeanspp(points, centroids, seed, stream=None):
    """K-Means++ initial centroids (the reference's init_centroids with
    std::mt19937(seed)) from device points [n, d] into device centroids [k, d]."""
    n, d = points.shape
    check(load().mxk_init_kmeanspp(n, d, centroids.shape[0], _ptr(points), _ptr(centroids), seed & 0xffffffff,
                                   _stream(stream)))


def gemm_tiles_multiplied(reset=False):
    """128 x 192 tiles multiplied by the MX GEMM on the current device since the
    last reset (pruned tiles excluded)."""
    v = ctypes.c_ulonglong(0)
    check(load().mxk_gemm_tiles_multiplied(ctypes.byref(v), 1 if reset else 0))
    return v.value


def gemm_rows_processed(reset=False):
    """Point rows processed by the MX GEMM on the current device since the last
    reset (rows whose labels the loop's bounds proved are not counted)."""
    v = ctypes.c_ulonglong(0)
    check(load().mxk_gemm_rows_processed(ctypes.byref(v), 1 if reset else 0))
    return v.value


def release_workspace():
    """Return the kmeans workspace kept by the library's pool on the current
    device to the driver."""
    check(load().mxk_release_workspace())


def check_mxfp8_scale_codec(result, stream=None):
    """Exhaustive device check of the fused quantizer's MXFP8 scale rule against
    ue8m0(amax / 448); result: 2 int64 device words (count, first pattern)."""
    check(load().mxk_check_mxfp8_scale_codec(_ptr(result), _stream(stream)))


def check_wait_timeout(limit_cycles, outcome, stream=None):
    """Run the bounded-wait self-check (an mbarrier nothing arrives on); returns
    the status the library reports (MXK_ERR_TIMEOUT expected) without raising.
    outcome: 2 int32 device words, 0 = that warp's wait gave up."""
    return load().mxk_check_wait_timeout(int(limit_cycles), _ptr(outcome), _stream(stream))


def gemm_mx(bits, m, n, k, a, a_scales, b, b_scales, out, stream=None):
    check(load().mxk_gemm_mx(bits, m, n, k, _ptr(a), _ptr(a_scales), _ptr(b), _ptr(b_scales), _ptr(out),
                             _stream(stream)))


def gemm_fp32(a, b, out, stream=None):
    check(load().mxk_gemm_fp32(a.shape[0], b.shape[0], a.shape[1], _ptr(a), _ptr(b), _ptr(out), _stream(stream)))


def assign_clusters(rows, k, point_norms, centroid_norms, dots, labels, gaps, pid=None, stream=None):
    check(load().mxk_assign_clusters(rows, k, _ptr(point_norms), _ptr(centroid_norms), _ptr(dots), _ptr(pid),
                                     _ptr(labels), _ptr(gaps), _stream(stream)))


def assign_mx_fused(bits, rows, k, d, a, a_scales, b, b_scales, point_norms, centroid_norms, labels, gaps=None,
                    pid=None, start_hint=None, stream=None):
    check(load().mxk_assign_mx_fused(bits, rows, k, d, _ptr(a), _ptr(a_scales), _ptr(b), _ptr(b_scales),
                                     _ptr(point_norms), _ptr(centroid_norms), _ptr(pid), _ptr(labels), _ptr(gaps),
                                     _ptr(start_hint), _stream(stream)))


def assign_f32_fused(rows, k, d, points, b, b_scales, point_norms, centroid_norms, labels, gaps=None, pid=None,
                     start_hint=None, stream=None):
    check(load().mxk_assign_f32_fused(rows, k, d, _ptr(points), points.shape[0], _ptr(b), _ptr(b_scales),
                                      _ptr(point_norms), _ptr(centroid_norms), _ptr(pid), _ptr(labels), _ptr(gaps),
                                      _ptr(start_hint), _stream(stream)))


def update_centroids(points, labels, old_centroids, centroids, counts, stream=None):
    check(load().mxk_update_centroids(points.shape[0], points.shape[1], centroids.shape[0], _ptr(points),
                                      _ptr(labels), _ptr(old_centroids), _ptr(centroids), _ptr(counts),
                                      _stream(stream)))


def centroid_shift(previous, current, device_sum, stream=None):
    out = ctypes.c_float(0.0)
    check(load().mxk_centroid_shift(previous.numel(), _ptr(previous), _ptr(current), _ptr(device_sum),
                                    ctypes.cast(ctypes.pointer(out), ctypes.c_void_p), _stream(stream)))
    return out.value


def kmeans_mixed(points, centroids, labels, options=None, stream=None, cache_points=False):
    """Run the Lloyd loop in place on device tensors; returns the iteration count.
    cache_points: quantize the points once per call instead of every iteration
    (mxk_kmeans_mixed_cached; same results, reported separately)."""
    opts = options or Options()
    iters = ctypes.c_int(0)
    fn = load().mxk_kmeans_mixed_cached if cache_points else load().mxk_kmeans_mixed
    check(fn(points.shape[0], points.shape[1], centroids.shape[0], _ptr(points), _ptr(centroids), _ptr(labels),
             ctypes.byref(opts), ctypes.byref(iters), _stream(stream)))
    return iters.value


def set_precision_policy(policy):
    """0: the reference's select_precision (always MXFP8, the default); 1: the
    candidate it computes and discards (test hook for the 4/6/8 groups)."""
    check(load().mxk_set_precision_policy(int(policy)))


def trace_next_call(max_iterations, centroids=None, labels=None, group_sizes=None):
    """Arm a trace of the next Lloyd call on the current device: per iteration i <
    max_iterations, centroids[i] <- the centroids it assigns against, labels[i] <-
    its labels, group_sizes[i] <- its (MXFP4, MXFP6, MXFP8) group rows.  The
    tensors are device tensors of shape [max_iterations, ...] (or None)."""
    t = Trace(None if centroids is None else centroids.data_ptr(),
              None if labels is None else labels.data_ptr(),
              None if group_sizes is None else group_sizes.data_ptr(), int(max_iterations))
    check(load().mxk_trace_next_call(ctypes.byref(t)))


def comm_unique_id():
    buf = ctypes.create_string_buffer(128)
    check(load().mxk_comm_unique_id(buf))
    return buf.raw


class Comm:
    """NCCL communicator of one rank (mxk_comm_init / mxk_comm_destroy)."""

    def __init__(self, nranks, rank, unique_id):
        self.handle = ctypes.c_void_p()
        check(load().mxk_comm_init(ctypes.byref(self.handle), nranks, rank, unique_id))

    def close(self):
        if self.handle:
            check(load().mxk_comm_destroy(self.handle))
            self.handle = ctypes.c_void_p()


def inject_rank_failure(rank, iteration):
    """Test hook: the sharded loop of `rank` leaves with an error when it reaches
    `iteration` (rank < 0 disarms)."""
    check(load().mxk_inject_rank_failure(int(rank), int(iteration)))


def shard_rows(n, world, rank):
    """Rows of one rank in the row-sharded path: contiguous shards of n // world
    rows, the first n % world ranks one row more.  -> (first_row, row_count)."""
    if n < 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError(f"shard_rows: bad arguments n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


def bootstrap_comm(group=None):
    """This rank's NCCL communicator for kmeans_mixed_sharded.  Rank 0 creates the
    unique id and broadcasts it over an initialized torch.distributed process group
    (any backend, so a gloo group on the host works); a rank that never joins makes
    the broadcast fail with the group's timeout instead of hanging.  -> Comm"""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    uid = [comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    return Comm(world, rank, uid[0])


def kmeans_mixed_sharded(comm, points, centroids, labels, options=None, stream=None):
    opts = options or Options()
    iters = ctypes.c_int(0)
    check(load().mxk_kmeans_mixed_sharded(comm.handle, points.shape[0], points.shape[1], centroids.shape[0],
                                          _ptr(points), _ptr(centroids), _ptr(labels), ctypes.byref(opts),
                                          ctypes.byref(iters), _stream(stream)))
    return iters.value


def profile_enable(on=True):
    check(load().mxk_profile_enable(1 if on else 0))


def profile_read():
    """{kernel name: (launches, total_ms)} for the current device since profile_enable()."""
    count = ctypes.c_int(0)
    check(load().mxk_profile_read(None, 0, ctypes.byref(count)))
    arr = (KernelStat * max(count.value, 1))()
    check(load().mxk_profile_read(arr, count.value, ctypes.byref(count)))
    return {arr[i].name.decode(): (arr[i].launches, arr[i].total_ms) for i in range(count.value)}


def _np(a):
    return ctypes.c_void_p(a.ctypes.data)


def kmeans_mixed_multi(points, centroids, labels, options, num_gpus):
    """kmeans_mixed over num_gpus GPUs of this node from HOST numpy arrays
    (points n x d float32, centroids k x d float32 in/out, labels n int32 out)."""
    import numpy as np
    for a, t in ((points, np.float32), (centroids, np.float32), (labels, np.int32)):
        if a.dtype != t or not a.flags.c_contiguous:
            raise TypeError("kmeans_mixed_multi: contiguous float32 points/centroids and int32 labels required")
    it = ctypes.c_int(0)
    check(load().mxk_kmeans_mixed_multi(points.shape[0], points.shape[1], centroids.shape[0], _np(points),
                                        _np(centroids), _np(labels), ctypes.byref(options), num_gpus,
                                        ctypes.byref(it)))
    return it.value


def host_init_kmeanspp(points, k, seed):
    """K-Means++ on a host float32 array [n, d] (same selections as the reference)."""
    import numpy as np
    p = np.ascontiguousarray(points, np.float32)
    out = np.empty((k, p.shape[1]), np.float32)
    check(load().mxk_host_init_kmeanspp(_np(p), p.shape[0], p.shape[1], k, seed, _np(out)))
    return out


def host_init_farthest(points, k):
    import numpy as np
    p = np.ascontiguousarray(points, np.float32)
    out = np.empty((k, p.shape[1]), np.float32)
    check(load().mxk_host_init_farthest(_np(p), p.shape[0], p.shape[1], k, _np(out)))
    return out


def host_read_points(path, n, d, padded_d, threads=None, chunk_bytes=0):
    """The reference's CSV reader (parallel); threads/chunk_bytes only change
    how the file is split, never the result."""
    import numpy as np
    out = np.empty((n, padded_d), np.float32)
    if threads is None and not chunk_bytes:
        check(load().mxk_host_read_points(str(path).encode(), n, d, padded_d, _np(out)))
    else:
        check(load().mxk_host_read_points_ex(str(path).encode(), n, d, padded_d, threads or 0, chunk_bytes,
                                             _np(out)))
    return out


def host_read_points_f32(path, n, d, padded_d):
    """Raw little-endian float32 rows (n x d, no header), zero padded."""
    import numpy as np
    out = np.empty((n, padded_d), np.float32)
    check(load().mxk_host_read_points_f32(str(path).encode(), n, d, padded_d, _np(out)))
    return out


def launch_count():
    return load().mxk_launch_count()
