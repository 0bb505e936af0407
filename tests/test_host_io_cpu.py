"""Host side of the CLI (mxk_host_* in include/mxk.h) against the reference's
own include/host_utils.hpp (compiled into oracle/_ref/libref_host.so) and the
committed golden selections: K-Means++ and farthest-first initialisation pick
the same rows; the CSV reader accepts and rejects the same files
(tests/host_checks.cpp:41-68)."""
import ctypes
import os

import numpy as np
import pytest

from conftest import REFERENCE_DIR, ROOT

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
        if not os.path.isdir(REFERENCE_DIR):
            pytest.skip("oracle/_ref not built and the reference checkout is absent")
        orc.build_ref()
        lib = orc.ref_lib("libref_host.so")
    return lib


# (the last case is above the size where the per-point distances run on all
# host threads)
@pytest.mark.parametrize("seed,n,d,k", [(1, 1000, 64, 32), (9, 3000, 128, 64), (123, 257, 7, 12),
                                        (5, 20011, 64, 24)])
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


# ---- parallel CSV reader against the reference's own read_points -----------
#
# The reader splits the file into chunks at line boundaries and parses them on
# several threads, with an exact fast path for plain decimals.  Whatever the
# chunking, it must accept and reject the same files as the reference's
# sequential reader, with the same message, and produce the same floats bit for
# bit (std::stof's correctly rounded results, -0 included).

def _ref_read(ref_host, path, n, d, dp):
    out = np.zeros((n, dp), np.float32)
    msg = ctypes.create_string_buffer(512)
    rc = ref_host.ref_read_points_msg(str(path).encode(), n, d, dp, ctypes.c_void_p(out.ctypes.data), msg, 512)
    return rc, out, msg.value.decode()


def _ours(mxk, path, n, d, dp, threads=None, chunk=0):
    try:
        return 0, mxk.host_read_points(path, n, d, dp, threads=threads, chunk_bytes=chunk), ""
    except ValueError as e:
        return 1, None, e.message


def _same(ref, got):
    rc, out, msg = ref
    grc, gout, gmsg = got
    assert grc == rc, (msg, gmsg)
    if rc == 0:
        assert np.array_equal(gout.view(np.uint32), out.view(np.uint32))
    else:
        assert gmsg == msg


@pytest.mark.parametrize("text,n,ok", CSV_CASES)
@pytest.mark.parametrize("chunk", [1, 3, 7])
def test_csv_reader_chunked_matches_reference(mxk, ref_host, tmp_path, text, n, ok, chunk):
    p = tmp_path / "pts.csv"
    p.write_text(text)
    _same(_ref_read(ref_host, p, n, 2, 128), _ours(mxk, p, n, 2, 128, threads=3, chunk=chunk))


TRICKY = ["0", "-0", "+0", "-0.0", "0.000", "1", "-1", "+1", "1.", ".5", "-.5", "5e0", "1e-3", "1E+3", " 7",
          "\t7", "7 ", "7\t", "7\r", "  -3.25  ", "1e-38", "1.17549435e-38", "1.1754942e-38", "1e-40", "1e-45",
          "0e-99", "0e999999", "3.4028235e38", "3.4028236e38", "3.40282357e38", "1e39", "-1e39", "16777217",
          "16777219", "33554435", "0.1", "0.2", "0.3", "123456789012345678", "1234567890123456789",
          "12345678901234567890", "9007199254740993", "0.1000000000000000055511151231257827", "0x1p3", "0X1.8p1",
          "0x", "inf", "-inf", "nan", "NaN", "infinity", "", " ", "e5", "1e", "1e+", "1.2.3", "--1", "+-1", "1x",
          "1 2", ".", "-", "\v7", "\f7", "7\v", "1e22", "1e23", "9e22", "4.5e-23", "1e-22", "2e-22",
          "00000000000000000000001.5", "1.50000000000000000000000", "0.000000000000000000000000000001"]


def test_csv_reader_tricky_cells_match_reference(mxk, ref_host, tmp_path):
    for i, cell in enumerate(TRICKY):
        p = tmp_path / f"c{i}.csv"
        with open(p, "w", newline="") as f:
            f.write("a,b,label\n" + f"{cell},2.5,x\n" + f"-1,{cell},y\n")
        for chunk in (0, 4):
            _same(_ref_read(ref_host, p, 2, 2, 128), _ours(mxk, p, 2, 2, 128, threads=2, chunk=chunk))


def _random_decimals(g, count):
    """Plain decimals of 1-19 significant digits and powers of ten across the
    float range: the fast path's whole domain and its edges."""
    out = []
    for _ in range(count):
        nd = int(g.integers(1, 20))
        digits = "".join(str(int(v)) for v in g.integers(0, 10, nd))
        sign = g.choice(["", "-", "+"], p=[0.6, 0.35, 0.05])
        form = int(g.integers(0, 3))
        e = int(g.integers(-48, 40))
        if form == 0:  # d.ddd e+-x
            s = f"{sign}{digits[0]}.{digits[1:]}e{e}"
        elif form == 1:  # ddd.ddd
            cut = int(g.integers(0, nd + 1))
            s = f"{sign}{digits[:cut]}.{digits[cut:]}" if cut < nd else f"{sign}{digits}"
            if s in (sign + ".", "."):
                s = sign + "0"
        else:  # ddd e+-x
            s = f"{sign}{digits}E{e:+d}"
        out.append(s)
    return out


def test_csv_reader_random_decimals_bit_exact(mxk, ref_host, tmp_path):
    """About 200k random plain decimals, parsed by the reference (std::stof per
    cell) and by the parallel reader (fast path + strtof), compared bit for bit,
    including which ones are rejected (denormal and overflowing values)."""
    g = np.random.default_rng(123)
    d = 64
    for trial in range(4):
        n = 800
        cells = _random_decimals(g, n * d)
        p = tmp_path / f"r{trial}.csv"
        with open(p, "w") as f:
            f.write(",".join(f"f{j}" for j in range(d)) + "\n")
            for r in range(n):
                f.write(",".join(cells[r * d:(r + 1) * d]) + "\n")
        ref = _ref_read(ref_host, p, n, d, 128)
        if ref[0]:
            # a rejected value stops the reference at its first one; compare
            # that, then each row separately so the accepted cells count too
            _same(ref, _ours(mxk, p, n, d, 128, threads=4))
            for r in range(n):
                q = tmp_path / "row.csv"
                q.write_text(",".join(f"f{j}" for j in range(d)) + "\n" + ",".join(cells[r * d:(r + 1) * d]) + "\n")
                _same(_ref_read(ref_host, q, 1, d, 128), _ours(mxk, q, 1, d, 128, threads=1))
        else:
            _same(ref, _ours(mxk, p, n, d, 128, threads=4, chunk=997))


def test_csv_reader_fast_path_domain_exhaustive_mantissas(mxk, ref_host, tmp_path):
    """Mantissas up to 2^53 times every power of ten the fast path takes
    (1e-22..1e22), plus integers on and next to float rounding midpoints, where
    rounding the correctly rounded double to float could differ from strtof."""
    g = np.random.default_rng(7)
    cells = []
    for e in range(-22, 23):
        for m in g.integers(1, 2 ** 53, 40, dtype=np.int64).tolist() + [2 ** 53, 2 ** 53 - 1, 1, 9, 10 ** 15]:
            cells.append(f"{m}e{e}")
    for k in range(24, 54):
        for off in (-1, 0, 1):
            base = (1 << k) + (1 << (k - 24)) * 1  # float midpoint between 2^k and its successor
            cells.append(str(base + off))
            cells.append(str(3 * (1 << k) + (1 << (k - 23)) + off))
    d = 8
    while len(cells) % d:
        cells.append("1")
    n = len(cells) // d
    p = tmp_path / "m.csv"
    with open(p, "w") as f:
        f.write(",".join("x" * 1 for _ in range(d)) + "\n")
        for r in range(n):
            f.write(",".join(cells[r * d:(r + 1) * d]) + "\n")
    ref = _ref_read(ref_host, p, n, d, 128)
    got = _ours(mxk, p, n, d, 128, threads=4, chunk=513)
    if ref[0] == 0:
        _same(ref, got)
    else:  # values beyond the float range are rejected: check row by row
        for r in range(n):
            q = tmp_path / "row.csv"
            q.write_text(",".join("x" for _ in range(d)) + "\n" + ",".join(cells[r * d:(r + 1) * d]) + "\n")
            _same(_ref_read(ref_host, q, 1, d, 128), _ours(mxk, q, 1, d, 128, threads=1))


def test_csv_reader_error_row_independent_of_chunking(mxk, ref_host, tmp_path):
    """Several bad lines in different chunks: the first in file order is the one
    reported, with the reference's data row number (blank lines not counted)."""
    g = np.random.default_rng(3)
    d, n = 5, 3000
    x = g.standard_normal((n, d)).astype(np.float32)
    lines = ["a,b,c,d,e"]
    for r in range(n):
        lines.append(",".join(repr(float(v)) for v in x[r]))
        if r % 97 == 0:
            lines.append("  \r")
    good = "\n".join(lines) + "\n"
    p = tmp_path / "ok.csv"
    p.write_text(good)
    ref = _ref_read(ref_host, p, n, d, 8)
    assert ref[0] == 0
    for threads, chunk in [(1, 0), (8, 64), (5, 1)]:
        _same(ref, _ours(mxk, p, n, d, 8, threads=threads, chunk=chunk))
    # n too small / too large
    for nn in (n - 1, n + 1):
        _same(_ref_read(ref_host, p, nn, d, 8), _ours(mxk, p, nn, d, 8, threads=8, chunk=64))
    bad = list(lines)
    bad[2500] = bad[2500] + ",9"          # wrong column count, late
    bad[1800] = bad[1800].replace(",", ",1e-41,", 1).rsplit(",", 1)[0]  # denormal, earlier
    bad[2900] = "1,2,3,4,nan"
    q = tmp_path / "bad.csv"
    q.write_text("\n".join(bad) + "\n")
    ref = _ref_read(ref_host, q, n, d, 8)
    assert ref[0] == 1 and "Invalid feature" in ref[2]
    for threads, chunk in [(1, 0), (8, 64), (3, 5)]:
        _same(ref, _ours(mxk, q, n, d, 8, threads=threads, chunk=chunk))


def test_csv_reader_nul_and_binary_junk(mxk, ref_host, tmp_path):
    p = tmp_path / "nul.csv"
    p.write_bytes(b"a,b\n1\x00,2\n")
    _same(_ref_read(ref_host, p, 1, 2, 4), _ours(mxk, p, 1, 2, 4, threads=2, chunk=2))
    p.write_bytes(b"a,b\n1,2\n\x00\n")
    _same(_ref_read(ref_host, p, 1, 2, 4), _ours(mxk, p, 1, 2, 4, threads=2, chunk=2))
    p.write_bytes(b"a,b\n1,2")  # no final newline
    _same(_ref_read(ref_host, p, 1, 2, 4), _ours(mxk, p, 1, 2, 4, threads=2, chunk=1))
    d = tmp_path / "dir"
    d.mkdir()
    _same(_ref_read(ref_host, d, 1, 2, 4), _ours(mxk, d, 1, 2, 4))
    _same(_ref_read(ref_host, tmp_path / "missing.csv", 1, 2, 4), _ours(mxk, tmp_path / "missing.csv", 1, 2, 4))


# ---- binary float32 input ---------------------------------------------------

def test_f32_reader(mxk, tmp_path):
    g = np.random.default_rng(5)
    n, d = 1001, 96
    x = g.standard_normal((n, d)).astype(np.float32)
    x[3, 4] = -0.0
    p = tmp_path / "pts.f32"
    x.astype("<f4").tofile(p)
    got = mxk.host_read_points_f32(p, n, d, 128)
    assert np.array_equal(got[:, :d].view(np.uint32), x.view(np.uint32))
    assert not got[:, d:].any()
    assert np.array_equal(mxk.host_read_points_f32(p, n, d, d), x)
    with pytest.raises(ValueError, match="exactly n \\* d float32"):
        mxk.host_read_points_f32(p, n + 1, d, 128)
    x[700, 5] = np.nan
    x[900, 0] = np.inf
    x.tofile(p)
    with pytest.raises(ValueError, match="Invalid feature at data row 701, column 6"):
        mxk.host_read_points_f32(p, n, d, 128)
    with pytest.raises(ValueError, match="Cannot open input"):
        mxk.host_read_points_f32(tmp_path / "none.f32", n, d, 128)


# ---- label file -------------------------------------------------------------

_REF_WRITER = r"""
import ctypes, sys
lib = ctypes.CDLL(sys.argv[1])
data = open(sys.argv[2], "rb").read()
n = len(data) // 4
arr = (ctypes.c_int * max(n, 1)).from_buffer_copy(data or bytes(4))
lib.ref_write_labels.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int64]
sys.exit(lib.ref_write_labels(sys.argv[3].encode(), ctypes.cast(arr, ctypes.c_void_p), n))
"""


def test_label_writer_bytes_match_reference(mxk, orc, ref_host, tmp_path):
    """Labels formatted on several threads in blocks: the file is byte for byte
    the reference's ofstream output (header, one decimal label per line),
    including negative and extreme values and sizes across block boundaries.
    The reference's writer runs in a child process that loads nothing but
    ctypes and the reference library (in a process that has loaded numpy's
    bundled runtime libraries first, its ofstream faults)."""
    import subprocess
    import sys
    g = np.random.default_rng(1)
    ref_so = os.path.join(orc.REF_DIR, "libref_host.so")
    script = tmp_path / "ref_writer.py"
    script.write_text(_REF_WRITER)
    for n in (0, 1, 7, (1 << 20) - 1, (1 << 20) + 3, 3 * (1 << 20) + 5):
        lab = g.integers(0, 2048, n).astype(np.int32)
        if n > 4:
            lab[:4] = [np.iinfo(np.int32).min, np.iinfo(np.int32).max, -1, 0]
        a, b, raw = tmp_path / "ours.csv", tmp_path / "ref.csv", tmp_path / "labels.bin"
        assert mxk.load().mxk_host_write_labels(str(a).encode(), mxk._np(lab) if n else None, n) == mxk.OK
        expected = ("clusters\n" + "".join(f"{v}\n" for v in lab.tolist())).encode()
        assert a.read_bytes() == expected
        if n < (1 << 21):
            lab.astype("<i4").tofile(raw)
            r = subprocess.run([sys.executable, str(script), ref_so, str(raw), str(b)], capture_output=True)
            assert r.returncode == 0, r.stderr
            assert a.read_bytes() == b.read_bytes()
    d = tmp_path / "adir"
    d.mkdir()
    assert mxk.load().mxk_host_write_labels(str(d).encode(), None, 0) == mxk.ERR_INVALID
    assert b"Cannot open output" in mxk.load().mxk_last_error()
