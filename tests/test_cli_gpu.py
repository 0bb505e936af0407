"""The mxkmeans CLI end to end (reference src/main.cu): CSV in, GPU
initialisation, Lloyd, label file and stdout record out.  The same run is
replayed through the reference's own CSV reader and K-Means++ / farthest-first
(oracle/_ref/libref_host.so) and this library's kmeans_mixed; integer-valued
points keep every sum exact, so the labels must agree exactly.  The same points
given as a raw float32 (.f32) file give the same labels."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, blobs

pytestmark = pytest.mark.gpu

CLI = os.path.join(ROOT, "mx-kmeans_b200", "mxkmeans")


@pytest.mark.parametrize("init", ["kmeans++", "farthest"])
def test_cli_matches_reference_host_path(torch_cuda, mxk, orc, tmp_path, init):
    torch = torch_cuda
    ref = orc.ref_lib("libref_host.so")
    assert ref is not None, "oracle/_ref/libref_host.so is missing"
    n, d, k, seed = 3000, 96, 12, 5
    x = np.rint(blobs(n, d, k, seed=21, spread=8.0, sigma=1.0, pad_to=1))[:, :d].astype(np.float32)
    csv = tmp_path / "points.csv"
    with open(csv, "w") as f:
        f.write(",".join(f"f{j}" for j in range(d)) + ",label\n")
        for row in x:
            f.write(",".join(str(int(v)) for v in row) + ",0\n")
    out = tmp_path / "labels.csv"
    r = subprocess.run([CLI, "-n", str(n), "-d", str(d), "-k", str(k), "-i", str(csv), "-o", str(out), "-m", "25",
                        "-t", "0", "-s", str(seed), "--init", init], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    rec = r.stdout.strip().splitlines()[-1].split(",")
    assert rec[:3] == [str(n), str(d), str(k)]
    iters = int(rec[4])
    lines = open(out).read().split()
    assert lines[0] == "clusters"
    labels_cli = np.array(lines[1:], np.int32)

    dp = 128
    pts = np.zeros((n, dp), np.float32)
    ref.ref_read_points.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    assert ref.ref_read_points(str(csv).encode(), n, d, dp, pts.ctypes.data) == 0
    c0 = np.zeros((k, dp), np.float32)
    if init == "farthest":
        ref.ref_init_farthest.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        ref.ref_init_farthest(pts.ctypes.data, n, dp, k, c0.ctypes.data)
    else:
        ref.ref_init_kmeanspp.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_uint32, ctypes.c_void_p]
        ref.ref_init_kmeanspp(pts.ctypes.data, n, dp, k, seed, c0.ctypes.data)
    xt = torch.from_numpy(pts).cuda()
    ct = torch.from_numpy(c0).cuda()
    lab = torch.empty(n, dtype=torch.int32, device="cuda")
    it = mxk.kmeans_mixed(xt, ct, lab, mxk.Options(max_iterations=25, tolerance=0.0))
    assert it == iters
    assert np.array_equal(lab.cpu().numpy(), labels_cli)

    # the same points as raw float32 rows (.f32 input): same run, same labels
    raw = tmp_path / "points.f32"
    x.astype("<f4").tofile(raw)
    out2 = tmp_path / "labels2.csv"
    r2 = subprocess.run([CLI, "-n", str(n), "-d", str(d), "-k", str(k), "-i", str(raw), "-o", str(out2), "-m", "25",
                         "-t", "0", "-s", str(seed), "--init", init], capture_output=True, text=True, timeout=300)
    assert r2.returncode == 0, r2.stderr
    assert r2.stdout.strip().splitlines()[-1].split(",")[4] == str(iters)
    assert open(out2).read() == open(out).read()
