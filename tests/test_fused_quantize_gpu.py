"""The in-kernel point quantization of the fused assignment (mxk_assign_f32_fused)
equals quantize_rows followed by the fused assignment on pre-quantized rows:
identical MXFP8 bytes, so identical labels and gaps."""
import numpy as np
import pytest

from conftest import blobs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k,seed,with_pid", [(5000, 300, 1, True), (70000, 2048, 2, True), (129, 7, 3, False),
                                               (1000, 200, 4, False)])
def test_f32_fused_equals_quantize_then_assign(torch_cuda, mxk, n, k, seed, with_pid):
    torch = torch_cuda
    d = 128
    x = blobs(n, d, 24, seed=seed)
    x[:7] *= np.float32(2.0 ** -30)   # tiny rows (small UE8M0 scales)
    x[7:9] = 0.0                      # all-zero rows (scale 1.0)
    x[9, :5] = np.float32(1e30)       # saturating values
    x[10] *= np.float32(2.0 ** -125)  # block maxima below 2^-117: scale from the division
    g = np.random.default_rng(seed)
    c = x[g.choice(n, k, replace=False)].copy()
    c[0, 3] = np.float32(2.0 ** -20)
    X = torch.from_numpy(x).cuda()
    C = torch.from_numpy(c).cuda()
    rows = n
    pid = torch.from_numpy(g.permutation(n).astype(np.int32)).cuda() if with_pid else None
    qc = torch.empty(k * d, dtype=torch.uint8, device="cuda"); sc = torch.empty(k * d // 32, dtype=torch.uint8, device="cuda")
    mxk.quantize_rows(8, C, qc, sc)
    pn = torch.empty(n, device="cuda"); cn = torch.empty(k, device="cuda")
    mxk.compute_l2_norm(X, pn); mxk.compute_l2_norm(C, cn)
    # reference path: quantize the rows (in pid order) then assign
    qx = torch.empty(rows * d, dtype=torch.uint8, device="cuda"); sx = torch.empty(rows * d // 32, dtype=torch.uint8, device="cuda")
    mxk.quantize_rows(8, X, qx, sx, pid=pid, rows=rows)
    lab_ref = torch.full((n,), -7, dtype=torch.int32, device="cuda"); gap_ref = torch.zeros(n, device="cuda")
    mxk.assign_mx_fused(8, rows, k, d, qx, sx, qc, sc, pn, cn, lab_ref, gap_ref, pid=pid)
    lab = torch.full((n,), -7, dtype=torch.int32, device="cuda"); gap = torch.zeros(n, device="cuda")
    mxk.assign_f32_fused(rows, k, d, X, qc, sc, pn, cn, lab, gap, pid=pid)
    lab_ng = torch.full((n,), -7, dtype=torch.int32, device="cuda")
    mxk.assign_f32_fused(rows, k, d, X, qc, sc, pn, cn, lab_ng, None, pid=pid, start_hint=lab_ref)
    torch.cuda.synchronize()
    assert torch.equal(lab, lab_ref)
    # bit-exact, NaN where both are NaN (the 1e30 row's norm is infinite)
    torch.testing.assert_close(gap, gap_ref, rtol=0, atol=0, equal_nan=True)
    assert torch.equal(lab_ng, lab_ref)


def test_f32_fused_rejects_other_shapes(torch_cuda, mxk):
    torch = torch_cuda
    x = torch.zeros((10, 256), device="cuda")
    q = torch.zeros(4 * 256, dtype=torch.uint8, device="cuda"); s = torch.zeros(4 * 8, dtype=torch.uint8, device="cuda")
    n = torch.zeros(10, device="cuda"); c = torch.zeros(4, device="cuda")
    lab = torch.zeros(10, dtype=torch.int32, device="cuda")
    with pytest.raises(mxk.MxkInvalidArgument):
        mxk.assign_f32_fused(10, 4, 256, x, q, s, n, c, lab)


def test_mxfp8_scale_codec_exhaustive(torch_cuda, mxk):
    """The quantizer's division-free scale rule equals ue8m0(amax / 448) with the
    IEEE division for all 2^32 float32 bit patterns."""
    torch = torch_cuda
    res = torch.zeros(2, dtype=torch.int64, device="cuda")
    mxk.check_mxfp8_scale_codec(res)
    torch.cuda.synchronize()
    count, first = res.cpu().tolist()
    assert count == 0, f"{count} disagreements, first at bit pattern {first & 0xffffffff:#010x}"
    assert first == -1
