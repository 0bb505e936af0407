"""K1 parity: MX quantization on the GPU vs the CPU oracle, bit for bit.

Reference behaviour: src/kernels/quantize.cu:13-72 (scales, RNE conversion,
packing, per-row max squared error); pinned by tests/cuda_checks.cu:56-73.
"""
import numpy as np
import pytest

from conftest import reference_fixture_a, reference_fixture_b

pytestmark = pytest.mark.gpu


def _gpu_quantize(torch, mxk, bits, x, pid=None, errors=True):
    dev = torch.device("cuda:0")
    xt = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    rows = x.shape[0] if pid is None else len(pid)
    d = x.shape[1]
    values = torch.zeros(rows * d * bits // 8, dtype=torch.uint8, device=dev)
    scales = torch.zeros(rows * (d // 32), dtype=torch.uint8, device=dev)
    err = torch.zeros(rows, dtype=torch.float32, device=dev) if errors else None
    pid_t = None if pid is None else torch.from_numpy(np.asarray(pid, np.int32)).to(dev)
    mxk.quantize_rows(bits, xt, values, scales, pid=pid_t, max_errors=err, rows=rows)
    torch.cuda.synchronize()
    return (values.cpu().numpy().reshape(rows, -1), scales.cpu().numpy().reshape(rows, -1),
            None if err is None else err.cpu().numpy())


@pytest.mark.parametrize("bits", [8, 6, 4])
def test_reference_fixture_bit_exact(torch_cuda, mxk, orc, bits):
    # tests/cuda_checks.cu:35-73: 131 x 256 sin fixture, reversed pid.
    a = reference_fixture_a()
    pid = np.arange(a.shape[0] - 1, -1, -1, dtype=np.int32)
    gv, gs, ge = _gpu_quantize(torch_cuda, mxk, bits, a, pid)
    ov, os_, oe = orc.quantize_rows(bits, a, pid, errors=True)
    assert np.array_equal(gs, os_), "UE8M0 scales differ"
    assert np.array_equal(gv, ov), "packed values differ"
    assert np.array_equal(ge.view(np.uint32), oe.view(np.uint32)), "max squared errors differ"


def test_centroid_fixture_mxfp8(torch_cuda, mxk, orc):
    b = reference_fixture_b()
    gv, gs, _ = _gpu_quantize(torch_cuda, mxk, 8, b, errors=False)
    ov, os_, _ = orc.quantize_rows(8, b)
    assert np.array_equal(gs, os_) and np.array_equal(gv, ov)


@pytest.mark.parametrize("bits", [8, 6, 4])
def test_edge_values(torch_cuda, mxk, orc, bits):
    # zero blocks (scale 1), negative zero, subnormals, tiny and huge magnitudes,
    # exact ties of the target grid, values just below/above the scale boundary.
    d = 128
    rows = []
    rows.append(np.zeros(d, np.float32))
    r = np.zeros(d, np.float32); r[::2] = -0.0; rows.append(r)
    rows.append(np.full(d, np.float32(1.4e-45)))
    rows.append((np.arange(d, dtype=np.float32) - 64) * np.float32(1e-39))
    rows.append((np.arange(d, dtype=np.float32) - 64) * np.float32(5e36))  # up to 3.2e38, finite
    rows.append(np.linspace(-448, 448, d).astype(np.float32))
    rows.append(np.linspace(-7.5, 7.5, d).astype(np.float32))
    rows.append(np.linspace(-6, 6, d).astype(np.float32))
    rows.append(np.full(d, np.float32(447.9)))
    rows.append(np.full(d, np.float32(448.0 * 2 ** -30)))
    g = np.random.default_rng(3)
    for scale in (1e-30, 1e-3, 1.0, 1e3, 1e30):
        rows.append((g.standard_normal(d) * scale).astype(np.float32))
    # halfway points of the E4M3 grid at several binades
    e4 = np.array([1.0625, 1.1875, 3.3125, 0.5078125, 13.0, 14.0, 15.0], np.float32)
    rows.append(np.resize(np.concatenate([e4, -e4, [448.0]]).astype(np.float32), d))
    x = np.stack(rows).astype(np.float32)
    assert np.all(np.isfinite(x))
    gv, gs, ge = _gpu_quantize(torch_cuda, mxk, bits, x)
    ov, os_, oe = orc.quantize_rows(bits, x, errors=True)
    bad = np.nonzero(np.any(gs != os_, axis=1) | np.any(gv != ov, axis=1))[0]
    assert bad.size == 0, f"rows {bad[:5]}: gpu scales {gs[bad[:2]]} oracle {os_[bad[:2]]}"
    assert np.array_equal(ge.view(np.uint32), oe.view(np.uint32))


@pytest.mark.parametrize("bits,d", [(8, 128), (8, 768), (6, 256), (4, 384)])
def test_random_rows(torch_cuda, mxk, orc, bits, d):
    g = np.random.default_rng(bits * 1000 + d)
    n = 4099
    x = (g.standard_normal((n, d)) * np.exp2(g.integers(-20, 20, size=(n, d // 32)).repeat(32, axis=1))).astype(
        np.float32)
    gv, gs, ge = _gpu_quantize(torch_cuda, mxk, bits, x)
    ov, os_, oe = orc.quantize_rows(bits, x, errors=True)
    assert np.array_equal(gs, os_)
    assert np.array_equal(gv, ov)
    assert np.array_equal(ge.view(np.uint32), oe.view(np.uint32))


def test_large_shape_sampled(torch_cuda, mxk, orc):
    # Full-size property: 2^21 rows x 128 (the benchmarked shape has 2^23); every row
    # checked through a checksum, 4096 sampled rows checked byte for byte.
    torch = torch_cuda
    n, d = 1 << 21, 128
    gen = torch.Generator(device="cuda:0").manual_seed(5)
    xt = torch.randn((n, d), generator=gen, device="cuda:0") * 3.0
    values = torch.empty(n * d, dtype=torch.uint8, device="cuda:0")
    scales = torch.empty(n * d // 32, dtype=torch.uint8, device="cuda:0")
    mxk.quantize_rows(8, xt, values, scales)
    torch.cuda.synchronize()
    idx = np.sort(np.random.default_rng(1).choice(n, 4096, replace=False))
    xs = xt[torch.from_numpy(idx).cuda()].cpu().numpy()
    ov, os_, _ = orc.quantize_rows(8, xs)
    gv = values.view(n, d)[torch.from_numpy(idx).cuda()].cpu().numpy()
    gs = scales.view(n, d // 32)[torch.from_numpy(idx).cuda()].cpu().numpy()
    assert np.array_equal(gv, ov) and np.array_equal(gs, os_)
    # every scale byte is a plausible power of two for N(0, 9) data
    s_all = scales.cpu().numpy()
    assert s_all.min() >= 110 and s_all.max() <= 127


def test_rejects_bad_bits(torch_cuda, mxk):
    x = torch_cuda.zeros((4, 32), device="cuda:0")
    v = torch_cuda.zeros(4 * 32, dtype=torch_cuda.uint8, device="cuda:0")
    s = torch_cuda.zeros(4, dtype=torch_cuda.uint8, device="cuda:0")
    with pytest.raises(ValueError, match="Precision must be 4, 6, or 8"):
        mxk.quantize_rows(5, x, v, s)
