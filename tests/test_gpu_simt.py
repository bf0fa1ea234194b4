"""GPU parity of the simt kernels (package kernels) against the oracle and the
golden vectors, in the pattern of simt/parity_test.go: the device result
must equal gpu.RunCPU's (restated by the oracle) on the same bytes.

Bit-exact: every kernel except FIR, whose fma order is the reference
device's and is held to the kernels' 1e-5 bound against the emulator order
(simt/parity_test.go:181) and bit-exact against the oracle's fma order.
Each kernel also runs on unaligned slices (scalar path), ragged lengths and
grids that cover fewer threads than the output (only covered indices move).
"""
import numpy as np
import pytest

import oracle_lib as O
from tolerance import assert_agree, assert_close, assert_equal, max_ulp

torch = pytest.importorskip("torch")
from simtgo_b200 import simt  # noqa: E402
from simtgo_b200._lib import AliasError, BlockSizeError, LengthError  # noqa: E402

pytestmark = pytest.mark.gpu


def dev(a, offset=0):
    """numpy -> CUDA tensor; offset>0 makes the data start `offset` elements
    past a 256-byte-aligned allocation (an unaligned slice)."""
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a)
    if offset == 0:
        return t.cuda()
    buf = torch.empty(a.size + offset, dtype=t.dtype, device="cuda")
    view = buf[offset:]
    view.copy_(t.cuda())
    return view


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def normal(n, seed):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


SIZES = [1, 3, 31, 255, 257, 4099, 1 << 16, (1 << 20) + 13]


# ---- golden vectors (the reference's own kernels on the same inputs) --------

@pytest.mark.parametrize("tag", ["full", "ragged", "partial"])
def test_vecadd_golden(golden, tag):
    g = golden(f"vecadd_{tag}")
    grid, block = (int(v) for v in g["geom"])
    c = dev(g["c0"])
    simt.build("VecAdd").launch(grid, block, c, dev(g["a"]), dev(g["b"]))
    assert_agree("vecadd", host(c), g["c"])


def test_scale_golden(golden):
    g = golden("scale")
    y = dev(np.zeros_like(g["y"]))
    simt.build("Scale").launch(*g["geom"], y, dev(g["x"]), float(g["k"]))
    assert_agree("scale", host(y), g["y"])


def test_magnitude_golden(golden):
    g = golden("magnitude")
    m = dev(np.zeros_like(g["mag"]))
    simt.build("Magnitude").launch(*g["geom"], m, dev(g["re"]), dev(g["im"]))
    assert_agree("magnitude", host(m), g["mag"])


def test_magnitudefast_golden(golden):
    g = golden("magnitudefast")
    m = dev(np.zeros_like(g["mag"]))
    simt.build("MagnitudeFast").launch(*g["geom"], m, dev(g["re"]), dev(g["im"]),
                                       float(g["scale"]))
    assert_agree("magnitudefast", host(m), g["mag"])


def test_softclip_golden(golden):
    g = golden("softclip")
    y = dev(np.zeros_like(g["y"]))
    simt.build("Softclip").launch(*g["geom"], y, dev(g["x"]), float(g["threshold"]))
    assert_agree("softclip", host(y), g["y"])


def test_classify_golden(golden):
    g = golden("classify")
    out = dev(np.zeros_like(g["out"]))
    simt.build("Classify").launch(*g["geom"], out, dev(g["x"]), dev(g["edges"]))
    assert_agree("classify", host(out), g["out"])


def test_bandgain_golden(golden):
    g = golden("bandgain")
    y = dev(np.zeros_like(g["y"]))
    cfg = simt.Shape(float(g["floor_gain"]), int(g["count"]), float(g["bias"]))
    simt.build("BandGain").launch(*g["geom"], y, dev(g["x"]), dev(g["bands"].reshape(-1)), cfg)
    assert_agree("bandgain", host(y), g["y"])


def test_quantize_golden(golden):
    g = golden("quantize")
    n = len(g["x"])
    code, energy = dev(np.zeros(n, np.int32)), dev(np.zeros(n, np.int64))
    clipped = dev(np.zeros(n, np.bool_))
    simt.build("Quantize").launch(*g["geom"], code, energy, clipped, dev(g["x"]),
                                  float(g["step"]), int(g["seed"]))
    assert_equal("code", host(code), g["code"])
    assert_equal("energy", host(energy), g["energy"])
    assert_equal("clipped", host(clipped).astype(np.uint8), g["clipped"])


@pytest.mark.parametrize("tag", ["pattern", "short"])
def test_gray_golden(golden, tag):
    g = golden(f"gray_{tag}")
    out = dev(g["out0"])
    simt.build("Gray").launch(*g["geom"], out, dev(g["rgb"]))
    assert_equal("gray", host(out), g["out"])


@pytest.mark.parametrize("tag", ["formula", "zipf"])
def test_histogram_golden(golden, tag):
    g = golden(f"histogram_{tag}")
    bins = dev(g["bins0"])
    simt.build("Histogram").launch(*g["geom"], bins, dev(g["x"]))
    assert_equal("bins", host(bins), g["bins"])


@pytest.mark.parametrize("tag", ["full", "partial"])
def test_transpose_golden(golden, tag):
    g = golden(f"transpose_{tag}")
    w, h, gx, gy = (int(v) for v in g["geom"])
    out = dev(g["out0"])
    simt.build("Transpose").launch_dim((gx, gy), (16, 16), out, dev(g["inp"]), w, h)
    assert_equal("transpose", host(out), g["out"])


@pytest.mark.parametrize("tag", ["formula", "normal"])
def test_warpreduce_golden(golden, tag):
    g = golden(f"warpreduce_{tag}")
    out = dev(np.zeros_like(g["out"]))
    simt.build("WarpReduceSum").launch(*g["geom"], out, dev(g["x"]))
    assert_agree("warpreduce", host(out), g["out"])


@pytest.mark.parametrize("tag", ["box33", "rand31", "taps65", "partial"])
def test_fir_golden(golden, tag):
    g = golden(f"fir_{tag}")
    y = dev(g["y0"])
    simt.build("FIR").launch(*g["geom"], y, dev(g["x"]), dev(g["h"]))
    got = host(y)
    # The golden run is the emulator's order (each product rounded).
    assert_close("fir vs reference build", got, g["y"], 1e-5)
    rc, want = O.fir(g["x"], g["h"], *g["geom"], fused=True)
    want[int(g["geom"][0]) * 256:] = g["y0"][int(g["geom"][0]) * 256:]
    assert rc == 0
    assert_agree("fir vs fma oracle", got, want)


# ---- randomised parity against the oracle ---------------------------------

@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("offset", [0, 1])
def test_vecadd_parity(n, offset):
    a, b = normal(n, 1), normal(n, 2)
    rc, want = O.vecadd(a, b, (n + 255) // 256, 256)
    assert rc == 0
    c = dev(np.zeros(n, np.float32), offset)
    simt.build("VecAdd").launch_n(n, 256, c, dev(a, offset), dev(b, offset))
    assert_agree("vecadd", host(c), want)


@pytest.mark.parametrize("n", SIZES)
def test_scale_parity(n):
    x = normal(n, 3)
    for offset in (0, 3):
        rc, want = O.scale(x, -1.75, (n + 127) // 128, 128)
        y = dev(np.zeros(n, np.float32), offset)
        simt.build("Scale").launch_n(n, 128, y, dev(x, offset), -1.75)
        assert_agree("scale", host(y), want)


@pytest.mark.parametrize("n", SIZES)
def test_magnitude_parity(n):
    re, im = normal(n, 4) * 3, normal(n, 5)
    rc, want = O.magnitude(re, im, (n + 255) // 256, 256)
    m = dev(np.zeros(n, np.float32))
    simt.build("Magnitude").launch_n(n, 256, m, dev(re), dev(im))
    assert_agree("magnitude", host(m), want)


def test_magnitude_wide_range():
    """Exponents across the whole float32 range: the fast path's domain edge
    (2^-60, 2^60), subnormals, overflow to the float64 path, and exact ties."""
    rng = np.random.default_rng(6)
    n = 1 << 20
    e1 = rng.integers(-150, 128, n).astype(np.float64)
    e2 = e1 + rng.integers(-30, 30, n)
    re = (rng.uniform(1, 2, n) * np.exp2(e1)).astype(np.float32)
    im = (rng.uniform(1, 2, n) * np.exp2(np.clip(e2, -150, 127))).astype(np.float32)
    re[:6] = [3, 0, 5, 1e-45, 3.4e38, 2.0 ** -60]
    im[:6] = [4, 0, 12, 1e-45, 3.4e38, 2.0 ** 60]
    rc, want = O.magnitude(re, im, n // 256, 256)
    m = dev(np.zeros(n, np.float32))
    simt.build("Magnitude").launch_n(n, 256, m, dev(re), dev(im))
    got = host(m)
    assert_agree("magnitude", got, want)
    assert got[0] == 5 and got[2] == 13


@pytest.mark.parametrize("n", SIZES)
def test_magnitudefast_parity(n):
    re, im = normal(n, 7), normal(n, 8)
    rc, want = O.magnitudefast(re, im, 3.0, (n + 255) // 256, 256)
    m = dev(np.zeros(n, np.float32), 1 if n % 2 else 0)
    simt.build("MagnitudeFast").launch_n(n, 256, m, dev(re), dev(im), 3.0)
    assert_agree("magnitudefast", host(m), want)


@pytest.mark.parametrize("n", [1, 5, 4097, 1 << 20])
def test_magnitudefast_interleaved(n):
    from simtgo_b200 import _lib
    import ctypes as C
    z = normal(2 * n, 9)
    rc, want = O.magnitudefast_interleaved(z, 3.0, (n + 255) // 256, 256)
    rc2, planar = O.magnitudefast(z[0::2].copy(), z[1::2].copy(), 3.0, (n + 255) // 256, 256)
    assert_agree("interleaved oracle == planar oracle", want, planar)
    m, dz = dev(np.zeros(n, np.float32)), dev(z)
    L = _lib.load()
    _lib.check(L.simtgo_MagnitudeFast_interleaved(C.c_void_p(m.data_ptr()), n,
                                                  C.c_void_p(dz.data_ptr()), 2 * n, 3.0,
                                                  (n + 255) // 256, 256, None))
    _lib.check(L.simtgo_stream_sync(None))
    assert_agree("magnitudefast_interleaved", host(m), want)


@pytest.mark.parametrize("n", SIZES)
def test_softclip_parity(n):
    x = normal(n, 10) * 2
    rc, want = O.softclip(x, 0.5, (n + 255) // 256, 256)
    y = dev(np.zeros(n, np.float32))
    simt.build("Softclip").launch_n(n, 256, y, dev(x), 0.5)
    assert_agree("softclip", host(y), want)


@pytest.mark.parametrize("edges", [[0.1, 0.25, 0.5, 0.8, 1.2, 1.8, 2.5], [], [0.7],
                                   [0.1, 0.2, 0.3], list(np.linspace(0.01, 3, 300))])
def test_classify_parity(edges):
    n = 70001
    e = np.array(edges, np.float32)
    x = normal(n, 11) * 1.5
    rc, want = O.classify(x, e, (n + 127) // 128, 128)
    out = dev(np.zeros(n, np.float32))
    simt.build("Classify").launch_n(n, 128, out, dev(x), dev(e) if len(e) else
                                    torch.empty(0, device="cuda"))
    assert_agree("classify", host(out), want)


@pytest.mark.parametrize("nb", [3, 7, 37, 1500])
def test_bandgain_unsorted_curve(nb):
    """First match in order on an unsorted curve with repeated and NaN
    uppers (shadowed bands, a NaN band first), NaN and infinite samples:
    the register, shared-memory and in-order search paths all agree with
    the emulator."""
    n = 20011
    rng = np.random.default_rng(40 + nb)
    ups = rng.uniform(-2, 2, nb).astype(np.float32)
    ups[0] = np.nan
    if nb > 2:
        ups[2] = ups[1]
    bands = [(float(u), float(gn)) for u, gn in zip(ups, rng.uniform(0, 3, nb))]
    x = normal(n, 41)
    x[:4] = [np.nan, np.inf, -np.inf, 0.0]
    rc, want = O.bandgain(x, bands, 0.125, 3, 0.001, (n + 255) // 256, 256)
    y = dev(np.zeros(n, np.float32))
    simt.build("BandGain").launch_n(n, 256, y, dev(x), simt.bands_tensor(bands),
                                    simt.Shape(0.125, 3, 0.001))
    assert_agree("bandgain", host(y), want)


@pytest.mark.parametrize("nb", [0, 1, 4, 6, 100, 1500])
def test_bandgain_parity(nb):
    n = 50003
    rng = np.random.default_rng(12)
    ups = np.sort(rng.uniform(-2, 2, nb)).astype(np.float32)
    bands = [(float(u), float(gn)) for u, gn in zip(ups, rng.uniform(0, 3, nb))]
    x = normal(n, 13)
    rc, want = O.bandgain(x, bands, 0.125, 3, 0.001, (n + 255) // 256, 256)
    y = dev(np.zeros(n, np.float32))
    bt = simt.bands_tensor(bands) if nb else torch.empty(0, device="cuda")
    simt.build("BandGain").launch_n(n, 256, y, dev(x), bt, simt.Shape(0.125, 3, 0.001))
    assert_agree("bandgain", host(y), want)


@pytest.mark.parametrize("step", [0.3, -0.5, 2.0 ** -20, 2.0 ** 100, 2.0 ** 127, 2.0 ** -149])
def test_quantize_steps(step):
    """x/step rounded as the emulator does for steps of every kind: not a
    power of two, negative, tiny and huge powers of two (subnormal and
    overflowing quotients, the smallest subnormal step), with zeros,
    infinities and NaN among the samples."""
    n = 4099
    x = normal(n, 15) * 4
    x[:10] = [np.inf, -np.inf, np.nan, 0.0, -0.0, 1e-38, -1e-45, 3e38, -3e38, 1.5e-39]
    rc, code, energy, clipped = O.quantize(x, step, 12345, (n + 255) // 256, 256)
    dc, de = dev(np.zeros(n, np.int32)), dev(np.zeros(n, np.int64))
    dk = dev(np.zeros(n, np.bool_))
    simt.build("Quantize").launch_n(n, 256, dc, de, dk, dev(x), step, 12345)
    assert_equal("code", host(dc), code)
    assert_equal("energy", host(de), energy)
    assert_equal("clipped", host(dk).astype(np.uint8), clipped)


@pytest.mark.parametrize("n", SIZES)
def test_quantize_parity(n):
    x = normal(n, 14) * 4
    if n > 8:
        x[:8] = [np.inf, -np.inf, np.nan, 3e9, -3e9, 31.99, -32.01, 0.0]
    rc, code, energy, clipped = O.quantize(x, 0.25, 0x9E3779B9, (n + 255) // 256, 256)
    dc, de = dev(np.zeros(n, np.int32)), dev(np.zeros(n, np.int64))
    dk = dev(np.zeros(n, np.bool_))
    simt.build("Quantize").launch_n(n, 256, dc, de, dk, dev(x), 0.25, 0x9E3779B9)
    assert_equal("code", host(dc), code)
    assert_equal("energy", host(de), energy)
    assert_equal("clipped", host(dk).astype(np.uint8), clipped)
    # simt/parity_test.go:389-396: energy = q^2, and a clipped sample sits at
    # a rail. (A sample can also land on 127 without clipping: 31.99/0.25
    # plus a negative dither truncates to 127.)
    assert (energy == code.astype(np.int64) ** 2).all()
    assert ((code[clipped == 1] == 127) | (code[clipped == 1] == -128)).all()


@pytest.mark.parametrize("npx,short", [(1, 0), (15, 0), (17, 1), (4096, 0), (33177600 // 64, 2),
                                       (100003, 5)])
def test_gray_parity(npx, short):
    rng = np.random.default_rng(15)
    rgb = rng.integers(0, 256, 3 * npx - short, dtype=np.uint8)
    rc, want = O.gray(rgb, npx, (npx + 255) // 256, 256)
    out = dev(np.zeros(npx, np.uint8))
    simt.build("Gray").launch_n(npx, 256, out, dev(rgb))
    assert_equal("gray", host(out), want)


def test_gray_full_frame():
    """7680x4320 interleaved RGB, uniform bytes: the Gray workload."""
    npx = 7680 * 4320
    rgb = np.random.default_rng(10).integers(0, 256, 3 * npx, dtype=np.uint8)
    rgb[:6] = [255, 255, 255, 0, 0, 0]
    rc, want = O.gray(rgb, npx, (npx + 255) // 256, 256)
    out = dev(np.zeros(npx, np.uint8))
    simt.build("Gray").launch_n(npx, 256, out, dev(rgb))
    got = host(out)
    assert got[0] == 255 and got[1] == 0
    assert_equal("gray", got, want)


@pytest.mark.parametrize("n", [1, 7, 1000, 1 << 16, (1 << 22) + 3])
@pytest.mark.parametrize("dist", ["uniform", "zipf", "wide"])
def test_histogram_parity(n, dist):
    rng = np.random.default_rng(16)
    if dist == "uniform":
        x = rng.integers(0, 256, n, dtype=np.int32)
    elif dist == "zipf":
        p = (np.arange(256) + 1.0) ** -1.2
        x = np.searchsorted(np.cumsum(p / p.sum()), rng.random(n)).astype(np.int32)
    else:
        x = rng.integers(-300, 600, n, dtype=np.int32)
    bins0 = rng.integers(0, 100, 256, dtype=np.int32)
    rc, want = O.histogram(x, 256, (n + 255) // 256, 256, bins=bins0)
    b = dev(bins0)
    simt.build("Histogram").launch_n(n, 256, b, dev(x, 1 if n % 2 else 0))
    assert_equal("bins", host(b), want)


def test_histogram_dyn_known_answer():
    """TestDynamicSharedTileParity (simt/shared_parity_cuda_test.go:146-178):
    x[i] = i*i % 311 - 8, n = 2^15, 192 bins through LaunchShared."""
    n = 1 << 15
    i = np.arange(n, dtype=np.int64)
    x = ((i * i) % 311 - 8).astype(np.int32)
    b = dev(np.zeros(192, np.int32))
    simt.build("HistogramDyn").launch_shared((n + 255) // 256, 256, 192, b, dev(x))
    want = np.bincount(x[(x >= 0) & (x < 192)], minlength=192).astype(np.int32)
    assert_equal("bins", host(b), want)


@pytest.mark.parametrize("tile,nbins", [(1, 1), (192, 192), (256, 300), (1000, 600),
                                        (5000, 5000), (33000, 10), (57000, 57000)])
@pytest.mark.parametrize("offset", [0, 1])
def test_histogram_dyn_parity(tile, nbins, offset):
    """Launch-sized tiles from 1 to ~57 K bins (one private table per warp
    down to one per block), bins shorter and longer than the tile, samples
    outside the tile, a grid covering part of x, unaligned x; the counts
    are added to bins that start non-zero."""
    rng = np.random.default_rng(tile + nbins + offset)
    n = 200003
    x = rng.integers(-10, tile + 10, n, dtype=np.int32)
    bins0 = rng.integers(0, 100, nbins, dtype=np.int32)
    grid = n // 256 - 3
    rc, want = O.histogram_dyn(x, nbins, tile, grid, 256, bins=bins0)
    assert rc == 0
    b = dev(bins0)
    simt.build("HistogramDyn").launch_shared(grid, 256, tile, b, dev(x, offset))
    assert_equal("bins", host(b), want)


def test_histogram_dyn_tile_too_large():
    """A tile beyond a block's shared memory is a SharedMemoryError before
    the launch (simt/shared_parity_cuda_test.go:216-227)."""
    b = dev(np.zeros(8, np.int32))
    with pytest.raises(simt.SharedMemoryError):
        simt.build("HistogramDyn").launch_shared(1, 32, 1 << 20, b, dev(np.zeros(8, np.int32)))


def test_histogram_short_bins_and_partial_grid():
    x = np.random.default_rng(17).integers(0, 256, 100000, dtype=np.int32)
    rc, want = O.histogram(x, 100, 37, 512)
    b = dev(np.zeros(100, np.int32))
    simt.build("Histogram").launch(37, 512, b, dev(x))
    assert_equal("bins", host(b), want)


@pytest.mark.parametrize("w,h", [(1, 1), (133, 71), (64, 64), (100, 300), (1024, 4), (4, 1024),
                                 (1000, 1003)])
def test_transpose_parity(w, h):
    inp = normal(w * h, 18)
    gx, gy = (w + 15) // 16, (h + 15) // 16
    for gxx, gyy in [(gx, gy), (max(1, gx // 2), gy), (gx, max(1, gy // 3))]:
        rc, want = O.transpose(inp, w, h, gxx, gyy)
        out = dev(np.zeros(w * h, np.float32))
        simt.build("Transpose").launch_dim((gxx, gyy), (16, 16), out, dev(inp), w, h)
        assert_equal("transpose", host(out), want)


def test_transpose_16k():
    """The 16384x16384 workload (1 GiB each way), checked against the
    obvious loop via numpy."""
    n = 16384
    inp = np.random.default_rng(9).uniform(-1, 1, n * n).astype(np.float32)
    din = dev(inp)
    out = torch.empty(n * n, dtype=torch.float32, device="cuda")
    simt.build("Transpose").launch_dim((n // 16, n // 16), (16, 16), out, din, n, n)
    got = host(out).reshape(n, n)
    assert np.array_equal(got, inp.reshape(n, n).T)


@pytest.mark.parametrize("n", [1, 31, 32, 33, 37 * 128 + 53, 1 << 16, (1 << 20) + 96,
                               (1 << 22) + 5])
def test_warpreduce_parity(n):
    x = normal(n, 19)
    grid = (n + 127) // 128
    for out_len, offset in [(grid * 4, 0), (grid * 4 + 9, 0), (max(1, grid), 1)]:
        rc, want = O.warpreducesum(x, out_len, grid)
        out = dev(np.full(out_len, 7.0, np.float32))
        simt.build("WarpReduceSum").launch(grid, 128, out, dev(x, offset))
        got = host(out)
        covered = min(out_len, grid * 4)
        assert_agree("warpreduce", got[:covered], want[:covered])
        assert (got[covered:] == 7.0).all()


@pytest.mark.parametrize("n,taps", [(1, 1), (300, 3), (4099, 31), (1 << 15, 33), (70000, 65),
                                    ((1 << 20), 31), ((1 << 20) + 77, 17)])
def test_fir_parity(n, taps):
    rng = np.random.default_rng(20)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    h = rng.uniform(-1, 1, taps).astype(np.float32)
    h = (h / max(1.0, abs(float(h.sum())))).astype(np.float32)
    grid = (n + 255) // 256
    rc, want_fma = O.fir(x, h, grid, fused=True)
    rc, want_cpu = O.fir(x, h, grid, fused=False)
    for offset in (0, 1):
        y = dev(np.zeros(n, np.float32), offset)
        simt.build("FIR").launch_n(n, 256, y, dev(x, offset), dev(h))
        got = host(y)
        assert_agree("fir vs fma-order oracle", got, want_fma)
        assert_close("fir vs gpu.RunCPU order", got, want_cpu, 1e-5)


def test_fir_independent_reference():
    """simt/parity_test.go:141-181: 2^15 samples, 33 taps of 1/33, against
    the plain loop; the device within 1e-5."""
    n = 1 << 15
    x = normal(n, 1)
    h = np.full(33, 1 / 33, np.float32)
    ref = np.zeros(n, np.float32)
    for k in range(33):
        ref[k:] = (ref[k:] + np.float32(h[k]) * x[: n - k]).astype(np.float32)
    y = dev(np.zeros(n, np.float32))
    simt.build("FIR").launch_n(n, 256, y, dev(x), dev(h))
    assert_close("gpu vs reference loop", host(y), ref, 1e-5)


def test_fir_zero_taps_and_partial_grid():
    x = normal(5000, 21)
    y = dev(np.full(5000, 9.0, np.float32))
    simt.build("FIR").launch(3, 256, y, dev(x), torch.empty(0, device="cuda"))
    got = host(y)
    assert (got[:768] == 0).all() and (got[768:] == 9.0).all()


# ---- the launch contract on a device -------------------------------------------

def test_errors_on_device():
    x = dev(normal(64, 22))
    with pytest.raises(BlockSizeError):
        simt.build("FIR").launch(1, 128, x, x, x)
    with pytest.raises(AliasError):
        simt.build("VecAdd").launch(1, 64, x, x, dev(normal(64, 23)))
    with pytest.raises(LengthError):
        simt.build("VecAdd").launch(1, 64, x, dev(normal(32, 1)), dev(normal(64, 1)))
    with pytest.raises(simt.ArgCountError):
        simt.build("Scale").launch(1, 64, x, x)
    with pytest.raises(TypeError):
        simt.build("Histogram").launch(1, 64, dev(np.zeros(256, np.int32)), x)


def test_launch_on_stream_is_async_then_syncs():
    n = 1 << 20
    a, b = normal(n, 24), normal(n, 25)
    s = torch.cuda.Stream()
    c = dev(np.zeros(n, np.float32))
    da, db = dev(a), dev(b)
    torch.cuda.synchronize()
    simt.build("VecAdd").launch_on(s, (n + 255) // 256, 256, c, da, db)
    simt.stream_sync(s)
    assert_agree("vecadd on stream", c.cpu().numpy(), (a + b).astype(np.float32))


def test_magnitudefast_max_ulp_logged():
    """simt/parity_test.go:1314: the reference's fast-math build is within
    1e-5; this implementation is exact, 0 ulp from the emulator."""
    n = 1 << 14
    re, im = normal(n, 1), normal(n, 2)
    rc, want = O.magnitudefast(re, im, 3.0, n // 256, 256)
    m = dev(np.zeros(n, np.float32))
    simt.build("MagnitudeFast").launch_n(n, 256, m, dev(re), dev(im), 3.0)
    assert max_ulp(host(m), want) == 0
