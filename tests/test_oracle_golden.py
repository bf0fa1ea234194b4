"""Pins the oracle: its results must equal the golden vectors that the
reference's own generated kernels (kernels/prebuilt/*.cu, built for the host)
produced on the same inputs. CPU only."""
import numpy as np
import pytest

import oracle_lib as O
from tolerance import assert_agree, assert_equal


@pytest.mark.parametrize("tag", ["full", "ragged", "partial"])
def test_vecadd(golden, tag):
    g = golden(f"vecadd_{tag}")
    grid, block = g["geom"]
    c = g["c0"].copy()
    rc = O.oracle().oracle_vecadd(O.f32p(c), len(c), O.f32p(g["a"]), len(g["a"]), O.f32p(g["b"]),
                                  len(g["b"]), O._i64(grid), O._i64(block))
    assert rc == 0
    assert_agree("vecadd", c, g["c"])


def test_scale(golden):
    g = golden("scale")
    rc, y = O.scale(g["x"], float(g["k"]), *g["geom"])
    assert rc == 0
    assert_agree("scale", y, g["y"])


def test_magnitude(golden):
    g = golden("magnitude")
    rc, m = O.magnitude(g["re"], g["im"], *g["geom"])
    assert rc == 0
    # The reference's host build calls glibc hypotf; gpu.Hypot is math.Hypot
    # rounded to float32. Both are correctly rounded on every sample here.
    assert_agree("magnitude", m, g["mag"])


def test_magnitudefast(golden):
    g = golden("magnitudefast")
    rc, m = O.magnitudefast(g["re"], g["im"], float(g["scale"]), *g["geom"])
    assert rc == 0
    assert_agree("magnitudefast", m, g["mag"])


def test_softclip(golden):
    g = golden("softclip")
    rc, y = O.softclip(g["x"], float(g["threshold"]), *g["geom"])
    assert rc == 0
    assert_agree("softclip", y, g["y"])


def test_classify(golden):
    g = golden("classify")
    rc, out = O.classify(g["x"], g["edges"], *g["geom"])
    assert rc == 0
    assert_agree("classify", out, g["out"])


def test_bandgain(golden):
    g = golden("bandgain")
    bands = [tuple(b) for b in g["bands"]]
    rc, y = O.bandgain(g["x"], bands, float(g["floor_gain"]), int(g["count"]), float(g["bias"]),
                       *g["geom"])
    assert rc == 0
    assert_agree("bandgain", y, g["y"])


def test_quantize(golden):
    g = golden("quantize")
    rc, code, energy, clipped = O.quantize(g["x"], float(g["step"]), int(g["seed"]), *g["geom"])
    assert rc == 0
    assert_equal("code", code, g["code"])
    assert_equal("energy", energy, g["energy"])
    assert_equal("clipped", clipped, g["clipped"])


@pytest.mark.parametrize("tag", ["pattern", "short"])
def test_gray(golden, tag):
    g = golden(f"gray_{tag}")
    out = g["out0"].copy()
    grid, block = g["geom"]
    rc = O.oracle().oracle_gray(O.u8p(out), len(out), O.u8p(g["rgb"]), len(g["rgb"]),
                                O._i64(grid), O._i64(block))
    assert rc == 0
    assert_equal("gray", out, g["out"])


@pytest.mark.parametrize("tag", ["formula", "zipf"])
def test_histogram(golden, tag):
    g = golden(f"histogram_{tag}")
    rc, bins = O.histogram(g["x"], len(g["bins0"]), *g["geom"], bins=g["bins0"])
    assert rc == 0
    assert_equal("bins", bins, g["bins"])


@pytest.mark.parametrize("tag", ["full", "partial"])
def test_transpose(golden, tag):
    g = golden(f"transpose_{tag}")
    w, h, gx, gy = (int(v) for v in g["geom"])
    out = g["out0"].copy()
    rc = O.oracle().oracle_transpose(O.f32p(out), len(out), O.f32p(g["inp"]), len(g["inp"]), w,
                                     h, O._i64(gx), O._i64(gy), O._i64(16), O._i64(16))
    assert rc == 0
    assert_equal("transpose", out, g["out"])


@pytest.mark.parametrize("tag", ["formula", "normal"])
def test_warpreduce(golden, tag):
    g = golden(f"warpreduce_{tag}")
    grid, block = g["geom"]
    rc, out = O.warpreducesum(g["x"], len(g["out"]), grid, block)
    assert rc == 0
    assert_agree("warpreduce", out, g["out"])


@pytest.mark.parametrize("tag", ["box33", "rand31", "taps65", "partial"])
def test_fir(golden, tag):
    g = golden(f"fir_{tag}")
    grid, block = g["geom"]
    y = g["y0"].copy()
    rc = O.oracle().oracle_fir(O.f32p(y), len(y), O.f32p(g["x"]), len(g["x"]), O.f32p(g["h"]),
                               len(g["h"]), O._i64(grid), O._i64(block))
    assert rc == 0
    assert_agree("fir", y, g["y"])


def test_histogram_dyn_known_answer():
    """The DynProbe parity test's input (simt/shared_parity_cuda_test.go:
    156-160): x[i] = i*i % 311 - 8, n = 2^15, a 192-bin launch-sized tile;
    the oracle's counts equal a direct count, and with a 256-bin tile it
    agrees with the fixed Histogram."""
    n = 1 << 15
    i = np.arange(n, dtype=np.int64)
    x = ((i * i) % 311 - 8).astype(np.int32)
    rc, got = O.histogram_dyn(x, 192, 192, (n + 255) // 256, 256)
    assert rc == 0
    want = np.bincount(x[(x >= 0) & (x < 192)], minlength=192).astype(np.int32)
    assert_equal("histogram_dyn", got, want)
    rc, h256 = O.histogram(x, 300, (n + 255) // 256, 256)
    rc2, d256 = O.histogram_dyn(x, 300, 256, (n + 255) // 256, 256)
    assert rc == rc2 == 0
    assert_equal("dyn vs fixed", d256, h256)
    # bins shorter than the tile keep only their own; a tile shorter than
    # the bins leaves the rest untouched.
    rc, short = O.histogram_dyn(x, 50, 192, (n + 255) // 256, 256)
    assert_equal("short bins", short, want[:50])
    rc, wide = O.histogram_dyn(x, 400, 100, (n + 255) // 256, 256)
    assert_equal("short tile", wide[:100], want[:100])
    assert not wide[100:].any()
