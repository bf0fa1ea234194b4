"""Generates the golden vectors in tests/golden/*.npz.

Each case feeds seeded inputs to the REFERENCE's own generated kernels
(kernels/prebuilt/*.cu of CWBudde/simtgo) compiled for the host by
oracle/Makefile (`make -C oracle ref`, which reads the reference tree named
by the SIMTGO_REFERENCE environment variable) and
stores inputs, launch geometry and outputs. The reference publishes no
numeric golden vectors, so these pin the oracle to the reference's code; the
shapes and special values follow the reference's own parity tests
(simt/parity_test.go, simt/shared_parity_cuda_test.go,
simt/warp_parity_cuda_test.go).

Run with the reference tree:  SIMTGO_REFERENCE=<tree> python tests/golden/make_golden.py
The .npz files are committed; the GPU tests only read them.
"""
from __future__ import annotations

import ctypes as C
import pathlib
import subprocess
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import oracle_lib as O  # noqa: E402

f32, i32 = C.c_float, C.c_int32


def normal(n, seed):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


def specials():
    """Values the float kernels must agree on bit for bit (or as NaN)."""
    return np.array([0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 1e-45, -1e-45, 1.17549435e-38, 3.4e38,
                     -3.4e38, np.inf, -np.inf, np.nan, 2.5, 1e-20, 65504.0, 1e20, -7.25, 0.1],
                    np.float32)


def with_specials(x):
    s = specials()
    x = x.copy()
    x[: len(s)] = s
    return x


def save(name, **arrays):
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print("wrote", name, {k: v.shape for k, v in arrays.items()})


def grid_for(n, block):
    return (n + block - 1) // block


def main():
    subprocess.run(["make", "-C", str(O.ORACLE_DIR), "ref"], check=True)
    O.set_threads(8)
    R = O.ref()

    # VecAdd: 2^16, block 256 (simt/parity_test.go:59), plus a ragged n and a
    # launch covering fewer threads than c_len.
    for tag, n, block, grid in [("full", 1 << 16, 256, grid_for(1 << 16, 256)),
                                ("ragged", 4099, 128, grid_for(4099, 128)),
                                ("partial", 5000, 256, 7)]:
        a, b = with_specials(normal(n, 1)), normal(n, 2)
        c = np.full(n, 7.0, np.float32)
        R.ref_VecAdd(O.f32p(c), n, O.f32p(a), n, O.f32p(b), n, grid, block)
        save(f"vecadd_{tag}", a=a, b=b, c0=np.full(n, 7.0, np.float32), c=c,
             geom=np.array([grid, block]))

    # Scale: 2^14, block 128, factor 0.75 (simt/parity_test.go:88).
    n = 1 << 14
    x = with_specials(normal(n, 3))
    y = np.zeros(n, np.float32)
    R.ref_Scale(O.f32p(y), n, O.f32p(x), n, f32(0.75), grid_for(n, 128), 128)
    save("scale", x=x, y=y, k=np.float32(0.75), geom=np.array([grid_for(n, 128), 128]))

    # Magnitude and MagnitudeFast (simt/parity_test.go:113, :1314, scale 3).
    re, im = with_specials(normal(n, 4)), normal(n, 5)
    im[:20] = specials()[::-1]
    m = np.zeros(n, np.float32)
    R.ref_Magnitude(O.f32p(m), n, O.f32p(re), n, O.f32p(im), n, grid_for(n, 256), 256)
    save("magnitude", re=re, im=im, mag=m, geom=np.array([grid_for(n, 256), 256]))
    mf = np.zeros(n, np.float32)
    R.ref_MagnitudeFast(O.f32p(mf), n, O.f32p(re), n, O.f32p(im), n, f32(3.0),
                        grid_for(n, 256), 256)
    save("magnitudefast", re=re, im=im, mag=mf, scale=np.float32(3.0),
         geom=np.array([grid_for(n, 256), 256]))

    # Softclip, threshold 0.5 (simt/parity_test.go:252).
    x = with_specials(normal(n, 6))
    y = np.zeros(n, np.float32)
    R.ref_Softclip(O.f32p(y), n, O.f32p(x), n, f32(0.5), grid_for(n, 256), 256)
    save("softclip", x=x, y=y, threshold=np.float32(0.5), geom=np.array([grid_for(n, 256), 256]))

    # Classify with the reference's edges, block 128 (simt/parity_test.go:189).
    edges = np.array([0.1, 0.25, 0.5, 0.8, 1.2, 1.8, 2.5], np.float32)
    x = with_specials(normal(n, 7) * 1.5)
    out = np.zeros(n, np.float32)
    R.ref_Classify(O.f32p(out), n, O.f32p(x), n, O.f32p(edges), len(edges),
                   grid_for(n, 128), 128)
    save("classify", x=x, edges=edges, out=out, geom=np.array([grid_for(n, 128), 128]))

    # BandGain with the reference's bands and Shape (simt/parity_test.go:439).
    bands = [(-0.5, 0.25), (0.0, 0.5), (0.5, 1.0), (1.0, 2.0)]
    barr = O.bands_array(bands)
    cfg = O.Shape(0.125, 3, 0.001)
    x = with_specials(normal(n, 8))
    y = np.zeros(n, np.float32)
    R.ref_BandGain(O.f32p(y), n, O.f32p(x), n, barr, len(bands), C.byref(cfg),
                   grid_for(n, 256), 256)
    save("bandgain", x=x, bands=np.array(bands, np.float32), floor_gain=np.float32(0.125),
         count=np.int32(3), bias=np.float64(0.001), y=y, geom=np.array([grid_for(n, 256), 256]))

    # Quantize, step 0.05, seed 0x9e3779b9 (simt/parity_test.go:374), plus
    # values past the int32 range.
    x = with_specials(normal(n, 9))
    x[20:24] = [3e9, -3e9, 1e10, -2147483648.0]
    code = np.zeros(n, np.int32)
    energy = np.zeros(n, np.int64)
    clipped = np.zeros(n, np.uint8)
    R.ref_Quantize(O.i32p(code), n, O.i64p(energy), n, O.u8p(clipped), n, O.f32p(x), n,
                   f32(0.05), C.c_uint32(0x9E3779B9), grid_for(n, 256), 256)
    save("quantize", x=x, step=np.float32(0.05), seed=np.uint32(0x9E3779B9), code=code,
         energy=energy, clipped=clipped, geom=np.array([grid_for(n, 256), 256]))

    # Gray: the reference's pattern with a white and a black pixel
    # (simt/parity_test.go:744-759), and a short rgb buffer.
    for tag, npx, rgb_len in [("pattern", 1 << 14, 3 << 14), ("short", 5003, 3 * 5003 - 4)]:
        i = np.arange(3 * npx, dtype=np.int64)
        rgb = ((i * 37 + i // 251) % 256).astype(np.uint8)
        rgb[0:3] = 255
        rgb[3:6] = 0
        rgb = rgb[:rgb_len].copy()
        out = np.full(npx, 0xAB, np.uint8)
        R.ref_Gray(O.u8p(out), npx, O.u8p(rgb), rgb_len, grid_for(npx, 256), 256)
        save(f"gray_{tag}", rgb=rgb, out0=np.full(npx, 0xAB, np.uint8), out=out,
             geom=np.array([grid_for(npx, 256), 256]))

    # Histogram: x = i*i % 311 - 8 over 2^15 (simt/shared_parity_cuda_test.go:84),
    # and a Zipf(1.2) draw into 200 bins with a partial grid.
    nh = 1 << 15
    ii = np.arange(nh, dtype=np.int64)
    xh = ((ii * ii) % 311 - 8).astype(np.int32)
    bins = np.zeros(256, np.int32)
    R.ref_Histogram(O.i32p(bins), 256, O.i32p(xh), nh, grid_for(nh, 256), 256)
    save("histogram_formula", x=xh, bins0=np.zeros(256, np.int32), bins=bins,
         geom=np.array([grid_for(nh, 256), 256]))
    p = (np.arange(256) + 1.0) ** -1.2
    cdf = np.cumsum(p / p.sum())
    u = np.random.default_rng(5).random(nh)
    xz = np.searchsorted(cdf, u).astype(np.int32)
    xz[:4] = [-1, 256, 1000, -(2 ** 31)]
    bins0 = np.arange(200, dtype=np.int32)
    bins = bins0.copy()
    R.ref_Histogram(O.i32p(bins), 200, O.i32p(xz), nh, 100, 128)
    save("histogram_zipf", x=xz, bins0=bins0, bins=bins, geom=np.array([100, 128]))

    # Transpose 133x71 (simt/parity_test.go:303) and a partially covered grid.
    for tag, w, h, gx, gy in [("full", 133, 71, 9, 5), ("partial", 133, 71, 5, 3)]:
        inp = normal(w * h, 10)
        out = np.full(w * h, -1.0, np.float32)
        R.ref_Transpose(O.f32p(out), w * h, O.f32p(inp), w * h, w, h, gx, gy)
        save(f"transpose_{tag}", inp=inp, out0=np.full(w * h, -1.0, np.float32), out=out,
             geom=np.array([w, h, gx, gy]))

    # WarpReduceSum: n = 37*128+53 with x = i%17-8 (simt/warp_parity_cuda_test.go:35),
    # and normal values, where the addition tree decides the bits.
    nw = 37 * 128 + 53
    gw = grid_for(nw, 128)
    for tag, x in [("formula", (np.arange(nw) % 17 - 8).astype(np.float32)),
                   ("normal", normal(nw, 11))]:
        out = np.zeros(gw * 4, np.float32)
        R.ref_WarpReduceSum(O.f32p(out), gw * 4, O.f32p(x), nw, gw)
        save(f"warpreduce_{tag}", x=x, out=out, geom=np.array([gw, 128]))

    # FIR: 2^15 samples, 33 taps of 1/33 (simt/parity_test.go:141); 31 random
    # taps over a ragged length; the largest tap count the tile holds; and a
    # grid covering fewer outputs than y_len.
    rng = np.random.default_rng(2)
    h31 = rng.uniform(-1, 1, 31).astype(np.float32)
    h31 = (h31 / h31.sum()).astype(np.float32)
    cases = [("box33", normal(1 << 15, 12), np.full(33, 1 / 33, np.float32), None),
             ("rand31", np.random.default_rng(1).uniform(-1, 1, 4099).astype(np.float32), h31,
              None),
             ("taps65", normal(3000, 13), normal(65, 14) / 8, None),
             ("partial", normal(5000, 15), h31, 9)]
    for tag, x, hh, grid in cases:
        n = len(x)
        grid = grid_for(n, 256) if grid is None else grid
        y = np.full(n, 5.0, np.float32)
        R.ref_FIR(O.f32p(y), n, O.f32p(x), n, O.f32p(hh), len(hh), grid)
        save(f"fir_{tag}", x=x, h=hh, y0=np.full(n, 5.0, np.float32), y=y,
             geom=np.array([grid, 256]))


if __name__ == "__main__":
    main()
