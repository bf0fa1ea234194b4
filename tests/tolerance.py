"""The reference's comparison rules (internal/tolerance/tolerance.go), restated.

close(): |got - want| <= tol * max(|want|, 1)   (tolerance.go:51, Close64)
agree(): bit equality first; NaN agrees only with NaN; infinities and the two
         zeros are compared exactly; only finite pairs reach the bound
         (tolerance.go:102-150, Agree / agree64).
equal(): exact equality for integers, bytes and bools (tolerance.go:79).

The float kernels that reproduce gpu.RunCPU bit for bit are checked with
tol = 0 through agree(), so only a NaN payload may differ (CUDA's canonical
NaN is 0x7fffffff; Go's math.NaN() rounds to 0x7fc00000).
"""
from __future__ import annotations

import numpy as np


def agree_mask(got, want, tol: float):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    g32 = np.asarray(got, np.float32).view(np.uint32)
    w32 = np.asarray(want, np.float32).view(np.uint32)
    same = g32 == w32
    both_nan = np.isnan(got) & np.isnan(want)
    finite = np.isfinite(got) & np.isfinite(want)
    zeros = (got == 0) & (want == 0)
    with np.errstate(invalid="ignore", over="ignore"):
        bound = tol * np.maximum(np.abs(want), 1.0)
        within = finite & ~zeros & (np.abs(got - want) <= bound)
    return same | both_nan | within


def assert_agree(name, got, want, tol: float = 0.0):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{name}: shape {got.shape}, want {want.shape}"
    ok = agree_mask(got, want, tol)
    if not ok.all():
        i = int(np.flatnonzero(~ok)[0])
        raise AssertionError(
            f"{name} element {i}: got {got[i]!r} ({np.float32(got[i]).view(np.uint32):#010x}), "
            f"want {want[i]!r} ({np.float32(want[i]).view(np.uint32):#010x}), "
            f"{int((~ok).sum())} of {ok.size} differ (tol {tol})")


def assert_close(name, got, want, tol: float):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{name}: shape {got.shape}, want {want.shape}"
    d = np.abs(got - want)
    bound = tol * np.maximum(np.abs(want), 1.0)
    bad = ~(d <= bound)
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{name} element {i}: got {got[i]}, want {want[i]} "
                             f"(|delta| {d[i]:g}, bound {bound[i]:g}); {int(bad.sum())} differ")


def assert_equal(name, got, want):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{name}: shape {got.shape}, want {want.shape}"
    bad = got != want
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{name} element {i}: got {got[i]!r}, want {want[i]!r}; "
                             f"{int(bad.sum())} of {bad.size} differ")


def max_ulp(got, want):
    """Largest distance in float32 units in the last place over finite pairs."""
    g = np.asarray(got, np.float32)
    w = np.asarray(want, np.float32)
    m = np.isfinite(g) & np.isfinite(w)
    if not m.any():
        return 0

    def key(a):
        i = a.view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)

    return int(np.max(np.abs(key(g[m]) - key(w[m]))))
