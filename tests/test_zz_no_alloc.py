"""simtgo_tile_run_stepwise_noalloc through the C ABI.

The allocation-free stepwise run exists for callers that cannot allocate
device memory (a real-time processing callback with a deadline, where
cudaMalloc may synchronise the device for an unbounded time; a framework
whose pool owns the device). It keeps the intermediate node values in the
library's fixed 16 MiB scratch array instead. Here it must give exactly what
the existing device-resident entry point (simtgo_tile_run) gives, on two
different graphs called one after the other (the second run inherits the
first one's scratch contents), and on the first graph again; and refuse
graphs whose intermediates do not fit, and host inputs.

This file is collected last so a failure here leaves every other test run.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
from simtgo_b200 import _lib, tile  # noqa: E402

pytestmark = pytest.mark.gpu
P = C.c_void_p


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def run_existing(L, g, root, n):
    out = torch.empty(n, device="cuda")
    _lib.check(L.simtgo_tile_run(g._h, root.node, P(out.data_ptr()), n, None))
    _lib.check(L.simtgo_stream_sync(None))
    return out.cpu().numpy()


def run_noalloc(L, g, root, n):
    out = torch.full((n,), float("nan"), device="cuda")
    _lib.check(L.simtgo_tile_run_stepwise_noalloc(g._h, root.node, P(out.data_ptr()), n, None))
    _lib.check(L.simtgo_stream_sync(None))
    return out.cpu().numpy()


def twelve(n, seed):
    rng = np.random.default_rng(seed)
    g = tile.New()
    a, b, c = (g.InputDevice(dev(rng.uniform(-4, 4, n))) for _ in range(3))
    s = tile.Scale(a, 0.5)
    ab = tile.Abs(b)
    out = tile.Mul(tile.Hypot(tile.Add(tile.Mul(s, tile.Sqrt(ab)), c),
                              tile.FIR(s, np.full(31, 1 / 31, np.float32))), ab)
    return g, out


def pipeline(n, seed):
    rng = np.random.default_rng(seed)
    g = tile.New()
    re, im = (g.InputDevice(dev(rng.standard_normal(n))) for _ in range(2))
    out = tile.Hypot(tile.FIR(tile.Scale(re, 0.5), np.full(17, 1 / 17, np.float32)), im)
    return g, out


def same(name, got, want):
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


def test_matches_existing_entry_on_consecutive_calls():
    L = _lib.load()
    n1, n2 = 100003, 70001
    g1, o1 = twelve(n1, 1)
    g2, o2 = pipeline(n2, 2)
    want1 = run_existing(L, g1, o1, n1)
    want2 = run_existing(L, g2, o2, n2)
    same("first call, 12-node graph", run_noalloc(L, g1, o1, n1), want1)
    same("second call, another graph", run_noalloc(L, g2, o2, n2), want2)
    same("third call, first graph again", run_noalloc(L, g1, o1, n1), want1)


def test_input_root_and_single_step_match_existing_entry():
    # A graph whose root is one of its device inputs has no step to run; the
    # output must still receive the input's values, as simtgo_tile_run gives.
    L = _lib.load()
    n = 50021
    rng = np.random.default_rng(4)
    g = tile.New()
    a = g.InputDevice(dev(rng.uniform(-4, 4, n)))
    same("input root", run_noalloc(L, g, a, n), run_existing(L, g, a, n))
    s = tile.Scale(a, -1.5)
    same("Scale of an input", run_noalloc(L, g, s, n), run_existing(L, g, s, n))
    same("input root again", run_noalloc(L, g, a, n), run_existing(L, g, a, n))


def test_refuses_what_does_not_fit():
    L = _lib.load()
    # 7 intermediate nodes of 1M floats each: 7M floats > the 4M-float scratch.
    g, out = twelve(1 << 20, 3)
    dst = torch.empty(1 << 20, device="cuda")
    rc = L.simtgo_tile_run_stepwise_noalloc(g._h, out.node, P(dst.data_ptr()), 1 << 20, None)
    assert rc == _lib.ESIZE
    assert "16 MiB" in L.simtgo_last_error().decode()
    # Host inputs would need an upload, i.e. an allocation.
    g = tile.New()
    out = tile.Scale(g.Input(np.ones(64, np.float32)), 2.0)
    dst = torch.empty(64, device="cuda")
    assert L.simtgo_tile_run_stepwise_noalloc(g._h, out.node, P(dst.data_ptr()), 64,
                                              None) == _lib.EARG
