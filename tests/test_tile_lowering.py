"""The tile track's lowering, checked on the CPU: the library's listing of
the fused program (Tensor.Source, tile/run.go:10) is executed here by a
small emulator of the device interpreter's instruction set -- 8 register
slots, per-position values, windows staged with zeros outside the signal,
fma accumulation in tap order -- and must reproduce the oracle's node-by-node
evaluation bit for bit. This pins register allocation, hoisted loads,
in-place reuse and the window programs without a GPU."""
import ctypes
import re

import numpy as np
import pytest

import oracle_lib as O
from simtgo_b200 import tile

f32 = np.float32
_libm = ctypes.CDLL("libm.so.6")
_libm.fmaf.restype = ctypes.c_float
_libm.fmaf.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]


def _fmaf(a, b, c):
    return _libm.fmaf(a, b, c)


def emulate(listing, inputs, n, halo=0):
    """inputs[k]: the data of in<k> over positions [-halo, n)."""
    progs, cur = {}, None
    taps_of = {}
    for line in listing.splitlines():
        if not line or line.startswith(";"):
            continue
        m = re.match(r"window (\d+) taps (\d+) node (\d+)", line)
        if m:
            cur = ("w", int(m.group(1)))
            taps_of[int(m.group(1))] = int(m.group(2))
            progs[cur] = []
            continue
        if line == "main":
            cur = ("main",)
            progs[cur] = []
            continue
        pc, op, *args = line.split()
        progs[cur].append((op, args))
    span = n + halo

    def run(prog, tiles, taps_vals):
        r = [None] * 8
        out = None
        for op, a in prog:
            idx = lambda s: int(s.lstrip("rinw"))  # noqa: E731
            if op == "load":
                r[idx(a[0])] = inputs[idx(a[1])].astype(f32).copy()
            elif op == "scale":
                r[idx(a[0])] = (f32(float.fromhex(a[1])) * r[idx(a[0])]).astype(f32)
            elif op == "sqrt":
                r[idx(a[0])] = np.sqrt(r[idx(a[0])].astype(np.float64)).astype(f32)
            elif op == "abs":
                r[idx(a[0])] = np.abs(r[idx(a[0])])
            elif op == "mov":
                r[idx(a[0])] = r[idx(a[1])].copy()
            elif op in ("add", "mul"):
                d, s = idx(a[0]), idx(a[1])
                r[d] = (r[d] + r[s] if op == "add" else r[d] * r[s]).astype(f32)
            elif op == "hypot":
                d, s = idx(a[0]), idx(a[1])
                r[d] = np.array([O.oracle().oracle_hypot(float(u), float(v))
                                 for u, v in zip(r[d], r[s])], f32)
            elif op == "firacc":
                d, w = idx(a[0]), idx(a[1])
                t = tiles[w]
                acc = np.zeros(span, f32)
                for k in range(taps_of[w]):
                    shifted = np.zeros(span, f32)   # samples before the signal read 0
                    shifted[k:] = t[: span - k]
                    hk = float(taps_vals[w][k])
                    acc = np.array([_fmaf(hk, float(x), float(y)) for x, y in zip(shifted, acc)],
                                   f32)
                r[d] = acc
            elif op == "store":
                out = r[idx(a[0])]
            elif op == "stage":
                v = r[idx(a[0])].copy()
                out = v
            elif op == "end":
                break
        return out

    return progs, run


def run_listing(listing, inputs, n, taps_vals, halo=0):
    progs, run = emulate(listing, inputs, n, halo)
    tiles = {}
    for key in sorted(k for k in progs if k[0] == "w"):
        tiles[key[1]] = run(progs[key], tiles, taps_vals)   # signal over [-halo, n)
    out = run(progs[("main",)], tiles, taps_vals)
    return out[halo:]


def twelve(g, a, b, c, h):
    s = tile.Scale(a, 0.5)
    ab = tile.Abs(b)
    q = tile.Sqrt(ab)
    m = tile.Mul(s, q)
    d = tile.Add(m, c)
    f = tile.FIR(s, h)
    y = tile.Hypot(d, f)
    return tile.Mul(y, ab)


def oracle_twelve(a, b, c, h, n, halo):
    nodes = [{"kind": "input", "data": a}, {"kind": "input", "data": b},
             {"kind": "input", "data": c}, {"kind": "scale", "a": 0, "scale": 0.5},
             {"kind": "abs", "a": 1}, {"kind": "sqrt", "a": 4}, {"kind": "mul", "a": 3, "b": 5},
             {"kind": "add", "a": 6, "b": 2}, {"kind": "input", "data": h},
             {"kind": "fir", "a": 3, "taps": h}, {"kind": "hypot", "a": 7, "b": 9},
             {"kind": "mul", "a": 10, "b": 4}]
    rc, out = O.tile_eval(nodes, 11, n, halo)
    assert rc == 0
    return out


@pytest.mark.parametrize("halo", [0, 8])
def test_twelve_node_listing_matches_oracle(halo):
    n = 300
    rng = np.random.default_rng(1)
    a, b, c = (rng.uniform(-4, 4, n + halo).astype(f32) for _ in range(3))
    h = (rng.uniform(-1, 1, 9) / 5).astype(f32)
    g = tile.New()
    root = twelve(g, *(g.Input(v[halo:]) for v in (a, b, c)), h)
    src = root.Source()
    assert src.count("window ") == 1 and "main" in src
    # in<k> -> node id, in listing order
    node_of = [int(m) for m in re.findall(r"; in\d+ = node (\d+)", src)]
    data = {0: a, 1: b, 2: c}
    got = run_listing(src, [data[i] for i in node_of], n, {0: h}, halo)
    want = oracle_twelve(a, b, c, h, n, halo)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_register_reuse_under_pressure():
    """A graph with many simultaneously live values forces unhoisted loads
    and in-place reuse; the listing still computes the oracle's values."""
    n = 64
    rng = np.random.default_rng(2)
    xs = [rng.uniform(0.5, 2, n).astype(f32) for _ in range(12)]
    g = tile.New()
    ts = [g.Input(x) for x in xs]
    # ((x0*x1)+(x2*x3)) ... pairwise, then each pair product reused twice
    prods = [tile.Mul(ts[i], ts[i + 1]) for i in range(0, 12, 2)]
    sums = [tile.Add(prods[i], prods[(i + 1) % 6]) for i in range(6)]
    acc = sums[0]
    for s in sums[1:]:
        acc = tile.Hypot(acc, s)
    src = acc.Source()
    node_of = [int(m) for m in re.findall(r"; in\d+ = node (\d+)", src)]
    got = run_listing(src, [xs[i] for i in node_of], n, {})
    # oracle node table in creation order
    nodes = [{"kind": "input", "data": x} for x in xs]
    pid = list(range(12, 18))
    for i in range(0, 12, 2):
        nodes.append({"kind": "mul", "a": i, "b": i + 1})
    for i in range(6):
        nodes.append({"kind": "add", "a": pid[i], "b": pid[(i + 1) % 6]})
    prev = 18
    for j in range(19, 24):
        nodes.append({"kind": "hypot", "a": prev, "b": j})
        prev = len(nodes) - 1
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
    assert rc == 0 and acc.node == len(nodes) - 1
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_source_of_an_error_graph_raises():
    g = tile.New()
    out = tile.Add(g.Input(np.zeros(3)), g.Input(np.zeros(4)))
    with pytest.raises(Exception, match="does not match"):
        out.Source()
