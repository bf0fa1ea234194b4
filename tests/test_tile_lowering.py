"""The tile track's lowering, checked on the CPU: the library's listing of
the fused program (Tensor.Source, tile/run.go:10) is executed here by a
small emulator of the device interpreter's accumulator machine -- one
accumulator, operands in inputs, temporaries and window tiles, per-position
values, windows staged with zeros outside the signal, fma accumulation in
tap order -- and must reproduce the oracle's node-by-node evaluation bit for
bit. This pins evaluation order, temporaries, operand reuse and the window
programs without a GPU."""
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
        pc, _, rest = line.partition(" ")
        for step in rest.split(" | "):   # the steps one device instruction fuses
            op, *args = step.split()
            progs[cur].append((op, args))
    span = n + halo

    def run(prog, tiles, taps_vals):
        acc = None
        temps = {}
        out = None

        def val(m):
            if m == "acc":
                return acc
            k = int(m[1:] if m[0] in "tw" else m[2:])
            return {"i": inputs, "t": temps, "w": tiles}[m[0]][k].astype(f32)

        for op, a in prog:
            if op == "lda":
                acc = val(a[0]).copy()
            elif op == "sta":
                temps[int(a[0][1:])] = acc.copy()
            elif op == "scale":
                acc = (f32(float.fromhex(a[0])) * acc).astype(f32)
            elif op == "sqrt":
                acc = np.sqrt(acc.astype(np.float64)).astype(f32)
            elif op == "abs":
                acc = np.abs(acc)
            elif op in ("add", "mul"):
                m = val(a[0])
                acc = (acc + m if op == "add" else acc * m).astype(f32)
            elif op == "hypot":
                m = val(a[0])
                acc = np.array([O.oracle().oracle_hypot(float(u), float(v))
                                for u, v in zip(acc, m)], f32)
            elif op == "firacc":
                w = int(a[0][1:])
                t = tiles[w]
                s = np.zeros(span, f32)
                for k in range(taps_of[w]):
                    shifted = np.zeros(span, f32)   # samples before the signal read 0
                    shifted[k:] = t[: span - k]
                    hk = float(taps_vals[w][k])
                    s = np.array([_fmaf(hk, float(x), float(y)) for x, y in zip(shifted, s)], f32)
                acc = s
            elif op in ("store", "stage"):
                out = acc.copy()
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
    """A graph with many simultaneously live values needs several
    temporaries at once; the listing still computes the oracle's values."""
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


def _random_graph(seed, n, halo, chained=False):
    """A random DAG over the track's seven operations with shared values,
    x-op-x nodes and up to two windows (none inside another; with chained,
    up to three, windows of windows allowed): the tile graph and the
    oracle's node table, in the same creation order."""
    rng = np.random.default_rng(seed)
    g = tile.New()
    if chained:
        g.AllowChainedWindows()
    nodes, ts, has_fir, values = [], [], [], []

    def add(t, nd, fir):
        assert t.node == len(nodes)
        values.append(len(nodes))
        nodes.append(nd)
        ts.append(t)
        has_fir.append(fir)

    for _ in range(int(rng.integers(1, 4))):
        d = rng.uniform(-4, 4, n + halo).astype(f32)
        add(g.Input(d[halo:]), {"kind": "input", "data": d}, False)
    windows = 0
    for _ in range(int(rng.integers(4, 14))):
        pick = lambda: values[int(rng.integers(0, len(values)))]  # noqa: E731
        kind = rng.choice(["scale", "abs", "sqrtabs", "add", "mul", "hypot", "fir"])
        i = pick()
        if kind == "fir":
            if windows == (3 if chained else 2) or (has_fir[i] and not chained):
                kind = "abs"
            else:
                windows += 1
                h = (rng.uniform(-1, 1, int(rng.integers(1, 12))) / 4).astype(f32)
                add_taps = len(nodes)
                t = tile.FIR(ts[i], h)
                nodes.append({"kind": "input", "data": h})
                ts.append(None)
                has_fir.append(False)
                assert t.node == add_taps + 1
                add(t, {"kind": "fir", "a": i, "taps": h}, True)
                continue
        if kind == "scale":
            k = float(rng.choice([0.5, -1.25, 3.0, -0.1]))
            add(tile.Scale(ts[i], k), {"kind": "scale", "a": i, "scale": k}, has_fir[i])
        elif kind == "abs":
            add(tile.Abs(ts[i]), {"kind": "abs", "a": i}, has_fir[i])
        elif kind == "sqrtabs":
            add(tile.Abs(ts[i]), {"kind": "abs", "a": i}, has_fir[i])
            j = len(ts) - 1
            add(tile.Sqrt(ts[j]), {"kind": "sqrt", "a": j}, has_fir[i])
        else:
            j = i if rng.random() < 0.2 else pick()
            op = {"add": tile.Add, "mul": tile.Mul, "hypot": tile.Hypot}[kind]
            add(op(ts[i], ts[j]), {"kind": kind, "a": i, "b": j}, has_fir[i] or has_fir[j])
    return ts[values[-1]], nodes


def _chained_graph(seed, n, halo):
    """Two or three windows each reading the one before (chains), sometimes
    a second window over the same inner one (a diamond), mixed with inputs:
    the tile graph (chained windows allowed) and the oracle's node table."""
    rng = np.random.default_rng(seed)
    g = tile.New().AllowChainedWindows()
    nodes = []

    def rec(t, nd):
        assert t.node == len(nodes), (t.node, len(nodes))
        nodes.append(nd)
        return t

    def fir(t, h):
        nodes.append({"kind": "input", "data": h})   # the taps node
        return rec(tile.FIR(t, h), {"kind": "fir", "a": t.node, "taps": h})

    def binop(name, x, y):
        op = {"add": tile.Add, "mul": tile.Mul, "hypot": tile.Hypot}[name]
        return rec(op(x, y), {"kind": name, "a": x.node, "b": y.node})

    ins = []
    for _ in range(2):
        d = rng.uniform(-4, 4, n + halo).astype(f32)
        ins.append(rec(g.Input(d[halo:]), {"kind": "input", "data": d}))
    a, b = ins
    cur = binop(str(rng.choice(["add", "mul"])), a, b)
    wins = []
    for _ in range(int(rng.integers(2, 4))):
        h = (rng.uniform(-1, 1, int(rng.integers(1, 20))) / 4).astype(f32)
        w = fir(cur, h)
        wins.append(w)
        pick = int(rng.integers(0, 3))
        if pick == 0:
            cur = w
        elif pick == 1:
            cur = binop("add", w, a)
        else:
            cur = rec(tile.Abs(w), {"kind": "abs", "a": w.node})
            cur = binop("mul", cur, b)
    root = cur
    if rng.random() < 0.5:   # a diamond: another window over the first one
        h = (rng.uniform(-1, 1, int(rng.integers(1, 12))) / 4).astype(f32)
        root = binop("add", root, fir(wins[0], h))
    return root, nodes


@pytest.mark.parametrize("seed", range(16))
def test_chained_windows_listing_matches_oracle(seed):
    """Windows of windows (the opt-in): each window's program reads the
    windows inside it (firacc), and the emulated listing equals the oracle's
    node-by-node evaluation, halo included."""
    n, halo = 40, (12 if seed % 2 else 0)
    root, nodes = _chained_graph(seed, n, halo)
    assert root.g.Err() is None
    src = root.Source()
    assert any(b.startswith("window") and "firacc" in b
               for b in re.split(r"\n(?=window|main)", src)), src
    src = root.Source()
    node_of = [int(m) for m in re.findall(r"; in\d+ = node (\d+)", src)]
    taps = {}
    for m in re.finditer(r"window (\d+) taps \d+ node (\d+)", src):
        taps[int(m.group(1))] = nodes[int(m.group(2))]["taps"]
    got = run_listing(src, [nodes[i]["data"] for i in node_of], n, taps, halo)
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, halo)
    assert rc == 0
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_chained_window_opt_in_only():
    """The reference's rejection stays the default; the opt-in accepts."""
    x = np.ones(8, f32)
    g = tile.New()
    inner = tile.FIR(g.Input(x), np.ones(3, f32))
    tile.FIR(inner, np.ones(2, f32))
    assert "chaining windowed" in str(g.Err())
    g2 = tile.New().AllowChainedWindows()
    inner = tile.FIR(g2.Input(x), np.ones(3, f32))
    out = tile.FIR(tile.Add(inner, inner), np.ones(2, f32))
    assert g2.Err() is None
    assert "window 1 taps 2" in out.Source()


@pytest.mark.parametrize("seed", range(24))
def test_random_graph_listing_matches_oracle(seed):
    n, halo = 40, (8 if seed % 3 == 0 else 0)
    root, nodes = _random_graph(seed, n, halo)
    src = root.Source()
    node_of = [int(m) for m in re.findall(r"; in\d+ = node (\d+)", src)]
    taps = {}
    for m in re.finditer(r"window (\d+) taps \d+ node (\d+)", src):
        taps[int(m.group(1))] = nodes[int(m.group(2))]["taps"]
    got = run_listing(src, [nodes[i]["data"] for i in node_of], n, taps, halo)
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, halo)
    assert rc == 0
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_chain_of_eight_full_windows():
    """The deepest chain the kernel stages: eight 64-tap windows each reading
    the one before (heads of 68 to 544 samples), emulated against the
    oracle with a halo."""
    n, halo = 60, 16   # the emulator wants the span longer than the taps
    rng = np.random.default_rng(8)
    g = tile.New().AllowChainedWindows()
    d = rng.uniform(-1, 1, n + halo).astype(f32)
    cur = g.Input(d[halo:])
    nodes = [{"kind": "input", "data": d}]
    for _ in range(8):
        h = (rng.uniform(-1, 1, 64) / 16).astype(f32)
        nodes.append({"kind": "input", "data": h})
        a = cur.node
        cur = tile.FIR(cur, h)
        nodes.append({"kind": "fir", "a": a, "taps": h})
        assert cur.node == len(nodes) - 1
    assert g.Err() is None
    src = cur.Source()
    assert src.count("window ") == 8
    node_of = [int(m) for m in re.findall(r"; in\d+ = node (\d+)", src)]
    taps = {}
    for m in re.finditer(r"window (\d+) taps \d+ node (\d+)", src):
        taps[int(m.group(1))] = nodes[int(m.group(2))]["taps"]
    got = run_listing(src, [nodes[i]["data"] for i in node_of], n, taps, halo)
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, halo)
    assert rc == 0
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
