"""GPU parity of the tile track (package tile): the fused interpreter against
the oracle's node-by-node evaluation, the stepwise path against the fused
one, and the reference's own pipeline test (tile/tile_test.go:53-99)."""
import math

import numpy as np
import pytest

import oracle_lib as O
from test_abi import twelve_node_graph
from tolerance import assert_agree, assert_close

torch = pytest.importorskip("torch")
from simtgo_b200 import tile  # noqa: E402
from simtgo_b200._lib import AliasError  # noqa: E402

pytestmark = pytest.mark.gpu


def normal(n, seed):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


class Recorder:
    """Builds the same graph in the library and as an oracle node table."""

    def __init__(self, device_inputs=False):
        self.g = tile.New()
        self.nodes = []
        self.dev = device_inputs
        self.keep = []

    def input(self, xs):
        xs = np.asarray(xs, np.float32)
        if self.dev:
            t = torch.from_numpy(xs).cuda()
            self.keep.append(t)
            r = self.g.InputDevice(t)
        else:
            r = self.g.Input(xs)
        self.nodes.append({"kind": "input", "data": xs})
        return r

    def _add(self, r, **nd):
        assert r.node == len(self.nodes), (r.node, len(self.nodes))
        self.nodes.append(nd)
        return r

    def scale(self, a, k):
        return self._add(tile.Scale(a, k), kind="scale", a=a.node, scale=k)

    def add(self, a, b):
        return self._add(tile.Add(a, b), kind="add", a=a.node, b=b.node)

    def mul(self, a, b):
        return self._add(tile.Mul(a, b), kind="mul", a=a.node, b=b.node)

    def hypot(self, a, b):
        return self._add(tile.Hypot(a, b), kind="hypot", a=a.node, b=b.node)

    def sqrt(self, a):
        return self._add(tile.Sqrt(a), kind="sqrt", a=a.node)

    def abs(self, a):
        return self._add(tile.Abs(a), kind="abs", a=a.node)

    def fir(self, a, h):
        h = np.asarray(h, np.float32)
        r = tile.FIR(a, h)
        self.nodes.append({"kind": "input", "data": h})   # the taps node
        return self._add(r, kind="fir", a=a.node, taps=h)

    def want(self, root, n, halo=0):
        rc, out = O.tile_eval(self.nodes, root.node, n, halo)
        assert rc == 0
        return out


def build_twelve(rec, n, seed=6):
    rng = np.random.default_rng(seed)
    a, b, c = (rec.input(rng.uniform(-4, 4, n).astype(np.float32)) for _ in range(3))
    h = np.full(31, 1 / 31, np.float32)
    s = rec.scale(a, 0.5)
    ab = rec.abs(b)
    q = rec.sqrt(ab)
    m = rec.mul(s, q)
    d = rec.add(m, c)
    f = rec.fir(s, h)
    y = rec.hypot(d, f)
    return rec.mul(y, ab)


@pytest.mark.parametrize("n", [1, 5, 255, 1024, 1025, 4099, 1 << 16, (1 << 20) + 3])
def test_twelve_node_graph(n):
    rec = Recorder()
    out = build_twelve(rec, n)
    assert rec.g.Err() is None
    got = out.Materialize()
    assert_agree("fused vs oracle", got, rec.want(out, n))
    step, launches = out.MaterializeStepwise()
    assert launches == 8  # scale, abs, sqrt, mul, add, fir, hypot, mul
    assert_agree("stepwise vs fused", step, got)


def test_reference_pipeline():
    """tile/tile_test.go:53-99: Hypot(FIR(Scale(re, 0.5), h), im), 2^14
    samples, 17 taps of 1/17; fused vs a float64 reference at 1e-5, stepwise
    vs fused at 1e-6, 3 launches."""
    n = 1 << 14
    re, im = normal(n, 1), normal(n, 2)
    h = np.full(17, 1 / 17, np.float32)
    g = tile.New()
    filtered = tile.FIR(tile.Scale(g.Input(re), 0.5), h)
    out = tile.Hypot(filtered, g.Input(im))
    got = out.Materialize()
    want = np.zeros(n, np.float32)
    for i in range(n):
        acc = np.float32(0)
        for k in range(17):
            if i - k >= 0:
                acc = np.float32(acc + np.float32(h[k] * np.float32(0.5)) * re[i - k])
        want[i] = np.float32(math.hypot(float(acc), float(im[i])))
    assert_close("fused vs reference", got, want, 1e-5)
    step, launches = out.MaterializeStepwise()
    assert launches == 3
    assert_close("stepwise vs fused", step, got, 1e-6)


@pytest.mark.parametrize("taps", [1, 2, 3, 4, 5, 31, 63, 64])
def test_fir_node_taps(taps):
    n = 5000
    rec = Recorder()
    x = rec.input(normal(n, 3))
    h = normal(taps, 4) / taps
    out = rec.fir(x, h)
    assert_agree("fir node", out.Materialize(), rec.want(out, n))


def test_two_windows_and_shared_nodes():
    n = 20011
    rec = Recorder()
    a, b = rec.input(normal(n, 5)), rec.input(normal(n, 6))
    s = rec.sqrt(rec.abs(a))
    f1 = rec.fir(s, normal(7, 7))
    f2 = rec.fir(rec.add(a, b), normal(40, 8))
    m = rec.mul(f1, f2)
    out = rec.hypot(rec.add(m, s), rec.mul(a, a))
    assert_agree("two windows", out.Materialize(), rec.want(out, n))


def test_device_resident_run_and_alias():
    n = (1 << 18) + 7
    rec = Recorder(device_inputs=True)
    out = build_twelve(rec, n, seed=11)
    dout = torch.empty(n, dtype=torch.float32, device="cuda")
    out.Run(dout)
    torch.cuda.synchronize()
    assert_agree("device run", dout.cpu().numpy(), rec.want(out, n))
    with pytest.raises(AliasError, match="overlaps input p"):
        out.Run(rec.keep[0])


@pytest.mark.parametrize("halo", [0, 30, 32, 40])
def test_shard_with_halo(halo):
    """A shard of the graph: inputs carry `halo` preceding elements; the FIR
    reads them instead of zeros. Equal to the matching slice of the whole."""
    n_total, start = 9000, 4000
    n = 3000
    rng = np.random.default_rng(12)
    full = [rng.uniform(-4, 4, n_total).astype(np.float32) for _ in range(3)]
    # whole-signal reference
    whole = Recorder()
    out_w = build_twelve_inputs(whole, full)
    ref = whole.want(out_w, n_total)
    # the shard
    shard = Recorder(device_inputs=True)
    lo = start - halo
    out_s = build_twelve_inputs(shard, [x[lo:start + n] for x in full], n_override=n + halo)
    # rebuild with shard length n and halo-offset device inputs
    g = tile.New()
    keep = [torch.from_numpy(x[lo:start + n].copy()).cuda() for x in full]
    ins = [g.InputDevice(t[halo:]) for t in keep]
    root = twelve_node_graph(g, *ins, np.full(31, 1 / 31, np.float32))
    dout = torch.empty(n, dtype=torch.float32, device="cuda")
    root.Run(dout, halo=halo)
    torch.cuda.synchronize()
    got = dout.cpu().numpy()
    if halo >= 30:
        assert_agree("shard == slice of whole", got, ref[start:start + n])
    # and the oracle's own shard evaluation agrees in every case
    rc, want = O.tile_eval(shard.nodes, out_s.node, n, halo)
    assert rc == 0
    assert_agree("shard vs oracle shard", got, want)
    del out_s


def build_twelve_inputs(rec, xs, n_override=None):
    a, b, c = (rec.input(x) for x in xs)
    h = np.full(31, 1 / 31, np.float32)
    s = rec.scale(a, 0.5)
    ab = rec.abs(b)
    q = rec.sqrt(ab)
    m = rec.mul(s, q)
    d = rec.add(m, c)
    f = rec.fir(s, h)
    y = rec.hypot(d, f)
    return rec.mul(y, ab)


def test_input_only_and_unaligned():
    n = 1001
    x = normal(n + 1, 13)
    rec = Recorder()
    a = rec.input(x[1:])
    assert_agree("identity", a.Materialize(), x[1:])
    t = torch.from_numpy(x).cuda()
    g = tile.New()
    root = tile.Hypot(g.InputDevice(t[1:]), g.InputDevice(t[1:]))
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    root.Run(out)
    torch.cuda.synchronize()
    want = np.array([O.oracle().oracle_hypot(float(v), float(v)) for v in x[1:]], np.float32)
    assert_agree("unaligned device inputs", out.cpu().numpy(), want)


def test_hypot_wide_range():
    """The fused kernel's four-wide Hypot over exponents across the whole
    float32 range and both signs -- the fast path's domain edge (2^-60,
    2^60), zeros, subnormals, overflow, infinities and NaN -- bit for bit
    against the oracle's gpu.Hypot (kernels/kernels.go:29)."""
    rng = np.random.default_rng(16)
    n = (1 << 20) + 13
    e1 = rng.integers(-150, 128, n).astype(np.float64)
    e2 = np.clip(e1 + rng.integers(-40, 40, n), -150, 127)
    sx, sy = rng.choice([-1.0, 1.0], n), rng.choice([-1.0, 1.0], n)
    with np.errstate(over="ignore"):
        x = (sx * rng.uniform(1, 2, n) * np.exp2(e1)).astype(np.float32)
        y = (sy * rng.uniform(1, 2, n) * np.exp2(e2)).astype(np.float32)
    x[:14] = [3, 0, -5, 1e-45, 3.4e38, 2.0 ** -60, np.inf, np.nan, -0.0, 2.0 ** 60, 1.0, -np.inf,
              2.0 ** -61, 1e-40]
    y[:14] = [4, 0, 12, 1e-45, 3.4e38, 2.0 ** 60, np.nan, 1.0, 7.0, 2.0 ** -61, 0.0, np.nan,
              2.0 ** -61, 2.0 ** -59]
    rc, want = O.magnitude(x, y, (n + 255) // 256, 256)
    assert rc == 0
    g = tile.New()
    tx, ty = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tile.Hypot(g.InputDevice(tx), g.InputDevice(ty)).Run(out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert_agree("tile Hypot, wide range", got, want)
    assert got[0] == 5 and got[2] == 13 and got[10] == 1


def test_sqrt_every_float32():
    """The fused kernel's Sqrt over all 2^32 float32 bit patterns, in sixteen
    runs of 2^28, bit for bit against the correctly rounded float32 square
    root (gpu.Sqrt is float32(math.Sqrt(float64(x))), gpu/math.go:11-17, and
    that double rounding is exact for square roots); NaN agrees with NaN."""
    run = 1 << 28
    x = torch.empty(run, dtype=torch.float32, device="cuda")
    out = torch.empty(run, dtype=torch.float32, device="cuda")
    g = tile.New()
    root = tile.Sqrt(g.InputDevice(x))
    for r in range(16):
        bits = np.arange(r * run, (r + 1) * run, dtype=np.uint64).astype(np.uint32)
        xs = bits.view(np.float32)
        x.copy_(torch.from_numpy(xs))
        root.Run(out)
        got = out.cpu().numpy()
        with np.errstate(invalid="ignore"):
            want = np.sqrt(xs)
        bad = (got.view(np.uint32) != want.view(np.uint32)) & ~(np.isnan(got) & np.isnan(want))
        assert not bad.any(), (
            f"sqrt({xs[bad][0]!r} = {bits[bad][0]:#010x}): got {got[bad][0]!r}, want "
            f"{want[bad][0]!r}; {int(bad.sum())} of {run} in run {r} differ")


@pytest.mark.parametrize("seed", range(16))
def test_random_graphs(seed):
    """Random DAGs over the seven operations (shared values, x-op-x nodes,
    up to two windows) on the device, bit for bit against the oracle: 3001
    elements (one chunk per block) and 2^21+77 (several chunks per block, so
    the window heads are carried between chunks)."""
    from test_tile_lowering import _random_graph

    for n in (3001, (1 << 21) + 77):
        root, nodes = _random_graph(seed, n, 0)
        got = root.Materialize()
        rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
        assert rc == 0
        assert_agree(f"random graph {seed} n={n}", got, want)


@pytest.mark.parametrize("seed", [3, 7, 11, 19])
def test_random_graphs_unaligned_device_inputs(seed):
    """The same random DAGs with device inputs that start 4 bytes past a
    16-byte boundary and an output that does too: the interpreter reads the
    inputs from HBM itself (no bulk copies), several chunks per block."""
    from test_tile_lowering import _random_graph

    n = (1 << 21) + 77
    root, nodes = _random_graph(seed, n, 0)
    g = tile.New()
    keep, ids = [], {}
    for i, nd in enumerate(nodes):   # rebuild with device inputs, same node ids
        if nd["kind"] == "input" and not any(m.get("taps") is nd["data"] for m in nodes):
            buf = torch.empty(len(nd["data"]) + 1, device="cuda")
            buf[1:].copy_(torch.from_numpy(nd["data"]))
            keep.append(buf)
            ids[i] = g.InputDevice(buf[1:])
        elif nd["kind"] == "input":
            ids[i] = None  # a FIR's taps: created by tile.FIR below
        elif nd["kind"] == "fir":
            ids[i] = tile.FIR(ids[nd["a"]], nd["taps"])
        elif nd["kind"] == "scale":
            ids[i] = tile.Scale(ids[nd["a"]], nd["scale"])
        elif nd["kind"] in ("abs", "sqrt"):
            ids[i] = {"abs": tile.Abs, "sqrt": tile.Sqrt}[nd["kind"]](ids[nd["a"]])
        else:
            op = {"add": tile.Add, "mul": tile.Mul, "hypot": tile.Hypot}[nd["kind"]]
            ids[i] = op(ids[nd["a"]], ids[nd["b"]])
        assert ids[i] is None or ids[i].node == i
    last = ids[len(nodes) - 1]
    out_buf = torch.empty(n + 1, device="cuda")
    last.Run(out_buf[1:])
    torch.cuda.synchronize()
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
    assert rc == 0
    assert_agree(f"unaligned random graph {seed}", out_buf[1:].cpu().numpy(), want)


@pytest.mark.parametrize("seed", range(8))
def test_chained_windows(seed):
    """Windows of windows (the library's opt-in; the reference rejects
    them): fused on the device, bit for bit against the oracle's
    node-by-node evaluation, over one and several chunks per block (heads
    carried through every window of the chain), and equal to the stepwise
    path, which materialises each window before the next reads it."""
    from test_tile_lowering import _chained_graph

    for n in (3001, (1 << 21) + 77):
        root, nodes = _chained_graph(seed, n, 0)
        got = root.Materialize()
        rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
        assert rc == 0
        assert_agree(f"chained graph {seed} n={n}", got, want)
        if n == 3001:
            step, _ = root.MaterializeStepwise()
            assert_agree(f"chained graph {seed} stepwise", step, got)


@pytest.mark.parametrize("halo", [0, 40, 44])
def test_chained_windows_shard_halo(halo):
    """A shard of FIR(Add(FIR(a, h1), a), h2) with taps 17 and 21: with a
    halo of at least 16 + 20 samples its outputs equal the whole signal's
    from the shard's first element on; with none, the first shard's."""
    n_all, start = (1 << 20) + 500, 70000
    x = normal(n_all, 21)
    h1 = (np.arange(17, dtype=np.float32) / 60).astype(np.float32)
    h2 = (np.cos(np.arange(21, dtype=np.float32)) / 9).astype(np.float32)
    nodes = [{"kind": "input", "data": x}, {"kind": "input", "data": h1},
             {"kind": "fir", "a": 0, "taps": h1}, {"kind": "add", "a": 2, "b": 0},
             {"kind": "input", "data": h2}, {"kind": "fir", "a": 3, "taps": h2}]
    rc, whole = O.tile_eval(nodes, 5, n_all, 0)
    assert rc == 0
    s0 = start if halo else 0
    n = n_all - s0
    buf = torch.from_numpy(x[s0 - halo:].copy()).cuda()
    g = tile.New().AllowChainedWindows()
    a = g.InputDevice(buf[halo:])
    out = tile.FIR(tile.Add(tile.FIR(a, h1), a), h2)
    y = torch.empty(n, device="cuda")
    out.Run(y, halo=halo)
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32),
                                  whole[s0:].view(np.uint32))


def test_chained_windows_reduce():
    from test_tile_lowering import _chained_graph

    n = (1 << 20) + 3
    root, nodes = _chained_graph(5, n, 0)
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
    assert rc == 0
    got = tile.Sum(root).Materialize()
    assert np.float32(got).view(np.uint32) == O.tile_reduce(want, "sum")[0].view(np.uint32)
