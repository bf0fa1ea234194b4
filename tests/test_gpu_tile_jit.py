"""GPU parity of the tile track's specialised kernels (each program compiled
in as constants, tile_jit.cu) against the interpreter they replace and the
oracle, bit for bit: random graphs in every layout the launcher picks (bulk
and direct inputs, two and four groups per thread), windows carried across
chunks, shards with a halo, chained windows and the four reductions. The
other tile tests run in the default mode, which is the specialised path;
here each case runs in both modes."""
import numpy as np
import pytest

import oracle_lib as O
from tolerance import assert_agree

torch = pytest.importorskip("torch")
from simtgo_b200 import tile  # noqa: E402

pytestmark = pytest.mark.gpu

KINDS = {"sum": tile.Sum, "min": tile.Min, "max": tile.Max, "argmax": tile.ArgMax}


@pytest.fixture(autouse=True)
def restore_mode():
    mode = tile.JITInfo()[0]
    yield
    tile.SetJIT(mode)


def both(fn):
    """fn() with the interpreter (mode 0) and with the specialised kernel
    required (mode 2); checks that the second ran specialised launches."""
    tile.SetJIT(0)
    a = fn()
    tile.SetJIT(2)
    before = tile.JITInfo()[3]
    b = fn()
    assert tile.JITInfo()[3] > before, "no specialised kernel was launched"
    return a, b


def bits(x):
    return np.asarray(x, np.float32).view(np.uint32)


def test_nvrtc_is_there():
    mode, available, _, _, _ = tile.JITInfo()
    assert available, "libnvrtc could not be opened: tile programs would run interpreted"


@pytest.mark.parametrize("seed", range(8))
def test_random_graphs_both_modes(seed):
    from test_tile_lowering import _random_graph

    for n in (3001, (1 << 21) + 77):
        root, nodes = _random_graph(seed, n, 0)
        interp, spec = both(root.Materialize)
        assert np.array_equal(bits(interp), bits(spec)), f"seed {seed} n={n}"
        rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
        assert rc == 0
        assert_agree(f"specialised random graph {seed} n={n}", spec, want)


@pytest.mark.parametrize("seed", [3, 11])
def test_unaligned_device_inputs_both_modes(seed):
    """Inputs and output 4 bytes past a 16-byte boundary: the direct form
    (inputs read from HBM by the kernel itself)."""
    from test_tile_lowering import _random_graph

    n = (1 << 20) + 5
    root, nodes = _random_graph(seed, n, 0)
    g = tile.New()
    keep, ids = [], {}
    for i, nd in enumerate(nodes):
        if nd["kind"] == "input" and not any(m.get("taps") is nd["data"] for m in nodes):
            buf = torch.empty(len(nd["data"]) + 1, device="cuda")
            buf[1:].copy_(torch.from_numpy(nd["data"]))
            keep.append(buf)
            ids[i] = g.InputDevice(buf[1:])
        elif nd["kind"] == "input":
            ids[i] = None
        elif nd["kind"] == "fir":
            ids[i] = tile.FIR(ids[nd["a"]], nd["taps"])
        elif nd["kind"] == "scale":
            ids[i] = tile.Scale(ids[nd["a"]], nd["scale"])
        elif nd["kind"] in ("abs", "sqrt"):
            ids[i] = {"abs": tile.Abs, "sqrt": tile.Sqrt}[nd["kind"]](ids[nd["a"]])
        else:
            op = {"add": tile.Add, "mul": tile.Mul, "hypot": tile.Hypot}[nd["kind"]]
            ids[i] = op(ids[nd["a"]], ids[nd["b"]])
    last = ids[len(nodes) - 1]

    def run():
        out = torch.empty(n + 1, device="cuda")
        last.Run(out[1:])
        torch.cuda.synchronize()
        return out[1:].cpu().numpy()

    interp, spec = both(run)
    assert np.array_equal(bits(interp), bits(spec))
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
    assert rc == 0
    assert_agree(f"specialised unaligned graph {seed}", spec, want)


@pytest.mark.parametrize("halo", [0, 32, 40])
def test_shard_halo_both_modes(halo):
    """The twelve-node graph on a shard whose device inputs carry `halo`
    preceding samples (bulk copies for halo % 4 == 0, several chunks per
    block): the same slice of the whole signal in both modes."""
    from test_abi import twelve_node_graph

    n_total, start, n = 3 << 20, 1 << 20, (1 << 20) + 3
    rng = np.random.default_rng(12)
    full = [rng.uniform(-4, 4, n_total).astype(np.float32) for _ in range(3)]
    g = tile.New()
    keep = [torch.from_numpy(x[start - halo:start + n].copy()).cuda() for x in full]
    root = twelve_node_graph(g, *[g.InputDevice(t[halo:]) for t in keep],
                             np.full(31, 1 / 31, np.float32))

    def run():
        out = torch.empty(n, device="cuda")
        root.Run(out, halo=halo)
        torch.cuda.synchronize()
        return out.cpu().numpy()

    interp, spec = both(run)
    assert np.array_equal(bits(interp), bits(spec))


@pytest.mark.parametrize("seed", [0, 4])
def test_chained_windows_both_modes(seed):
    from test_tile_lowering import _chained_graph

    n = (1 << 20) + 333
    root, nodes = _chained_graph(seed, n, 0)
    interp, spec = both(root.Materialize)
    assert np.array_equal(bits(interp), bits(spec))
    rc, want = O.tile_eval(nodes, len(nodes) - 1, n, 0)
    assert rc == 0
    assert_agree(f"specialised chained windows {seed}", spec, want)


@pytest.mark.parametrize("kind", list(KINDS))
def test_reductions_both_modes(kind):
    from test_tile_lowering import _random_graph

    n = 3 * 4096 + 1001
    root, nodes = _random_graph(2, n, 0)
    def run():
        r = KINDS[kind](root).Materialize()
        return r if isinstance(r, tuple) else (None, r)   # (index, value)

    interp, spec = both(run)
    assert interp[0] == spec[0] and bits(interp[1]) == bits(spec[1]), (kind, interp, spec)


def test_kernel_from_disk_cache_runs(tmp_path):
    """A second process loads the first one's compiled kernel from the
    on-disk cache (no compilation) and computes the same bits."""
    import os
    import subprocess
    import sys

    prog = (
        "import sys, numpy as np\n"
        "from simtgo_b200 import tile\n"
        "tile.SetJIT(2)\n"
        "rng = np.random.default_rng(3)\n"
        "g = tile.New()\n"
        "a, b = (g.Input(rng.uniform(-4, 4, 100003).astype(np.float32)) for _ in range(2))\n"
        "t = tile.Hypot(tile.FIR(tile.Scale(a, 0.5), np.full(9, 1 / 9, np.float32)), b)\n"
        "out = t.Materialize()\n"
        "np.save(sys.argv[1], out)\n"
        "print(tile.JITInfo()[2], tile.JITInfo()[4])\n")
    env = dict(os.environ, SIMTGO_B200_CACHE=str(tmp_path / "cache"))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

    def run(name):
        out = subprocess.run([sys.executable, "-c", prog, str(tmp_path / name)], env=env,
                             cwd=root, check=True, capture_output=True, text=True).stdout.split()
        return int(out[0]), int(out[1]), np.load(tmp_path / (name + ".npy"))

    c1, h1, y1 = run("first")
    c2, h2, y2 = run("second")
    assert (c1, h1) == (1, 0) and (c2, h2) == (0, 1)
    assert np.array_equal(bits(y1), bits(y2))


@pytest.mark.parametrize("kind", list(KINDS))
def test_streaming_chains_both_modes(kind):
    """Reductions of a chain of steps on one aligned device input (the
    streaming path), with a NaN, a -0 and an infinity among the values: the
    chain compiled in as constants against the run-time chain, bit for bit
    (value and index). The oracle's tree pins the run-time chain in
    test_gpu_tile_reduce.py."""
    n = (1 << 21) + 1234
    rng = np.random.default_rng(7)
    xs = rng.uniform(-4, 4, n).astype(np.float32)
    xs[[5, 77777, n - 3]] = [np.nan, -0.0, np.inf]
    g = tile.New()
    keep = torch.from_numpy(xs).cuda()
    a = g.InputDevice(keep)
    chains = {
        "abs_scale": tile.Abs(tile.Scale(a, -2.0)),
        "sqrt_abs": tile.Sqrt(tile.Abs(a)),
        "mul_add": tile.Mul(tile.Add(a, a), tile.Add(a, a)),
        "scale_abs_scale": tile.Scale(tile.Abs(tile.Scale(a, 0.75)), -3.0),
    }
    for name, t in chains.items():
        def run():
            v = torch.empty(1, device="cuda")
            i = torch.empty(1, dtype=torch.int64, device="cuda")
            KINDS[kind](t).Run(v, i)
            torch.cuda.synchronize()
            return (int(i.item()) if kind == "argmax" else None), v.cpu().numpy()[0]

        interp, spec = both(run)
        assert interp[0] == spec[0] and bits(interp[1]) == bits(spec[1]), (kind, name)


def test_shutdown_unloads_and_relaunch_reloads():
    """simtgo_shutdown unloads the specialised kernels' modules; the next
    launch of the same graph loads its kernel again (from the on-disk cache,
    not a compilation) and computes the same bits."""
    from simtgo_b200 import _lib

    rng = np.random.default_rng(21)
    g = tile.New()
    a, b = (g.Input(rng.uniform(-4, 4, 70001).astype(np.float32)) for _ in range(2))
    t = tile.Add(tile.Hypot(a, b), tile.FIR(tile.Abs(a), np.full(13, 1 / 13, np.float32)))
    tile.SetJIT(2)
    y1 = t.Materialize()
    _, _, compiled, _, hits = tile.JITInfo()
    _lib.check(_lib.load().simtgo_shutdown())
    y2 = t.Materialize()
    _, _, compiled2, _, hits2 = tile.JITInfo()
    assert compiled2 == compiled and hits2 == hits + 1
    assert np.array_equal(bits(y1), bits(y2))


def test_without_nvrtc_falls_back_or_fails(tmp_path):
    """With libnvrtc unavailable, mode 1 runs the graph on the interpreter
    (no specialised launch, the same bits) and mode 2 refuses with an
    error; nothing crashes."""
    import os
    import subprocess
    import sys

    prog = (
        "import sys, numpy as np\n"
        "from simtgo_b200 import tile\n"
        "from simtgo_b200._lib import SimtgoError\n"
        "rng = np.random.default_rng(5)\n"
        "g = tile.New()\n"
        "a, b = (g.Input(rng.uniform(-4, 4, 50001).astype(np.float32)) for _ in range(2))\n"
        "t = tile.Mul(tile.FIR(a, np.full(7, 1 / 7, np.float32)), tile.Sqrt(tile.Abs(b)))\n"
        "np.save(sys.argv[1], t.Materialize())\n"
        "launches = tile.JITInfo()[3]\n"
        "tile.SetJIT(2)\n"
        "try:\n"
        "    t.Materialize()\n"
        "    refused = False\n"
        "except SimtgoError:\n"
        "    refused = True\n"
        "print(launches, refused)\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    base = dict(os.environ, SIMTGO_B200_CACHE="off")
    bad = dict(base, SIMTGO_NVRTC_LIB=str(tmp_path / "no_such_libnvrtc.so"))
    out = subprocess.run([sys.executable, "-c", prog, str(tmp_path / "interp")], env=bad,
                         cwd=root, check=True, capture_output=True, text=True).stdout.split()
    assert out == ["0", "True"]
    out = subprocess.run([sys.executable, "-c", prog, str(tmp_path / "spec")], env=base,
                         cwd=root, check=True, capture_output=True, text=True).stdout.split()
    assert out[0] != "0" and out[1] == "False"
    assert np.array_equal(bits(np.load(tmp_path / "interp.npy")),
                          bits(np.load(tmp_path / "spec.npy")))


def test_long_program_runs_on_the_interpreter():
    """A program of more than 32 device instructions runs on the
    interpreter in every mode (its compile would outgrow its run): no
    specialised launch, and the interpreter's bits."""
    rng = np.random.default_rng(9)
    g = tile.New()
    a, b = (g.Input(rng.uniform(-1, 1, 30001).astype(np.float32)) for _ in range(2))
    t = a
    for i in range(30):
        t = tile.Add(tile.Mul(t, b), a) if i % 2 else tile.Scale(t, 0.5)
    assert t.ProgramSize()[0] > 32
    tile.SetJIT(0)
    y0 = t.Materialize()
    tile.SetJIT(2)
    before = tile.JITInfo()[3]
    y2 = t.Materialize()
    assert tile.JITInfo()[3] == before
    assert np.array_equal(bits(y0), bits(y2))
