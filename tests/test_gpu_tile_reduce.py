"""GPU parity of the tile reductions (Sum, Min, Max, ArgMax; no counterpart
in the reference): the fused reduction against the oracle's restatement of
the library's stated tree, over the values the same graph materialises on
the device, bit for bit (value bits and ArgMax index). Sizes cover the empty
tensor, one partial chunk, exact and ragged chunk ends and three levels of
the tree; inputs cover NaN, signed zeros, infinities and ties across
chunks; graphs cover random DAGs with windows, the twelve-node graph, the
sharded form with a halo (one rank) and the host-input form."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O
from test_gpu_tile import Recorder, build_twelve, normal

torch = pytest.importorskip("torch")
from simtgo_b200 import _lib, tile  # noqa: E402

pytestmark = pytest.mark.gpu

KINDS = {"sum": tile.SUM, "min": tile.MIN, "max": tile.MAX, "argmax": tile.ARGMAX}


def _bits(v):
    return int(np.array(v, np.float32).view(np.uint32))


def run_device(t, kind):
    v = torch.full((1,), 12345.0, device="cuda")
    i = torch.full((1,), -7, dtype=torch.int64, device="cuda")
    tile.Reduction(t, KINDS[kind]).Run(v, i)
    torch.cuda.synchronize()
    return np.float32(v.item()), int(i.item())


def check(name, got, want, kind):
    assert _bits(got[0]) == _bits(want[0]), f"{name} {kind}: got {got[0]!r}, want {want[0]!r}"
    if kind == "argmax":
        assert got[1] == want[1], f"{name} argmax index: got {got[1]}, want {want[1]}"


@pytest.mark.parametrize("kind", list(KINDS))
@pytest.mark.parametrize("n", [0, 1, 5, 2047, 2048, 2049, 3 * 2048 + 1000, (1 << 22) + 3,
                               2048 * 2048 * 2 + 17])
def test_sizes_device_inputs(kind, n):
    rec = Recorder(device_inputs=True)
    a = rec.input(normal(n, n + 1) * 3)
    b = rec.input(normal(n, n + 2))
    t = rec.add(rec.mul(a, a), b)
    vals = torch.empty(n, device="cuda")
    if n:
        t.Run(vals)
    want = O.tile_reduce(vals.cpu().numpy(), kind)
    check(f"n={n}", run_device(t, kind), want, kind)


@pytest.mark.parametrize("kind", list(KINDS))
def test_edge_values(kind):
    n = 3 * 2048 + 11
    rng = np.random.default_rng(5)
    cases = {
        "nan": lambda x: x.__setitem__([100, 5000], np.nan),
        "zeros": lambda x: x.fill(0.0) or x.__setitem__(slice(0, None, 3), -0.0),
        "neg_zero_only": lambda x: x.fill(-0.0),
        "inf": lambda x: x.__setitem__([7, 4000], [np.inf, -np.inf]),
        "ties": lambda x: x.__setitem__([2100, 4200, 6000], 99.0),
        "all_neg_inf": lambda x: x.fill(-np.inf),
    }
    for name, plant in cases.items():
        x = rng.standard_normal(n).astype(np.float32)
        plant(x)
        rec = Recorder(device_inputs=True)
        t = rec.input(x)          # the identity graph: the values are x itself
        check(name, run_device(t, kind), O.tile_reduce(x, kind), kind)


@pytest.mark.parametrize("kind", list(KINDS))
@pytest.mark.parametrize("seed", range(6))
def test_random_graphs(kind, seed):
    """Random DAGs with windows (host inputs, the Materialize form), over
    one and many chunks per block."""
    from test_tile_lowering import _random_graph

    for n in (3001, (1 << 21) + 77):
        root, nodes = _random_graph(seed, n, 0)
        vals = root.Materialize()
        got = tile.Reduction(root, KINDS[kind]).Materialize()
        got = (got[1], got[0]) if kind == "argmax" else (got, None)
        check(f"seed {seed} n={n}", got, O.tile_reduce(vals, kind), kind)


def test_twelve_node_graph_sum_and_argmax():
    n = (1 << 22) + 5
    rec = Recorder(device_inputs=True)
    out = build_twelve(rec, n)
    vals = torch.empty(n, device="cuda")
    out.Run(vals)
    v = vals.cpu().numpy()
    for kind in ("sum", "argmax"):
        check("twelve", run_device(out, kind), O.tile_reduce(v, kind), kind)


@pytest.mark.parametrize("kind", ["sum", "argmax"])
def test_shard_single_rank_with_halo(kind):
    """reduce_shard on a one-rank communicator: the shard's FIR reads the
    halo samples in front of it, like simtgo_tile_run_shard."""
    L = _lib.load()
    uid = C.create_string_buffer(128)
    _lib.check(L.simtgo_comm_unique_id(uid))
    comm = C.c_void_p()
    _lib.check(L.simtgo_comm_init(C.byref(comm), uid, 1, 0))
    try:
        n, halo = (1 << 20) + 9, 12
        xs = normal(n + halo, 9)
        buf = torch.from_numpy(xs).cuda()
        h = (np.arange(1, 14, dtype=np.float32) / 50).astype(np.float32)
        g = tile.New()
        a = g.InputDevice(buf[halo:])
        t = tile.Add(tile.FIR(a, h), tile.Abs(a))
        assert tile.ShardRange(n, 1, 0) == (0, n)
        vals = torch.empty(n, device="cuda")
        t.Run(vals, halo=halo)
        want = O.tile_reduce(vals.cpu().numpy(), kind)
        v = torch.zeros(1, device="cuda")
        i = torch.zeros(1, dtype=torch.int64, device="cuda")
        tile.Reduction(t, KINDS[kind]).RunShard(comm, n, v, i, halo=halo)
        torch.cuda.synchronize()
        check("shard", (np.float32(v.item()), int(i.item())), want, kind)
        # A shard length that is not this rank's range is refused.
        g2 = tile.New()
        t2 = g2.InputDevice(buf[:n - 1])
        with pytest.raises(_lib.SimtgoError):
            tile.Reduction(t2, tile.SUM).RunShard(comm, n, v, i)
    finally:
        _lib.check(L.simtgo_comm_destroy(comm))


def test_arguments_refused():
    g = tile.New()
    x = torch.ones(10, device="cuda")
    t = g.InputDevice(x)
    v = torch.zeros(1, device="cuda")
    L = _lib.load()
    assert L.simtgo_tile_reduce(g._h, t.node, 9, C.c_void_p(v.data_ptr()), None, None) \
        == _lib.EARG
    assert L.simtgo_tile_reduce(g._h, t.node, tile.ARGMAX, C.c_void_p(v.data_ptr()), None,
                                None) == _lib.ENULL
    assert L.simtgo_tile_reduce(g._h, t.node, tile.SUM, None, None, None) == _lib.ENULL
