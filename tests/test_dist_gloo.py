"""The multi-rank host logic on CPU: two gloo ranks (one process each, as one
process per GPU) follow the shard plans of simtgo_b200.shard, compute their
part with the oracle, and exchange what the sharded workloads exchange:

  FIR        nothing on the data path (the halo is part of the shard);
             gathered only to check that the shards tile the whole output;
  Histogram  the 256 partial bins, summed with an all-reduce;
  tile       nothing (pure split), gathered for the check;
  reduction  the block partials of each rank's whole 2048-blocks,
             all-gathered, then the same tree on every rank.

Each result must equal the unsharded oracle run. Also: a rank that fails
between steps is seen by the other as a collective error within the
process group's timeout, never as a hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from simtgo_b200 import shard

WORLD = 2


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _signal(total):
    return np.random.default_rng(7).uniform(-1, 1, total).astype(np.float32)


def _worker_workloads(rank, port, q):
    import oracle_lib as O

    _init(rank, port)
    try:
        total, taps = 50021, 127
        x = _signal(total)
        h = (np.random.default_rng(8).uniform(-1, 1, taps) / 20).astype(np.float32)
        # FIR: this rank's plan, then its shard alone.
        p = shard.fir_plan(total, WORLD, rank, taps)
        assert p.halo == (0 if rank == 0 else 128)
        rc, y = O.fir_shard(x[p.in_lo:p.out_hi].copy(), p.halo, h, p.n)
        assert rc == 0
        parts = [None] * WORLD
        dist.all_gather_object(parts, (p.out_lo, y))
        # Histogram: local bins + all-reduce (the sum over ranks).
        xi = np.random.default_rng(9).integers(-5, 260, total, dtype=np.int32)
        hp = shard.histogram_plan(total, WORLD, rank)
        rc, b = O.histogram_shard(xi[hp.out_lo:hp.out_hi].copy())
        bins = torch.from_numpy(b.astype(np.int64))
        dist.all_reduce(bins)
        # Tile graph with a 31-tap window: pure split plus a halo.
        tp = shard.tile_plan(total, WORLD, rank, max_taps=31)
        ins = [np.random.default_rng(10 + k).uniform(-4, 4, total).astype(np.float32)
               for k in range(3)]
        hh = np.full(31, 1 / 31, np.float32)

        def nodes(data):
            a, bb, c = data
            return [{"kind": "input", "data": a}, {"kind": "input", "data": bb},
                    {"kind": "input", "data": c}, {"kind": "scale", "a": 0, "scale": 0.5},
                    {"kind": "abs", "a": 1}, {"kind": "sqrt", "a": 4},
                    {"kind": "mul", "a": 3, "b": 5}, {"kind": "add", "a": 6, "b": 2},
                    {"kind": "input", "data": hh}, {"kind": "fir", "a": 3, "taps": hh},
                    {"kind": "hypot", "a": 7, "b": 9}, {"kind": "mul", "a": 10, "b": 4}]

        rc, t = O.tile_eval(nodes([v[tp.in_lo:tp.out_hi] for v in ins]), 11, tp.n, tp.halo)
        tparts = [None] * WORLD
        dist.all_gather_object(tparts, (tp.out_lo, t))
        if rank == 0:
            rc, whole = O.fir_shard(x, 0, h, total)
            got = np.concatenate([v for _, v in sorted(parts, key=lambda z: z[0])])
            fir_ok = np.array_equal(got.view(np.uint32), whole.view(np.uint32))
            rc, wb = O.histogram_shard(xi)
            hist_ok = np.array_equal(bins.numpy().astype(np.int32), wb)
            rc, wt = O.tile_eval(nodes(ins), 11, total, 0)
            gt = np.concatenate([v for _, v in sorted(tparts, key=lambda z: z[0])])
            tile_ok = np.array_equal(gt.view(np.uint32), wt.view(np.uint32))
            q.put((fir_ok, hist_ok, tile_ok))
    finally:
        dist.destroy_process_group()


def _worker_reduce(rank, port, q):
    """The sharded tile reduction's exchange: each rank reduces its
    ShardRange slice (whole 2048-blocks) to block partials, pads them to the
    per-rank slot count with the identity, all-gathers the slots, and
    finishes the tree over the first m = ceil(total / 2048) of them."""
    import oracle_lib as O
    from simtgo_b200 import tile

    _init(rank, port)
    try:
        total = 9 * 2048 + 1234
        x = np.random.default_rng(12).standard_normal(total).astype(np.float32)
        x[5000] = 50.0
        s0, n = tile.ShardRange(total, WORLD, rank)
        _, per = tile.ShardRange(total, WORLD, 0)
        slots = per // 2048
        m = (total + 2047) // 2048
        ok = {}
        for kind in ("sum", "min", "max", "argmax"):
            pv, pi = O.tile_reduce_partials(x[s0:s0 + n], kind, idx_base=s0)
            ident, _ = O.tile_reduce(np.zeros(0, np.float32), kind)
            pad_v = np.concatenate([pv, np.full(slots - len(pv), ident, np.float32)])
            pad_i = np.concatenate([pi, np.full(slots - len(pi), -1, np.int64)])
            gv = [torch.zeros(slots, dtype=torch.float32) for _ in range(WORLD)]
            gi = [torch.zeros(slots, dtype=torch.int64) for _ in range(WORLD)]
            dist.all_gather(gv, torch.from_numpy(pad_v))
            dist.all_gather(gi, torch.from_numpy(pad_i))
            allv = torch.cat(gv).numpy()[:m]
            alli = torch.cat(gi).numpy()[:m]
            got = O.tile_reduce_levels(allv, alli, kind)
            want = O.tile_reduce(x, kind)
            ok[kind] = (got[0].view(np.uint32) == want[0].view(np.uint32)
                        and (kind != "argmax" or got[1] == want[1] == 5000))
        flags = [None] * WORLD
        dist.all_gather_object(flags, ok)
        if rank == 0:
            q.put(flags)
    finally:
        dist.destroy_process_group()


def _worker_dead_peer(rank, port, q):
    _init(rank, port, timeout_s=5)
    t = torch.ones(4)
    dist.all_reduce(t)          # step 1: both ranks
    if rank == 1:
        os._exit(0)             # rank 1 leaves between steps
    try:
        dist.all_reduce(t)      # step 2: rank 0 alone
        q.put("no error")
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        q.put(type(e).__name__)


def _run(fn, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=fn, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        return q.get(timeout=timeout)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()


def test_sharded_workloads_equal_whole():
    fir_ok, hist_ok, tile_ok = _run(_worker_workloads)
    assert fir_ok, "FIR shards do not tile the whole output"
    assert hist_ok, "all-reduced partial bins differ from the whole histogram"
    assert tile_ok, "tile graph shards differ from the whole"


def test_sharded_reduction_equals_whole():
    flags = _run(_worker_reduce)
    for rank, ok in enumerate(flags):
        assert all(ok.values()), (rank, ok)


def test_dead_peer_is_an_error_not_a_hang():
    outcome = _run(_worker_dead_peer, timeout=90)
    assert outcome != "no error"


@pytest.mark.parametrize("total,world", [(10, 3), (2 ** 31, 8), (5, 8), (1 << 28, 2)])
def test_split_covers_exactly(total, world):
    spans = [shard.split(total, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert max(hi - lo for lo, hi in spans) - min(hi - lo for lo, hi in spans) <= 1


def test_fir_plan_halo_alignment():
    p = shard.fir_plan(1 << 31, 8, 3, 127)
    assert p.halo == 128 and p.in_lo == p.out_lo - 128 and p.n == 1 << 28
    assert shard.fir_plan(1 << 31, 8, 0, 127).halo == 0
    assert shard.round_halo(31) == 32 and shard.round_halo(1) == 0


def test_chain_window_halo():
    # FIR(Add(FIR(a, 17 taps), a), 21 taps) reaches 16 + 20 samples below.
    assert shard.chain_window([17, 21]) == 37
    assert shard.round_halo(shard.chain_window([17, 21])) == 36
    p = shard.tile_plan(1 << 20, 4, 2, max_taps=shard.chain_window([17, 21]))
    assert p.halo == 36 and p.in_lo == p.out_lo - 36
    assert shard.chain_window([1, 1]) == 1 and shard.round_halo(1) == 0
