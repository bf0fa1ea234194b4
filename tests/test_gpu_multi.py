"""Multi-GPU tests of the histogram all-reduce, one process per GPU (skipped
with fewer than two GPUs): the fused NVLink kernel and the NCCL path agree
with the whole input's histogram on every rank, and a rank that never
arrives makes the others' bounded wait run out -- an error status read on
the host, no fault, the context still usable. NVLS is off (NCCL_NVLS_ENABLE
=0) and the kernels use plain peer stores."""
import ctypes as C
import multiprocessing as mp
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

WORLD = 2
TOTAL = (1 << 22) + 12345


def _whole():
    return np.random.default_rng(77).integers(-5, 300, TOTAL, dtype=np.int32)


def _whole_f32():
    return np.random.default_rng(78).standard_normal(TOTAL).astype(np.float32)


def _taps():
    return (np.arange(1, 12, dtype=np.float32) / 40).astype(np.float32)


def _child(rank, uid, mode, q, bar):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import torch as t

        from simtgo_b200 import _lib

        t.cuda.set_device(rank)
        L = _lib.load()
        P = C.c_void_p
        comm = P()
        _lib.check(L.simtgo_comm_init(C.byref(comm), C.create_string_buffer(uid, 128), WORLD,
                                      rank))
        x = _whole()
        per = (TOTAL + WORLD - 1) // WORLD
        xs = t.from_numpy(x[rank * per:(rank + 1) * per].copy()).cuda()
        out = {}
        if mode == "agree":
            for name in ("simtgo_Histogram_allreduce", "simtgo_Histogram_allreduce_fused"):
                for call in range(3):
                    b = t.full((300,), rank + call, dtype=t.int32, device="cuda")
                    _lib.check(getattr(L, name)(comm, P(b.data_ptr()), 300, P(xs.data_ptr()),
                                                xs.numel(), None))
                    _lib.check(L.simtgo_stream_sync(None))
                    out[(name, call)] = b.cpu().numpy()
            # The overwrite form: the starting values are ignored.
            for call in range(3):
                b = t.full((300,), 1000 + rank + call, dtype=t.int32, device="cuda")
                _lib.check(L.simtgo_Histogram_allreduce_fused_overwrite(
                    comm, P(b.data_ptr()), 300, P(xs.data_ptr()), xs.numel(), None))
                _lib.check(L.simtgo_stream_sync(None))
                out[("overwrite", call)] = b.cpu().numpy()
        elif mode == "reduce":  # the tile reductions over shards with a halo
            from simtgo_b200 import tile

            xf = _whole_f32()
            start, ln = tile.ShardRange(TOTAL, WORLD, rank)
            halo = min(start, 16)
            buf = t.from_numpy(xf[start - halo:start + ln].copy()).cuda()
            g = tile.New()
            a = g.InputDevice(buf[halo:])
            y = tile.Add(tile.FIR(a, _taps()), tile.Abs(a))
            for kind in (tile.SUM, tile.MIN, tile.MAX, tile.ARGMAX):
                v = t.zeros(1, device="cuda")
                i = t.zeros(1, dtype=t.int64, device="cuda")
                tile.Reduction(y, kind).RunShard(comm, TOTAL, v, i, halo=halo)
                t.cuda.synchronize()
                out[kind] = (float(v.item()), int(i.item()))
        else:  # "absent": rank 1 maps the buffers, then skips the second call
            b = t.zeros(256, dtype=t.int32, device="cuda")
            _lib.check(L.simtgo_Histogram_allreduce_fused(comm, P(b.data_ptr()), 256,
                                                          P(xs.data_ptr()), xs.numel(), None))
            _lib.check(L.simtgo_stream_sync(None))
            if rank == 0:
                b.zero_()
                _lib.check(L.simtgo_Histogram_allreduce_fused(comm, P(b.data_ptr()), 256,
                                                              P(xs.data_ptr()), xs.numel(),
                                                              None))
                out["status"] = L.simtgo_stream_sync(None)
                out["msg"] = L.simtgo_last_error().decode()
                out["after"] = int(t.ones(4, device="cuda").sum().item())  # context usable
            t.cuda.synchronize()
        q.put((rank, out, None))
        # No rank frees its exchange buffer while another may still store
        # into it: every rank's kernels are done before any comm is destroyed.
        bar.wait(timeout=120)
        L.simtgo_comm_destroy(comm)
    except Exception as e:  # noqa: BLE001
        q.put((rank, None, repr(e)))


def _run(mode):
    from simtgo_b200 import _lib

    L = _lib.load()
    uid = C.create_string_buffer(128)
    _lib.check(L.simtgo_comm_unique_id(uid))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    bar = ctx.Barrier(WORLD)
    procs = [ctx.Process(target=_child, args=(r, uid.raw, mode, q, bar)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, out, err = q.get(timeout=180)
            assert err is None, f"rank {rank}: {err}"
            results[rank] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return results


@pytest.fixture(scope="module", autouse=True)
def _need_gpus():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")


def test_fused_and_nccl_agree_with_the_whole():
    res = _run("agree")
    x = _whole()
    counts = np.bincount(x[(x >= 0) & (x < 256)], minlength=256).astype(np.int64)
    for call in range(3):
        start = sum(r + call for r in range(WORLD))
        want = np.full(300, start, np.int64)
        want[:256] += counts
        for rank in range(WORLD):
            for name in ("simtgo_Histogram_allreduce", "simtgo_Histogram_allreduce_fused"):
                np.testing.assert_array_equal(res[rank][(name, call)], want.astype(np.int32),
                                              err_msg=f"{name} call {call} rank {rank}")
            over = np.zeros(300, np.int64)
            over[:256] = counts
            np.testing.assert_array_equal(res[rank][("overwrite", call)], over.astype(np.int32),
                                          err_msg=f"overwrite call {call} rank {rank}")


def test_absent_rank_times_out_with_a_status():
    res = _run("absent")
    from simtgo_b200 import _lib

    assert res[0]["status"] == _lib.EDEVICE, res[0]
    assert "watchdog" in res[0]["msg"]
    assert res[0]["after"] == 4


def test_tile_reduce_shards_equal_the_whole():
    """Each rank reduces its shard (FIR over a 16-sample halo); after the
    all-gather of the block partials every rank holds the whole signal's
    result, bit for bit as the oracle's tree over the whole signal."""
    import oracle_lib as O

    res = _run("reduce")
    x = _whole_f32()
    h = _taps()
    nodes = [{"kind": "input", "data": x}, {"kind": "input", "data": h},
             {"kind": "fir", "a": 0, "taps": h}, {"kind": "abs", "a": 0},
             {"kind": "add", "a": 2, "b": 3}]
    rc, vals = O.tile_eval(nodes, 4, TOTAL, 0)
    assert rc == 0
    for kind, name in enumerate(("sum", "min", "max", "argmax")):
        wv, wi = O.tile_reduce(vals, name)
        for rank in range(WORLD):
            gv, gi = res[rank][kind]
            assert np.float32(gv).view(np.uint32) == np.float32(wv).view(np.uint32), \
                (name, rank, gv, wv)
            if name == "argmax":
                assert gi == wi, (rank, gi, wi)
