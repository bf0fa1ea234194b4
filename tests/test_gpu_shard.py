"""GPU tests of the long / sharded forms: simtgo_FIR_shard (64-bit extents,
up to 1024 taps, halos), simtgo_Histogram_shard and the single-rank
communicator path of simtgo_Histogram_allreduce. Full-size cases are checked
through properties that do not need the oracle at that size: shards
concatenate to the whole, totals are conserved, sampled outputs match."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O
from tolerance import assert_agree, assert_equal

torch = pytest.importorskip("torch")
from simtgo_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu
P = C.c_void_p


def fir_shard(y, x, halo, h):
    L = _lib.load()
    _lib.check(L.simtgo_FIR_shard(P(y.data_ptr()), y.numel(), P(x.data_ptr()), x.numel(), halo,
                                  P(h.data_ptr()), h.numel(), None))
    _lib.check(L.simtgo_stream_sync(None))


@pytest.mark.parametrize("n,taps,halo", [(1, 1, 0), (8192, 127, 0), (8193, 127, 126),
                                         (100000, 127, 126), (50000, 1024, 1023),
                                         (20000, 200, 50), (777, 9, 700), ((1 << 20) + 5, 31, 30)])
def test_fir_shard_parity(n, taps, halo):
    rng = np.random.default_rng(n + taps)
    x = rng.uniform(-1, 1, n + halo).astype(np.float32)
    h = rng.uniform(-1, 1, taps).astype(np.float32)
    h /= np.float32(max(1.0, abs(float(h.sum()))))
    rc, want = O.fir_shard(x, halo, h, n)
    assert rc == 0
    for off in (0, 1):
        xb = torch.empty(n + halo + off, device="cuda")
        xd = xb[off:]
        xd.copy_(torch.from_numpy(x))
        yd = torch.empty(n, device="cuda")
        fir_shard(yd, xd, halo, torch.from_numpy(h).cuda())
        assert_agree("fir_shard", yd.cpu().numpy(), want)


@pytest.mark.parametrize("n,taps,halo,short,pinned", [
    (1, 1, 0, 0, True), (5000, 127, 126, 0, True), ((1 << 22) + 12345, 127, 126, 0, True),
    ((1 << 23) + 3, 63, 0, 0, False), (3 * (1 << 22), 1024, 1023, 0, True),
    ((1 << 22) + 100, 31, 30, 5000, True), ((1 << 22) + 100, 31, 7, (1 << 22) + 60, True)])
def test_fir_shard_host_equals_device(n, taps, halo, short, pinned):
    """The host-memory form (chunks of 2^22 on three streams) gives the
    device form's bits: ragged chunk counts, halos shorter than taps-1,
    signals that end before the outputs do (zeros read past x), pinned and
    pageable buffers."""
    rng = np.random.default_rng(n + taps + halo)
    xl = n + halo - short
    x = rng.uniform(-1, 1, xl).astype(np.float32)
    h = (rng.uniform(-1, 1, taps) / taps).astype(np.float32)
    xt = torch.from_numpy(x)
    yt = torch.full((n,), np.nan, dtype=torch.float32)
    ht = torch.from_numpy(h)
    if pinned:
        xt, yt, ht = xt.pin_memory(), yt.pin_memory(), ht.pin_memory()
    L = _lib.load()
    s = torch.cuda.current_stream()
    _lib.check(L.simtgo_FIR_shard_host(P(yt.data_ptr()), n, P(xt.data_ptr()), xl, halo,
                                       P(ht.data_ptr()), taps, P(s.cuda_stream)))
    s.synchronize()
    _lib.check(L.simtgo_stream_sync(None))
    yd = torch.empty(n, device="cuda")
    fir_shard(yd, torch.from_numpy(x).cuda(), halo, torch.from_numpy(h).cuda())
    assert_equal("fir_shard_host", yt.numpy().view(np.uint32), yd.cpu().numpy().view(np.uint32))


def test_shutdown_releases_and_host_form_recovers():
    """simtgo_shutdown frees the host form's device buffers; the next call
    allocates them again and gives the same bits."""
    L = _lib.load()
    n, taps = (1 << 22) + 9, 63
    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.uniform(-1, 1, n).astype(np.float32)).pin_memory()
    h = torch.from_numpy((rng.uniform(-1, 1, taps) / taps).astype(np.float32)).pin_memory()
    outs = []
    for _ in range(2):
        y = torch.empty(n, dtype=torch.float32).pin_memory()
        _lib.check(L.simtgo_FIR_shard_host(P(y.data_ptr()), n, P(x.data_ptr()), n, 0,
                                           P(h.data_ptr()), taps, None))
        _lib.check(L.simtgo_stream_sync(None))
        outs.append(y.numpy().copy())
        _lib.check(L.simtgo_shutdown())
    assert_equal("after shutdown", outs[1].view(np.uint32), outs[0].view(np.uint32))


def test_fir_shards_concatenate_to_whole():
    """Eight shards of one signal, each with a 126-sample halo, equal the
    unsharded FIR over the whole (127 taps): the 2^31-sample workload's
    decomposition, at 2^24 samples."""
    n, taps, G = 1 << 24, 127, 8
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.uniform(-1, 1, n).astype(np.float32)).cuda()
    h = torch.from_numpy((rng.uniform(-1, 1, taps) / 10).astype(np.float32)).cuda()
    whole = torch.empty(n, device="cuda")
    fir_shard(whole, x, 0, h)
    per = n // G
    for g in range(G):
        lo = g * per
        halo = min(lo, taps - 1)
        y = torch.empty(per, device="cuda")
        fir_shard(y, x[lo - halo: lo + per], halo, h)
        assert torch.equal(y, whole[lo: lo + per]), f"shard {g}"
    # sampled outputs against the oracle
    xs, hs = x.cpu().numpy(), h.cpu().numpy()
    idx = np.random.default_rng(4).integers(0, n, 2000)
    ws = whole.cpu().numpy()
    for i in idx:
        lo = max(0, i - taps + 1)
        rc, w = O.fir_shard(xs[lo:i + 1].copy(), i - lo, hs, 1)
        assert_agree(f"sample {i}", ws[i:i + 1], w)


@pytest.mark.parametrize("n", [0, 5, 1 << 20, (1 << 24) + 1])
def test_histogram_shard(n):
    rng = np.random.default_rng(n)
    x = rng.integers(-10, 270, n, dtype=np.int32)
    rc, want = O.histogram_shard(x)
    bins = torch.zeros(256, dtype=torch.int32, device="cuda")
    xd = torch.from_numpy(x).cuda()
    L = _lib.load()
    _lib.check(L.simtgo_Histogram_shard(P(bins.data_ptr()), 256, P(xd.data_ptr()) if n else None,
                                        n, None))
    _lib.check(L.simtgo_stream_sync(None))
    assert_equal("bins", bins.cpu().numpy(), want)


def test_histogram_full_size_conserves_counts():
    """2^28 uniform int32 in [0,255] and a Zipf(1.2) draw: every sample is
    counted once (the bins sum to 2^28) and the bins equal numpy's."""
    n = 1 << 28
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randint(0, 256, (n,), dtype=torch.int32, device="cuda", generator=g)
    bins = torch.zeros(256, dtype=torch.int32, device="cuda")
    L = _lib.load()
    _lib.check(L.simtgo_Histogram_shard(P(bins.data_ptr()), 256, P(x.data_ptr()), n, None))
    _lib.check(L.simtgo_stream_sync(None))
    want = torch.bincount(x.long(), minlength=256).to(torch.int32)
    assert int(bins.sum()) == n
    assert torch.equal(bins, want)


def test_histogram_allreduce_single_rank():
    L = _lib.load()
    uid = C.create_string_buffer(128)
    _lib.check(L.simtgo_comm_unique_id(uid))
    comm = P()
    _lib.check(L.simtgo_comm_init(C.byref(comm), uid, 1, 0))
    try:
        x = torch.randint(0, 256, (1 << 20,), dtype=torch.int32, device="cuda")
        bins = torch.zeros(256, dtype=torch.int32, device="cuda")
        _lib.check(L.simtgo_Histogram_allreduce(comm, P(bins.data_ptr()), 256, P(x.data_ptr()),
                                                x.numel(), None))
        _lib.check(L.simtgo_stream_sync(None))
        assert torch.equal(bins, torch.bincount(x.long(), minlength=256).to(torch.int32))
    finally:
        _lib.check(L.simtgo_comm_destroy(comm))


@pytest.mark.parametrize("bins_len", [1, 100, 256, 1000, 4096])
def test_histogram_allreduce_fused_single_rank(bins_len):
    """The fused kernel with one rank (its own buffer is the only slot):
    five calls in a row (both slot halves, flags counting up) give the
    oracle's counts added to non-zero starting bins; bins past 256 keep
    their starting values; more than 4096 bins is refused."""
    L = _lib.load()
    uid = C.create_string_buffer(128)
    _lib.check(L.simtgo_comm_unique_id(uid))
    comm = P()
    _lib.check(L.simtgo_comm_init(C.byref(comm), uid, 1, 0))
    try:
        rng = np.random.default_rng(bins_len)
        for call in range(5):
            n = 100003 + 7 * call
            x = rng.integers(-20, 300, n, dtype=np.int32)
            bins0 = rng.integers(0, 50, bins_len, dtype=np.int32)
            rc, want = O.histogram_shard(x, bins_len, bins=bins0)
            assert rc == 0
            b = torch.from_numpy(bins0).cuda()
            xd = torch.from_numpy(x).cuda()
            _lib.check(L.simtgo_Histogram_allreduce_fused(comm, P(b.data_ptr()), bins_len,
                                                          P(xd.data_ptr()), n, None))
            _lib.check(L.simtgo_stream_sync(None))
            assert_equal(f"call {call}", b.cpu().numpy(), want)
            # The overwrite form counts into bins whatever they held.
            b = torch.from_numpy(bins0).cuda()
            _lib.check(L.simtgo_Histogram_allreduce_fused_overwrite(
                comm, P(b.data_ptr()), bins_len, P(xd.data_ptr()), n, None))
            _lib.check(L.simtgo_stream_sync(None))
            rc, fresh = O.histogram_shard(x, bins_len)
            assert_equal(f"overwrite call {call}", b.cpu().numpy(), fresh)
        big = torch.zeros(4097, dtype=torch.int32, device="cuda")
        assert L.simtgo_Histogram_allreduce_fused(comm, P(big.data_ptr()), 4097,
                                                  P(xd.data_ptr()), n, None) == _lib.ESIZE
    finally:
        _lib.check(L.simtgo_comm_destroy(comm))
