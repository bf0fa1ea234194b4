"""GPU parity at the benchmark workloads' full sizes, element for element
against the oracle (no sampling):

- the twelve-node tile graph over 3 x 2^28 inputs uniform[-4,4] with 31
  taps of 1/31 (tile/codegen.go:16-133), fused and as a shard with a halo;
- the 127-tap FIR over a 2^28-output shard whose input carries the 126
  preceding samples (kernels/fir.go:17-46);
- the signal chain: 2^28 interleaved N(0,1) complex samples through
  MagnitudeFast(scale 3) -> Softclip(0.5) -> Quantize(step 0.25, seed
  0x9e3779b9) -> WarpReduceSum of the Softclip output and of float32(code)
  (kernels/magnitudefast.go:20, softclip.go:25, quantize.go:16,
  warpreduce.go:21).

The oracle runs on every host core; each case takes seconds. The chunked
oracle itself is checked on the CPU against one whole evaluation.
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle_lib as O
from tolerance import assert_agree

torch = pytest.importorskip("torch")
from simtgo_b200 import _lib, simt, tile  # noqa: E402

P = C.c_void_p
FULL = 1 << 28


@pytest.fixture(autouse=True)
def _threads():
    O.set_threads(os.cpu_count() or 1)
    yield
    if torch.cuda.is_available():
        torch.cuda.empty_cache()


def same_bits(name, got, want):
    assert got.shape == want.shape, name
    bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, (f"{name}: {bad.size} of {got.size} differ; first at {bad[0]}: "
                           f"{got[bad[0]]!r} vs {want[bad[0]]!r}")


def twelve_nodes(a, b, c, taps):
    """The oracle's node table of the twelve-node graph, in creation order
    (the taps are an input node, as tile/tile.go:147 records them)."""
    return [{"kind": "input", "data": a}, {"kind": "input", "data": b},
            {"kind": "input", "data": c}, {"kind": "scale", "a": 0, "scale": 0.5},
            {"kind": "abs", "a": 1}, {"kind": "sqrt", "a": 4}, {"kind": "mul", "a": 3, "b": 5},
            {"kind": "add", "a": 6, "b": 2}, {"kind": "input", "data": taps},
            {"kind": "fir", "a": 3, "taps": taps}, {"kind": "hypot", "a": 7, "b": 9},
            {"kind": "mul", "a": 10, "b": 4}]


def twelve_graph(g, a, b, c, taps):
    s = tile.Scale(a, 0.5)
    ab = tile.Abs(b)
    out = tile.Mul(tile.Hypot(tile.Add(tile.Mul(s, tile.Sqrt(ab)), c), tile.FIR(s, taps)), ab)
    assert out.node == 11 and g.Err() is None
    return out


def test_chunked_oracle_equals_whole():
    """The chunked evaluation used below equals one whole evaluation."""
    n = 3 * 4096 + 17
    rng = np.random.default_rng(1)
    a, b, c = (rng.uniform(-4, 4, n).astype(np.float32) for _ in range(3))
    taps = np.full(31, 1 / 31, np.float32)
    nodes = twelve_nodes(a, b, c, taps)
    rc, whole = O.tile_eval(nodes, 11, n)
    assert rc == 0
    same_bits("chunked", O.tile_eval_chunked(nodes, 11, n, 30, chunk=4096), whole)


@pytest.mark.gpu
def test_twelve_node_graph_full_size():
    rng = [np.random.default_rng(s) for s in (6, 7, 8)]
    host = [r.uniform(-4, 4, FULL).astype(np.float32) for r in rng]
    taps = np.full(31, 1 / 31, np.float32)
    want = O.tile_eval_chunked(twelve_nodes(*host, taps), 11, FULL, 30)
    dev = [torch.from_numpy(h).cuda() for h in host]
    g = tile.New()
    out = twelve_graph(g, *(g.InputDevice(d) for d in dev), taps)
    y = torch.empty(FULL, device="cuda")
    out.Run(y)
    same_bits("twelve-node graph, 2^28, fused", y.cpu().numpy(), want)
    # The upper half as a shard whose inputs carry 32 preceding samples.
    half, halo = FULL // 2, 32
    g2 = tile.New()
    out2 = twelve_graph(g2, *(g2.InputDevice(d[half:]) for d in dev), taps)
    y2 = torch.empty(FULL - half, device="cuda")
    out2.Run(y2, halo=halo)
    same_bits("twelve-node graph, upper half as a shard", y2.cpu().numpy(), want[half:])


@pytest.mark.gpu
def test_fir_127_taps_full_shard():
    n, halo, taps = FULL, 126, 127
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, n + halo).astype(np.float32)
    h = rng.uniform(-1, 1, taps)
    h = (h / h.sum()).astype(np.float32)
    xd, hd = torch.from_numpy(x).cuda(), torch.from_numpy(h).cuda()
    y = torch.empty(n, device="cuda")
    L = _lib.load()
    _lib.check(L.simtgo_FIR_shard(P(y.data_ptr()), n, P(xd.data_ptr()), n + halo, halo,
                                  P(hd.data_ptr()), taps, None))
    _lib.check(L.simtgo_stream_sync(None))
    got = y.cpu().numpy()
    del y, xd
    rc, want = O.fir_shard(x, halo, h, n)
    assert rc == 0
    same_bits("FIR 127 taps, 2^28 outputs (device fma order)", got, want)
    # gpu.RunCPU's unfused order, within the kernels' 1e-5 (tolerance.go:51).
    rc, emu = O.fir_shard(x, halo, h, n, fused=False)
    assert rc == 0
    assert_agree("FIR 127 taps vs RunCPU order", got, emu, tol=1e-5)


@pytest.mark.gpu
def test_signal_chain_full_size():
    n = FULL
    grid = (n + 255) // 256
    z = np.random.default_rng(11).standard_normal(2 * n, dtype=np.float32)
    L = _lib.load()
    zd = torch.from_numpy(z).cuda()
    mag = torch.empty(n, device="cuda")
    _lib.check(L.simtgo_MagnitudeFast_interleaved(P(mag.data_ptr()), n, P(zd.data_ptr()), 2 * n,
                                                  3.0, grid, 256, None))
    del zd
    soft = torch.empty(n, device="cuda")
    simt.build("Softclip").launch(grid, 256, soft, mag, 0.5)
    code = torch.empty(n, dtype=torch.int32, device="cuda")
    energy = torch.empty(n, dtype=torch.int64, device="cuda")
    clipped = torch.empty(n, dtype=torch.bool, device="cuda")
    simt.build("Quantize").launch(grid, 256, code, energy, clipped, soft, 0.25, 0x9E3779B9)
    wr = simt.build("WarpReduceSum")
    sums = torch.empty(n // 32, device="cuda")
    wr.launch((n + 127) // 128, 128, sums, soft)
    csums = torch.empty(n // 32, device="cuda")
    wr.launch((n + 127) // 128, 128, csums, code.float())
    simt.stream_sync()

    rc, w_mag = O.magnitudefast_interleaved(z, 3.0, grid, 256)
    assert rc == 0
    del z
    same_bits("MagnitudeFast interleaved", mag.cpu().numpy(), w_mag)
    del mag
    rc, w_soft = O.softclip(w_mag, 0.5, grid, 256)
    assert rc == 0
    del w_mag
    same_bits("Softclip", soft.cpu().numpy(), w_soft)
    rc, w_code, w_energy, w_clipped = O.quantize(w_soft, 0.25, 0x9E3779B9, grid, 256)
    assert rc == 0
    assert np.array_equal(code.cpu().numpy(), w_code), "Quantize code"
    assert np.array_equal(energy.cpu().numpy(), w_energy), "Quantize energy"
    assert np.array_equal(clipped.cpu().numpy().view(np.uint8), w_clipped), "Quantize clipped"
    rc, w_sums = O.warpreducesum(w_soft, n // 32, (n + 127) // 128)
    assert rc == 0
    same_bits("WarpReduceSum of the Softclip output", sums.cpu().numpy(), w_sums)
    rc, w_csums = O.warpreducesum(w_code.astype(np.float32), n // 32, (n + 127) // 128)
    assert rc == 0
    same_bits("WarpReduceSum of float32(code)", csums.cpu().numpy(), w_csums)
    # The quantised chain's totals: every code is in [-128, 127] and its
    # energy is its square (kernels/quantize.go:30-41).
    assert w_code.min() >= -128 and w_code.max() <= 127
    assert np.array_equal(w_energy, w_code.astype(np.int64) ** 2)
