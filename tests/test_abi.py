"""The C ABI on the CPU: the library loads, exports every function that
include/*.h declares, and refuses -- before touching a device -- the launches
simt.Kernel.launch refuses (simt/kernel.go:488-514): wrong block sizes
(BlockSizeError), overlapping written slices (AliasError), slices shorter than
the launch reads (gpu.RunCPU's index-out-of-range), and the tile graph's
latched errors (tile/tile.go:78-149). No compute call is made here."""
import ctypes as C
import pathlib
import re
import subprocess

import numpy as np
import pytest

from simtgo_b200 import _lib, tile

ROOT = pathlib.Path(__file__).resolve().parent.parent


def header_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(simtgo_\w+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_exports_every_declared_function(lib):
    declared = header_functions()
    assert len(declared) >= 40
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.lib_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (simtgo_\w+)", out))
    assert declared <= exported, f"missing: {sorted(declared - exported)}"
    assert declared == set(_lib.exported_symbols())


def test_no_oracle_linked():
    out = subprocess.run(["ldd", str(_lib.lib_path())], capture_output=True, text=True).stdout
    assert "oracle" not in out and "libref" not in out
    syms = subprocess.run(["nm", "-D", str(_lib.lib_path())], capture_output=True,
                          text=True).stdout
    assert "oracle_" not in syms and "ref_" not in re.sub(r"\w+ref_\w*", "", syms)


def err(lib):
    return lib.simtgo_last_error().decode()


P = C.c_void_p


def test_block_size_contract(lib):
    # FIRBlock = 256, WarpReduceBlock = 128, TransposeTile^2 = 256.
    assert lib.simtgo_FIR(P(4096), 8, P(8192), 8, P(1 << 20), 3, 1, 128, None) == _lib.EBLOCK
    assert "requires block == 256, got 128" in err(lib)
    assert lib.simtgo_WarpReduceSum(P(4096), 4, P(8192), 64, 1, 256, None) == _lib.EBLOCK
    assert "requires block == 128, got 256" in err(lib)
    # simt/parity_test.go TestLaunchDimCountsTheWholeBlock: 16x8 is 128 threads.
    assert lib.simtgo_Transpose(P(4096), 16, P(8192), 16, 4, 4, 1, 1, 16, 8, None) == _lib.EBLOCK
    assert "requires block == 256, got 128" in err(lib)
    assert lib.simtgo_Transpose(P(4096), 16, P(8192), 16, 4, 4, 1, 1, 32, 8, None) == _lib.EBLOCK


def test_launch_geometry_refused(lib):
    assert lib.simtgo_VecAdd(P(4096), 8, P(8192), 8, P(1 << 20), 8, 0, 256, None) == _lib.ELAUNCH
    assert lib.simtgo_VecAdd(P(4096), 8, P(8192), 8, P(1 << 20), 8, 1, 2048, None) == _lib.ELAUNCH
    assert lib.simtgo_Scale(P(4096), 8, P(8192), 8, 1.0, 1, 0, None) == _lib.ELAUNCH


def test_alias_refused(lib):
    # c overlaps a: the kernel writes through c.
    rc = lib.simtgo_VecAdd(P(4096), 16, P(4096 + 32), 16, P(1 << 20), 16, 1, 256, None)
    assert rc == _lib.EALIAS
    assert "parameters c and a" in err(lib) and "writes through c" in err(lib)
    # Two read-only slices may share memory.
    rc = lib.simtgo_VecAdd(P(1 << 20), 16, P(4096), 16, P(4096), 16, 1, 256, None)
    assert rc != _lib.EALIAS
    # Quantize's three outputs must not overlap each other either.
    rc = lib.simtgo_Quantize(P(4096), 16, P(4096 + 8), 16, P(1 << 20), 16, P(1 << 21), 16, 0.25,
                             1, 1, 256, None)
    assert rc == _lib.EALIAS


def test_short_slices_refused(lib):
    rc = lib.simtgo_VecAdd(P(4096), 16, P(1 << 20), 8, P(1 << 21), 16, 1, 256, None)
    assert rc == _lib.ELENGTH and "index out of range" in err(lib)
    # A grid covering fewer threads than c_len reads only what it covers.
    rc = lib.simtgo_VecAdd(P(4096), 16, P(1 << 20), 8, P(1 << 21), 8, 1, 8, None)
    assert rc not in (_lib.ELENGTH, _lib.EALIAS)
    rc = lib.simtgo_Quantize(P(4096), 16, P(1 << 16), 8, P(1 << 20), 16, P(1 << 21), 16, 0.25, 1,
                             1, 256, None)
    assert rc == _lib.ELENGTH and "energy" in err(lib)
    rc = lib.simtgo_Transpose(P(4096), 9443, P(1 << 20), 9000, 133, 71, 9, 5, 16, 16, None)
    assert rc == _lib.ELENGTH and "in has" in err(lib)


def test_fir_taps_limit(lib):
    # 65 taps still fit the 320-sample tile; 66 do not (fir.go:24).
    rc = lib.simtgo_FIR(P(4096), 8, P(8192), 8, P(1 << 20), 66, 1, 256, None)
    assert rc == _lib.ETAPS
    rc = lib.simtgo_FIR_shard(P(4096), 8, P(8192), 8, 0, P(1 << 20), 1025, None)
    assert rc == _lib.ETAPS
    rc = lib.simtgo_FIR_shard(P(4096), 8, P(8192), 8, 0, P(1 << 20), 0, None)
    assert rc == _lib.ETAPS


def test_null_pointers_refused(lib):
    rc = lib.simtgo_VecAdd(None, 16, P(1 << 20), 16, P(1 << 21), 16, 1, 256, None)
    assert rc == _lib.ENULL
    rc = lib.simtgo_BandGain(P(4096), 8, P(8192), 8, None, 0, None, 1, 256, None)
    assert rc == _lib.ENULL


def test_empty_launch_is_a_no_op(lib):
    # A covered extent of zero elements touches nothing, device or not.
    assert lib.simtgo_VecAdd(P(4096), 0, P(8192), 0, P(1 << 20), 0, 1, 256, None) == 0
    assert lib.simtgo_Histogram(P(4096), 256, P(8192), 0, 1, 256, None) == 0
    assert lib.simtgo_FIR_shard(P(4096), 0, P(8192), 0, 0, P(1 << 20), 3, None) == 0


# ---- tile graph: recording and lowering need no device ---------------------

def test_tile_shape_mismatch():
    g = tile.New()
    out = tile.Add(g.Input(np.zeros(8)), g.Input(np.zeros(9)))
    e = g.Err()
    assert e is not None and "does not match" in str(e)
    with pytest.raises(_lib.GraphError, match="does not match"):
        out.Materialize()


def test_tile_chained_window_rejected():
    g = tile.New()
    h = [1, 2, 3]
    tile.FIR(tile.FIR(g.Input(np.zeros(1024)), h), h)
    assert "chaining windowed" in str(g.Err())


def test_tile_taps_bounds():
    g = tile.New()
    tile.FIR(g.Input(np.zeros(64)), np.ones(65))
    assert "65 taps is outside 1..64" in str(g.Err())
    g = tile.New()
    tile.FIR(g.Input(np.zeros(64)), [])
    assert "0 taps is outside 1..64" in str(g.Err())


def test_tile_first_error_is_kept():
    g = tile.New()
    a = g.Input(np.zeros(4))
    tile.Add(a, g.Input(np.zeros(5)))
    tile.FIR(tile.FIR(a, [1.0]), [1.0])
    assert "does not match" in str(g.Err())


def test_tile_different_graphs():
    g1, g2 = tile.New(), tile.New()
    tile.Add(g1.Input(np.zeros(4)), g2.Input(np.zeros(4)))
    assert "different graphs" in str(g1.Err())


def twelve_node_graph(g, a, b, c, h):
    """The 12-node DAG of the tile workload: every op of the track, the FIR
    taps counted as a node (tile/tile.go:147)."""
    s = tile.Scale(a, 0.5)
    ab = tile.Abs(b)
    q = tile.Sqrt(ab)
    m = tile.Mul(s, q)
    d = tile.Add(m, c)
    f = tile.FIR(s, h)
    y = tile.Hypot(d, f)
    return tile.Mul(y, ab)


def test_tile_lowering_is_one_program():
    n = 100
    g = tile.New()
    a, b, c = (g.Input(np.zeros(n)) for _ in range(3))
    out = twelve_node_graph(g, a, b, c, np.ones(31) / 31)
    assert g.Err() is None
    assert out.node == 11  # 12 nodes, ids 0..11
    instructions, inputs, windows = out.ProgramSize()
    assert inputs == 3 and windows == 1
    assert 0 < instructions < 40


def test_tile_wide_graph_falls_back_then_refuses():
    g = tile.New()
    xs = [g.Input(np.zeros(16)) for _ in range(20)]
    acc = xs[0]
    for x in xs[1:]:
        acc = tile.Add(acc, x)
    assert acc.ProgramSize()[1] == 20  # 20 inputs: loads not hoisted, still fits
    # A balanced tree of 512 leaves keeps ~10 partial sums alive.
    g = tile.New()
    level = [g.Input(np.zeros(16)) for _ in range(32)]
    while len(level) > 1:
        level = [tile.Mul(level[i], level[i + 1]) for i in range(0, len(level), 2)]
    assert level[0].ProgramSize()[1] == 32


def test_launch_shared_spelling_refused():
    """simt/shared_parity_cuda_test.go:185-213: a kernel with a launch-sized
    tile launched without a size, and one without such a tile handed a
    size, are refused before anything reaches the device."""
    from simtgo_b200 import simt

    dyn = simt.Kernel("HistogramDyn", simt.KERNELS["HistogramDyn"])
    plain = simt.Kernel("VecAdd", simt.KERNELS["VecAdd"])
    with pytest.raises(simt.DynamicSharedError) as e:
        dyn.launch(1, 32, None, None)
    assert e.value.dynamic
    with pytest.raises(simt.DynamicSharedError) as e:
        dyn.launch_on(object(), 1, 32, None, None)
    assert e.value.dynamic
    with pytest.raises(simt.DynamicSharedError) as e:
        plain.launch_shared(1, 32, 8, None, None, None)
    assert not e.value.dynamic


def test_tile_reduce_arguments_refused_on_the_host(lib):
    """The reductions' argument checks run before anything touches a
    device: an unknown kind, a missing value or ArgMax index, a graph error,
    a shard range outside the ranks."""
    g = lib.simtgo_tile_new()
    try:
        fake = C.c_void_p(0x1000)   # never dereferenced: every call below is refused first
        t = lib.simtgo_tile_input_device(g, fake, 64)
        assert lib.simtgo_tile_reduce(g, t, 9, fake, fake, None) == _lib.EARG
        assert lib.simtgo_tile_reduce(g, t, -1, fake, fake, None) == _lib.EARG
        assert lib.simtgo_tile_reduce(g, t, tile.SUM, None, None, None) == _lib.ENULL
        assert lib.simtgo_tile_reduce(g, t, tile.ARGMAX, fake, None, None) == _lib.ENULL
        assert lib.simtgo_tile_reduce(g, 99, tile.SUM, fake, None, None) == _lib.EARG
        v, i = C.c_float(), C.c_int64()
        assert lib.simtgo_tile_reduce_materialize(g, t, 7, C.byref(v), C.byref(i)) == _lib.EARG
        s0, n = C.c_int64(), C.c_int64()
        assert lib.simtgo_tile_shard_range(100, 0, 0, C.byref(s0), C.byref(n)) == _lib.EARG
        assert lib.simtgo_tile_shard_range(-1, 2, 0, C.byref(s0), C.byref(n)) == _lib.EARG
        assert lib.simtgo_tile_shard_range(100, 2, 0, None, C.byref(n)) == _lib.ENULL
        assert lib.simtgo_tile_allow_chained_windows(None, 1) == _lib.ENULL
    finally:
        lib.simtgo_tile_free(g)
    bad = lib.simtgo_tile_new()
    try:
        a = lib.simtgo_tile_input_device(bad, C.c_void_p(0x1000), 8)
        b = lib.simtgo_tile_input_device(bad, C.c_void_p(0x2000), 9)
        lib.simtgo_tile_add(bad, a, b)   # length mismatch: latched
        assert lib.simtgo_tile_reduce(bad, a, tile.SUM, C.c_void_p(0x1000), None,
                                      None) == _lib.EGRAPH
    finally:
        lib.simtgo_tile_free(bad)
