"""Test infrastructure: ctypes bindings for the oracle (oracle/liboracle.so)
and, when it was built, the reference's generated kernels compiled for the
host (oracle/_ref/libref.so).

Only tests, the smoke check and the benchmark's CPU-baseline leg import this
module. Every wrapper takes numpy arrays and returns numpy arrays (or the
status code), so a test reads like the reference's parity tests
(simt/parity_test.go): run the oracle, run the device, compare.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib
import subprocess

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent.parent
ORACLE_DIR = ROOT / "oracle"
ORACLE_SO = ORACLE_DIR / "liboracle.so"
REF_SO = ORACLE_DIR / "_ref" / "libref.so"

_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_i64p = C.POINTER(C.c_int64)
_u8p = C.POINTER(C.c_uint8)
_i32 = C.c_int32
_i64 = C.c_int64


def _ptr(a: np.ndarray | None, ty):
    if a is None:
        return C.cast(None, ty)
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ty)


class Band(C.Structure):
    """kernels/bandgain.go:9-12 Band."""

    _fields_ = [("upper", C.c_float), ("gain", C.c_float)]


class Shape(C.Structure):
    """kernels/bandgain.go:26-30 Shape."""

    _fields_ = [("floor_gain", C.c_float), ("count", C.c_int32), ("bias", C.c_double)]


class TileNode(C.Structure):
    _fields_ = [
        ("kind", C.c_int32),
        ("a", C.c_int32),
        ("b", C.c_int32),
        ("scale", C.c_float),
        ("data", _f32p),
        ("taps", _f32p),
        ("ntaps", C.c_int32),
    ]


def _build_oracle():
    if not ORACLE_SO.exists():
        subprocess.run(["make", "-C", str(ORACLE_DIR), "all"], check=True,
                       stdout=subprocess.DEVNULL)


_oracle = None
_ref = None


def oracle() -> C.CDLL:
    global _oracle
    if _oracle is None:
        _build_oracle()
        lib = C.CDLL(str(ORACLE_SO))
        lib.oracle_hypot.restype = C.c_float
        lib.oracle_hypot.argtypes = [C.c_float, C.c_float]
        _oracle = lib
    return _oracle


def ref():
    """The reference's own kernels built for the host, or None."""
    global _ref
    if _ref is None and REF_SO.exists():
        _ref = C.CDLL(str(REF_SO))
    return _ref


def set_threads(n: int):
    oracle().oracle_set_threads(int(n))
    r = ref()
    if r is not None:
        r.ref_set_workers(int(n))


# ---- oracle wrappers (mirror include/simtgo_b200.h minus the stream) -------

def vecadd(a, b, grid, block, n_out=None):
    n_out = len(a) if n_out is None else n_out
    c = np.zeros(n_out, np.float32)
    rc = oracle().oracle_vecadd(_ptr(c, _f32p), _i32(len(c)), _ptr(a, _f32p), _i32(len(a)),
                                _ptr(b, _f32p), _i32(len(b)), _i64(grid), _i64(block))
    return rc, c


def scale(x, k, grid, block):
    y = np.zeros(len(x), np.float32)
    rc = oracle().oracle_scale(_ptr(y, _f32p), _i32(len(y)), _ptr(x, _f32p), _i32(len(x)),
                               C.c_float(k), _i64(grid), _i64(block))
    return rc, y


def magnitude(re, im, grid, block):
    m = np.zeros(len(re), np.float32)
    rc = oracle().oracle_magnitude(_ptr(m, _f32p), _i32(len(m)), _ptr(re, _f32p), _i32(len(re)),
                                   _ptr(im, _f32p), _i32(len(im)), _i64(grid), _i64(block))
    return rc, m


def magnitudefast(re, im, s, grid, block):
    m = np.zeros(len(re), np.float32)
    rc = oracle().oracle_magnitudefast(_ptr(m, _f32p), _i32(len(m)), _ptr(re, _f32p),
                                       _i32(len(re)), _ptr(im, _f32p), _i32(len(im)),
                                       C.c_float(s), _i64(grid), _i64(block))
    return rc, m


def magnitudefast_interleaved(z, s, grid, block):
    m = np.zeros(len(z) // 2, np.float32)
    rc = oracle().oracle_magnitudefast_interleaved(_ptr(m, _f32p), _i32(len(m)), _ptr(z, _f32p),
                                                   _i32(len(z)), C.c_float(s), _i64(grid),
                                                   _i64(block))
    return rc, m


def softclip(x, t, grid, block):
    y = np.zeros(len(x), np.float32)
    rc = oracle().oracle_softclip(_ptr(y, _f32p), _i32(len(y)), _ptr(x, _f32p), _i32(len(x)),
                                  C.c_float(t), _i64(grid), _i64(block))
    return rc, y


def classify(x, edges, grid, block):
    out = np.zeros(len(x), np.float32)
    rc = oracle().oracle_classify(_ptr(out, _f32p), _i32(len(out)), _ptr(x, _f32p),
                                  _i32(len(x)), _ptr(edges, _f32p), _i32(len(edges)),
                                  _i64(grid), _i64(block))
    return rc, out


def bands_array(bands):
    arr = (Band * max(1, len(bands)))()
    for i, (u, g) in enumerate(bands):
        arr[i].upper, arr[i].gain = u, g
    return arr


def bandgain(x, bands, floor_gain, count, bias, grid, block):
    y = np.zeros(len(x), np.float32)
    arr = bands_array(bands)
    cfg = Shape(floor_gain, count, bias)
    rc = oracle().oracle_bandgain(_ptr(y, _f32p), _i32(len(y)), _ptr(x, _f32p), _i32(len(x)),
                                  arr, _i32(len(bands)), C.byref(cfg), _i64(grid), _i64(block))
    return rc, y


def quantize(x, step, seed, grid, block):
    n = len(x)
    code = np.zeros(n, np.int32)
    energy = np.zeros(n, np.int64)
    clipped = np.zeros(n, np.uint8)
    rc = oracle().oracle_quantize(_ptr(code, _i32p), _i32(n), _ptr(energy, _i64p), _i32(n),
                                  _ptr(clipped, _u8p), _i32(n), _ptr(x, _f32p), _i32(n),
                                  C.c_float(step), C.c_uint32(seed), _i64(grid), _i64(block))
    return rc, code, energy, clipped


def gray(rgb, n_out, grid, block):
    out = np.zeros(n_out, np.uint8)
    rc = oracle().oracle_gray(_ptr(out, _u8p), _i32(n_out), _ptr(rgb, _u8p), _i32(len(rgb)),
                              _i64(grid), _i64(block))
    return rc, out


def histogram(x, n_bins, grid, block, bins=None):
    bins = np.zeros(n_bins, np.int32) if bins is None else bins.copy()
    rc = oracle().oracle_histogram(_ptr(bins, _i32p), _i32(len(bins)), _ptr(x, _i32p),
                                   _i32(len(x)), _i64(grid), _i64(block))
    return rc, bins


def histogram_dyn(x, n_bins, tile, grid, block, bins=None):
    bins = np.zeros(n_bins, np.int32) if bins is None else bins.copy()
    rc = oracle().oracle_histogram_dyn(_ptr(bins, _i32p), _i32(len(bins)), _ptr(x, _i32p),
                                       _i32(len(x)), _i32(tile), _i64(grid), _i64(block))
    return rc, bins


def histogram_shard(x, n_bins=256, bins=None):
    bins = np.zeros(n_bins, np.int32) if bins is None else bins.copy()
    rc = oracle().oracle_histogram_shard(_ptr(bins, _i32p), _i32(len(bins)), _ptr(x, _i32p),
                                         _i64(len(x)))
    return rc, bins


def transpose(inp, w, h, gx, gy, bx=16, by=16, out_len=None):
    out = np.zeros(w * h if out_len is None else out_len, np.float32)
    rc = oracle().oracle_transpose(_ptr(out, _f32p), _i32(len(out)), _ptr(inp, _f32p),
                                   _i32(len(inp)), _i32(w), _i32(h), _i64(gx), _i64(gy),
                                   _i64(bx), _i64(by))
    return rc, out


def warpreducesum(x, n_out, grid, block=128):
    out = np.zeros(n_out, np.float32)
    rc = oracle().oracle_warpreducesum(_ptr(out, _f32p), _i32(n_out), _ptr(x, _f32p),
                                       _i32(len(x)), _i64(grid), _i64(block))
    return rc, out


def fir(x, h, grid, block=256, n_out=None, fused=False):
    y = np.zeros(len(x) if n_out is None else n_out, np.float32)
    fn = oracle().oracle_fir_fma if fused else oracle().oracle_fir
    rc = fn(_ptr(y, _f32p), _i32(len(y)), _ptr(x, _f32p), _i32(len(x)), _ptr(h, _f32p),
            _i32(len(h)), _i64(grid), _i64(block))
    return rc, y


def fir_shard(x, halo, h, n_out, fused=True):
    y = np.zeros(n_out, np.float32)
    fn = oracle().oracle_fir_shard if fused else oracle().oracle_fir_shard_runcpu
    rc = fn(_ptr(y, _f32p), _i64(n_out), _ptr(x, _f32p), _i64(len(x)), _i64(halo),
            _ptr(h, _f32p), _i32(len(h)))
    return rc, y


TILE_KINDS = {"input": 0, "scale": 1, "add": 2, "mul": 3, "sqrt": 4, "abs": 5, "hypot": 6,
              "fir": 7}


def tile_eval(nodes, root, n, halo=0):
    """nodes: list of dicts {kind, a, b, scale, data, taps} in creation order."""
    arr = (TileNode * len(nodes))()
    keep = []
    for i, nd in enumerate(nodes):
        arr[i].kind = TILE_KINDS[nd["kind"]]
        arr[i].a = nd.get("a", -1)
        arr[i].b = nd.get("b", -1)
        arr[i].scale = nd.get("scale", 0.0)
        if nd.get("data") is not None:
            d = np.ascontiguousarray(nd["data"], np.float32)
            keep.append(d)
            arr[i].data = _ptr(d, _f32p)
        if nd.get("taps") is not None:
            t = np.ascontiguousarray(nd["taps"], np.float32)
            keep.append(t)
            arr[i].taps = _ptr(t, _f32p)
            arr[i].ntaps = len(t)
    out = np.zeros(n, np.float32)
    rc = oracle().oracle_tile_eval(arr, _i32(len(nodes)), _i32(root), _ptr(out, _f32p), _i32(n),
                                   _i32(halo))
    return rc, out


def tile_eval_chunked(nodes, root, n, reach, chunk=1 << 22, threads=None):
    """tile_eval over n elements as independent chunks evaluated in parallel
    (the ctypes call releases the GIL): chunk c takes its inputs from
    [c0 - h, c0 + len) with h = min(reach, c0), so every window of the graph
    (reach = the most samples any output reads below itself) sees the same
    values as in one whole evaluation. Input nodes whose data has n elements
    are sliced; the others (taps) are passed whole."""
    from concurrent.futures import ThreadPoolExecutor

    out = np.empty(n, np.float32)
    starts = list(range(0, n, chunk))

    def one(c0):
        h = min(reach, c0)
        cn = min(chunk, n - c0)
        sub = []
        for nd in nodes:
            d = nd.get("data")
            if nd["kind"] == "input" and d is not None and len(d) == n:
                nd = dict(nd, data=d[c0 - h: c0 + cn])
            sub.append(nd)
        rc, o = tile_eval(sub, root, cn, h)
        assert rc == 0, rc
        out[c0: c0 + cn] = o

    with ThreadPoolExecutor(threads or os.cpu_count() or 1) as ex:
        list(ex.map(one, starts))
    return out


TILE_REDUCE = {"sum": 0, "min": 1, "max": 2, "argmax": 3}


def tile_reduce(x, kind, idx_base=0):
    """(value, index) of the library's tile reduction `kind` over x."""
    x = np.ascontiguousarray(x, np.float32)
    v, i = C.c_float(), C.c_int64()
    rc = oracle().oracle_tile_reduce(_ptr(x, _f32p), _i64(len(x)), _i32(TILE_REDUCE[kind]),
                                     _i64(idx_base), C.byref(v), C.byref(i))
    assert rc == 0, rc
    return np.float32(v.value), i.value


def tile_reduce_partials(x, kind, idx_base=0):
    """The first level: one (value, index) per block of 2048."""
    x = np.ascontiguousarray(x, np.float32)
    m = (len(x) + 2047) // 2048
    pv, pi = np.zeros(max(m, 1), np.float32), np.zeros(max(m, 1), np.int64)
    rc = oracle().oracle_tile_reduce_partials(_ptr(x, _f32p), _i64(len(x)),
                                              _i32(TILE_REDUCE[kind]), _i64(idx_base),
                                              _ptr(pv, _f32p), _ptr(pi, _i64p))
    assert rc == 0, rc
    return pv[:m], pi[:m]


def tile_reduce_levels(pv, pi, kind):
    pv = np.ascontiguousarray(pv, np.float32)
    pi = np.ascontiguousarray(pi, np.int64)
    v, i = C.c_float(), C.c_int64()
    rc = oracle().oracle_tile_reduce_levels(_ptr(pv, _f32p), _ptr(pi, _i64p), _i64(len(pv)),
                                            _i32(TILE_REDUCE[kind]), C.byref(v), C.byref(i))
    assert rc == 0, rc
    return np.float32(v.value), i.value


# ---- the reference's kernels built for the host (pinning only) -------------

def ref_call(name, *args):
    r = ref()
    if r is None:
        raise RuntimeError("oracle/_ref/libref.so was not built (needs the reference tree)")
    return getattr(r, "ref_" + name)(*args)


def f32p(a):
    return _ptr(a, _f32p)


def i32p(a):
    return _ptr(a, _i32p)


def i64p(a):
    return _ptr(a, _i64p)


def u8p(a):
    return _ptr(a, _u8p)


def build_env_threads() -> int:
    return int(os.environ.get("ORACLE_THREADS", "0")) or os.cpu_count() or 1
