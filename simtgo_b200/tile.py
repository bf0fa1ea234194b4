"""The tile track (package tile, tile/tile.go and tile/run.go) over
libsimtgo_b200.so. The graph is recorded and lowered in the library (C++);
this module only keeps the host arrays alive and spells the Go API:

    g = tile.New()
    out = tile.Hypot(tile.FIR(tile.Scale(g.Input(re), 0.5), h), g.Input(im))
    vals = out.Materialize()                 # tile/run.go:20
    vals, launches = out.MaterializeStepwise()   # tile/run.go:89

Device-resident values (the `dev` field of tile/tile.go:46):
    a = g.InputDevice(tensor)               # a CUDA float32 tensor
    out.Run(dev_out, stream)                 # no upload, no download

Reductions (no counterpart in the reference, whose plan lists them as the
tile track's next step), fused into the same single pass:
    total = tile.Sum(tile.Mul(x, x)).Materialize()
    i, v = tile.ArgMax(out).Materialize()
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import GraphError, check

BlockSize = 256   # tile/tile.go:22
MaxTaps = 64      # tile/tile.go:25


class Graph:
    """tile.Graph: records a pipeline; nothing runs until a materialisation."""

    def __init__(self):
        self._L = _lib.load()
        self._h = self._L.simtgo_tile_new()
        self._keep = []   # host arrays the library points at

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            self._L.simtgo_tile_free(h)

    def _t(self, node):
        return Tensor(self, node)

    def Input(self, xs) -> "Tensor":
        a = np.ascontiguousarray(xs, dtype=np.float32)
        self._keep.append(a)
        return self._t(self._L.simtgo_tile_input(self._h, a.ctypes.data_as(C.c_void_p), len(a)))

    def InputDevice(self, t) -> "Tensor":
        import torch

        if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32
                and t.is_contiguous()):
            raise TypeError("tile: InputDevice takes a contiguous CUDA float32 tensor")
        self._keep.append(t)
        return self._t(self._L.simtgo_tile_input_device(self._h, C.c_void_p(t.data_ptr()),
                                                        t.numel()))

    def AllowChainedWindows(self, allow: bool = True):
        """No counterpart in the reference (which rejects a FIR of an
        expression holding a FIR): FIRs recorded afterwards may be chained,
        each reading the inner one as if it had been materialised first."""
        check(self._L.simtgo_tile_allow_chained_windows(self._h, 1 if allow else 0))
        return self

    def Err(self):
        """tile/tile.go:163: the first error recorded while building, or None."""
        if self._L.simtgo_tile_err(self._h) == 0:
            return None
        return GraphError(_lib.EGRAPH, self._L.simtgo_tile_err_string(self._h).decode())


class Tensor:
    def __init__(self, g: Graph, node: int):
        self.g = g
        self.node = node

    def Len(self) -> int:
        return self.g._L.simtgo_tile_len(self.g._h, self.node)

    def ProgramSize(self):
        """(instructions, inputs, windows) of the fused program: the analogue
        of Tensor.Source (tile/run.go:10), which compiles without running."""
        a, b, c = C.c_int32(), C.c_int32(), C.c_int32()
        check(self.g._L.simtgo_tile_program_size(self.g._h, self.node, C.byref(a), C.byref(b),
                                                 C.byref(c)))
        return a.value, b.value, c.value

    def Source(self) -> str:
        """tile/run.go:10: the program this tensor would be computed by,
        without running it (the listing of the lowered accumulator-machine
        program, one fused device instruction per line)."""
        L, g = self.g._L, self.g._h
        need = L.simtgo_tile_source(g, self.node, None, 0)
        check(need if need < 0 else 0)
        buf = C.create_string_buffer(need)
        L.simtgo_tile_source(g, self.node, buf, need)
        return buf.value.decode()

    def JITSource(self, reduce: int = -1, groups: int = 4, bulk: bool = True,
                  compile: bool = False) -> str:
        """The source of this tensor's specialised kernel (the lowered
        program as compile-time constants, tile_jit.cu) for `groups` float4
        groups per thread and bulk-copied or directly read inputs; with
        compile=True NVRTC also compiles it (no GPU needed) and a failure
        raises. groups=0 with a reduction of a chain of steps on one input:
        the streaming reduction's kernel for that chain."""
        L, g = self.g._L, self.g._h
        need = L.simtgo_tile_jit_source(g, self.node, reduce, groups, int(bulk), int(compile),
                                        None, 0)
        check(need if need < 0 else 0)
        buf = C.create_string_buffer(need)
        L.simtgo_tile_jit_source(g, self.node, reduce, groups, int(bulk), 0, buf, need)
        return buf.value.decode()

    def Materialize(self) -> np.ndarray:
        out = np.empty(max(self.Len(), 0), np.float32)
        check(self.g._L.simtgo_tile_materialize(self.g._h, self.node,
                                                out.ctypes.data_as(C.c_void_p), len(out)))
        return out

    def MaterializeStepwise(self):
        out = np.empty(max(self.Len(), 0), np.float32)
        n = C.c_int32()
        check(self.g._L.simtgo_tile_materialize_stepwise(
            self.g._h, self.node, out.ctypes.data_as(C.c_void_p), len(out), C.byref(n)))
        return out, n.value

    def Run(self, dev_out, stream=None, halo: int = 0):
        """Device-resident run into dev_out (CUDA float32 tensor of Len()
        elements); asynchronous on stream. halo: see simtgo_tile_run_shard."""
        sp = getattr(stream, "cuda_stream", stream)
        check(self.g._L.simtgo_tile_run_shard(self.g._h, self.node,
                                              C.c_void_p(dev_out.data_ptr()), dev_out.numel(),
                                              int(halo), sp))


SUM, MIN, MAX, ARGMAX = 0, 1, 2, 3


class Reduction:
    """A tensor reduced to one value in the fused pass: Sum (float32, in the
    library's fixed tree order), Min and Max (Go's min/max: NaN wins, -0 <
    +0), ArgMax (the first index of the maximum, with the maximum)."""

    def __init__(self, t: Tensor, kind: int):
        self.t = t
        self.kind = kind

    def Materialize(self):
        """Host inputs uploaded, one fused kernel: the value, or for ArgMax
        (index, value)."""
        v, i = C.c_float(), C.c_int64()
        check(self.t.g._L.simtgo_tile_reduce_materialize(self.t.g._h, self.t.node, self.kind,
                                                         C.byref(v), C.byref(i)))
        val = np.float32(v.value)
        return (i.value, val) if self.kind == ARGMAX else val

    def Run(self, dev_value, dev_index=None, stream=None):
        """Device-resident: dev_value (a CUDA float32 tensor of >= 1
        element) and, for ArgMax, dev_index (CUDA int64); asynchronous."""
        sp = getattr(stream, "cuda_stream", stream)
        di = C.c_void_p(dev_index.data_ptr()) if dev_index is not None else None
        check(self.t.g._L.simtgo_tile_reduce(self.t.g._h, self.t.node, self.kind,
                                             C.c_void_p(dev_value.data_ptr()), di, sp))

    def RunShard(self, comm, n_total: int, dev_value, dev_index=None, halo: int = 0,
                 stream=None):
        """This rank's part of the reduction of a signal sharded as
        ShardRange(n_total, nranks, rank) says (a collective over comm, a
        simtgo_comm handle): every rank gets the whole signal's result."""
        sp = getattr(stream, "cuda_stream", stream)
        di = C.c_void_p(dev_index.data_ptr()) if dev_index is not None else None
        check(self.t.g._L.simtgo_tile_reduce_shard(self.t.g._h, self.t.node, self.kind, int(halo),
                                                   int(n_total), comm,
                                                   C.c_void_p(dev_value.data_ptr()), di, sp))


def Sum(t: Tensor) -> Reduction:
    return Reduction(t, SUM)


def Min(t: Tensor) -> Reduction:
    return Reduction(t, MIN)


def Max(t: Tensor) -> Reduction:
    return Reduction(t, MAX)


def ArgMax(t: Tensor) -> Reduction:
    return Reduction(t, ARGMAX)


def SetJIT(mode: int) -> None:
    """How fused programs run: 0 the interpreter only, 1 (default) each
    program's specialised kernel when libnvrtc can be opened, 2 the
    specialised kernel or an error (simtgo_tile_set_jit)."""
    check(_lib.load().simtgo_tile_set_jit(mode))


def JITInfo():
    """(mode, NVRTC available, programs compiled, specialised launches,
    kernels served by the on-disk cache) of this process."""
    m, a = C.c_int32(), C.c_int32()
    c, n, h = C.c_int64(), C.c_int64(), C.c_int64()
    check(_lib.load().simtgo_tile_jit_info(C.byref(m), C.byref(a), C.byref(c), C.byref(n),
                                           C.byref(h)))
    return m.value, bool(a.value), c.value, n.value, h.value


def ShardRange(n_total: int, nranks: int, rank: int):
    """(start, length) of rank's shard for Reduction.RunShard: whole blocks
    of 2048, the last ranks possibly empty."""
    s, n = C.c_int64(), C.c_int64()
    check(_lib.load().simtgo_tile_shard_range(int(n_total), int(nranks), int(rank), C.byref(s),
                                              C.byref(n)))
    return s.value, n.value


def New() -> Graph:
    return Graph()


def Add(a: Tensor, b: Tensor) -> Tensor:
    return a.g._t(a.g._L.simtgo_tile_add(a.g._h, a.node, _same(a, b)))


def Mul(a: Tensor, b: Tensor) -> Tensor:
    return a.g._t(a.g._L.simtgo_tile_mul(a.g._h, a.node, _same(a, b)))


def Hypot(a: Tensor, b: Tensor) -> Tensor:
    return a.g._t(a.g._L.simtgo_tile_hypot(a.g._h, a.node, _same(a, b)))


def Scale(a: Tensor, k: float) -> Tensor:
    return a.g._t(a.g._L.simtgo_tile_scale(a.g._h, a.node, float(k)))


def Sqrt(a: Tensor) -> Tensor:
    return a.g._t(a.g._L.simtgo_tile_sqrt(a.g._h, a.node))


def Abs(a: Tensor) -> Tensor:
    return a.g._t(a.g._L.simtgo_tile_abs(a.g._h, a.node))


def FIR(a: Tensor, h) -> Tensor:
    hh = np.ascontiguousarray(h, dtype=np.float32)
    return a.g._t(a.g._L.simtgo_tile_fir(a.g._h, a.node, hh.ctypes.data_as(C.c_void_p), len(hh)))


def _same(a: Tensor, b: Tensor) -> int:
    # Operands from different graphs: the library sees an id it cannot
    # trust, so pass one it will refuse ("operands come from different graphs").
    return b.node if a.g is b.g else -1


__all__ = ["New", "Graph", "Tensor", "Add", "Mul", "Hypot", "Scale", "Sqrt", "Abs", "FIR",
           "BlockSize", "MaxTaps", "Reduction", "Sum", "Min", "Max", "ArgMax", "ShardRange",
           "SUM", "MIN", "MAX", "ARGMAX"]
