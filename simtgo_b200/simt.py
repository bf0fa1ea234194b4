"""The simt launch surface (simt/kernel.go) over libsimtgo_b200.so.

    k = simt.build("FIR")                 # simt.Build(dev, simtgo.Kernels(), "FIR")
    k.launch_n(n, 256, y, x, h)           # Kernel.LaunchN
    k.launch(grid, block, y, x, h)        # Kernel.Launch (synchronous)
    k.launch_dim((gx, gy), (16, 16), out, inp, w, h)   # Kernel.LaunchDim
    k.launch_on(stream, grid, block, ...) # Kernel.LaunchOn (asynchronous)
    simt.build("HistogramDyn").launch_shared(grid, block, tile, bins, x)
                                          # Kernel.LaunchShared (launch-sized tile)

Arguments follow the Go kernel's parameters minus the gpu.Ctx: device
buffers (CUDA torch tensors: the device pointer and element count travel,
as cuda.Slice.KernelArgs flattens a slice) and scalars. Host-side checks
mirror Kernel.launch: the argument count (ArgCountError, kernel.go:293), the
element type of each slice, and -- inside the library -- the block size
(BlockSizeError) and overlapping written slices (AliasError).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib
from ._lib import Band, Shape, check

# Kernel name -> parameters (name, kind). kind: f32/i32/i64/u8/bool slices,
# "band" slice, scalars "f32s", "i32s", "u32s", "shape" (by value).
KERNELS = {
    "VecAdd": [("c", "f32"), ("a", "f32"), ("b", "f32")],
    "Scale": [("y", "f32"), ("x", "f32"), ("k", "f32s")],
    "Magnitude": [("mag", "f32"), ("re", "f32"), ("im", "f32")],
    "MagnitudeFast": [("mag", "f32"), ("re", "f32"), ("im", "f32"), ("scale", "f32s")],
    "Softclip": [("y", "f32"), ("x", "f32"), ("threshold", "f32s")],
    "Classify": [("out", "f32"), ("x", "f32"), ("edges", "f32")],
    "BandGain": [("y", "f32"), ("x", "f32"), ("bands", "band"), ("cfg", "shape")],
    "Quantize": [("code", "i32"), ("energy", "i64"), ("clipped", "bool"), ("x", "f32"),
                 ("step", "f32s"), ("seed", "u32s")],
    "Gray": [("out", "u8"), ("rgb", "u8")],
    "Histogram": [("bins", "i32"), ("x", "i32")],
    "Transpose": [("out", "f32"), ("in", "f32"), ("w", "i32s"), ("h", "i32s")],
    "WarpReduceSum": [("out", "f32"), ("x", "f32")],
    "FIR": [("y", "f32"), ("x", "f32"), ("h", "f32")],
    # The DynProbe body (simt/shared_parity_cuda_test.go:117-138): a histogram
    # whose int32 tile is sized at the launch (Kernel.LaunchShared).
    "HistogramDyn": [("bins", "i32"), ("x", "i32")],
}

# Kernels with a launch-sized shared tile: launched through launch_shared only.
DYNAMIC = {"HistogramDyn"}

# kernels.FIRBlock, WarpReduceBlock, TransposeTile^2 (AssumeBlockDim).
REQUIRED_BLOCK = {"FIR": 256, "WarpReduceSum": 128, "Transpose": 256}

_DTYPES = {"f32": "float32", "i32": "int32", "i64": "int64", "u8": "uint8", "bool": "bool",
           "band": None}


class ArgCountError(TypeError):
    """simt.ArgCountError (simt/kernel.go:266-284)."""


class DynamicSharedError(TypeError):
    """simt.DynamicSharedError (simt/kernel.go:236-250): a kernel with a
    launch-sized tile launched without a size (dynamic=True), or one without
    such a tile handed a size (dynamic=False)."""

    def __init__(self, msg, dynamic):
        super().__init__(msg)
        self.dynamic = dynamic


class SharedMemoryError(_lib.SimtgoError):
    """simt.SharedMemoryError: the tile exceeds a block's shared memory."""


def _slice(t, kind, kernel, pname):
    """(device pointer, element count) of a CUDA tensor, checked for type."""
    import torch

    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"simt: {kernel}: {pname} must be a CUDA tensor (a device slice)")
    if not t.is_contiguous():
        raise TypeError(f"simt: {kernel}: {pname} must be contiguous")
    if kind == "band":
        if t.dtype != torch.float32 or t.numel() % 2:
            raise TypeError(f"simt: {kernel}: {pname} must hold (upper, gain) float32 pairs")
        return t.data_ptr(), t.numel() // 2
    want = getattr(torch, _DTYPES[kind])
    if t.dtype != want:
        raise TypeError(f"simt: {kernel}: {pname} is {t.dtype}, the kernel takes []{kind}")
    return t.data_ptr(), t.numel()


def _stream_ptr(stream):
    if stream is None:
        return None
    return getattr(stream, "cuda_stream", stream)


@dataclass
class Kernel:
    """simt.Kernel (simt/kernel.go:15-53) for one of the hot-path kernels."""

    name: str
    params: list
    required_block: int = 0

    def _call(self, grid, block, args, stream, sync, tile=None):
        dynamic = self.name in DYNAMIC
        if dynamic and tile is None:
            raise DynamicSharedError(f"simt: {self.name} has a launch-sized shared tile; launch "
                                     "it with launch_shared", True)
        if not dynamic and tile is not None:
            raise DynamicSharedError(f"simt: {self.name} has no launch-sized shared tile; "
                                     "launch_shared hands it a size it has no parameter for",
                                     False)
        if len(args) != len(self.params):
            raise ArgCountError(f"simt: {self.name} takes {len(self.params)} launch "
                                f"argument(s), got {len(args)}")
        L = _lib.load()
        flat = []
        keep = []
        for (pname, kind), a in zip(self.params, args):
            if kind == "f32s":
                flat.append(C.c_float(float(a)))
            elif kind == "i32s":
                flat.append(C.c_int32(int(a)))
            elif kind == "u32s":
                flat.append(C.c_uint32(int(a) & 0xFFFFFFFF))
            elif kind == "shape":
                s = a if isinstance(a, Shape) else Shape(*a)
                keep.append(s)
                flat.append(C.byref(s))
            else:
                p, n = _slice(a, kind, self.name, pname)
                flat += [C.c_void_p(p), C.c_int32(n)]
        sp = _stream_ptr(stream)
        fn = getattr(L, "simtgo_" + self.name)
        if self.name == "Transpose":
            (gx, gy), (bx, by) = grid, block
            rc = fn(*flat, gx, gy, bx, by, sp)
        elif dynamic:
            rc = fn(*flat, int(tile), int(grid), int(block), sp)
        else:
            rc = fn(*flat, int(grid), int(block), sp)
        if dynamic and rc == _lib.ESIZE:
            raise SharedMemoryError(rc, L.simtgo_last_error().decode(errors="replace"))
        check(rc)
        if sync:
            check(L.simtgo_stream_sync(sp))

    def launch(self, grid, block, *args, stream=None):
        """Kernel.Launch: runs and waits (LaunchSync)."""
        if self.name == "Transpose":
            return self.launch_dim((grid, 1), (block, 1), *args, stream=stream)
        self._call(grid, block, args, stream, True)

    def launch_dim(self, grid, block, *args, stream=None):
        """Kernel.LaunchDim over a 2-D grid (Transpose) or 1-D tuples."""
        if self.name != "Transpose":
            gx, gy = (tuple(grid) + (1,))[:2]
            bx, by = (tuple(block) + (1,))[:2]
            if gy != 1 or by != 1:
                raise ValueError(f"simt: {self.name} reads one axis; launch it 1-D")
            return self._call(gx, bx, args, stream, True)
        self._call(tuple(grid)[:2], tuple(block)[:2], args, stream, True)

    def launch_n(self, n, block, *args, stream=None):
        """Kernel.LaunchN: enough blocks to cover n threads."""
        return self.launch((n + block - 1) // block, block, *args, stream=stream)

    def launch_shared(self, grid, block, tile, *args, stream=None):
        """Kernel.LaunchShared: runs with a tile of `tile` elements and waits."""
        self._call(grid, block, args, stream, True, tile=tile)

    def launch_on(self, stream, grid, block, *args):
        """Kernel.LaunchOn: queued on stream, not waited for."""
        if stream is None:
            raise ValueError(f"simt: {self.name}: LaunchOn needs a stream; use Launch for the "
                             "synchronous form")
        if self.name == "Transpose":
            return self._call(tuple(grid)[:2], tuple(block)[:2], args, stream, False)
        self._call(grid, block, args, stream, False)


def build(name: str) -> Kernel:
    """simt.Build for a kernel of package kernels: nothing to compile (the
    kernels are built ahead of time for sm_100a); checks the library and the
    device."""
    if name not in KERNELS:
        raise KeyError(f"simt: no kernel {name!r} in package kernels")
    L = _lib.load()
    sm, ma, mi = C.c_int32(), C.c_int32(), C.c_int32()
    check(L.simtgo_device_info(C.byref(sm), C.byref(ma), C.byref(mi)))
    return Kernel(name, KERNELS[name], REQUIRED_BLOCK.get(name, 0))


def stream_sync(stream=None):
    check(_lib.load().simtgo_stream_sync(_stream_ptr(stream)))


def bands_tensor(bands, device="cuda"):
    """[]Band as a device buffer of (upper, gain) float32 pairs."""
    import torch

    return torch.tensor([v for b in bands for v in b], dtype=torch.float32, device=device)


__all__ = ["build", "Kernel", "KERNELS", "Band", "Shape", "ArgCountError", "DynamicSharedError",
           "SharedMemoryError", "stream_sync", "bands_tensor"]
