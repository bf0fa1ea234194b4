"""ctypes binding of libsimtgo_b200.so (include/simtgo_b200.h).

The shared library is the product; this module only declares its symbols.
There is no fallback: if the library is missing or cannot be loaded, every
call raises. Set SIMTGO_B200_LIB to load a library from another path.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

PKG = pathlib.Path(__file__).resolve().parent
DEFAULT_LIB = PKG / "libsimtgo_b200.so"

SIMTGO_OK = 0
ENULL, ELENGTH, EBLOCK, EALIAS, ELAUNCH, ETAPS, EGRAPH, EDEVICE, ECOMM, ESIZE, EARG = (
    -1, -2, -3, -4, -5, -6, -7, -8, -9, -10, -11)

_vp = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_u32 = C.c_uint32
_f32 = C.c_float


class Band(C.Structure):
    """kernels/bandgain.go:9-12."""
    _fields_ = [("upper", C.c_float), ("gain", C.c_float)]


class Shape(C.Structure):
    """kernels/bandgain.go:26-30 (Floor, Count, Bias: 16 bytes)."""
    _fields_ = [("floor_gain", C.c_float), ("count", C.c_int32), ("bias", C.c_double)]


# name -> argtypes (restype is int unless listed in _RESTYPES)
_SIGS = {
    "simtgo_last_error": [],
    "simtgo_version": [],
    "simtgo_device_info": [C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_i32)],
    "simtgo_stream_sync": [_vp],
    "simtgo_shutdown": [],
    "simtgo_VecAdd": [_vp, _i32, _vp, _i32, _vp, _i32, _i32, _i32, _vp],
    "simtgo_Scale": [_vp, _i32, _vp, _i32, _f32, _i32, _i32, _vp],
    "simtgo_Magnitude": [_vp, _i32, _vp, _i32, _vp, _i32, _i32, _i32, _vp],
    "simtgo_MagnitudeFast": [_vp, _i32, _vp, _i32, _vp, _i32, _f32, _i32, _i32, _vp],
    "simtgo_MagnitudeFast_interleaved": [_vp, _i32, _vp, _i32, _f32, _i32, _i32, _vp],
    "simtgo_Softclip": [_vp, _i32, _vp, _i32, _f32, _i32, _i32, _vp],
    "simtgo_Classify": [_vp, _i32, _vp, _i32, _vp, _i32, _i32, _i32, _vp],
    "simtgo_BandGain": [_vp, _i32, _vp, _i32, _vp, _i32, C.POINTER(Shape), _i32, _i32, _vp],
    "simtgo_Quantize": [_vp, _i32, _vp, _i32, _vp, _i32, _vp, _i32, _f32, _u32, _i32, _i32, _vp],
    "simtgo_Gray": [_vp, _i32, _vp, _i32, _i32, _i32, _vp],
    "simtgo_Histogram": [_vp, _i32, _vp, _i32, _i32, _i32, _vp],
    "simtgo_HistogramDyn": [_vp, _i32, _vp, _i32, _i32, _i32, _i32, _vp],
    "simtgo_Transpose": [_vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp],
    "simtgo_WarpReduceSum": [_vp, _i32, _vp, _i32, _i32, _i32, _vp],
    "simtgo_FIR": [_vp, _i32, _vp, _i32, _vp, _i32, _i32, _i32, _vp],
    "simtgo_FIR_shard": [_vp, _i64, _vp, _i64, _i64, _vp, _i32, _vp],
    "simtgo_FIR_shard_host": [_vp, _i64, _vp, _i64, _i64, _vp, _i32, _vp],
    "simtgo_Histogram_shard": [_vp, _i32, _vp, _i64, _vp],
    "simtgo_comm_unique_id": [C.c_char_p],
    "simtgo_comm_init": [C.POINTER(_vp), C.c_char_p, _i32, _i32],
    "simtgo_comm_destroy": [_vp],
    "simtgo_comm_allreduce_i32": [_vp, _vp, _i32, _vp],
    "simtgo_Histogram_allreduce": [_vp, _vp, _i32, _vp, _i64, _vp],
    "simtgo_Histogram_allreduce_fused": [_vp, _vp, _i32, _vp, _i64, _vp],
    "simtgo_Histogram_allreduce_fused_overwrite": [_vp, _vp, _i32, _vp, _i64, _vp],
    "simtgo_tile_new": [],
    "simtgo_tile_free": [_vp],
    "simtgo_tile_input": [_vp, _vp, _i32],
    "simtgo_tile_input_device": [_vp, _vp, _i32],
    "simtgo_tile_add": [_vp, _i32, _i32],
    "simtgo_tile_mul": [_vp, _i32, _i32],
    "simtgo_tile_hypot": [_vp, _i32, _i32],
    "simtgo_tile_scale": [_vp, _i32, _f32],
    "simtgo_tile_sqrt": [_vp, _i32],
    "simtgo_tile_abs": [_vp, _i32],
    "simtgo_tile_fir": [_vp, _i32, _vp, _i32],
    "simtgo_tile_allow_chained_windows": [_vp, _i32],
    "simtgo_tile_len": [_vp, _i32],
    "simtgo_tile_err": [_vp],
    "simtgo_tile_err_string": [_vp],
    "simtgo_tile_program_size": [_vp, _i32, C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_i32)],
    "simtgo_tile_source": [_vp, _i32, C.c_char_p, _i32],
    "simtgo_tile_set_jit": [_i32],
    "simtgo_tile_jit_info": [C.POINTER(_i32), C.POINTER(_i32), C.POINTER(C.c_int64),
                             C.POINTER(C.c_int64), C.POINTER(C.c_int64)],
    "simtgo_tile_jit_source": [_vp, _i32, _i32, _i32, _i32, _i32, C.c_char_p, _i32],
    "simtgo_tile_materialize": [_vp, _i32, _vp, _i32],
    "simtgo_tile_materialize_stepwise": [_vp, _i32, _vp, _i32, C.POINTER(_i32)],
    "simtgo_tile_run": [_vp, _i32, _vp, _i32, _vp],
    "simtgo_tile_run_shard": [_vp, _i32, _vp, _i32, _i32, _vp],
    "simtgo_tile_run_stepwise_noalloc": [_vp, _i32, _vp, _i32, _vp],
    "simtgo_tile_reduce": [_vp, _i32, _i32, _vp, _vp, _vp],
    "simtgo_tile_reduce_materialize": [_vp, _i32, _i32, C.POINTER(C.c_float),
                                       C.POINTER(C.c_int64)],
    "simtgo_tile_shard_range": [C.c_int64, _i32, _i32, C.POINTER(C.c_int64),
                                C.POINTER(C.c_int64)],
    "simtgo_tile_reduce_shard": [_vp, _i32, _i32, _i32, C.c_int64, _vp, _vp, _vp, _vp],
}
_RESTYPES = {
    "simtgo_last_error": C.c_char_p,
    "simtgo_version": C.c_char_p,
    "simtgo_tile_new": _vp,
    "simtgo_tile_free": None,
    "simtgo_tile_err_string": C.c_char_p,
}

_lib = None


def lib_path() -> pathlib.Path:
    return pathlib.Path(os.environ.get("SIMTGO_B200_LIB", str(DEFAULT_LIB)))


def load() -> C.CDLL:
    """Loads the library (once). Raises if it is missing: there is no
    CPU fallback."""
    global _lib
    if _lib is None:
        p = lib_path()
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with `python -m simtgo_b200.build` "
                "(nvcc, sm_100a); simtgo_b200 has no CPU fallback")
        lib = C.CDLL(str(p))
        missing = [n for n in _SIGS if not hasattr(lib, n)]
        if missing:
            raise RuntimeError(f"{p} does not export {', '.join(missing)}")
        for name, args in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, C.c_int)
        _lib = lib
    return _lib


def exported_symbols():
    return list(_SIGS)


class SimtgoError(RuntimeError):
    """A non-zero status from the library, with its message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class BlockSizeError(SimtgoError):
    """simt.BlockSizeError (simt/kernel.go:220-229)."""


class AliasError(SimtgoError):
    """simt.AliasError / tile.AliasError."""


class LengthError(SimtgoError):
    """A slice shorter than the launch reads: gpu.RunCPU's index-out-of-range."""


class TapsError(SimtgoError):
    pass


class GraphError(SimtgoError):
    """A latched tile graph error (tile/tile.go:78-82)."""


_CLASSES = {EBLOCK: BlockSizeError, EALIAS: AliasError, ELENGTH: LengthError, ETAPS: TapsError,
            EGRAPH: GraphError}


def check(rc: int):
    if rc != 0:
        msg = load().simtgo_last_error().decode(errors="replace")
        raise _CLASSES.get(rc, SimtgoError)(rc, msg)
    return rc
