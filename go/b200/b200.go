// Package b200 binds libsimtgo_b200.so -- simtgo's data-parallel hot path
// (the kernels of package kernels and the tile track's fused graph) built
// for B200 (sm_100a) -- with purego, without cgo, the way simtgo already
// binds libcuda and libnvrtc (cuda/loader_cuda.go:169-189).
//
// Every function of include/simtgo_b200.h has one variable here, bound by
// Load. Device memory is passed as uintptr (a cuda.DevPtr from cuMemAlloc in
// the device's primary context, which the library's CUDA runtime shares),
// host memory as unsafe.Pointer or a typed pointer, and a stream as the
// uintptr of its CUstream (0: the legacy default stream). C int and int32_t
// are int32, int64_t int64, float float32; a status is an int32, 0 for
// success (Check turns it into an error carrying the library's message).
//
// Calls must come from the goroutine that holds the OS thread with the
// device's context current -- inside simtgo's Context.call
// (cuda/driver_cuda.go:221-230) -- like every other driver call simtgo makes.
package b200

import (
	"errors"
	"fmt"
	"os"
	"sync"
	"unsafe"

	"github.com/ebitengine/purego"
)

// Status codes (include/simtgo_b200.h). Positive values are a cudaError_t,
// or 1000 + an ncclResult_t, passed through.
const (
	OK      int32 = 0
	ENull   int32 = -1  // a null pointer where the extent needs memory
	ELength int32 = -2  // a slice too short for the covered extent (gpu.RunCPU would panic)
	EBlock  int32 = -3  // simt.BlockSizeError (simt/kernel.go:220-229)
	EAlias  int32 = -4  // simt.AliasError / tile.AliasError
	ELaunch int32 = -5  // a grid or block the driver would refuse
	ETaps   int32 = -6  // FIR taps outside what the kernel can stage
	EGraph  int32 = -7  // a latched tile graph error (tile/tile.go:78)
	EDevice int32 = -8  // no usable device, wrong architecture, or a bounded wait gave up
	EComm   int32 = -9  // communicator misuse, or NCCL not loadable
	ESize   int32 = -10 // a size beyond a documented library maximum
	EArg    int32 = -11 // any other refused argument
)

// Limits and reduction kinds (include/simtgo_b200.h).
const (
	FIRShardMaxTaps           = 1024
	TileBlockSize             = 256     // tile/tile.go:22
	TileMaxTaps               = 64      // tile/tile.go:25
	TileNoAllocScratchFloats  = 1 << 22 // simtgo_tile_run_stepwise_noalloc's fixed scratch
	TileSum             int32 = 0
	TileMin             int32 = 1
	TileMax             int32 = 2
	TileArgMax          int32 = 3
)

// Band mirrors kernels.Band (kernels/bandgain.go:9-12) and simtgo_band: 8 bytes.
type Band struct {
	Upper float32
	Gain  float32
}

// Shape mirrors kernels.Shape (kernels/bandgain.go:26-30) and simtgo_shape:
// 16 bytes (float32, int32, float64).
type Shape struct {
	Floor float32
	Count int32
	Bias  float64
}

// The library's entry points, one variable per function of
// include/simtgo_b200.h, bound by Load.
var (
	// Library-wide.
	LastError  func() string
	Version    func() string
	DeviceInfo func(smCount *int32, ccMajor *int32, ccMinor *int32) int32
	StreamSync func(stream uintptr) int32
	Shutdown   func() int32

	// Package kernels: (device pointer, int32 length) per slice, as
	// cuda.Slice.KernelArgs flattens them (cuda/slice_cuda.go:94), then the
	// launch's grid and block and the stream.
	VecAdd                   func(c uintptr, cLen int32, a uintptr, aLen int32, b uintptr, bLen int32, grid int32, block int32, stream uintptr) int32
	Scale                    func(y uintptr, yLen int32, x uintptr, xLen int32, k float32, grid int32, block int32, stream uintptr) int32
	Magnitude                func(mag uintptr, magLen int32, re uintptr, reLen int32, im uintptr, imLen int32, grid int32, block int32, stream uintptr) int32
	MagnitudeFast            func(mag uintptr, magLen int32, re uintptr, reLen int32, im uintptr, imLen int32, scale float32, grid int32, block int32, stream uintptr) int32
	MagnitudeFastInterleaved func(mag uintptr, magLen int32, z uintptr, zLen int32, scale float32, grid int32, block int32, stream uintptr) int32
	Softclip                 func(y uintptr, yLen int32, x uintptr, xLen int32, threshold float32, grid int32, block int32, stream uintptr) int32
	Classify                 func(out uintptr, outLen int32, x uintptr, xLen int32, edges uintptr, edgesLen int32, grid int32, block int32, stream uintptr) int32
	BandGain                 func(y uintptr, yLen int32, x uintptr, xLen int32, bands uintptr, bandsLen int32, cfg *Shape, grid int32, block int32, stream uintptr) int32
	Quantize                 func(code uintptr, codeLen int32, energy uintptr, energyLen int32, clipped uintptr, clippedLen int32, x uintptr, xLen int32, step float32, seed uint32, grid int32, block int32, stream uintptr) int32
	Gray                     func(out uintptr, outLen int32, rgb uintptr, rgbLen int32, grid int32, block int32, stream uintptr) int32
	Histogram                func(bins uintptr, binsLen int32, x uintptr, xLen int32, grid int32, block int32, stream uintptr) int32
	HistogramDyn             func(bins uintptr, binsLen int32, x uintptr, xLen int32, tileLen int32, grid int32, block int32, stream uintptr) int32
	Transpose                func(out uintptr, outLen int32, in uintptr, inLen int32, w int32, h int32, gridX int32, gridY int32, blockX int32, blockY int32, stream uintptr) int32
	WarpReduceSum            func(out uintptr, outLen int32, x uintptr, xLen int32, grid int32, block int32, stream uintptr) int32
	FIR                      func(y uintptr, yLen int32, x uintptr, xLen int32, h uintptr, hLen int32, grid int32, block int32, stream uintptr) int32

	// The long and sharded forms (64-bit extents).
	FIRShard       func(y uintptr, yLen int64, x uintptr, xLen int64, halo int64, h uintptr, taps int32, stream uintptr) int32
	FIRShardHost   func(y unsafe.Pointer, yLen int64, x unsafe.Pointer, xLen int64, halo int64, h unsafe.Pointer, taps int32, stream uintptr) int32
	HistogramShard func(bins uintptr, binsLen int32, x uintptr, xLen int64, stream uintptr) int32

	// The communicator and the sharded histogram's all-reduce.
	CommUniqueID                    func(outID *[128]byte) int32
	CommInit                        func(out *uintptr, id *[128]byte, nranks int32, rank int32) int32
	CommDestroy                     func(comm uintptr) int32
	CommAllreduceI32                func(comm uintptr, buf uintptr, n int32, stream uintptr) int32
	HistogramAllreduce              func(comm uintptr, bins uintptr, binsLen int32, x uintptr, xLen int64, stream uintptr) int32
	HistogramAllreduceFused         func(comm uintptr, bins uintptr, binsLen int32, x uintptr, xLen int64, stream uintptr) int32
	HistogramAllreduceFusedOverwrite func(comm uintptr, bins uintptr, binsLen int32, x uintptr, xLen int64, stream uintptr) int32

	// The tile track (package tile): a graph handle is a uintptr, a tensor
	// its node id (int32, -1 on a latched error).
	TileNew                   func() uintptr
	TileFree                  func(g uintptr)
	TileInput                 func(g uintptr, host unsafe.Pointer, n int32) int32
	TileInputDevice           func(g uintptr, dev uintptr, n int32) int32
	TileAdd                   func(g uintptr, a int32, b int32) int32
	TileMul                   func(g uintptr, a int32, b int32) int32
	TileHypot                 func(g uintptr, a int32, b int32) int32
	TileScale                 func(g uintptr, a int32, k float32) int32
	TileSqrt                  func(g uintptr, a int32) int32
	TileAbs                   func(g uintptr, a int32) int32
	TileFIR                   func(g uintptr, a int32, h unsafe.Pointer, taps int32) int32
	TileAllowChainedWindows   func(g uintptr, allow int32) int32
	TileLen                   func(g uintptr, t int32) int32
	TileErr                   func(g uintptr) int32
	TileErrString             func(g uintptr) string
	TileProgramSize           func(g uintptr, t int32, nInstructions *int32, nInputs *int32, nWindows *int32) int32
	TileSource                func(g uintptr, t int32, buf unsafe.Pointer, capacity int32) int32
	TileSetJIT                func(mode int32) int32
	TileJITInfo               func(mode *int32, available *int32, compiled *int64, launches *int64, cacheHits *int64) int32
	TileJITSource             func(g uintptr, t int32, reduce int32, groups int32, bulk int32, compile int32, buf unsafe.Pointer, capacity int32) int32
	TileMaterialize           func(g uintptr, t int32, hostOut unsafe.Pointer, outLen int32) int32
	TileMaterializeStepwise   func(g uintptr, t int32, hostOut unsafe.Pointer, outLen int32, launches *int32) int32
	TileRun                   func(g uintptr, t int32, devOut uintptr, outLen int32, stream uintptr) int32
	TileRunShard              func(g uintptr, t int32, devOut uintptr, outLen int32, halo int32, stream uintptr) int32
	TileRunStepwiseNoalloc    func(g uintptr, t int32, devOut uintptr, outLen int32, stream uintptr) int32
	TileReduce                func(g uintptr, t int32, kind int32, devValue uintptr, devIndex uintptr, stream uintptr) int32
	TileReduceMaterialize     func(g uintptr, t int32, kind int32, value *float32, index *int64) int32
	TileShardRange            func(nTotal int64, nranks int32, rank int32, start *int64, length *int64) int32
	TileReduceShard           func(g uintptr, t int32, kind int32, halo int32, nTotal int64, comm uintptr, devValue uintptr, devIndex uintptr, stream uintptr) int32
)

var (
	loadOnce sync.Once
	loadErr  error
)

// Load opens the library (SIMTGO_B200_LIB overrides path) and binds every
// entry point. Later calls return the first call's result.
func Load(path string) error {
	loadOnce.Do(func() {
		if p := os.Getenv("SIMTGO_B200_LIB"); p != "" {
			path = p
		}
		h, err := purego.Dlopen(path, purego.RTLD_NOW|purego.RTLD_GLOBAL)
		if err != nil {
			loadErr = fmt.Errorf("b200: %w", err)
			return
		}
		bind(h)
	})
	return loadErr
}

func bind(h uintptr) {
	purego.RegisterLibFunc(&LastError, h, "simtgo_last_error")
	purego.RegisterLibFunc(&Version, h, "simtgo_version")
	purego.RegisterLibFunc(&DeviceInfo, h, "simtgo_device_info")
	purego.RegisterLibFunc(&StreamSync, h, "simtgo_stream_sync")
	purego.RegisterLibFunc(&Shutdown, h, "simtgo_shutdown")

	purego.RegisterLibFunc(&VecAdd, h, "simtgo_VecAdd")
	purego.RegisterLibFunc(&Scale, h, "simtgo_Scale")
	purego.RegisterLibFunc(&Magnitude, h, "simtgo_Magnitude")
	purego.RegisterLibFunc(&MagnitudeFast, h, "simtgo_MagnitudeFast")
	purego.RegisterLibFunc(&MagnitudeFastInterleaved, h, "simtgo_MagnitudeFast_interleaved")
	purego.RegisterLibFunc(&Softclip, h, "simtgo_Softclip")
	purego.RegisterLibFunc(&Classify, h, "simtgo_Classify")
	purego.RegisterLibFunc(&BandGain, h, "simtgo_BandGain")
	purego.RegisterLibFunc(&Quantize, h, "simtgo_Quantize")
	purego.RegisterLibFunc(&Gray, h, "simtgo_Gray")
	purego.RegisterLibFunc(&Histogram, h, "simtgo_Histogram")
	purego.RegisterLibFunc(&HistogramDyn, h, "simtgo_HistogramDyn")
	purego.RegisterLibFunc(&Transpose, h, "simtgo_Transpose")
	purego.RegisterLibFunc(&WarpReduceSum, h, "simtgo_WarpReduceSum")
	purego.RegisterLibFunc(&FIR, h, "simtgo_FIR")

	purego.RegisterLibFunc(&FIRShard, h, "simtgo_FIR_shard")
	purego.RegisterLibFunc(&FIRShardHost, h, "simtgo_FIR_shard_host")
	purego.RegisterLibFunc(&HistogramShard, h, "simtgo_Histogram_shard")

	purego.RegisterLibFunc(&CommUniqueID, h, "simtgo_comm_unique_id")
	purego.RegisterLibFunc(&CommInit, h, "simtgo_comm_init")
	purego.RegisterLibFunc(&CommDestroy, h, "simtgo_comm_destroy")
	purego.RegisterLibFunc(&CommAllreduceI32, h, "simtgo_comm_allreduce_i32")
	purego.RegisterLibFunc(&HistogramAllreduce, h, "simtgo_Histogram_allreduce")
	purego.RegisterLibFunc(&HistogramAllreduceFused, h, "simtgo_Histogram_allreduce_fused")
	purego.RegisterLibFunc(&HistogramAllreduceFusedOverwrite, h, "simtgo_Histogram_allreduce_fused_overwrite")

	purego.RegisterLibFunc(&TileNew, h, "simtgo_tile_new")
	purego.RegisterLibFunc(&TileFree, h, "simtgo_tile_free")
	purego.RegisterLibFunc(&TileInput, h, "simtgo_tile_input")
	purego.RegisterLibFunc(&TileInputDevice, h, "simtgo_tile_input_device")
	purego.RegisterLibFunc(&TileAdd, h, "simtgo_tile_add")
	purego.RegisterLibFunc(&TileMul, h, "simtgo_tile_mul")
	purego.RegisterLibFunc(&TileHypot, h, "simtgo_tile_hypot")
	purego.RegisterLibFunc(&TileScale, h, "simtgo_tile_scale")
	purego.RegisterLibFunc(&TileSqrt, h, "simtgo_tile_sqrt")
	purego.RegisterLibFunc(&TileAbs, h, "simtgo_tile_abs")
	purego.RegisterLibFunc(&TileFIR, h, "simtgo_tile_fir")
	purego.RegisterLibFunc(&TileAllowChainedWindows, h, "simtgo_tile_allow_chained_windows")
	purego.RegisterLibFunc(&TileLen, h, "simtgo_tile_len")
	purego.RegisterLibFunc(&TileErr, h, "simtgo_tile_err")
	purego.RegisterLibFunc(&TileErrString, h, "simtgo_tile_err_string")
	purego.RegisterLibFunc(&TileProgramSize, h, "simtgo_tile_program_size")
	purego.RegisterLibFunc(&TileSource, h, "simtgo_tile_source")
	purego.RegisterLibFunc(&TileSetJIT, h, "simtgo_tile_set_jit")
	purego.RegisterLibFunc(&TileJITInfo, h, "simtgo_tile_jit_info")
	purego.RegisterLibFunc(&TileJITSource, h, "simtgo_tile_jit_source")
	purego.RegisterLibFunc(&TileMaterialize, h, "simtgo_tile_materialize")
	purego.RegisterLibFunc(&TileMaterializeStepwise, h, "simtgo_tile_materialize_stepwise")
	purego.RegisterLibFunc(&TileRun, h, "simtgo_tile_run")
	purego.RegisterLibFunc(&TileRunShard, h, "simtgo_tile_run_shard")
	purego.RegisterLibFunc(&TileRunStepwiseNoalloc, h, "simtgo_tile_run_stepwise_noalloc")
	purego.RegisterLibFunc(&TileReduce, h, "simtgo_tile_reduce")
	purego.RegisterLibFunc(&TileReduceMaterialize, h, "simtgo_tile_reduce_materialize")
	purego.RegisterLibFunc(&TileShardRange, h, "simtgo_tile_shard_range")
	purego.RegisterLibFunc(&TileReduceShard, h, "simtgo_tile_reduce_shard")
}

// Sentinels for the library's own codes, so that callers can map them onto
// simtgo's error types with errors.Is (BlockSizeError, AliasError, ...).
var (
	ErrNull   = errors.New("b200: null pointer")
	ErrLength = errors.New("b200: slice too short")
	ErrBlock  = errors.New("b200: block size")
	ErrAlias  = errors.New("b200: aliased slices")
	ErrLaunch = errors.New("b200: launch configuration")
	ErrTaps   = errors.New("b200: taps")
	ErrGraph  = errors.New("b200: tile graph")
	ErrDevice = errors.New("b200: device")
	ErrComm   = errors.New("b200: communicator")
	ErrSize   = errors.New("b200: size limit")
	ErrArg    = errors.New("b200: argument")
)

var sentinel = map[int32]error{
	ENull: ErrNull, ELength: ErrLength, EBlock: ErrBlock, EAlias: ErrAlias, ELaunch: ErrLaunch,
	ETaps: ErrTaps, EGraph: ErrGraph, EDevice: ErrDevice, EComm: ErrComm, ESize: ErrSize,
	EArg: ErrArg,
}

// Error is a non-zero status with the library's message for it.
type Error struct {
	Code int32
	Msg  string
}

func (e *Error) Error() string { return fmt.Sprintf("simtgo_b200 [%d]: %s", e.Code, e.Msg) }

// Is matches the sentinel of the error's code.
func (e *Error) Is(target error) bool { return sentinel[e.Code] == target }

// Check returns nil for a zero status, else an *Error with the calling
// thread's message (read before any other library call on the thread).
func Check(rc int32) error {
	if rc == OK {
		return nil
	}
	return &Error{Code: rc, Msg: LastError()}
}
