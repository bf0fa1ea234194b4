/*
 * simtgo_b200.h -- C ABI of libsimtgo_b200.so, the B200 (sm_100a) kernels for
 * simtgo's data-parallel hot path.
 *
 * The library replaces the device half of two call sites in simtgo:
 *
 *   simt:  Kernel.launch -> cuda.Function.LaunchSync / Launch
 *          (simt/kernel.go:488-514, cuda/driver_cuda.go:546, cuda/stream_cuda.go:270)
 *   tile:  Tensor.run -> jit.Load + LaunchSync   (tile/run.go:37-83)
 *
 * Every symbol is a plain C function over plain pointers, sizes and a stream
 * handle, so it can be bound by purego (no cgo), ctypes, or a C/C++ caller.
 *
 * Conventions
 * -----------
 * - Slices travel as (pointer, int32 length) pairs, exactly as
 *   cuda.Slice.KernelArgs flattens them (cuda/slice_cuda.go:94) and in the
 *   parameter order of the generated kernel (kernels/prebuilt/<K>.cu).
 *   Output and input pointers are DEVICE pointers in the current CUDA
 *   context (simtgo's cuMemAlloc'd DevPtrs in the primary context qualify).
 * - grid and block are the launch geometry the caller asked for. The kernels
 *   here choose their own B200 geometry, but the covered extent grid*block
 *   is honoured: a thread index the original launch did not cover writes
 *   nothing, exactly as in gpu.RunCPU (gpu/gpu.go:270-306).
 * - stream is a cudaStream_t (NULL = the legacy default stream). Every entry
 *   point is asynchronous on that stream; simtgo_stream_sync() is the
 *   synchronous tail simt.Kernel.Launch adds (LaunchSync) and reports
 *   sticky device errors.
 * - Return value: 0 on success; a negative SIMTGO_E* code for an argument
 *   the host refused before anything was launched; a positive value is a
 *   cudaError_t (or ncclResult_t + 1000 for the communicator calls) passed
 *   through. simtgo_last_error() returns the calling thread's message for
 *   the most recent failure.
 * - Nothing here traps the device. Bounds that gpu.RunCPU would turn into an
 *   index-out-of-range panic are refused on the host with SIMTGO_ELENGTH.
 */
#ifndef SIMTGO_B200_H
#define SIMTGO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
    SIMTGO_OK = 0,
    SIMTGO_ENULL = -1,     /* a null pointer where the extent needs memory   */
    SIMTGO_ELENGTH = -2,   /* a slice too short for the covered extent: the
                              access gpu.RunCPU would panic on               */
    SIMTGO_EBLOCK = -3,    /* simt.BlockSizeError (simt/kernel.go:220-229)   */
    SIMTGO_EALIAS = -4,    /* simt.AliasError / tile.AliasError
                              (simt/kernel.go:251-264, tile/alias.go:17-23) */
    SIMTGO_ELAUNCH = -5,   /* grid/block the driver would refuse             */
    SIMTGO_ETAPS = -6,     /* FIR taps outside what the kernel can stage     */
    SIMTGO_EGRAPH = -7,    /* a latched tile graph error (tile/tile.go:78)   */
    SIMTGO_EDEVICE = -8,   /* no usable CUDA device / wrong architecture     */
    SIMTGO_ECOMM = -9,     /* communicator misuse or NCCL not loadable       */
    SIMTGO_ESIZE = -10,    /* a size beyond a documented library maximum     */
    SIMTGO_EARG = -11      /* any other refused argument                     */
};

/* Message for the calling thread's most recent failure ("" if none). */
const char* simtgo_last_error(void);
/* Library version string. */
const char* simtgo_version(void);
/* Names the device the library would launch on and checks it is sm_100.
 * Writes the SM count and the device's compute capability. */
int simtgo_device_info(int32_t* sm_count, int32_t* cc_major, int32_t* cc_minor);
/* cudaStreamSynchronize(stream); the synchronous tail of simt.Kernel.Launch. */
int simtgo_stream_sync(void* stream);
/* Frees the library's private device resources: the buffers, streams and
 * events of simtgo_FIR_shard_host on every device that used it, the freed
 * scratch the tile reductions' memory pool keeps mapped, and the modules of
 * the specialised tile kernels (a later launch loads them again, from the
 * on-disk cache when it has them). Call with no
 * library work in flight (e.g. before the process or the Go context ends);
 * later calls allocate afresh. Caller-owned buffers and communicators
 * (simtgo_comm_destroy) are not touched; the fixed 16 MiB scratch of
 * simtgo_tile_run_stepwise_noalloc lives as long as the loaded module. */
int simtgo_shutdown(void);

/* ---- the simt kernels (package kernels) -------------------------------- */

/* kernels/kernels.go:12 VecAdd; generated kernels/prebuilt/VecAdd.cu.
 * c[i] = a[i] + b[i] for i < min(c_len, grid*block). Bit-exact. */
int simtgo_VecAdd(float* c, int32_t c_len, const float* a, int32_t a_len,
                  const float* b, int32_t b_len,
                  int32_t grid, int32_t block, void* stream);

/* kernels/kernels.go:29 Scale; Scale.cu. y[i] = k*x[i]. Bit-exact. */
int simtgo_Scale(float* y, int32_t y_len, const float* x, int32_t x_len, float k,
                 int32_t grid, int32_t block, void* stream);

/* kernels/kernels.go:21 Magnitude; Magnitude.cu. mag[i] = gpu.Hypot(re[i], im[i])
 * with gpu.Hypot = float32(math.Hypot(float64, float64)) (gpu/math.go:17).
 * Bit-exact with the emulator's definition. */
int simtgo_Magnitude(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                     const float* im, int32_t im_len,
                     int32_t grid, int32_t block, void* stream);

/* kernels/magnitudefast.go:20 MagnitudeFast; MagnitudeFast.cu.
 * mag[i] = Sqrt(re*re + im*im) / scale, each operation rounded to nearest
 * (the gpu.RunCPU result, so bit-exact with it; the reference's
 * --use_fast_math build is within its documented 1e-5 of this). */
int simtgo_MagnitudeFast(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                         const float* im, int32_t im_len, float scale,
                         int32_t grid, int32_t block, void* stream);

/* MagnitudeFast over interleaved complex samples z = (re0, im0, re1, im1, ...).
 * z_len counts floats; element i reads z[2i], z[2i+1]. Same arithmetic as
 * simtgo_MagnitudeFast with re[i] = z[2i], im[i] = z[2i+1]. No counterpart
 * signature in the reference (its MagnitudeFast is planar); the signal-chain
 * workload stores complex values interleaved. */
int simtgo_MagnitudeFast_interleaved(float* mag, int32_t mag_len, const float* z,
                                     int32_t z_len, float scale,
                                     int32_t grid, int32_t block, void* stream);

/* kernels/softclip.go:11-30 Softclip; Softclip.cu. Bit-exact. */
int simtgo_Softclip(float* y, int32_t y_len, const float* x, int32_t x_len,
                    float threshold, int32_t grid, int32_t block, void* stream);

/* kernels/classify.go:14-56 Classify; Classify.cu. edges is a device slice.
 * Bit-exact with gpu.RunCPU (gain*v and bias*0.001 rounded separately). */
int simtgo_Classify(float* out, int32_t out_len, const float* x, int32_t x_len,
                    const float* edges, int32_t edges_len,
                    int32_t grid, int32_t block, void* stream);

/* kernels/bandgain.go:9-12 Band (8 bytes) and :26-30 Shape (16 bytes). */
typedef struct simtgo_band { float upper; float gain; } simtgo_band;
typedef struct simtgo_shape { float floor_gain; int32_t count; double bias; } simtgo_shape;

/* kernels/bandgain.go:42-76 BandGain; BandGain.cu. bands is a device slice;
 * cfg is a HOST pointer to the Shape the reference passes by value.
 * Bit-exact with gpu.RunCPU (float64 steps rounded separately). */
int simtgo_BandGain(float* y, int32_t y_len, const float* x, int32_t x_len,
                    const simtgo_band* bands, int32_t bands_len, const simtgo_shape* cfg,
                    int32_t grid, int32_t block, void* stream);

/* kernels/quantize.go:16-45 Quantize; Quantize.cu. clipped is Go's []bool
 * (one byte, 0 or 1). A float->int32 conversion out of range (or NaN) gives
 * INT32_MIN, as amd64 CVTTSS2SL does under gpu.RunCPU. Bit-exact. */
int simtgo_Quantize(int32_t* code, int32_t code_len, int64_t* energy, int32_t energy_len,
                    uint8_t* clipped, int32_t clipped_len, const float* x, int32_t x_len,
                    float step, uint32_t seed, int32_t grid, int32_t block, void* stream);

/* kernels/gray.go:34-55 Gray; Gray.cu. Bit-exact. */
int simtgo_Gray(uint8_t* out, int32_t out_len, const uint8_t* rgb, int32_t rgb_len,
                int32_t grid, int32_t block, void* stream);

/* kernels/histogram.go:23-50 Histogram; Histogram.cu. ADDS the counts of
 * x[i] in [0,256) (i < min(x_len, grid*block)) into bins[k], k < bins_len;
 * callers zero bins first, as the reference's test does. Exact. */
int simtgo_Histogram(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                     int32_t grid, int32_t block, void* stream);

/* simt Kernel.LaunchShared (simt/kernel.go:444-481) with a launch-sized
 * int32 tile of tile_len elements, on the DynProbe body
 * (simt/shared_parity_cuda_test.go:117-138): ADDS the counts of x[i] in
 * [0, tile_len), i < min(x_len, grid*block), into bins[k] for
 * k < min(tile_len, bins_len); other samples are dropped. A tile larger than
 * a block's shared memory (~57 K elements on B200) is refused before the
 * launch with SIMTGO_ESIZE (simt.SharedMemoryError). Exact. */
int simtgo_HistogramDyn(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                        int32_t tile_len, int32_t grid, int32_t block, void* stream);

/* kernels/transpose.go:15-38 Transpose; Transpose.cu. out[x*h+y] = in[y*w+x]
 * for x < min(w, 16*grid_x), y < min(h, 16*grid_y). block_x*block_y must be
 * 256 (AssumeBlockDim(TransposeTile*TransposeTile)). Exact. */
int simtgo_Transpose(float* out, int32_t out_len, const float* in, int32_t in_len,
                     int32_t w, int32_t h, int32_t grid_x, int32_t grid_y,
                     int32_t block_x, int32_t block_y, void* stream);

/* kernels/warpreduce.go:21-43 WarpReduceSum; WarpReduceSum.cu. block must be
 * 128. out[w] = the shuffle-down tree sum of x[32w..32w+31] (missing samples
 * are 0) for w < min(out_len, grid*4). Bit-exact (same addition tree). */
int simtgo_WarpReduceSum(float* out, int32_t out_len, const float* x, int32_t x_len,
                         int32_t grid, int32_t block, void* stream);

/* kernels/fir.go:17-46 FIR; FIR.cu. block must be 256 (FIRBlock). y[n] =
 * sum_k h[k]*x[n-k], x zero outside [0, x_len), for n < min(y_len, 256*grid).
 * The accumulation is fma(h[k], x, acc) for k = 0..taps-1 in order: bit-exact
 * with the reference's device code (nvcc contracts `acc += h*x`), within 1e-5
 * of gpu.RunCPU (kernels' tolerance). taps = h_len may be 0..65 (the staged
 * tile is FIRBlock+FIRMaxTaps samples); more is SIMTGO_ETAPS. */
int simtgo_FIR(float* y, int32_t y_len, const float* x, int32_t x_len,
               const float* h, int32_t h_len,
               int32_t grid, int32_t block, void* stream);

/* ---- sharded / large-extent forms -------------------------------------- */

/* Maximum taps of simtgo_FIR_shard. */
#define SIMTGO_FIR_SHARD_MAX_TAPS 1024

/* One shard of a long FIR (the 2^31-sample, 127-tap workload): the FIR of
 * kernels/fir.go:17 with 64-bit extents and up to SIMTGO_FIR_SHARD_MAX_TAPS
 * taps. y[j], j < y_len, is output (g0 + j) of the whole signal; x holds the
 * `halo` samples that precede the shard followed by the shard's own, so
 * x[halo + j] is sample g0 + j. Samples before x[0] or at/after x[x_len] read
 * as zero (shard 0 passes halo = 0). Same fma order as simtgo_FIR. h is a
 * device pointer. No counterpart in the reference, which has no multi-GPU
 * support; it generalises kernels/fir.go:17-46. */
int simtgo_FIR_shard(float* y, int64_t y_len, const float* x, int64_t x_len, int64_t halo,
                     const float* h, int32_t taps, void* stream);

/* simtgo_FIR_shard with y, x and h in host memory (pinned for full speed;
 * pageable memory works): the shard streams through the GPU in chunks of
 * 2^22 outputs on three internal streams, so the upload of one chunk, the
 * kernel of the next and the download of the one before overlap. The calling
 * thread only enqueues: y is complete when `stream` reaches the point of the
 * call (as with cudaMemcpyAsync). The library keeps three 48 MB sets of
 * device buffers per device for it, allocated on first use; calls are
 * serialised. No counterpart in the reference: it is the cuda.Upload ->
 * FIR -> Download sequence of one shard, pipelined. */
int simtgo_FIR_shard_host(float* y, int64_t y_len, const float* x, int64_t x_len, int64_t halo,
                          const float* h, int32_t taps, void* stream);

/* kernels/histogram.go:23 over a 64-bit extent: adds the counts of every
 * x[i], i < x_len, into bins[k], k < bins_len. */
int simtgo_Histogram_shard(int32_t* bins, int32_t bins_len, const int32_t* x, int64_t x_len,
                           void* stream);

/* ---- communicator (histogram partial bins -> one result on every rank) -- */

typedef struct simtgo_comm simtgo_comm;
/* 128-byte NCCL unique id, created on one rank and shared by the caller. */
int simtgo_comm_unique_id(uint8_t out_id[128]);
/* One rank of a communicator over the current device. NCCL is dlopen'ed
 * (libnccl.so.2, the process's already-loaded copy if there is one). */
int simtgo_comm_init(simtgo_comm** out, const uint8_t id[128], int32_t nranks, int32_t rank);
int simtgo_comm_destroy(simtgo_comm* comm);
/* In-place sum all-reduce of n int32 on stream. */
int simtgo_comm_allreduce_i32(simtgo_comm* comm, int32_t* buf, int32_t n, void* stream);
/* Histogram of this rank's shard added into bins, then the bins summed over
 * all ranks, so every rank ends with the histogram of the whole input. */
int simtgo_Histogram_allreduce(simtgo_comm* comm, int32_t* bins, int32_t bins_len,
                               const int32_t* x, int64_t x_len, void* stream);
/* The same result in ONE kernel over NVLink peer memory instead of a local
 * histogram followed by an NCCL all-reduce: the grid counts its shard, its
 * last block stores this rank's bins (its own plus the counts) into a slot
 * of every rank's exchange buffer, raises a flag on each rank (system-scope
 * release), waits for every rank's flag (acquire) and sums the slots into
 * bins. bins_len <= 4096 (more is SIMTGO_ESIZE). A collective: every rank
 * calls it, in the same order; the first call maps every rank's exchange
 * buffer with CUDA IPC (handles shared by an NCCL all-gather). The wait is
 * bounded (about a second): a rank that does not arrive leaves the others'
 * bins unchanged and raises the watchdog, which simtgo_stream_sync reports
 * as SIMTGO_EDEVICE. */
int simtgo_Histogram_allreduce_fused(simtgo_comm* comm, int32_t* bins, int32_t bins_len,
                                     const int32_t* x, int64_t x_len, void* stream);
/* No counterpart in the reference (which adds into bins, as the entry above
 * does): the same exchange with the incoming bins read as zero, so that
 * every rank ends with the counts of the whole input without zeroing bins
 * first -- the zeroing launch of a repeated sharded histogram folded into
 * the kernel. Same limits, collective order and bounded wait. */
int simtgo_Histogram_allreduce_fused_overwrite(simtgo_comm* comm, int32_t* bins,
                                               int32_t bins_len, const int32_t* x, int64_t x_len,
                                               void* stream);

/* ---- the tile track (package tile) -------------------------------------- */

/* tile/tile.go:22 BlockSize and :25 MaxTaps. */
#define SIMTGO_TILE_BLOCK_SIZE 256
#define SIMTGO_TILE_MAX_TAPS 64

typedef struct simtgo_tile_graph simtgo_tile_graph;
/* A tensor handle is the node id within its graph (>= 0). */
typedef int32_t simtgo_tensor;

/* tile/tile.go:60 New. The graph records operations; nothing touches the
 * device until a materialisation. */
simtgo_tile_graph* simtgo_tile_new(void);
void simtgo_tile_free(simtgo_tile_graph* g);
/* tile/tile.go:86 Input: host data, uploaded on materialisation. The graph
 * keeps the pointer, not a copy: the data must outlive the graph's use. */
simtgo_tensor simtgo_tile_input(simtgo_tile_graph* g, const float* host, int32_t n);
/* Device-resident input (the `dev` field of tile/tile.go:46): no upload. */
simtgo_tensor simtgo_tile_input_device(simtgo_tile_graph* g, const float* dev, int32_t n);
/* tile/tile.go:105-149. On a latched error each returns its first operand,
 * as the reference does; simtgo_tile_err() reports the first error. */
simtgo_tensor simtgo_tile_add(simtgo_tile_graph* g, simtgo_tensor a, simtgo_tensor b);
simtgo_tensor simtgo_tile_mul(simtgo_tile_graph* g, simtgo_tensor a, simtgo_tensor b);
simtgo_tensor simtgo_tile_hypot(simtgo_tile_graph* g, simtgo_tensor a, simtgo_tensor b);
simtgo_tensor simtgo_tile_scale(simtgo_tile_graph* g, simtgo_tensor a, float k);
simtgo_tensor simtgo_tile_sqrt(simtgo_tile_graph* g, simtgo_tensor a);
simtgo_tensor simtgo_tile_abs(simtgo_tile_graph* g, simtgo_tensor a);
/* tile/tile.go:135 FIR: h is HOST memory of `taps` floats (copied). */
simtgo_tensor simtgo_tile_fir(simtgo_tile_graph* g, simtgo_tensor a, const float* h, int32_t taps);
/* No counterpart in the reference, which rejects a FIR whose input contains
 * a FIR (tile/tile.go:141-146, pinned by TestChainedWindowRejected) and
 * lists chained windows as future work (PLAN.md, Phase 6). With allow != 0,
 * FIRs recorded afterwards on this graph may be chained: each window reads
 * the one inside it as zero outside [-halo, n), exactly as if the inner one
 * had been materialised first (MaterializeStepwise gives the same bits). A
 * sharded run is exact at the shard's edge when halo covers the sum of
 * taps-1 along the longest chain. The default (0) keeps the reference's
 * error. */
int simtgo_tile_allow_chained_windows(simtgo_tile_graph* g, int32_t allow);
/* tile/tile.go:63 Tensor.Len. -1 for a handle that is not in the graph. */
int32_t simtgo_tile_len(const simtgo_tile_graph* g, simtgo_tensor t);
/* tile/tile.go:163 Err: SIMTGO_OK or SIMTGO_EGRAPH; the message is in
 * simtgo_tile_err_string. */
int simtgo_tile_err(const simtgo_tile_graph* g);
const char* simtgo_tile_err_string(const simtgo_tile_graph* g);
/* Number of device instructions the fused program for t has (the analogue of
 * Tensor.Source, tile/run.go:10: it compiles without running). */
int simtgo_tile_program_size(simtgo_tile_graph* g, simtgo_tensor t, int32_t* n_instructions,
                             int32_t* n_inputs, int32_t* n_windows);

/* tile/run.go:10 Tensor.Source: the program the tensor would be computed by,
 * as text, without running anything -- here the listing of the lowered
 * accumulator-machine program (one fused device instruction per line, its
 * steps separated by " | "). Writes at most cap bytes
 * (NUL-terminated) and returns the size the whole listing needs, or a
 * negative status. */
int32_t simtgo_tile_source(simtgo_tile_graph* g, simtgo_tensor t, char* buf, int32_t cap);

/* Specialised kernels (tile/run.go:38 run -> internal/jit/jit.go Load: the
 * reference compiles each distinct graph with NVRTC and caches the result).
 * Every launch of a fused program of up to 32 device instructions
 * (simtgo_tile_program_size) -- materialise, run, shards, reductions,
 * stepwise steps -- runs the program's own specialised kernel: the lowered
 * program compiled in as constants (NVRTC, sm_100a, on first use of each
 * distinct program per device, then cached for the life of the process),
 * computing the same bits as the interpreter it replaces. Longer programs
 * run on the interpreter in every mode (their compile time grows faster
 * than their length, while their dispatch is spread over more work). Mode 0: the
 * interpreter only; 1 (the default, or SIMTGO_TILE_JIT=1 in the environment
 * before the first tile launch): specialise, or interpret when libnvrtc
 * cannot be opened (libnvrtc.so.12, or the library SIMTGO_NVRTC_LIB names);
 * 2: specialise or fail with SIMTGO_EDEVICE. A first launch
 * of a new program compiles (about a second) before it enqueues, so make it
 * before any stream capture. */
int simtgo_tile_set_jit(int32_t mode);
/* The mode, whether libnvrtc could be opened, how many programs were
 * compiled and specialised launches made in this process, and how many
 * kernels came from the on-disk cache instead of a compilation (compiled
 * cubins are kept in $SIMTGO_B200_CACHE, else $XDG_CACHE_HOME/simtgo_b200,
 * else ~/.cache/simtgo_b200; SIMTGO_B200_CACHE=off disables it; an entry is
 * served only when its stored identity -- source, headers, options, NVRTC
 * version -- matches byte for byte). Any pointer may be NULL. */
int simtgo_tile_jit_info(int32_t* mode, int32_t* available, int64_t* compiled,
                         int64_t* launches, int64_t* cache_hits);
/* The specialised kernel's source for t (reduce: -1 or a SIMTGO_TILE_*
 * reduction) with `groups` (2 or 4) float4 groups per thread and bulk-copied
 * (bulk != 0) or directly read inputs, written like simtgo_tile_source; with
 * compile != 0 it is compiled too (no GPU needed) and a failure returned.
 * groups 0 (with a reduction of a chain of Scale, Sqrt, Abs, x+x, x*x steps
 * on one input) gives the streaming reduction's kernel for that chain
 * instead, the steps compiled in as constants; bulk is then ignored. */
int32_t simtgo_tile_jit_source(simtgo_tile_graph* g, simtgo_tensor t, int32_t reduce,
                               int32_t groups, int32_t bulk, int32_t compile, char* buf,
                               int32_t cap);

/* tile/run.go:20 Materialize: upload host inputs, run the one fused kernel,
 * download into host_out (out_len == Len(t)), free what the call allocated.
 * Synchronous. */
int simtgo_tile_materialize(simtgo_tile_graph* g, simtgo_tensor t, float* host_out,
                            int32_t out_len);
/* tile/run.go:89 MaterializeStepwise: one kernel per operation node with a
 * device temporary between each; writes the launch count. Synchronous. */
int simtgo_tile_materialize_stepwise(simtgo_tile_graph* g, simtgo_tensor t, float* host_out,
                                     int32_t out_len, int32_t* launches);
/* Device-resident run (tile/run.go:37 `run` without the uploads): every input
 * must be a device input; out is a device buffer of Len(t) floats.
 * Asynchronous on stream. The output may not overlap an input
 * (tile/alias.go:42). */
int simtgo_tile_run(simtgo_tile_graph* g, simtgo_tensor t, float* dev_out, int32_t out_len,
                    void* stream);
/* One shard of the graph's elementwise split: every device input points at
 * the shard's first own element and has `halo` valid elements in front of
 * it (ptr[-halo .. -1], the samples preceding the shard; halo = 0 on the
 * first shard); window (FIR) nodes read them instead of zeros. Without a FIR
 * node, halo may be 0 on every shard. */
int simtgo_tile_run_shard(simtgo_tile_graph* g, simtgo_tensor t, float* dev_out,
                          int32_t out_len, int32_t halo, void* stream);

/* No counterpart in the reference. MaterializeStepwise's computation
 * (tile/run.go:89: one kernel per operation node) for callers that cannot
 * allocate device memory -- e.g. a real-time signal-processing callback
 * with a fixed deadline, where cudaMalloc/cudaFree may synchronise the
 * whole device and take unbounded time, or an application whose memory pool
 * owns the device and forbids outside allocations. It allocates no device
 * memory: every input must be a device input (simtgo_tile_input_device),
 * the caller passes dev_out (out_len == Len(t)), and the intermediate node
 * values live in a fixed scratch array inside the library of
 * SIMTGO_TILE_NOALLOC_SCRATCH_FLOATS floats (16 MiB), which every GPU that
 * loads the library holds until the process exits. A graph whose
 * intermediate nodes need more (each node's length rounded up to 64 floats,
 * summed over the nodes other than t) is refused with SIMTGO_ESIZE. The
 * first call on a device resolves the array's device address (once per
 * device, with that device current), so it should come before any stream
 * capture begins on that device. Every call uses the same array and
 * leaves its values there; each node's region is written in full before it
 * is read, so nothing needs clearing. Calls that overlap on the GPU (two
 * streams, or two host threads) race on the array. Its steps always run in
 * the precompiled interpreter, never in a specialised kernel (loading one
 * allocates device memory for its code). Asynchronous on stream; the
 * result equals simtgo_tile_run's bit for bit. */
#define SIMTGO_TILE_NOALLOC_SCRATCH_FLOATS (1 << 22)
int simtgo_tile_run_stepwise_noalloc(simtgo_tile_graph* g, simtgo_tensor t, float* dev_out,
                                     int32_t out_len, void* stream);

/* ---- tile reductions (no counterpart in the reference) --------------------
 * The reference's tile track has no reductions; its plan lists sum, min, max
 * and argmax "with the shared-memory + warp pattern" as the next step
 * (PLAN.md, Phase 6, "Reductions"). Here a reduction consumes the fused
 * graph's values inside the same single pass over HBM (no output array is
 * written) and yields one value:
 *   SIMTGO_TILE_SUM     the float32 sum, in the fixed order below (a NaN
 *                       result is written as 0x7fc00000);
 *   SIMTGO_TILE_MIN,    Go's min / max: NaN (written as 0x7fc00000) if any
 *   SIMTGO_TILE_MAX     element is NaN, and -0 < +0;
 *   SIMTGO_TILE_ARGMAX  the first index whose value is MAX bit for bit (+0
 *                       wins over -0, the first NaN wins), with that value.
 * Empty tensors give SUM +0, MIN +Inf, MAX -Inf, ARGMAX index -1 (value -Inf).
 * Summation order: the values are cut into blocks of 2048, zero-padded past
 * the end. Block b's partial is ((w0+w1)+(w2+w3))+((w4+w5)+(w6+w7)), where
 * w_k is the butterfly sum of t_l over lanes l = 0..31 (each lane adds the
 * lane l^16, then l^8, l^4, l^2, l^1) and
 *   t_l = ((x[e]+x[e+1]) + (x[e+2]+x[e+3])) + ((x[f]+x[f+1]) + (x[f+2]+x[f+3])),
 *   e = 2048 b + 4 (32 k + l), f = e + 1024.
 * While more than one partial remains, the partials are reduced the same
 * way, as values of their own. So the sum is reproducible bit for bit, on one
 * GPU or sharded (simtgo_tile_reduce_shard). */
#define SIMTGO_TILE_SUM 0
#define SIMTGO_TILE_MIN 1
#define SIMTGO_TILE_MAX 2
#define SIMTGO_TILE_ARGMAX 3
/* Reduces t (every input a device input) into dev_value (one float) and,
 * for ARGMAX, dev_index (one int64; may be null for the other kinds).
 * Asynchronous on stream; allocates its partials stream-ordered
 * (cudaMallocAsync) and frees them the same way. */
int simtgo_tile_reduce(simtgo_tile_graph* g, simtgo_tensor t, int32_t kind, float* dev_value,
                       int64_t* dev_index, void* stream);
/* The same with host inputs uploaded and host results (Materialize's
 * counterpart). Synchronous. */
int simtgo_tile_reduce_materialize(simtgo_tile_graph* g, simtgo_tensor t, int32_t kind,
                                   float* value, int64_t* index);
/* The shard of a signal of n_total elements that rank `rank` of `nranks`
 * holds for simtgo_tile_reduce_shard: [rank*per, min(n_total, (rank+1)*per))
 * with per = ceil(ceil(n_total / nranks) / 2048) * 2048 (whole blocks of
 * the summation order; trailing ranks may hold nothing). */
int simtgo_tile_shard_range(int64_t n_total, int32_t nranks, int32_t rank, int64_t* start,
                            int64_t* len);
/* One rank's part of the reduction of a graph sharded over the ranks of
 * comm (a collective: every rank calls it, in the same order). Len(t) must
 * be this rank's simtgo_tile_shard_range length; device inputs carry `halo`
 * preceding samples as in simtgo_tile_run_shard. Each rank computes the
 * partials of its own blocks, an NCCL all-gather assembles every block's
 * partial on every rank, and each rank finishes the same tree: the result
 * equals simtgo_tile_reduce over the whole signal, bit for bit, on every
 * rank; ARGMAX indices are global. Asynchronous on stream. As with any NCCL
 * collective, the ranks must agree: a rank whose arguments are refused
 * returns before the all-gather, and its peers' all-gather then waits for
 * it, so a caller validates the split (simtgo_tile_shard_range) on every
 * rank before calling. */
int simtgo_tile_reduce_shard(simtgo_tile_graph* g, simtgo_tensor t, int32_t kind, int32_t halo,
                             int64_t n_total, simtgo_comm* comm, float* dev_value,
                             int64_t* dev_index, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SIMTGO_B200_H */
