// fir.cu -- FIR (kernels/fir.go:17-46) and its long, sharded form.
//
// y[j] = sum_k h[k] * x[j + halo - k], x read as zero outside [0, x_len),
// accumulated as acc = fma(h[k], x, acc) for k = 0, 1, ..., taps-1: the
// order and rounding of the reference's device code, where nvcc contracts
// `acc += h[k] * tile[...]` (kernels/prebuilt/FIR.cu:24-27).
//
// B200 design. Each warp produces 640 consecutive outputs on its own: lane l
// owns 20 consecutive outputs, so every sample it loads from shared memory
// feeds up to 20 fused multiply-adds from registers (the reference does one
// output per thread, with one shared load and one global tap load per
// multiply-add):
//  * the warp's signal span (its outputs plus the taps-1 halo) arrives by
//    one 1-D bulk copy (cp.async.bulk, TMA) into a LINEAR shared tile of the
//    warp's own, completing on the warp's own mbarrier, so no instruction
//    waits for more than one warp (no block barrier);
//  * 20 outputs per lane put lane l's window 80 bytes after lane l-1's
//    (5 x 16 B, odd), so the eight lanes of each 16-byte load phase hit
//    eight different bank groups: conflict-free without any swizzle or
//    padding, and every window load is base + a compile-time offset;
//  * taps go in chunks of 8: a chunk needs 27 samples per lane, eight
//    16-byte shared loads aligned down, and two broadcast tap loads, then
//    20 x 8 FFMA with every operand in a register; up to four chunks (and
//    the last, partial one) share one register window (a ring of eight
//    float4s), so each chunk after the first loads only the two float4s its
//    taps reach below the others (measured 9% faster than a fresh window
//    per chunk);
//  * the window's alignment within a 16-byte chunk, (D - 7) mod 4, is the
//    same for every warp and chunk, so it is a template parameter;
//  * the outputs leave from registers as 16-byte streaming stores.
// Blocks hold 8 warps (2 for short signals, so that they spread over every SM).
// At 127 taps the kernel is bound by FP32 FMA issue, not by HBM.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tma.cuh"

using namespace sgd;

namespace {

// Threads per block: kWide for long signals, kNarrow for signals with
// fewer than four waves of wide blocks (a 2^20-sample signal fills 205 wide
// blocks of 5120 outputs on 148 SMs, but 1366 narrow ones of 768). Both
// are sized for a 64-register budget: 4 wide or 16 narrow blocks per SM.
constexpr int kWide = 256;
constexpr int kNarrow = 64;
__host__ __device__ constexpr int min_blocks(int nt) { return 1024 / nt; }
// Outputs per lane (KPT): lane windows are 4*KPT bytes apart, so KPT/4 must
// be odd for the 8 lanes of a 16-byte load phase to hit 8 different bank
// groups. 20 for long signals (with 4 blocks per SM it measured fastest of
// 20/28/36/44: the FFMA rate depends on how the accumulators and the window
// share the register file, not only on reuse); 12 for signals under one
// wave of wide blocks, whose launches are too short for their warps'
// load-compute-store chains to overlap: more, shorter chains (a 2^20-sample,
// 31-tap launch 4.50 -> 4.07 us; at 2^22 samples 20 per lane stays ahead).
constexpr int kKptLong = 20;
constexpr int kKptShort = 12;
__host__ __device__ constexpr bool kpt_ok(int kpt) { return kpt % 4 == 0 && (kpt / 4) % 2 == 1; }
static_assert(kpt_ok(kKptLong) && kpt_ok(kKptShort), "lane stride must be odd x 16 B");
constexpr int kChunk = 8;  // taps per register chunk
// A chunk's window, KPT + 7 + SH floats, in float4s: the register ring's size.
__host__ __device__ constexpr int ring_of(int kpt) { return (kpt + 10 + 3) / 4; }
static_assert(ring_of(kKptLong) == 8 && ring_of(kKptShort) == 6, "ring sizes");
// Ring slot of window float4 q (q may be negative).
__host__ __device__ constexpr int ring_slot(int q, int ring) { return ((q % ring) + ring) % ring; }
__host__ __device__ constexpr int tile_out(int nt) { return nt * kKptLong; }  // outputs per wide block

struct FirGeom {
    int64_t y_len;   // outputs of this launch
    int64_t x_len;   // samples in x
    int64_t halo;    // x[halo + j] is the sample of output j
    int32_t taps;
    int32_t taps_pad;  // taps rounded up to kChunk
    int32_t D;         // tile index of the sample of a block's first output
    int32_t tile;      // floats in the shared tile (multiple of 4)
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// NC whole chunks (8 NC taps), and with TAIL a last chunk of nk < 8 taps,
// from one register window: chunk c's window float4 i is w4[i - 2c] (w4 = w
// as float4, the window of chunk 0; output r at tap u of a chunk reads its
// float SH + 7 + r - u), kept in ring slot (i - 2c) mod RING, so each chunk
// after the first loads only its two new float4s.
template <int SH, int NC, bool TAIL, int KPT>
__device__ __forceinline__ void fir_ring(const float* __restrict__ w, const float* hs,
                                         float (&acc)[KPT], int nk = 0) {
    constexpr int RING = ring_of(KPT);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    float4 R[RING];
#pragma unroll
    for (int q = 0; q < RING; q++) R[q] = w4[q];
#pragma unroll
    for (int c = 0; c < NC; c++) {
        if (c > 0) {
            R[ring_slot(-2 * c, RING)] = w4[-2 * c];
            R[ring_slot(1 - 2 * c, RING)] = w4[1 - 2 * c];
        }
        const float4 ha = *reinterpret_cast<const float4*>(hs + 8 * c);
        const float4 hb = *reinterpret_cast<const float4*>(hs + 8 * c + 4);
        const float hv[kChunk] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
#pragma unroll
        for (int r = 0; r < KPT; r++)
#pragma unroll
            for (int u = 0; u < kChunk; u++) {
                const int j = SH + 7 + r - u;
                const float4& q = R[ring_slot((j >> 2) - 2 * c, RING)];
                const float s = (j & 3) == 0 ? q.x : (j & 3) == 1 ? q.y : (j & 3) == 2 ? q.z : q.w;
                acc[r] = __fmaf_rn(hv[u], s, acc[r]);
            }
    }
    if (TAIL) {  // chunk NC, with nk < 8 taps (the taps past them are zero padding)
        constexpr int c = NC;
        if (c > 0) {
            R[ring_slot(-2 * c, RING)] = w4[-2 * c];
            R[ring_slot(1 - 2 * c, RING)] = w4[1 - 2 * c];
        }
        const float4 ha = *reinterpret_cast<const float4*>(hs + 8 * c);
        const float4 hb = *reinterpret_cast<const float4*>(hs + 8 * c + 4);
        const float hv[kChunk] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
#pragma unroll
        for (int u = 0; u < kChunk - 1; u++)
            if (u < nk) {
#pragma unroll
                for (int r = 0; r < KPT; r++) {
                    const int j = SH + 7 + r - u;
                    const float4& q = R[ring_slot((j >> 2) - 2 * c, RING)];
                    const float s = (j & 3) == 0 ? q.x : (j & 3) == 1 ? q.y : (j & 3) == 2 ? q.z : q.w;
                    acc[r] = __fmaf_rn(hv[u], s, acc[r]);
                }
            }
    }
}

// Warp tile t = outputs [ob, ob + 32 KPT), ob = 32 KPT t. The warp's shared
// tile holds samples [A, A + tile) of x (x-index = j + halo for output j),
// A = ob + halo - D, zero outside [0, x_len). Output ob + KPT l + r at tap k
// reads tile index D + KPT l + r - k, with D = taps + 6 + ((halo - taps - 6)
// mod 4), so A is a multiple of 4 (16-byte aligned when x is) and the window
// of the last, partial chunk (up to 7 taps past the end) stays inside.
__host__ __device__ constexpr int warp_out(int kpt) { return 32 * kpt; }

template <int SH, int NT, int KPT>
__global__ void __launch_bounds__(NT, min_blocks(NT)) k_fir(float* __restrict__ y,
                                                            const float* __restrict__ x,
                                                            const float* __restrict__ h, FirGeom g,
                                                            int64_t nwt, bool bulk_in,
                                                            bool vec_out, uint32_t* wd) {
    constexpr int kWarpOut = warp_out(KPT);
    __shared__ __align__(8) uint64_t bars[NT / 32];
    extern __shared__ float4 dyn4[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t t = (int64_t)blockIdx.x * (NT / 32) + wid;
    // Programmatic dependent launch: wait for the grids this one depends on
    // (their writes visible) before touching memory.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (t >= nwt) return;
    // The warp's region: its copy of the taps, then its signal tile.
    float* const hs = reinterpret_cast<float*>(dyn4) + wid * (g.taps_pad + g.tile);
    float* const tile = hs + g.taps_pad;
    uint64_t* const bar = &bars[wid];
    const int64_t A = t * kWarpOut + g.halo - g.D;
    // [c0, c1) arrives by bulk copy; the lanes fill the rest: samples before
    // x (zeros), and from c1 on (a ragged last 1-3 samples, zeros past x, or
    // everything when x is not 16-byte aligned).
    const int64_t c0 = max(A, (int64_t)0);
    const int64_t end = min(A + g.tile, g.x_len);
    const int64_t c1 = bulk_in && end > c0 ? c0 + ((end - c0) & ~int64_t(3)) : c0;
    if (c1 > c0 && lane == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(bar, (uint32_t)((c1 - c0) * 4));
        bulk_load(tile + (c0 - A), x + c0, (uint32_t)((c1 - c0) * 4), bar);
    }
    for (int k = lane; k < g.taps_pad; k += 32) hs[k] = k < g.taps ? h[k] : 0.0f;
    for (int64_t i = lane; i < c0 - A; i += 32) tile[i] = 0.0f;
    for (int64_t i = (c1 - A) + lane; i < g.tile; i += 32) {
        const int64_t p = A + i;
        tile[i] = (p >= 0 && p < g.x_len) ? x[p] : 0.0f;
    }
    __syncwarp();  // the barrier's initialisation and the lanes' fills
    // Gave up waiting (the watchdog is raised): nothing else is in flight.
    if (c1 > c0 && !mbar_wait(bar, 0, wd)) return;
    __syncwarp();

    float acc[KPT];
#pragma unroll
    for (int r = 0; r < KPT; r++) acc[r] = 0.0f;
    // Window start at chunk k0: D - 7 - SH + KPT lane - k0 (a multiple of 4).
    const float* w = tile + (g.D - 7 - SH) + KPT * lane;
    int k0 = 0;
    for (; k0 + 4 * kChunk <= g.taps; k0 += 4 * kChunk)
        fir_ring<SH, 4, false, KPT>(w - k0, hs + k0, acc);
    const int nk = (g.taps - k0) % kChunk;
    if (nk) {
        switch ((g.taps - k0) / kChunk) {
            case 3: fir_ring<SH, 3, true, KPT>(w - k0, hs + k0, acc, nk); break;
            case 2: fir_ring<SH, 2, true, KPT>(w - k0, hs + k0, acc, nk); break;
            case 1: fir_ring<SH, 1, true, KPT>(w - k0, hs + k0, acc, nk); break;
            default: fir_ring<SH, 0, true, KPT>(w - k0, hs + k0, acc, nk); break;
        }
    } else {
        switch ((g.taps - k0) / kChunk) {
            case 3: fir_ring<SH, 3, false, KPT>(w - k0, hs + k0, acc); break;
            case 2: fir_ring<SH, 2, false, KPT>(w - k0, hs + k0, acc); break;
            case 1: fir_ring<SH, 1, false, KPT>(w - k0, hs + k0, acc); break;
            default: break;
        }
    }

    // Let the next grid start launching once every block is this far: its
    // blocks take the SMs as this grid's finish (launched before the FMAs,
    // they held SM slots through the whole of a short launch: 2^20 samples
    // x 31 taps 4.1 -> 4.8 us per launch; released here, 3.9 us).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t ob = t * kWarpOut + KPT * lane;
    if (vec_out && (t + 1) * kWarpOut <= g.y_len) {
#pragma unroll
        for (int c = 0; c < KPT / 4; c++)
            st_stream_f4(y + ob + 4 * c,
                         make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]));
    } else {
#pragma unroll
        for (int r = 0; r < KPT; r++)
            if (ob + r < g.y_len) y[ob + r] = acc[r];
    }
}

using FirKernel = void (*)(float*, const float*, const float*, FirGeom, int64_t, bool, bool,
                           uint32_t*);

template <int NT, int KPT>
constexpr FirKernel kFirKernels[4] = {k_fir<0, NT, KPT>, k_fir<1, NT, KPT>, k_fir<2, NT, KPT>,
                                      k_fir<3, NT, KPT>};

// Each kernel may take the opt-in maximum of dynamic shared memory less 1 KB
// (its static mbarriers); set once per device (a bit per device, for the
// twelve kernels).
int fir_dyn_max(const sg::DevInfo* d) { return d->max_smem_optin - 1024; }
std::atomic<uint64_t> g_fir_configured[12];

int fir_configure(const sg::DevInfo* d, int slot, FirKernel kern) {
    const uint64_t bit = 1ull << (d->device & 63);
    if (g_fir_configured[slot].load(std::memory_order_acquire) & bit) return 0;
    const int rc = sg::cuda_status(cudaFuncSetAttribute(kern,
                                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                        fir_dyn_max(d)),
                                   "cudaFuncSetAttribute(FIR)");
    if (rc == 0) g_fir_configured[slot].fetch_or(bit, std::memory_order_acq_rel);
    return rc;
}

int launch_fir(const char* K, float* y, int64_t y_len, const float* x, int64_t x_len,
               int64_t halo, const float* h, int32_t taps, void* stream) {
    const sg::DevInfo* d;
    int rc;
    if ((rc = sg::current_device(&d))) return rc;
    if (y_len <= 0) return 0;
    // Narrow blocks while wide ones would make fewer than four waves.
    const int64_t wide_waves =
        sg::ceil_div(y_len, (int64_t)tile_out(kWide)) / ((int64_t)d->sms * min_blocks(kWide));
    const bool narrow = wide_waves < 4;
    const bool short_chains = wide_waves < 1;  // 12 outputs per lane
    const int nt = narrow ? kNarrow : kWide;
    const int kpt = short_chains ? kKptShort : kKptLong;
    FirGeom g;
    g.y_len = y_len;
    g.x_len = x_len;
    g.halo = halo;
    g.taps = taps;
    g.taps_pad = (int32_t)sg::ceil_div(std::max(taps, 1), kChunk) * kChunk;
    // ob is a multiple of 4, so D (and with it SH) is the same for every warp.
    const int64_t m = (((halo - taps - 6) % 4) + 4) % 4;
    g.D = (int32_t)(taps + 6 + m);
    // The window loads of the last lane reach a few floats past the last
    // sample its outputs use (whole 16-byte loads): 8 floats of slack.
    g.tile = (int32_t)sg::ceil_div(g.D + warp_out(kpt) + 8, 4) * 4;
    const int sh = (g.D - 7) % 4;

    const FirKernel kern = short_chains ? kFirKernels<kNarrow, kKptShort>[sh]
                           : narrow     ? kFirKernels<kNarrow, kKptLong>[sh]
                                        : kFirKernels<kWide, kKptLong>[sh];
    const size_t smem = (size_t)(nt / 32) * (g.tile + g.taps_pad) * sizeof(float);
    if (smem > (size_t)fir_dyn_max(d))
        return sg::fail(SIMTGO_ESIZE, "%s: %d taps need %zu bytes of shared memory", K, taps,
                        smem);
    if ((rc = fir_configure(d, (short_chains ? 8 : narrow ? 4 : 0) + sh, kern))) return rc;
    const int64_t nwt = sg::ceil_div(y_len, (int64_t)warp_out(kpt));
    const int64_t blocks = sg::ceil_div(nwt, (int64_t)(nt / 32));
    if (blocks > 0x7fffffffLL) return sg::fail(SIMTGO_ESIZE, "%s: y_len too large", K);
    sg::before_launch();
    // Launched with programmatic stream serialisation (PDL): a launch that
    // follows another kernel on the stream starts while that one drains,
    // and waits in griddepcontrol.wait before touching memory.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(nt);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return sg::cuda_status(cudaLaunchKernelEx(&cfg, kern, y, x, h, g, nwt, sg::aligned16(x),
                                              sg::aligned16(y), sg::watchdog_device_ptr()),
                           K);
}

// ---- the shard from host memory ----------------------------------------------
// simtgo_FIR_shard_host streams a shard that lives in host memory through the
// GPU in chunks: chunk j's input (with the taps-1 samples before it) goes up,
// the kernel runs, and its output comes down, on one of kPipe streams, so the
// upload of one chunk, the kernel of the next and the download of the one
// before overlap (the two copy directions run at once). The device buffers
// are kept per device and reused by later calls; calls are serialised.
constexpr int kPipe = 3;
constexpr int64_t kPipeChunk = 1 << 22;  // outputs per chunk (16 MB)
constexpr int64_t kPipePad = SIMTGO_FIR_SHARD_MAX_TAPS;  // >= taps-1, keeps 16-byte alignment

struct HostPipe {
    float* xbuf[kPipe] = {};  // kPipePad + kPipeChunk samples
    float* ybuf[kPipe] = {};
    float* hbuf[kPipe] = {};
    cudaStream_t st[kPipe] = {};
    cudaEvent_t ev[kPipe] = {};
    bool ready = false;
};

HostPipe g_pipes[64];
std::mutex g_pipe_mu;  // serialises simtgo_FIR_shard_host and simtgo_shutdown

int host_pipe(int device, HostPipe** out) {
    if (device < 0 || device >= 64) return sg::fail(SIMTGO_EDEVICE, "FIR_shard_host: device %d", device);
    HostPipe& P = g_pipes[device];
    if (!P.ready) {
        int rc;
        for (int s = 0; s < kPipe; s++) {
            if ((rc = sg::cuda_status(cudaMalloc(&P.xbuf[s], (kPipePad + kPipeChunk) * 4), "cudaMalloc")) ||
                (rc = sg::cuda_status(cudaMalloc(&P.ybuf[s], kPipeChunk * 4), "cudaMalloc")) ||
                (rc = sg::cuda_status(cudaMalloc(&P.hbuf[s], SIMTGO_FIR_SHARD_MAX_TAPS * 4), "cudaMalloc")) ||
                (rc = sg::cuda_status(cudaStreamCreateWithFlags(&P.st[s], cudaStreamNonBlocking),
                                      "cudaStreamCreate")) ||
                (rc = sg::cuda_status(cudaEventCreateWithFlags(&P.ev[s], cudaEventDisableTiming),
                                      "cudaEventCreate")))
                return rc;
        }
        P.ready = true;
    }
    *out = &P;
    return 0;
}

}  // namespace

namespace sg {
// Frees every device's host-pipe resources (simtgo_shutdown).
int fir_host_release() {
    std::lock_guard<std::mutex> lock(g_pipe_mu);
    int prev = 0, rc = 0;
    cudaGetDevice(&prev);
    for (int dev = 0; dev < 64; dev++) {
        HostPipe& P = g_pipes[dev];
        if (!P.ready) continue;
        int r = cuda_status(cudaSetDevice(dev), "cudaSetDevice");
        for (int s = 0; s < kPipe && !r; s++) {
            if (P.st[s]) r = cuda_status(cudaStreamSynchronize(P.st[s]), "cudaStreamSynchronize");
            if (!r && P.ev[s]) r = cuda_status(cudaEventDestroy(P.ev[s]), "cudaEventDestroy");
            if (!r && P.st[s]) r = cuda_status(cudaStreamDestroy(P.st[s]), "cudaStreamDestroy");
            if (!r) r = cuda_status(cudaFree(P.xbuf[s]), "cudaFree");
            if (!r) r = cuda_status(cudaFree(P.ybuf[s]), "cudaFree");
            if (!r) r = cuda_status(cudaFree(P.hbuf[s]), "cudaFree");
        }
        if (!r) P = HostPipe();
        if (r && !rc) rc = r;
    }
    cudaSetDevice(prev);
    return rc;
}
}  // namespace sg

namespace {

}  // namespace

extern "C" {

int simtgo_FIR(float* y, int32_t y_len, const float* x, int32_t x_len, const float* h,
               int32_t h_len, int32_t grid, int32_t block, void* stream) {
    const char* K = "FIR";
    sg::clear_error();
    int64_t nt;
    int rc;
    if (y_len < 0 || x_len < 0) return sg::fail(SIMTGO_EARG, "simt: %s: negative length", K);
    if ((rc = sg::launch_extent_1d(K, grid, block, 256, &nt))) return rc;
    // The staged tile is FIRBlock + FIRMaxTaps = 320 samples (fir.go:24);
    // its halo holds taps-1 of them.
    if (h_len < 0 || h_len > 65)
        return sg::fail(SIMTGO_ETAPS,
                        "simt: FIR: %d taps do not fit the %d-sample tile (FIRBlock %d + "
                        "FIRMaxTaps %d); gpu.RunCPU panics: index out of range",
                        h_len, 320, 256, 64);
    const int64_t m = std::min<int64_t>(y_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_ptr(K, "y", y, m)) || (rc = sg::check_ptr(K, "x", x, x_len)) ||
        (rc = sg::check_ptr(K, "h", h, h_len)))
        return rc;
    if ((rc = sg::check_alias(K, {{"y", y, 4LL * y_len, true},
                                  {"x", x, 4LL * x_len, false},
                                  {"h", h, 4LL * h_len, false}})))
        return rc;
    if (h_len == 0) {
        // No taps: every covered output is the empty sum, +0.
        return sg::cuda_status(cudaMemsetAsync(y, 0, (size_t)m * 4, (cudaStream_t)stream), K);
    }
    return launch_fir(K, y, m, x, x_len, 0, h, h_len, stream);
}

int simtgo_FIR_shard(float* y, int64_t y_len, const float* x, int64_t x_len, int64_t halo,
                     const float* h, int32_t taps, void* stream) {
    const char* K = "FIR_shard";
    sg::clear_error();
    int rc;
    if (y_len < 0 || x_len < 0 || halo < 0)
        return sg::fail(SIMTGO_EARG, "%s: negative length or halo", K);
    if (taps < 1 || taps > SIMTGO_FIR_SHARD_MAX_TAPS)
        return sg::fail(SIMTGO_ETAPS, "%s: %d taps is outside 1..%d", K, taps,
                        SIMTGO_FIR_SHARD_MAX_TAPS);
    if (y_len == 0) return 0;
    if ((rc = sg::check_ptr(K, "y", y, y_len)) || (rc = sg::check_ptr(K, "x", x, x_len)) ||
        (rc = sg::check_ptr(K, "h", h, taps)))
        return rc;
    if ((rc = sg::check_alias(K, {{"y", y, 4 * y_len, true},
                                  {"x", x, 4 * x_len, false},
                                  {"h", h, 4LL * taps, false}})))
        return rc;
    return launch_fir(K, y, y_len, x, x_len, halo, h, taps, stream);
}

int simtgo_FIR_shard_host(float* y, int64_t y_len, const float* x, int64_t x_len, int64_t halo,
                          const float* h, int32_t taps, void* stream) {
    const char* K = "FIR_shard_host";
    sg::clear_error();
    int rc;
    if (y_len < 0 || x_len < 0 || halo < 0 || halo > x_len)
        return sg::fail(SIMTGO_EARG, "%s: negative length or halo, or halo past x", K);
    if (taps < 1 || taps > SIMTGO_FIR_SHARD_MAX_TAPS)
        return sg::fail(SIMTGO_ETAPS, "%s: %d taps is outside 1..%d", K, taps,
                        SIMTGO_FIR_SHARD_MAX_TAPS);
    if (y_len == 0) return 0;
    if ((rc = sg::check_ptr(K, "y", y, y_len)) || (rc = sg::check_ptr(K, "x", x, x_len)) ||
        (rc = sg::check_ptr(K, "h", h, taps)))
        return rc;
    const sg::DevInfo* d;
    if ((rc = sg::current_device(&d))) return rc;
    std::lock_guard<std::mutex> lock(g_pipe_mu);
    HostPipe* P;
    if ((rc = host_pipe(d->device, &P))) return rc;
    cudaStream_t caller = (cudaStream_t)stream;
    cudaEvent_t start = P->ev[0];
    if ((rc = sg::cuda_status(cudaEventRecord(start, caller), K))) return rc;
    for (int s = 0; s < kPipe; s++) {
        if ((rc = sg::cuda_status(cudaStreamWaitEvent(P->st[s], start, 0), K)) ||
            (rc = sg::cuda_status(cudaMemcpyAsync(P->hbuf[s], h, (size_t)taps * 4,
                                                  cudaMemcpyHostToDevice, P->st[s]), K)))
            return rc;
    }
    const int64_t body = x_len - halo;  // samples of the shard itself
    const int64_t H = taps - 1;
    for (int64_t j = 0, o0 = 0; o0 < y_len; j++, o0 += kPipeChunk) {
        const int s = (int)(j % kPipe);
        const int64_t cn = std::min<int64_t>(kPipeChunk, y_len - o0);
        // The chunk reads shard positions [o0 - hj, o0 + cn), x[halo + p];
        // those at or past the end of x (body) read as zero and are not
        // copied. hj <= halo + o0, so the start is inside x.
        const int64_t hj = std::min<int64_t>(H, halo + o0);
        const int64_t nx = std::max<int64_t>(0, std::min<int64_t>(o0 + cn, body) - (o0 - hj));
        // xd is 16-byte aligned (the kernel's bulk-copy path) whatever hj is.
        float* xd = P->xbuf[s] + kPipePad - ((hj + 3) & ~int64_t(3));
        if (nx > 0 &&
            (rc = sg::cuda_status(cudaMemcpyAsync(xd, x + halo + o0 - hj, (size_t)nx * 4,
                                                  cudaMemcpyHostToDevice, P->st[s]), K)))
            return rc;
        if ((rc = launch_fir(K, P->ybuf[s], cn, xd, nx, hj, P->hbuf[s], taps, P->st[s])))
            return rc;
        if ((rc = sg::cuda_status(cudaMemcpyAsync(y + o0, P->ybuf[s], (size_t)cn * 4,
                                                  cudaMemcpyDeviceToHost, P->st[s]), K)))
            return rc;
    }
    // The caller's stream continues once every chunk is down.
    for (int s = 0; s < kPipe; s++) {
        if ((rc = sg::cuda_status(cudaEventRecord(P->ev[s], P->st[s]), K)) ||
            (rc = sg::cuda_status(cudaStreamWaitEvent(caller, P->ev[s], 0), K)))
            return rc;
    }
    return 0;
}

}  // extern "C"
