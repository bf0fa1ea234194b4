// fir.cu -- FIR (kernels/fir.go:17-46) and its long, sharded form.
//
// y[j] = sum_k h[k] * x[j + halo - k], x read as zero outside [0, x_len),
// accumulated as acc = fma(h[k], x, acc) for k = 0, 1, ..., taps-1: the
// order and rounding of the reference's device code, where nvcc contracts
// `acc += h[k] * tile[...]` (kernels/prebuilt/FIR.cu:24-27).
//
// B200 design. A 256-thread block produces 8192 consecutive outputs; thread
// t owns 32 consecutive outputs, so every loaded sample feeds up to 32
// fused multiply-adds from registers (the reference does one output per
// thread, one shared load and one global tap load per multiply-add):
//  * the block's signal span (its outputs plus a taps-1 halo) arrives by
//    2-D TMA in 32-row boxes of 32 floats, 128-byte swizzled, so a row of 32
//    samples is one 128-byte line and the chunk order within each row is
//    permuted by the row index;
//  * taps are staged once per block in shared memory and read as broadcast
//    16-byte loads, eight per chunk;
//  * per chunk of 8 taps a thread loads the 39 samples its 32 outputs need
//    as eleven 16-byte loads -- conflict-free because lane t reads row t
//    plus a common offset and the swizzle spreads those rows over all banks
//    -- then issues 8 x 32 FFMA with every operand in a register;
//  * the window's alignment within a 16-byte chunk, (D - 7) mod 4, is the
//    same for every block and chunk, so it is a template parameter and all
//    register indices are compile-time.
// At 127 taps the kernel is bound by FP32 FMA issue, not by HBM.
#include <algorithm>

#include "common.cuh"
#include "tma.cuh"

using namespace sgd;

namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 32;                      // outputs per thread
constexpr int kTileOut = kThreads * kPerThread;     // 8192 outputs per block
constexpr int kChunk = 8;                           // taps per register chunk
constexpr int kWin = 44;                            // window floats (11 x 16 B)
constexpr int kBoxRows = 32;                        // TMA box: 32 rows x 32 floats
constexpr uint32_t kBoxBytes = kBoxRows * 128;

struct FirGeom {
    int64_t y_len;   // outputs of this launch
    int64_t x_len;   // samples in x
    int64_t halo;    // x[halo + j] is the sample of output j
    int32_t taps;
    int32_t taps_pad;   // taps rounded up to kChunk
    int32_t D;          // tile position of output ob + 0 at tap 0 (same for every block)
    int32_t rows;       // shared rows staged per block (multiple of kBoxRows)
    int64_t full_rows;  // x_len / 32: rows the tensor map covers
};

// Rows of the staged tile a given tap count needs (see the header comment
// of k_fir for the bounds).
inline int tile_rows(int taps) {
    const int need = (taps + 8258) / 32 + 1;
    return (int)sg::ceil_div(need, kBoxRows) * kBoxRows;
}

template <int SH>
__device__ __forceinline__ void fir_chunk(const uint8_t* tile, const float* hs, int k0, int nk,
                                          int s4, float2 (&acc)[kPerThread / 2]) {
    // Window floats wv[i] = tile position s4 + i, i < 44.
    float wv[kWin];
#pragma unroll
    for (int c = 0; c < kWin / 4; c++) {
        const int pos = s4 + 4 * c;
        const float4 q =
            *reinterpret_cast<const float4*>(tile + swz128((uint32_t)pos >> 5, ((uint32_t)pos & 31u) >> 2));
        wv[4 * c] = q.x;
        wv[4 * c + 1] = q.y;
        wv[4 * c + 2] = q.z;
        wv[4 * c + 3] = q.w;
    }
    const float4 ha = *reinterpret_cast<const float4*>(hs + k0);
    const float4 hb = *reinterpret_cast<const float4*>(hs + k0 + 4);
    const float hv[kChunk] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
    // Outputs 2i and 2i+1 advance together through one packed FP32 FMA
    // (fma.rn.f32x2): each lane is exactly fmaf, so every output keeps its
    // own k-ordered chain while the FMA work takes half the issue slots.
#pragma unroll
    for (int u = 0; u < kChunk; u++) {
        if (nk == kChunk || u < nk) {
            const float2 hh = make_float2(hv[u], hv[u]);
#pragma unroll
            for (int i = 0; i < kPerThread / 2; i++)
                acc[i] = __ffma2_rn(hh,
                                    make_float2(wv[SH + 7 - u + 2 * i], wv[SH + 8 - u + 2 * i]),
                                    acc[i]);
        }
    }
}

// One block = outputs [ob, ob + 8192). Tile row 0 is signal row R0 =
// (ob + halo - D) / 32; output ob + 32t + r at tap k reads tile position
// D + 32t + r - k, with D = a + (taps-1) + 32 and a = (halo - (taps-1)) mod 32,
// so positions stay >= 22 (a spare row absorbs the last, partial chunk) and
// below 32*rows.
template <int SH>
__global__ void __launch_bounds__(kThreads, 2) k_fir(const __grid_constant__ CUtensorMap map,
                                                      bool use_tma, float* __restrict__ y,
                                                      const float* __restrict__ x,
                                                      const float* __restrict__ h, FirGeom g,
                                                      bool vec_out, uint32_t* wd) {
    __shared__ __align__(8) uint64_t bar;
    extern __shared__ uint8_t dyn_smem[];
    uint8_t* tile = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
    float* hs = reinterpret_cast<float*>(tile + (size_t)g.rows * 128);
    const int tid = threadIdx.x;
    const int64_t ob = (int64_t)blockIdx.x * kTileOut;
    const int64_t R0 = (ob + g.halo - g.D) / 32;  // exact: ob + halo - D = 0 mod 32

    if (use_tma) {
        if (tid == 0) {
            mbar_init(&bar, 1);
            fence_mbar_init();
        }
        __syncthreads();  // no thread may test the barrier before it exists
        if (tid == 0) {
            mbar_arrive_expect_tx(&bar, (uint32_t)g.rows * 128u);
            for (int b = 0; b < g.rows / kBoxRows; b++)
                tma_load_2d(tile + b * kBoxBytes, &map, &bar, 0, (int32_t)(R0 + b * kBoxRows));
        }
    } else {
        // Unaligned or very short signal: stage with guarded loads.
        for (int i = tid; i < g.rows * 32; i += kThreads) {
            const int row = i >> 5, col = i & 31;
            const int64_t src = (R0 + row) * 32 + col;
            const float v = (src >= 0 && src < g.x_len) ? x[src] : 0.0f;
            *reinterpret_cast<float*>(tile + swz128(row, col >> 2) + (col & 3) * 4) = v;
        }
    }
    for (int k = tid; k < g.taps_pad; k += kThreads) hs[k] = k < g.taps ? h[k] : 0.0f;
    if (use_tma) {
        if (!mbar_wait(&bar, 0, wd)) return;
        // The tensor map covers whole rows only; the signal's ragged last row
        // (x_len mod 32 samples) was zero-filled and is patched here.
        const int64_t rem = g.x_len - g.full_rows * 32;
        const int64_t prow = g.full_rows - R0;
        if (rem > 0 && prow >= 0 && prow < g.rows && tid < rem) {
            *reinterpret_cast<float*>(tile + swz128((uint32_t)prow, tid >> 2) + (tid & 3) * 4) =
                x[g.full_rows * 32 + tid];
        }
    }
    __syncthreads();

    float2 acc[kPerThread / 2];  // acc[i] = outputs (2i, 2i+1) of this thread
#pragma unroll
    for (int i = 0; i < kPerThread / 2; i++) acc[i] = make_float2(0.0f, 0.0f);
    const int sbase = g.D + 32 * tid - 7 - SH;  // s4 at k0 = 0
    for (int k0 = 0; k0 < g.taps; k0 += kChunk)
        fir_chunk<SH>(tile, hs, k0, min(kChunk, g.taps - k0), sbase - k0, acc);

    const int64_t j0 = ob + (int64_t)kPerThread * tid;
    if (vec_out && j0 + kPerThread <= g.y_len) {
#pragma unroll
        for (int c = 0; c < kPerThread / 4; c++)
            st_stream_f4(y + j0 + 4 * c, make_float4(acc[2 * c].x, acc[2 * c].y,
                                                     acc[2 * c + 1].x, acc[2 * c + 1].y));
    } else {
#pragma unroll
        for (int r = 0; r < kPerThread; r++)
            if (j0 + r < g.y_len) y[j0 + r] = (r & 1) ? acc[r / 2].y : acc[r / 2].x;
    }
}

using FirKernel = void (*)(const CUtensorMap, bool, float*, const float*, const float*, FirGeom,
                           bool, uint32_t*);

int launch_fir(const char* K, float* y, int64_t y_len, const float* x, int64_t x_len,
               int64_t halo, const float* h, int32_t taps, void* stream) {
    const sg::DevInfo* d;
    int rc;
    if ((rc = sg::current_device(&d))) return rc;
    if (y_len <= 0) return 0;
    FirGeom g;
    g.y_len = y_len;
    g.x_len = x_len;
    g.halo = halo;
    g.taps = taps;
    g.taps_pad = (int32_t)sg::ceil_div(std::max(taps, 1), kChunk) * kChunk;
    const int64_t a = (((halo - (taps - 1)) % 32) + 32) % 32;
    g.D = (int32_t)(a + (taps - 1) + 32);
    g.rows = tile_rows(taps);
    g.full_rows = x_len / 32;
    const int sh = (int)(((g.D - 7) % 4 + 4) % 4);

    CUtensorMap map;
    bool use_tma = sg::aligned16(x) && g.full_rows >= 1;
    if (use_tma) {
        if ((rc = sg::tma_encode_2d(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, x, 32,
                                    (uint64_t)g.full_rows, 128, 32, kBoxRows,
                                    CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
    } else {
        memset(&map, 0, sizeof map);
    }
    static const FirKernel kernels[4] = {k_fir<0>, k_fir<1>, k_fir<2>, k_fir<3>};
    const FirKernel kern = kernels[sh];
    const size_t smem = 1024 + (size_t)g.rows * 128 + (size_t)g.taps_pad * 4;
    rc = sg::cuda_status(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
        "cudaFuncSetAttribute(FIR)");
    if (rc) return rc;
    const int64_t blocks = sg::ceil_div(y_len, kTileOut);
    if (blocks > 0x7fffffffLL) return sg::fail(SIMTGO_ESIZE, "%s: y_len too large", K);
    sg::before_launch();
    kern<<<(unsigned)blocks, kThreads, smem, (cudaStream_t)stream>>>(
        map, use_tma, y, x, h, g, sg::aligned16(y), sg::watchdog_device_ptr());
    return sg::launch_status(K);
}

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

}  // extern "C"
