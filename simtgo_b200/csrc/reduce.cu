// reduce.cu -- the two reducing kernels of package kernels:
// WarpReduceSum (kernels/warpreduce.go:21-43) and Histogram
// (kernels/histogram.go:23-50).
//
// WarpReduceSum: the reference gives each warp 32 samples and folds them with
// five __shfl_down_sync steps (offsets 16, 8, 4, 2, 1). Here one thread owns
// one group of 32: TMA copies tiles of 256 groups (32 KB) into shared memory
// with the 128-byte swizzle, double-buffered, so a thread reads its group as
// eight conflict-free 16-byte chunks and forms the very same addition tree
// in registers (lane l + lane l+16, then +8, +4, +2, +1), bit for bit.
// Output stores are coalesced (one float per thread).
//
// Histogram: a persistent grid; each warp owns a private 256-bin table in
// shared memory (no contention between warps), 16-byte loads of four
// samples, shared-memory atomics, and one global atomic per non-zero bin per
// block at the end. Samples outside [0, 256) are dropped (histogram.go:38);
// bins past bins_len are not written.
#include <algorithm>

#include "common.cuh"
#include "histogram.cuh"
#include "tma.cuh"

using namespace sgd;

namespace {

// ---- WarpReduceSum -----------------------------------------------------------
constexpr int kWrRows = 256;                     // groups per tile (= threads)
constexpr uint32_t kWrTileBytes = kWrRows * 128;  // 32 KB
constexpr int kWrStages = 2;

__device__ __forceinline__ float tree32(const float (&v)[32]) {
    float a[16], b[8], c[4], d[2];
#pragma unroll
    for (int l = 0; l < 16; l++) a[l] = __fadd_rn(v[l], v[l + 16]);
#pragma unroll
    for (int l = 0; l < 8; l++) b[l] = __fadd_rn(a[l], a[l + 8]);
#pragma unroll
    for (int l = 0; l < 4; l++) c[l] = __fadd_rn(b[l], b[l + 4]);
#pragma unroll
    for (int l = 0; l < 2; l++) d[l] = __fadd_rn(c[l], c[l + 2]);
    return __fadd_rn(d[0], d[1]);
}

__global__ void __launch_bounds__(kWrRows) k_warpreduce_tma(const __grid_constant__ CUtensorMap map,
                                                            float* __restrict__ out,
                                                            int64_t rows, uint32_t* wd) {
    __shared__ __align__(8) uint64_t bars[kWrStages];
    extern __shared__ uint8_t dyn_smem[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x;
    const int64_t ntiles = (rows + kWrRows - 1) / kWrRows;

    if (tid == 0) {
        for (int s = 0; s < kWrStages; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int s = 0; s < kWrStages; s++) {
            const int64_t t = blockIdx.x + (int64_t)s * gridDim.x;
            if (t < ntiles) {
                mbar_arrive_expect_tx(&bars[s], kWrTileBytes);
                tma_load_2d(tiles + s * kWrTileBytes, &map, &bars[s], 0, (int32_t)(t * kWrRows));
            }
        }
    }
    int it = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, it++) {
        const int s = it % kWrStages;
        if (!mbar_wait(&bars[s], (uint32_t)((it / kWrStages) & 1), wd)) {
            // Gave up (the watchdog is raised): the other stage's copy, if
            // one is in flight, lands (bounded wait) before the block exits.
            if (t + gridDim.x < ntiles)
                mbar_wait(&bars[(it + 1) % kWrStages], (uint32_t)(((it + 1) / kWrStages) & 1), wd);
            return;
        }
        const int64_t row = t * kWrRows + tid;
        if (row < rows) {
            const uint8_t* tile = tiles + s * kWrTileBytes;
            float v[32];
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float4 q = *reinterpret_cast<const float4*>(tile + swz128(tid, c));
                v[4 * c] = q.x;
                v[4 * c + 1] = q.y;
                v[4 * c + 2] = q.z;
                v[4 * c + 3] = q.w;
            }
            out[row] = tree32(v);
        }
        __syncthreads();  // every thread is done with stage s
        if (tid == 0) {
            const int64_t tn = t + (int64_t)kWrStages * gridDim.x;
            if (tn < ntiles) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&bars[s], kWrTileBytes);
                tma_load_2d(tiles + s * kWrTileBytes, &map, &bars[s], 0, (int32_t)(tn * kWrRows));
            }
        }
    }
}

// Groups [r0, r1) with plain guarded loads: the ragged tail of the input
// (groups that reach past x_len read zeros there), groups past the input,
// and whole inputs whose pointer is not 16-byte aligned.
__global__ void __launch_bounds__(256) k_warpreduce_rows(float* __restrict__ out,
                                                         const float* __restrict__ x,
                                                         int64_t x_len, int64_t r0, int64_t r1) {
    for (int64_t r = r0 + global_tid(); r < r1; r += grid_threads()) {
        float v[32];
#pragma unroll
        for (int l = 0; l < 32; l++) {
            const int64_t i = 32 * r + l;
            v[l] = i < x_len ? x[i] : 0.0f;
        }
        out[r] = tree32(v);
    }
}

// ---- Histogram -----------------------------------------------------------------
constexpr int kBins = kHistBins;

__global__ void __launch_bounds__(kHistThreads) k_histogram(int* __restrict__ bins, int n_bins,
                                                            const int* __restrict__ x, int64_t m,
                                                            bool vec) {
    __shared__ int sh[kHistWarps][kBins];
    for (int k = threadIdx.x; k < kHistWarps * kBins; k += blockDim.x) (&sh[0][0])[k] = 0;
    __syncthreads();
    int* mine = sh[threadIdx.x / 32];
    hist_count(x, m, vec, [&](int v) {
        if ((unsigned)v < (unsigned)kBins) atomicAdd(mine + v, 1);
    });
    __syncthreads();
    for (int k = threadIdx.x; k < kBins; k += blockDim.x) {
        int c = 0;
#pragma unroll
        for (int w = 0; w < kHistWarps; w++) c += sh[w][k];
        if (c != 0 && k < n_bins) atomicAdd(bins + k, c);
    }
}

int launch_histogram(const char* K, int32_t* bins, int32_t bins_len, const int32_t* x, int64_t m,
                     const sg::DevInfo* d, void* stream) {
    if (m <= 0 || bins_len <= 0) return 0;
    const int64_t want = sg::ceil_div(sg::ceil_div(m, 16), kHistThreads);
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)d->sms * 2));
    sg::before_launch();
    k_histogram<<<blocks, kHistThreads, 0, (cudaStream_t)stream>>>(bins, bins_len, x, m,
                                                                   sg::aligned16(x));
    return sg::launch_status(K);
}

// ---- Histogram with a launch-sized tile -----------------------------------------
// simt Kernel.LaunchShared (simt/kernel.go:444-481) on the DynProbe body
// (simt/shared_parity_cuda_test.go:117-138): tile_len bins sized at the
// launch. `copies` private tables per block in dynamic shared memory (one
// per warp while they fit 64 KB, fewer for wide tiles); the same persistent
// grid and 16-byte loads as k_histogram; one global atomic per non-zero bin
// k < min(tile_len, n_bins) per block.
__global__ void __launch_bounds__(kHistThreads) k_histogram_dyn(int* __restrict__ bins,
                                                                int n_bins,
                                                                const int* __restrict__ x,
                                                                int64_t m, int tile, int copies,
                                                                bool vec) {
    extern __shared__ int shd[];
    for (int k = threadIdx.x; k < copies * tile; k += blockDim.x) shd[k] = 0;
    __syncthreads();
    int* mine = shd + ((threadIdx.x / 32) % copies) * tile;
    hist_count(x, m, vec, [&](int v) {
        if ((unsigned)v < (unsigned)tile) atomicAdd(mine + v, 1);
    });
    __syncthreads();
    const int kmax = min(tile, n_bins);
    for (int k = threadIdx.x; k < kmax; k += blockDim.x) {
        int c = 0;
        for (int w = 0; w < copies; w++) c += shd[w * tile + k];
        if (c != 0) atomicAdd(bins + k, c);
    }
}

}  // namespace

namespace sg {
// Shared with comm.cu: the local half of simtgo_Histogram_allreduce.
int histogram_local(const char* K, int32_t* bins, int32_t bins_len, const int32_t* x,
                    int64_t x_len, void* stream) {
    const DevInfo* d;
    int rc;
    if (bins_len < 0 || x_len < 0) return fail(SIMTGO_EARG, "%s: a length is negative", K);
    if ((rc = check_ptr(K, "bins", bins, bins_len)) || (rc = check_ptr(K, "x", x, x_len)))
        return rc;
    if ((rc = check_alias(K, {{"bins", bins, 4LL * bins_len, true}, {"x", x, 4 * x_len, false}})))
        return rc;
    if ((rc = current_device(&d))) return rc;
    return launch_histogram(K, bins, bins_len, x, x_len, d, stream);
}
}  // namespace sg

extern "C" {

int simtgo_WarpReduceSum(float* out, int32_t out_len, const float* x, int32_t x_len, int32_t grid,
                         int32_t block, void* stream) {
    const char* K = "WarpReduceSum";
    sg::clear_error();
    int64_t nt;
    const sg::DevInfo* d;
    int rc;
    if (out_len < 0 || x_len < 0) return sg::fail(SIMTGO_EARG, "simt: %s: negative length", K);
    if ((rc = sg::launch_extent_1d(K, grid, block, 128, &nt))) return rc;
    const int64_t m = std::min<int64_t>(out_len, nt / 32);
    if (m <= 0) return 0;
    if ((rc = sg::check_ptr(K, "out", out, m)) || (rc = sg::check_ptr(K, "x", x, x_len))) return rc;
    if ((rc = sg::check_alias(K, {{"out", out, 4LL * out_len, true}, {"x", x, 4LL * x_len, false}})))
        return rc;
    if ((rc = sg::current_device(&d))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t full = x_len / 32;
    int64_t tma_rows = std::min<int64_t>(m, full);
    if (!sg::aligned16(x)) tma_rows = 0;
    if (tma_rows > 0) {
        CUtensorMap map;
        if ((rc = sg::tma_encode_2d(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, x, 32, (uint64_t)full,
                                    128, 32, kWrRows, CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
        const size_t smem = (size_t)kWrStages * kWrTileBytes + 1024;
        static bool attr_set[64] = {};
        if (!attr_set[d->device & 63]) {
            rc = sg::cuda_status(cudaFuncSetAttribute(k_warpreduce_tma,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      (int)smem),
                                 "cudaFuncSetAttribute(WarpReduceSum)");
            if (rc) return rc;
            attr_set[d->device & 63] = true;
        }
        const int64_t ntiles = sg::ceil_div(tma_rows, kWrRows);
        const int blocks = (int)std::min<int64_t>(ntiles, (int64_t)d->sms * 3);
        sg::before_launch();
        k_warpreduce_tma<<<blocks, kWrRows, smem, s>>>(map, out, tma_rows,
                                                       sg::watchdog_device_ptr());
        if ((rc = sg::launch_status(K))) return rc;
    }
    if (tma_rows < m) {
        const int64_t rows = m - tma_rows;
        const int blocks = (int)std::max<int64_t>(
            1, std::min<int64_t>(sg::ceil_div(rows, 256), (int64_t)d->sms * 4));
        sg::before_launch();
        k_warpreduce_rows<<<blocks, 256, 0, s>>>(out, x, x_len, tma_rows, m);
        if ((rc = sg::launch_status(K))) return rc;
    }
    return 0;
}

int simtgo_Histogram(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                     int32_t grid, int32_t block, void* stream) {
    const char* K = "Histogram";
    sg::clear_error();
    int64_t nt;
    const sg::DevInfo* d;
    int rc;
    if (bins_len < 0 || x_len < 0) return sg::fail(SIMTGO_EARG, "simt: %s: negative length", K);
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(x_len, nt);
    if (m <= 0 || bins_len == 0) return 0;
    if ((rc = sg::check_ptr(K, "bins", bins, bins_len)) || (rc = sg::check_ptr(K, "x", x, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"bins", bins, 4LL * bins_len, true},
                                  {"x", x, 4LL * x_len, false}})))
        return rc;
    if ((rc = sg::current_device(&d))) return rc;
    return launch_histogram(K, bins, bins_len, x, m, d, stream);
}

int simtgo_HistogramDyn(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                        int32_t tile_len, int32_t grid, int32_t block, void* stream) {
    const char* K = "HistogramDyn";
    sg::clear_error();
    int64_t nt;
    const sg::DevInfo* d;
    int rc;
    if (bins_len < 0 || x_len < 0 || tile_len < 0)
        return sg::fail(SIMTGO_EARG, "simt: %s: negative length or tile", K);
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    if ((rc = sg::current_device(&d))) return rc;
    // simt.SharedMemoryError (simt/shared_parity_cuda_test.go:216-227): a
    // tile larger than a block's shared memory is refused before the launch.
    const int64_t limit = (d->max_smem_optin - 1024) / 4;
    if (tile_len > limit)
        return sg::fail(SIMTGO_ESIZE,
                        "simt: %s: a shared tile of %d int32 elements (%lld bytes) exceeds the "
                        "%lld bytes a block can have",
                        K, tile_len, 4LL * tile_len, 4LL * limit);
    const int64_t m = std::min<int64_t>(x_len, nt);
    if (m <= 0 || bins_len == 0 || tile_len == 0) return 0;
    if ((rc = sg::check_ptr(K, "bins", bins, bins_len)) || (rc = sg::check_ptr(K, "x", x, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"bins", bins, 4LL * bins_len, true},
                                  {"x", x, 4LL * x_len, false}})))
        return rc;
    int copies = kHistWarps;
    while (copies > 1 && (int64_t)copies * tile_len * 4 > 64 * 1024) copies /= 2;
    const size_t smem = (size_t)copies * tile_len * 4;
    if (smem > 48 * 1024 &&
        (rc = sg::cuda_status(cudaFuncSetAttribute(k_histogram_dyn,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem),
                              "cudaFuncSetAttribute(HistogramDyn)")))
        return rc;
    // Enough samples per block that the per-block flush of the tile (one
    // atomic per non-zero bin) stays small next to the counting.
    const int64_t want = std::min(sg::ceil_div(sg::ceil_div(m, 16), kHistThreads),
                                  sg::ceil_div(m, 8LL * tile_len));
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)d->sms * 2));
    sg::before_launch();
    k_histogram_dyn<<<blocks, kHistThreads, smem, (cudaStream_t)stream>>>(
        bins, bins_len, x, m, tile_len, copies, sg::aligned16(x));
    return sg::launch_status(K);
}

int simtgo_Histogram_shard(int32_t* bins, int32_t bins_len, const int32_t* x, int64_t x_len,
                           void* stream) {
    sg::clear_error();
    return sg::histogram_local("Histogram_shard", bins, bins_len, x, x_len, stream);
}

}  // extern "C"
