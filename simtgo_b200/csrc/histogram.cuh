// histogram.cuh -- the counting loop the histogram kernels share (reduce.cu:
// Histogram and the launch-sized-tile form; comm.cu: the fused histogram +
// all-reduce): a persistent grid over x[0, m), 16-byte loads of four int32
// samples (four loads in flight per thread) when x is 16-byte aligned, and
// add(v) per sample.
#pragma once

#include "common.cuh"

namespace sgd {

constexpr int kHistThreads = 512;
constexpr int kHistWarps = kHistThreads / 32;
constexpr int kHistBins = 256;  // kernels/histogram.go: 256 bins

template <class Add>
__device__ __forceinline__ void hist_count(const int* __restrict__ x, int64_t m, bool vec,
                                           Add add) {
    const int64_t stride = grid_threads();
    int64_t done = 0;
    if (vec) {
        const int64_t nvec = m / 4;
        int64_t v = global_tid();
        for (; v + 3 * stride < nvec; v += 4 * stride) {
            int4 q[4];
#pragma unroll
            for (int u = 0; u < 4; u++) q[u] = ld_stream_i4(x + 4 * (v + u * stride));
#pragma unroll
            for (int u = 0; u < 4; u++) {
                add(q[u].x);
                add(q[u].y);
                add(q[u].z);
                add(q[u].w);
            }
        }
        for (; v < nvec; v += stride) {
            const int4 q = ld_stream_i4(x + 4 * v);
            add(q.x);
            add(q.y);
            add(q.z);
            add(q.w);
        }
        done = nvec * 4;
    }
    for (int64_t i = done + global_tid(); i < m; i += stride) add(x[i]);
}

}  // namespace sgd
