/*
 * ref_driver.cpp -- TEST INFRASTRUCTURE ONLY. Compiles the reference's
 * generated kernels (kernels/prebuilt/*.cu, included from the reference tree
 * by oracle/Makefile's -I) for the host and exposes one ref_<Kernel>(...)
 * launcher each, with the kernel's own parameters plus the launch geometry.
 *
 * Kernels with no barrier or warp exchange run their threads one after the
 * other. FIR, Histogram, Transpose and WarpReduceSum run each block's threads
 * as coroutines (see ref_shim.h). Blocks are spread over worker threads, as
 * gpu.RunCPU spreads them over goroutines (gpu/gpu.go:319-356).
 *
 * Built with -ffp-contract=off, so float expressions round each operation,
 * as the amd64 emulator does (hostrun.go:386 uses the same flag).
 */
#include <ucontext.h>

#include <atomic>
#include <cstdlib>
#include <functional>
#include <thread>
#include <vector>

thread_local shim_uint3 threadIdx;
thread_local shim_uint3 blockIdx;
thread_local shim_dim3 blockDim;
thread_local shim_dim3 gridDim;

#include "BandGain.cu"
#include "Classify.cu"
#include "FIR.cu"
#include "Gray.cu"
#include "Histogram.cu"
#include "Magnitude.cu"
#include "MagnitudeFast.cu"
#include "Quantize.cu"
#include "Scale.cu"
#include "Softclip.cu"
#include "Transpose.cu"
#include "VecAdd.cu"
#include "WarpReduceSum.cu"

namespace {

constexpr size_t kStack = 64 * 1024;

struct BlockSched {
    std::vector<ucontext_t> ctx;
    std::vector<char> stacks;
    std::vector<unsigned char> done;
    std::vector<shim_uint3> tid;
    ucontext_t main_ctx;
    int cur = 0;
    const std::function<void()>* body = nullptr;
    float slots[1024];
};

thread_local BlockSched* g_sched = nullptr;

void co_entry() {
    BlockSched* s = g_sched;
    (*s->body)();
    s->done[s->cur] = 1;
}

int g_workers = 1;

/* Run every block of the grid; `coop` selects coroutine threads. */
void launch(shim_dim3 grid, shim_dim3 block, bool coop, const std::function<void()>& body) {
    const long nblocks = (long)grid.x * grid.y * grid.z;
    const int nthreads = (int)(block.x * block.y * block.z);
    if (nblocks <= 0 || nthreads <= 0) return;
    int workers = g_workers < 1 ? 1 : g_workers;
    if (workers > nblocks) workers = (int)nblocks;
    std::atomic<long> next{0};
    auto worker = [&]() {
        gridDim = grid;
        blockDim = block;
        BlockSched sched;
        if (coop) {
            sched.ctx.resize(nthreads);
            sched.stacks.resize((size_t)nthreads * kStack);
            sched.done.resize(nthreads);
            sched.tid.resize(nthreads);
            sched.body = &body;
        }
        g_sched = &sched;
        for (;;) {
            long b = next.fetch_add(1);
            if (b >= nblocks) break;
            blockIdx.x = (unsigned)(b % grid.x);
            blockIdx.y = (unsigned)((b / grid.x) % grid.y);
            blockIdx.z = (unsigned)(b / ((long)grid.x * grid.y));
            int t = 0;
            for (unsigned z = 0; z < block.z; z++)
                for (unsigned y = 0; y < block.y; y++)
                    for (unsigned x = 0; x < block.x; x++, t++) {
                        shim_uint3 id{x, y, z};
                        if (!coop) {
                            threadIdx = id;
                            body();
                        } else {
                            sched.tid[t] = id;
                        }
                    }
            if (!coop) continue;
            for (int i = 0; i < nthreads; i++) {
                getcontext(&sched.ctx[i]);
                sched.ctx[i].uc_stack.ss_sp = &sched.stacks[(size_t)i * kStack];
                sched.ctx[i].uc_stack.ss_size = kStack;
                sched.ctx[i].uc_link = &sched.main_ctx;
                makecontext(&sched.ctx[i], co_entry, 0);
                sched.done[i] = 0;
            }
            bool alive = true;
            while (alive) {
                alive = false;
                for (int i = 0; i < nthreads; i++) {
                    if (sched.done[i]) continue;
                    threadIdx = sched.tid[i];
                    sched.cur = i;
                    swapcontext(&sched.main_ctx, &sched.ctx[i]);
                    if (!sched.done[i]) alive = true;
                }
            }
        }
        g_sched = nullptr;
    };
    if (workers == 1) {
        worker();
        return;
    }
    std::vector<std::thread> th;
    for (int w = 0; w < workers; w++) th.emplace_back(worker);
    for (auto& t : th) t.join();
}

shim_dim3 d1(int n) { return shim_dim3{(unsigned)n, 1u, 1u}; }

}  // namespace

void __syncthreads() {
    BlockSched* s = g_sched;
    swapcontext(&s->ctx[s->cur], &s->main_ctx);
}

int atomicAdd(int* p, int v) { return __atomic_fetch_add(p, v, __ATOMIC_RELAXED); }

float __shfl_down_sync(unsigned, float v, int delta) {
    BlockSched* s = g_sched;
    int tid = (int)(threadIdx.x + blockDim.x * (threadIdx.y + blockDim.y * threadIdx.z));
    s->slots[tid] = v;
    __syncthreads();
    int lane = tid % 32;
    float r = (lane + delta < 32) ? s->slots[tid + delta] : v;
    __syncthreads();
    return r;
}

extern "C" {

void ref_set_workers(int n) { g_workers = n < 1 ? 1 : n; }

void ref_VecAdd(float* c, int c_len, const float* a, int a_len, const float* b, int b_len,
                int grid, int block) {
    launch(d1(grid), d1(block), false, [&] { VecAdd(c, c_len, a, a_len, b, b_len); });
}
void ref_Scale(float* y, int y_len, const float* x, int x_len, float k, int grid, int block) {
    launch(d1(grid), d1(block), false, [&] { Scale(y, y_len, x, x_len, k); });
}
void ref_Magnitude(float* m, int m_len, const float* re, int re_len, const float* im, int im_len,
                   int grid, int block) {
    launch(d1(grid), d1(block), false, [&] { Magnitude(m, m_len, re, re_len, im, im_len); });
}
void ref_MagnitudeFast(float* m, int m_len, const float* re, int re_len, const float* im,
                       int im_len, float scale, int grid, int block) {
    launch(d1(grid), d1(block), false,
           [&] { MagnitudeFast(m, m_len, re, re_len, im, im_len, scale); });
}
void ref_Softclip(float* y, int y_len, const float* x, int x_len, float t, int grid, int block) {
    launch(d1(grid), d1(block), false, [&] { Softclip(y, y_len, x, x_len, t); });
}
void ref_Classify(float* out, int out_len, const float* x, int x_len, const float* e, int e_len,
                  int grid, int block) {
    launch(d1(grid), d1(block), false, [&] { Classify(out, out_len, x, x_len, e, e_len); });
}
void ref_BandGain(float* y, int y_len, const float* x, int x_len, const Band* bands,
                  int bands_len, const Shape* cfg, int grid, int block) {
    Shape s = *cfg;
    launch(d1(grid), d1(block), false,
           [&] { BandGain(y, y_len, x, x_len, bands, bands_len, s); });
}
void ref_Quantize(int* code, int code_len, long long* energy, int energy_len, bool* clipped,
                  int clipped_len, const float* x, int x_len, float step, unsigned seed,
                  int grid, int block) {
    launch(d1(grid), d1(block), false, [&] {
        Quantize(code, code_len, energy, energy_len, clipped, clipped_len, x, x_len, step, seed);
    });
}
void ref_Gray(unsigned char* out, int out_len, const unsigned char* rgb, int rgb_len, int grid,
              int block) {
    launch(d1(grid), d1(block), false, [&] { Gray(out, out_len, rgb, rgb_len); });
}
void ref_Histogram(int* bins, int bins_len, const int* x, int x_len, int grid, int block) {
    launch(d1(grid), d1(block), true, [&] { Histogram(bins, bins_len, x, x_len); });
}
void ref_Transpose(float* out, int out_len, const float* in, int in_len, int w, int h, int gx,
                   int gy) {
    launch(shim_dim3{(unsigned)gx, (unsigned)gy, 1u}, shim_dim3{16u, 16u, 1u}, true,
           [&] { Transpose(out, out_len, in, in_len, w, h); });
}
void ref_WarpReduceSum(float* out, int out_len, const float* x, int x_len, int grid) {
    launch(d1(grid), d1(128), true, [&] { WarpReduceSum(out, out_len, x, x_len); });
}
void ref_FIR(float* y, int y_len, const float* x, int x_len, const float* h, int h_len,
             int grid) {
    launch(d1(grid), d1(256), true, [&] { FIR(y, y_len, x, x_len, h, h_len); });
}

}  // extern "C"
