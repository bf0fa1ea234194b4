/*
 * ref_shim.h -- TEST INFRASTRUCTURE ONLY. Force-included (g++ -include) in
 * front of the reference's generated CUDA C (kernels/prebuilt/*.cu) so that
 * those sources, unmodified and read where they lie, compile as host C++.
 *
 * This is the technique simtgo itself uses for its host oracle
 * (internal/fuzz/hostrun/hostrun.go:1-50, driver.go:27-93), extended to the
 * cooperative kernels: every CUDA thread of a block is a ucontext coroutine
 * on one OS thread; __syncthreads() yields to the block's scheduler, which
 * resumes each thread in turn, so all threads meet at every barrier.
 * __shared__ arrays become static thread_local (one copy per worker thread =
 * per block in flight), which is what makes them shared by the coroutines.
 */
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

struct shim_uint3 {
    unsigned x, y, z;
};
typedef shim_uint3 shim_dim3;

extern thread_local shim_uint3 threadIdx;
extern thread_local shim_uint3 blockIdx;
extern thread_local shim_dim3 blockDim;
extern thread_local shim_dim3 gridDim;

#define __global__
#define __device__
#define __shared__ static thread_local
#define __restrict__ __restrict

void __syncthreads();
int atomicAdd(int* p, int v);
float __shfl_down_sync(unsigned mask, float v, int delta);

using std::fabs;
using std::sqrt;
