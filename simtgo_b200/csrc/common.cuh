// common.cuh -- shared host/device plumbing of libsimtgo_b200.so: status
// codes and messages, per-device properties, the launch-contract checks that
// simt.Kernel.launch makes on the host (simt/kernel.go:488-514), and the
// 128-bit streaming load/store helpers the memory-bound kernels share.
#pragma once

// Under run-time compilation (a tile graph's specialised kernel, tile_jit.cu)
// only the device helpers below are compiled; the JIT's prelude supplies the
// integer types.
#ifndef __CUDACC_RTC__
#include <cuda_runtime.h>
#include <stdint.h>

#include <initializer_list>

#include "../../include/simtgo_b200.h"

namespace sg {

// ---- status and messages -------------------------------------------------
// Records a message for the calling thread and returns code.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// 0 for cudaSuccess; otherwise records "<what>: <cuda error string>" and
// returns the cudaError_t value (positive).
int cuda_status(cudaError_t e, const char* what);
// Clears the calling thread's message.
void clear_error();

// ---- device properties -----------------------------------------------------
struct DevInfo {
    int device = -1;
    int sms = 0;
    int cc_major = 0, cc_minor = 0;
    int max_smem_optin = 0;
    int smem_per_sm = 0;
};
// Properties of the current device (cached). Returns 0 or a status code.
int current_device(const DevInfo** out);

// ---- the watchdog flag -----------------------------------------------------
// Every bounded spin (mbarrier, peer flag) that gives up sets a bit here and
// returns instead of hanging; simtgo_stream_sync reports it.
enum : uint32_t {
    WATCHDOG_TMA = 1u,
    WATCHDOG_PEER = 2u,
};
uint32_t* watchdog_device_ptr();  // device address of the flag word (current device)
int watchdog_check_and_clear(uint32_t* bits);

// Private resources released by simtgo_shutdown (fir.cu).
int fir_host_release();
int tile_pool_release();  // trims the tile reductions' scratch pools (simtgo_shutdown)
int tile_jit_release();   // unloads the specialised tile kernels' modules (simtgo_shutdown)

// ---- launch-contract checks (simt/kernel.go:293-369, :488-514) -------------
// The covered thread extent of a 1-D launch, or a status code. Refuses what
// cuLaunchKernel refuses (grid or block <= 0, block > 1024) and, if
// required_block != 0, a block of another size (simt.BlockSizeError).
int launch_extent_1d(const char* kernel, int32_t grid, int32_t block, int32_t required_block,
                     int64_t* threads);

struct Span {
    const char* name;
    const void* ptr;
    int64_t bytes;
    bool written;
};
// simt.AliasError: two slices overlap and the kernel writes through one.
int check_alias(const char* kernel, std::initializer_list<Span> spans);
// SIMTGO_ENULL for a null pointer that the extent needs.
int check_ptr(const char* kernel, const char* name, const void* p, int64_t need);
// SIMTGO_ELENGTH where gpu.RunCPU would index past the slice.
int check_len(const char* kernel, const char* name, int64_t len, int64_t need);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Discards an error left behind by some earlier runtime call of this
// thread (someone else's), so launch_status reports only the launch that
// follows. Sticky errors survive this and are reported all the same.
inline void before_launch() { (void)cudaGetLastError(); }
// Launch-error check after a <<<>>> launch.
int launch_status(const char* kernel);

}  // namespace sg
#endif  // __CUDACC_RTC__

// ---- device helpers ----------------------------------------------------------
namespace sgd {

// 128-bit load of read-only data that is streamed once: no L1 allocation.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
    float4 v;
    asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p));
    return v;
}
__device__ __forceinline__ int4 ld_stream_i4(const void* p) {
    int4 v;
    asm("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}
// 128-bit streaming store (evict-first).
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_stream_i4(void* p, int4 v) {
    asm volatile("st.global.cs.v4.s32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ int64_t global_tid() {
    return (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
}
__device__ __forceinline__ int64_t grid_threads() { return (int64_t)gridDim.x * blockDim.x; }

// Sets a bit of the device's watchdog word (sg::watchdog_device_ptr()).
__device__ __forceinline__ void watchdog_raise(uint32_t* wd, uint32_t bit) {
    if (wd) atomicOr(wd, bit);
}

}  // namespace sgd
