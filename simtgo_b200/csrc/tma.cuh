// tma.cuh -- Tensor Memory Accelerator plumbing for sm_100a: host-side
// tensor-map encoding (cuTensorMapEncodeTiled, reached through the runtime's
// driver entry point so the library needs no link against libcuda) and
// device-side mbarrier / cp.async.bulk.tensor wrappers in inline PTX.
//
// No load here is a cluster-multicast load: every tensor map covers this GPU's
// own memory and every CTA fetches its own tiles.
#pragma once
#ifndef __CUDACC_RTC__  // run-time compilation (tile_jit.cu) brings its own prelude
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#endif

#include "common.cuh"

#ifndef __CUDACC_RTC__
namespace sg {

// Encodes a 2-D tiled map over a row-major array of `rows` rows of `inner`
// elements (`row_bytes` apart), box = box_inner x box_rows, with `swizzle`.
// Returns 0, or SIMTGO_EARG/SIMTGO_EDEVICE with a message.
int tma_encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                  uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMapSwizzle swizzle);

}  // namespace sg
#endif

namespace sgd {

// Spins of a bounded mbarrier wait before the kernel gives up and raises
// the watchdog. Each try_wait suspends the thread for a while in hardware,
// so this is seconds, far beyond any real copy.
constexpr uint32_t kMbarSpinLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Makes initialised barriers visible to the async proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of bar to complete; false (and the watchdog
// raised) if it did not within kMbarSpinLimit tries.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* wd) {
    for (uint32_t i = 0; i < kMbarSpinLimit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    watchdog_raise(wd, 1u /* sg::WATCHDOG_TMA */);
    return false;
}

// 2-D tiled TMA load of the box at (x = inner coordinate, y = row) into
// shared memory, completing on bar. x must be a multiple of 16 bytes'
// worth of elements; y may be negative or past the end (zero fill).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Byte offset of float4 chunk `chunk` (0..7) of row `row` in a 128-byte-row
// tile written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (tile base 1024-byte
// aligned): the chunk index is XORed with the row index modulo 8.
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace sgd
