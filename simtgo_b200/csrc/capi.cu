// capi.cu -- library-wide entry points and the host helpers of common.cuh:
// thread-local error messages, the per-device property cache, the watchdog
// word, and the launch-contract checks simt.Kernel.launch makes
// (simt/kernel.go:293-369, :488-514).
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace {
thread_local char t_msg[1024] = "";

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
sg::DevInfo g_dev[kMaxDevices];
uint32_t* g_wd_ptr[kMaxDevices];
}  // namespace

// One flag word per device (each device that loads the module gets its own).
__device__ uint32_t g_watchdog_word;

namespace sg {

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof t_msg, fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { t_msg[0] = 0; }

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 0;
    snprintf(t_msg, sizeof t_msg, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return (int)e;
}

int launch_status(const char* kernel) {
    return cuda_status(cudaGetLastError(), kernel);
}

int current_device(const DevInfo** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(SIMTGO_EDEVICE, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevInfo& d = g_dev[dev];
    if (d.device < 0) {
        cudaDeviceProp p;
        e = cudaGetDeviceProperties(&p, dev);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
        if (p.major != 10 || p.minor != 0)
            return fail(SIMTGO_EDEVICE,
                        "device %d is sm_%d%d (%s); libsimtgo_b200 is built for sm_100a (B200)",
                        dev, p.major, p.minor, p.name);
        d.sms = p.multiProcessorCount;
        d.cc_major = p.major;
        d.cc_minor = p.minor;
        d.max_smem_optin = (int)p.sharedMemPerBlockOptin;
        d.smem_per_sm = (int)p.sharedMemPerMultiprocessor;
        d.device = dev;
    }
    *out = &d;
    return 0;
}

uint32_t* watchdog_device_ptr() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!g_wd_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_watchdog_word) != cudaSuccess) return nullptr;
        g_wd_ptr[dev] = (uint32_t*)p;
    }
    return g_wd_ptr[dev];
}

int watchdog_check_and_clear(uint32_t* bits) {
    *bits = 0;
    uint32_t* p = watchdog_device_ptr();
    if (!p) return 0;
    uint32_t v = 0;
    cudaError_t e = cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_status(e, "reading the watchdog word");
    if (v) {
        uint32_t z = 0;
        e = cudaMemcpy(p, &z, sizeof z, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_status(e, "clearing the watchdog word");
    }
    *bits = v;
    return 0;
}

int launch_extent_1d(const char* kernel, int32_t grid, int32_t block, int32_t required_block,
                     int64_t* threads) {
    if (block <= 0 || block > 1024)
        return fail(SIMTGO_ELAUNCH, "simt: %s: a block of %d threads is not launchable", kernel,
                    block);
    if (required_block != 0 && block != required_block)
        return fail(SIMTGO_EBLOCK, "simt: %s requires block == %d, got %d", kernel,
                    required_block, block);
    if (grid <= 0)
        return fail(SIMTGO_ELAUNCH, "simt: %s: a grid of %d blocks is not launchable", kernel,
                    grid);
    *threads = (int64_t)grid * block;
    return 0;
}

int check_alias(const char* kernel, std::initializer_list<Span> spans) {
    const Span* v = spans.begin();
    size_t n = spans.size();
    for (size_t i = 0; i < n; i++) {
        if (!v[i].ptr || v[i].bytes <= 0) continue;
        for (size_t j = i + 1; j < n; j++) {
            if (!v[j].ptr || v[j].bytes <= 0) continue;
            if (!v[i].written && !v[j].written) continue;  // restrict allows shared reads
            uintptr_t a0 = (uintptr_t)v[i].ptr, a1 = a0 + (uintptr_t)v[i].bytes;
            uintptr_t b0 = (uintptr_t)v[j].ptr, b1 = b0 + (uintptr_t)v[j].bytes;
            if (a0 >= b1 || b0 >= a1) continue;
            const Span& w = v[i].written ? v[i] : v[j];
            const Span& o = v[i].written ? v[j] : v[i];
            return fail(SIMTGO_EALIAS,
                        "simt: %s: parameters %s and %s were given overlapping device memory, "
                        "and the kernel writes through %s; the generated C declares every "
                        "pointer __restrict__, which promises that they do not overlap",
                        kernel, w.name, o.name, w.name);
        }
    }
    return 0;
}

int check_ptr(const char* kernel, const char* name, const void* p, int64_t need) {
    if (need > 0 && p == nullptr)
        return fail(SIMTGO_ENULL, "simt: %s: %s is null but %lld elements are accessed", kernel,
                    name, (long long)need);
    return 0;
}

int check_len(const char* kernel, const char* name, int64_t len, int64_t need) {
    if (len < need)
        return fail(SIMTGO_ELENGTH,
                    "simt: %s: %s has %lld elements but the launch reads or writes %lld "
                    "(gpu.RunCPU panics: index out of range)",
                    kernel, name, (long long)len, (long long)need);
    return 0;
}

}  // namespace sg

extern "C" {

const char* simtgo_last_error(void) { return t_msg; }

const char* simtgo_version(void) { return "simtgo_b200 0.2.0 (sm_100a; tile programs specialised by NVRTC)"; }

int simtgo_shutdown(void) {
    sg::clear_error();
    const int rc = sg::fir_host_release();
    const int rc2 = sg::tile_pool_release();
    const int rc3 = sg::tile_jit_release();
    return rc ? rc : rc2 ? rc2 : rc3;
}

int simtgo_device_info(int32_t* sm_count, int32_t* cc_major, int32_t* cc_minor) {
    const sg::DevInfo* d = nullptr;
    int rc = sg::current_device(&d);
    if (rc) return rc;
    if (sm_count) *sm_count = d->sms;
    if (cc_major) *cc_major = d->cc_major;
    if (cc_minor) *cc_minor = d->cc_minor;
    return 0;
}

int simtgo_stream_sync(void* stream) {
    int rc = sg::cuda_status(cudaStreamSynchronize((cudaStream_t)stream), "cudaStreamSynchronize");
    if (rc) return rc;
    uint32_t bits = 0;
    rc = sg::watchdog_check_and_clear(&bits);
    if (rc) return rc;
    if (bits)
        return sg::fail(SIMTGO_EDEVICE,
                        "a kernel gave up a bounded wait (watchdog bits %#x): an asynchronous "
                        "copy or a peer did not arrive; its outputs are incomplete",
                        bits);
    return 0;
}

}  // extern "C"
