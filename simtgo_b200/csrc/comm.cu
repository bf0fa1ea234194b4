// comm.cu -- the communicator behind simtgo_Histogram_allreduce: per-rank
// partial bins summed over ranks with an NCCL all-reduce on NVLink/NVSwitch,
// and simtgo_Histogram_allreduce_fused, which does the local histogram and
// the exchange in ONE kernel over NVLink peer memory: the grid counts into
// per-warp shared tables and a device-wide partial; the last block to
// finish stores this rank's bins into a slot of every rank's exchange buffer
// (peer stores over NVLink, mapped with CUDA IPC at first use), raises a
// flag on each rank with a system-scope release, waits (bounded) for every
// rank's flag with an acquire, and sums the slots into bins. Slots alternate
// between two halves by call parity and flags carry a call counter, so no
// reset or extra barrier is needed between calls.
//
// NCCL is dlopen'ed (libnccl.so.2, the process's copy if one is already
// loaded -- e.g. torch's), so the library has no link-time NCCL dependency,
// in the spirit of simtgo's purego loader (cuda/loader_cuda.go:36-73).
// The reference has no multi-GPU support at all; this is new.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "histogram.cuh"

using namespace sgd;

namespace sg {
int histogram_local(const char* K, int32_t* bins, int32_t bins_len, const int32_t* x,
                    int64_t x_len, void* stream);
}

namespace {

struct Nccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

std::once_flag g_once;
Nccl g_nccl;

void load_nccl() {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    g_nccl.GetUniqueId = (decltype(g_nccl.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    g_nccl.CommInitRank = (decltype(g_nccl.CommInitRank))dlsym(h, "ncclCommInitRank");
    g_nccl.CommDestroy = (decltype(g_nccl.CommDestroy))dlsym(h, "ncclCommDestroy");
    g_nccl.AllReduce = (decltype(g_nccl.AllReduce))dlsym(h, "ncclAllReduce");
    g_nccl.AllGather = (decltype(g_nccl.AllGather))dlsym(h, "ncclAllGather");
    g_nccl.GetErrorString = (decltype(g_nccl.GetErrorString))dlsym(h, "ncclGetErrorString");
    g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy &&
                g_nccl.AllReduce && g_nccl.AllGather && g_nccl.GetErrorString;
}

int need_nccl() {
    std::call_once(g_once, load_nccl);
    if (!g_nccl.ok) return sg::fail(SIMTGO_ECOMM, "libnccl.so.2 could not be loaded");
    return 0;
}

int nccl_status(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return 0;
    return sg::fail(1000 + (int)r, "%s: %s", what, g_nccl.GetErrorString(r));
}

// ---- the fused histogram + all-reduce ---------------------------------------
constexpr int kP2PCap = 4096;                // bins per rank slot
constexpr uint32_t kPeerSpin = 1u << 22;     // bounded wait (x 256 ns sleeps: ~1 s)

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Exchange buffer of one rank: slots[2][nranks][kP2PCap] int32, then
// nranks flags (uint32). Byte offset of the flags:
__host__ __device__ constexpr size_t p2p_flags_offset(int nranks) {
    return ((size_t)2 * nranks * kP2PCap * 4 + 127) / 128 * 128;
}

__global__ void __launch_bounds__(kHistThreads) k_hist_allreduce(
    int* __restrict__ bins, int bins_len, const int* __restrict__ x, int64_t m, bool vec,
    int* part, char* const* __restrict__ peers, char* mine, int rank, int nranks, uint32_t epoch,
    bool overwrite, uint32_t* wd) {
    __shared__ int sh[kHistWarps][kHistBins];
    __shared__ int last, failed;
    for (int k = threadIdx.x; k < kHistWarps * kHistBins; k += blockDim.x) (&sh[0][0])[k] = 0;
    __syncthreads();
    int* tab = sh[threadIdx.x / 32];
    hist_count(x, m, vec, [&](int v) {
        if ((unsigned)v < (unsigned)kHistBins) atomicAdd(tab + v, 1);
    });
    __syncthreads();
    for (int k = threadIdx.x; k < kHistBins; k += blockDim.x) {
        int c = 0;
#pragma unroll
        for (int w = 0; w < kHistWarps; w++) c += sh[w][k];
        if (c != 0) atomicAdd(part + k, c);
    }
    // The last block to finish sees every block's partial counts.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        last = atomicAdd(reinterpret_cast<unsigned*>(part + kHistBins), 1u) == gridDim.x - 1;
        failed = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int par = (int)(epoch & 1u);
    // This rank's bins (the caller's plus its counts, or with overwrite its
    // counts alone) into its slot on every rank, over NVLink for the peers.
    for (int k = threadIdx.x; k < bins_len; k += blockDim.x) {
        const int v = (overwrite ? 0 : bins[k]) + (k < kHistBins ? __ldcg(part + k) : 0);
        for (int r = 0; r < nranks; r++)
            reinterpret_cast<int*>(peers[r])[((size_t)par * nranks + rank) * kP2PCap + k] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < nranks) {
        uint32_t* flags = reinterpret_cast<uint32_t*>(peers[threadIdx.x] + p2p_flags_offset(nranks));
        st_release_sys(flags + rank, epoch);
        // Wait for rank threadIdx.x's slot in this rank's buffer.
        const uint32_t* mine_flag =
            reinterpret_cast<const uint32_t*>(mine + p2p_flags_offset(nranks)) + threadIdx.x;
        uint32_t i = 0;
        while ((int)(ld_acquire_sys(mine_flag) - epoch) < 0) {
            if (++i > kPeerSpin) {
                failed = 1;
                watchdog_raise(wd, 2u /* sg::WATCHDOG_PEER */);
                break;
            }
            __nanosleep(256);
        }
    }
    __syncthreads();
    if (!failed) {
        const int* slots = reinterpret_cast<const int*>(mine) + (size_t)par * nranks * kP2PCap;
        for (int k = threadIdx.x; k < bins_len; k += blockDim.x) {
            int sum = 0;
            for (int r = 0; r < nranks; r++) sum += __ldcv(slots + (size_t)r * kP2PCap + k);
            bins[k] = sum;
        }
    }
    // Ready for the next call.
    for (int k = threadIdx.x; k < kHistBins; k += blockDim.x) part[k] = 0;
    if (threadIdx.x == 0) part[kHistBins] = 0;
}

}  // namespace

struct simtgo_comm {
    ncclComm_t comm;
    int nranks, rank, device;
    // NVLink peer-to-peer state of the fused histogram all-reduce (first use).
    bool p2p = false;
    char* xb = nullptr;               // this rank's exchange buffer
    std::vector<char*> peer;          // every rank's buffer mapped here (peer[rank] == xb)
    char** d_peer = nullptr;          // the same, on the device
    int* part = nullptr;              // kHistBins partial counts + the block counter
    uint32_t epoch = 0;               // calls so far (the flags' value)
};

namespace {

// Maps every rank's exchange buffer into this process (a collective: every
// rank calls it on its first fused call).
int p2p_setup(simtgo_comm* c, cudaStream_t s) {
    const size_t bytes = p2p_flags_offset(c->nranks) + (size_t)c->nranks * 4;
    int rc;
    if ((rc = sg::cuda_status(cudaMalloc(&c->xb, bytes), "cudaMalloc(exchange)")) ||
        (rc = sg::cuda_status(cudaMemset(c->xb, 0, bytes), "cudaMemset(exchange)")) ||
        (rc = sg::cuda_status(cudaMalloc(&c->part, (kHistBins + 1) * sizeof(int)), "cudaMalloc")) ||
        (rc = sg::cuda_status(cudaMemset(c->part, 0, (kHistBins + 1) * sizeof(int)), "cudaMemset")))
        return rc;
    cudaIpcMemHandle_t mine;
    if ((rc = sg::cuda_status(cudaIpcGetMemHandle(&mine, c->xb), "cudaIpcGetMemHandle"))) return rc;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
    char* d_h = nullptr;
    if ((rc = sg::cuda_status(cudaMalloc(&d_h, 64 * (c->nranks + 1)), "cudaMalloc")) ||
        (rc = sg::cuda_status(cudaMemcpy(d_h, &mine, 64, cudaMemcpyHostToDevice), "handle up")))
        return rc;
    rc = nccl_status(g_nccl.AllGather(d_h, d_h + 64, 64, ncclUint8, c->comm, s), "ncclAllGather");
    std::vector<cudaIpcMemHandle_t> all(c->nranks);
    if (!rc) rc = sg::cuda_status(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (!rc)
        rc = sg::cuda_status(cudaMemcpy(all.data(), d_h + 64, 64 * c->nranks,
                                        cudaMemcpyDeviceToHost), "handles down");
    cudaFree(d_h);
    if (rc) return rc;
    c->peer.assign(c->nranks, nullptr);
    for (int r = 0; r < c->nranks; r++) {
        if (r == c->rank) {
            c->peer[r] = c->xb;
            continue;
        }
        void* p = nullptr;
        if ((rc = sg::cuda_status(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess),
                                  "cudaIpcOpenMemHandle")))
            return rc;
        c->peer[r] = (char*)p;
    }
    if ((rc = sg::cuda_status(cudaMalloc(&c->d_peer, sizeof(char*) * c->nranks), "cudaMalloc")) ||
        (rc = sg::cuda_status(cudaMemcpy(c->d_peer, c->peer.data(), sizeof(char*) * c->nranks,
                                         cudaMemcpyHostToDevice), "peers up")))
        return rc;
    c->p2p = true;
    return 0;
}

void p2p_release(simtgo_comm* c) {
    for (int r = 0; r < (int)c->peer.size(); r++)
        if (r != c->rank && c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]);
    if (c->d_peer) cudaFree(c->d_peer);
    if (c->part) cudaFree(c->part);
    if (c->xb) cudaFree(c->xb);
}

}  // namespace

namespace sg {
// The communicator's size and this process's rank.
int comm_rank(const simtgo_comm* c, int* nranks, int* rank) {
    if (!c) return sg::fail(SIMTGO_ECOMM, "null communicator");
    *nranks = c->nranks;
    *rank = c->rank;
    return 0;
}
// NCCL all-gather of `bytes` bytes from every rank into recv (rank order).
int comm_allgather(simtgo_comm* c, const void* send, void* recv, size_t bytes, cudaStream_t s) {
    int rc;
    if ((rc = need_nccl())) return rc;
    return nccl_status(g_nccl.AllGather(send, recv, bytes, ncclUint8, c->comm, s),
                       "ncclAllGather");
}
}  // namespace sg

extern "C" {

int simtgo_comm_unique_id(uint8_t out_id[128]) {
    sg::clear_error();
    int rc;
    if ((rc = need_nccl())) return rc;
    if (!out_id) return sg::fail(SIMTGO_ENULL, "comm_unique_id: null output");
    ncclUniqueId id;
    if ((rc = nccl_status(g_nccl.GetUniqueId(&id), "ncclGetUniqueId"))) return rc;
    static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out_id, &id, 128);
    return 0;
}

int simtgo_comm_init(simtgo_comm** out, const uint8_t id[128], int32_t nranks, int32_t rank) {
    sg::clear_error();
    int rc;
    if ((rc = need_nccl())) return rc;
    if (!out || !id) return sg::fail(SIMTGO_ENULL, "comm_init: null argument");
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return sg::fail(SIMTGO_ECOMM, "comm_init: rank %d of %d", rank, nranks);
    int dev = -1;
    if ((rc = sg::cuda_status(cudaGetDevice(&dev), "cudaGetDevice"))) return rc;
    ncclUniqueId uid;
    memcpy(&uid, id, 128);
    ncclComm_t c;
    if ((rc = nccl_status(g_nccl.CommInitRank(&c, nranks, uid, rank), "ncclCommInitRank")))
        return rc;
    simtgo_comm* cm = new simtgo_comm();
    cm->comm = c;
    cm->nranks = nranks;
    cm->rank = rank;
    cm->device = dev;
    *out = cm;
    return 0;
}

int simtgo_comm_destroy(simtgo_comm* comm) {
    sg::clear_error();
    if (!comm) return 0;
    int rc = need_nccl();
    p2p_release(comm);
    if (!rc) rc = nccl_status(g_nccl.CommDestroy(comm->comm), "ncclCommDestroy");
    delete comm;
    return rc;
}

int simtgo_comm_allreduce_i32(simtgo_comm* comm, int32_t* buf, int32_t n, void* stream) {
    sg::clear_error();
    int rc;
    if (!comm) return sg::fail(SIMTGO_ECOMM, "allreduce: null communicator");
    if ((rc = need_nccl())) return rc;
    if (n < 0) return sg::fail(SIMTGO_EARG, "allreduce: negative count");
    if (n > 0 && !buf) return sg::fail(SIMTGO_ENULL, "allreduce: null buffer");
    return nccl_status(g_nccl.AllReduce(buf, buf, (size_t)n, ncclInt32, ncclSum, comm->comm,
                                        (cudaStream_t)stream),
                       "ncclAllReduce");
}

int simtgo_Histogram_allreduce(simtgo_comm* comm, int32_t* bins, int32_t bins_len,
                               const int32_t* x, int64_t x_len, void* stream) {
    sg::clear_error();
    int rc;
    if (!comm) return sg::fail(SIMTGO_ECOMM, "Histogram_allreduce: null communicator");
    if ((rc = sg::histogram_local("Histogram_allreduce", bins, bins_len, x, x_len, stream)))
        return rc;
    return simtgo_comm_allreduce_i32(comm, bins, bins_len, stream);
}

}  // extern "C"

namespace {

int hist_allreduce_fused(const char* K, simtgo_comm* comm, int32_t* bins, int32_t bins_len,
                         const int32_t* x, int64_t x_len, bool overwrite, void* stream) {
    sg::clear_error();
    int rc;
    if (!comm) return sg::fail(SIMTGO_ECOMM, "%s: null communicator", K);
    if ((rc = need_nccl())) return rc;
    if (bins_len < 0 || x_len < 0) return sg::fail(SIMTGO_EARG, "%s: a length is negative", K);
    if (bins_len > kP2PCap)
        return sg::fail(SIMTGO_ESIZE, "%s: %d bins exceed the %d of an exchange slot; use "
                        "simtgo_Histogram_allreduce", K, bins_len, kP2PCap);
    if ((rc = sg::check_ptr(K, "bins", bins, bins_len)) || (rc = sg::check_ptr(K, "x", x, x_len)))
        return rc;
    if ((rc = sg::check_alias(K, {{"bins", bins, 4LL * bins_len, true}, {"x", x, 4 * x_len, false}})))
        return rc;
    const sg::DevInfo* d;
    if ((rc = sg::current_device(&d))) return rc;
    if (d->device != comm->device)
        return sg::fail(SIMTGO_ECOMM, "%s: the communicator belongs to device %d, not %d", K,
                        comm->device, d->device);
    cudaStream_t s = (cudaStream_t)stream;
    if (!comm->p2p && (rc = p2p_setup(comm, s))) return rc;
    comm->epoch++;
    const int64_t want = sg::ceil_div(sg::ceil_div(std::max<int64_t>(x_len, 1), 16), kHistThreads);
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)d->sms * 2));
    sg::before_launch();
    k_hist_allreduce<<<blocks, kHistThreads, 0, s>>>(
        bins, bins_len, x, x_len, sg::aligned16(x), comm->part, comm->d_peer, comm->xb,
        comm->rank, comm->nranks, comm->epoch, overwrite, sg::watchdog_device_ptr());
    return sg::launch_status(K);
}

}  // namespace

extern "C" {

int simtgo_Histogram_allreduce_fused(simtgo_comm* comm, int32_t* bins, int32_t bins_len,
                                     const int32_t* x, int64_t x_len, void* stream) {
    return hist_allreduce_fused("Histogram_allreduce_fused", comm, bins, bins_len, x, x_len,
                                false, stream);
}

int simtgo_Histogram_allreduce_fused_overwrite(simtgo_comm* comm, int32_t* bins,
                                               int32_t bins_len, const int32_t* x, int64_t x_len,
                                               void* stream) {
    return hist_allreduce_fused("Histogram_allreduce_fused_overwrite", comm, bins, bins_len, x,
                                x_len, true, stream);
}

}  // extern "C"
