// comm.cu -- the communicator behind simtgo_Histogram_allreduce: per-rank
// partial bins summed over ranks with an NCCL all-reduce on NVLink/NVSwitch.
//
// NCCL is dlopen'ed (libnccl.so.2, the process's copy if one is already
// loaded -- e.g. torch's), so the library has no link-time NCCL dependency,
// in the spirit of simtgo's purego loader (cuda/loader_cuda.go:36-73).
// The reference has no multi-GPU support at all; this is new.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

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
    g_nccl.GetErrorString = (decltype(g_nccl.GetErrorString))dlsym(h, "ncclGetErrorString");
    g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy &&
                g_nccl.AllReduce && g_nccl.GetErrorString;
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

}  // namespace

struct simtgo_comm {
    ncclComm_t comm;
    int nranks, rank, device;
};

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
    *out = new simtgo_comm{c, nranks, rank, dev};
    return 0;
}

int simtgo_comm_destroy(simtgo_comm* comm) {
    sg::clear_error();
    if (!comm) return 0;
    int rc = need_nccl();
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
