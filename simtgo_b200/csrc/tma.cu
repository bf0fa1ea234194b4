// tma.cu -- host half of tma.cuh: cuTensorMapEncodeTiled through the CUDA
// runtime's driver entry point.
#include <cudaTypedefs.h>

#include <mutex>

#include "tma.cuh"

namespace sg {

namespace {
std::once_flag g_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

void resolve() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

int tma_encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                  uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMapSwizzle swizzle) {
    std::call_once(g_once, resolve);
    if (!g_encode) return fail(SIMTGO_EDEVICE, "cuTensorMapEncodeTiled is not available");
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(SIMTGO_EARG, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return 0;
}

}  // namespace sg
