// Launch side of the persistent decode step (step_persistent.cuh): one
// instantiation per head width (M = head_dim / 32) and query-group size (RG),
// each launched cooperatively so that all CTAs of the grid are resident at
// once (the dataflow waits between CTAs rely on it).

#include <cuda_runtime.h>

#include "step_persistent.cuh"
#include "vrt_internal.hpp"
#include "vrt_kernels.hpp"

namespace vrt {

template <int M, int RG>
static cudaError_t ps_limits_t(uint32_t* max_dynamic, int* blocks_per_sm, uint32_t smem) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa{};
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, ps_step_kernel<M, RG>);
    if (e != cudaSuccess) return e;
    const int dyn = optin - static_cast<int>(fa.sharedSizeBytes);
    *max_dynamic = static_cast<uint32_t>(dyn);
    e = cudaFuncSetAttribute(ps_step_kernel<M, RG>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess || !blocks_per_sm) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, ps_step_kernel<M, RG>, kPsThreads,
                                                         smem ? smem : static_cast<size_t>(dyn));
}

template <int M, int RG>
static cudaError_t ps_launch_t(const PsParams& p, uint32_t grid, uint32_t smem, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kPsThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, ps_step_kernel<M, RG>, p);
}

#define VRT_PS_DISPATCH(CALL)                                                                  \
    VRT_PS_CASE(2, 1, CALL) VRT_PS_CASE(2, 2, CALL) VRT_PS_CASE(2, 4, CALL) VRT_PS_CASE(2, 8, CALL) \
    VRT_PS_CASE(4, 1, CALL) VRT_PS_CASE(4, 2, CALL) VRT_PS_CASE(4, 4, CALL) VRT_PS_CASE(4, 8, CALL) \
    VRT_PS_CASE(8, 1, CALL) VRT_PS_CASE(8, 2, CALL) VRT_PS_CASE(8, 4, CALL) VRT_PS_CASE(8, 8, CALL)

cudaError_t ps_limits(uint32_t hd, uint32_t rg, uint32_t smem, uint32_t* max_dynamic, int* blocks_per_sm) {
    const uint32_t m = hd / 32;
#define VRT_PS_CASE(MM, RR, CALL) \
    if (m == MM && rg == RR) return ps_limits_t<MM, RR>(max_dynamic, blocks_per_sm, smem);
    VRT_PS_DISPATCH(0)
#undef VRT_PS_CASE
    return cudaErrorInvalidValue;
}

cudaError_t ps_launch(const PsParams& p, uint32_t grid, uint32_t smem, cudaStream_t s) {
    const uint32_t m = p.hd / 32;
#define VRT_PS_CASE(MM, RR, CALL) \
    if (m == MM && p.rg == RR) return ps_launch_t<MM, RR>(p, grid, smem, s);
    VRT_PS_DISPATCH(0)
#undef VRT_PS_CASE
    return cudaErrorInvalidValue;
}

}  // namespace vrt
