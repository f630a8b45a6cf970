// Host-side internals shared by the runtime translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <mutex>
#include <string>
#include <unordered_map>

#include "vortexrt_b200.h"

struct vrt_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaDeviceProp prop{};
    unsigned long long* d_key = nullptr;  // argmax scratch
    void* ws = nullptr;                   // tensor-core GEMM operand scratch, grown on demand
    size_t ws_bytes = 0;
    std::mutex mu;
    std::unordered_map<void*, size_t> allocs;
};

namespace vrt {

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();
int cuda_fail(cudaError_t e, const char* what, const char* file, int line);

#define VRT_CUDA(call)                                                          \
    do {                                                                        \
        cudaError_t e_ = (call);                                                \
        if (e_ != cudaSuccess) return ::vrt::cuda_fail(e_, #call, __FILE__, __LINE__); \
    } while (0)

#define VRT_TRY(call)                    \
    do {                                 \
        int rc_ = (call);                \
        if (rc_ != VRT_OK) return rc_;   \
    } while (0)

inline cudaStream_t as_stream(vrt_ctx* ctx, void* s) {
    return s ? static_cast<cudaStream_t>(s) : ctx->stream;
}

// Launch with optional programmatic-dependent-launch attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                   Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int check_device_ptr(vrt_ctx* ctx, const void* p, const char* what);

// Packed (Q8T) fast-path launches used by both the model and the C ABI.
struct GemvLaunch;
}  // namespace vrt
