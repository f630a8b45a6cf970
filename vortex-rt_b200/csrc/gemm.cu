// Host side of the tensor-core Q8_0 GEMM (gemm_q8t.cuh): TMA tensor maps for
// the fp16 hi/lo activation operands, the launcher used by the model's
// batched paths, and the packed-matrix C ABI entry points.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "gemm_q8t.cuh"
#include "vrt_internal.hpp"
#include "vrt_kernels.hpp"

namespace vrt {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(p);
        }
    });
    return fn;
}

// Tensor map over a row-major fp16 matrix [rows][cols] (cols % 64 == 0, base
// 16-byte aligned), box = 64 columns x box_rows rows (128 for the large-M
// GEMM, 16 for the small-M form), 128B swizzle; rows past the end read as zeros.
int make_f16_tmap(TmaMap* out, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    static_assert(sizeof(TmaMap) == sizeof(CUtensorMap), "tensor map size");
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(VRT_E_UNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
    if (cols % kGemmBK || reinterpret_cast<uintptr_t>(base) % 16) return fail(VRT_E_INVALID, "fp16 operand layout");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGemmBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VRT_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return VRT_OK;
}

template <int EPI>
static cudaError_t gemm_launch_t(const TmaMap& hi, const TmaMap& lo, const GemmParams& p, cudaStream_t s) {
    static uint64_t done = 0;  // devices whose attribute is set (bit per ordinal)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !(done & (1ull << dev))) {
        e = cudaFuncSetAttribute(q8t_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemBytes);
        if (e != cudaSuccess) return e;
        done |= 1ull << dev;
    }
    const dim3 grid(p.n / kGemmBN, (p.m + kGemmBM - 1) / kGemmBM);
    return launch(q8t_gemm_kernel<EPI>, grid, dim3(kGemmThreads), kGemmSmemBytes, s, false, hi, lo, p);
}

template <int EPI, int NTMAX>
static cudaError_t gemm_small_launch_t(const TmaMap& hi, const TmaMap& lo, const GemmParams& p, cudaStream_t s) {
    static uint64_t done = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    constexpr uint32_t smem = SmallGemmLayout<NTMAX>::kSmem;
    if (dev < 64 && !(done & (1ull << dev))) {
        e = cudaFuncSetAttribute(q8t_gemm_small_kernel<EPI, NTMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        done |= 1ull << dev;
    }
    const dim3 grid(p.n / kGemmBN, (p.m + p.nt - 1) / p.nt, p.ksplit);
    return launch(q8t_gemm_small_kernel<EPI, NTMAX>, grid, dim3(kGemmSmallThreads), smem, s, false, hi, lo, p);
}

template <int NTMAX>
static cudaError_t gemm_small_epi(int epi, const TmaMap& hi, const TmaMap& lo, const GemmParams& p, cudaStream_t s) {
    switch (epi) {
    case kGemmStore: return gemm_small_launch_t<kGemmStore, NTMAX>(hi, lo, p, s);
    case kGemmGeluSplit: return gemm_small_launch_t<kGemmGeluSplit, NTMAX>(hi, lo, p, s);
    case kGemmArgmax: return gemm_small_launch_t<kGemmArgmax, NTMAX>(hi, lo, p, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemm_q8t_small(int epi, const TmaMap& hi, const TmaMap& lo, const GemmParams& p, cudaStream_t s) {
    if (p.nt != 16 && p.nt != 32 && p.nt != 64 && p.nt != 128) return cudaErrorInvalidValue;
    if (p.ksplit == 0 || (p.ksplit > 1 && (!p.ws || !p.tickets))) return cudaErrorInvalidValue;
    if (p.nt > 64) return cudaErrorInvalidValue;  // more rows: the large-M kernel
    return gemm_small_epi<64>(epi, hi, lo, p, s);
}

// K splits for a small-M GEMM: enough CTAs for two per SM, at least two
// 128-column K tiles per split, at most 16 splits.
// K ranges per (weight tile, token tile) of the small-M GEMM: one CTA per SM
// is resident, so the cost of a split is modelled as waves x (K stages per
// CTA + a fixed cost per CTA: ring fill and drain, the partial's write-out
// and the last CTA's reduction), in 128-column stages.
uint32_t gemm_small_ksplit(uint32_t n, uint32_t m, uint32_t k, int sms) {
    constexpr double kFixedStages = 8.0;  // measured on 27B bs32: 2 -> +0%, 4 -> +3.5%, 8 -> +4.1% over 2 CTAs/SM
    const uint32_t tiles = (n / kGemmBN) * ((m + gemm_small_tile(m) - 1) / gemm_small_tile(m));
    const uint32_t kt = k / kTileCols;
    const uint32_t kmax = std::max(1u, std::min(kt / 2, 16u));
    uint32_t best = 1;
    double best_cost = 0.0;
    for (uint32_t ks = 1; ks <= kmax; ++ks) {
        const uint64_t waves = (static_cast<uint64_t>(tiles) * ks + sms - 1) / sms;
        const double cost = static_cast<double>(waves) * (static_cast<double>(kt) / ks + kFixedStages);
        if (ks == 1 || cost < best_cost) {
            best = ks;
            best_cost = cost;
        }
    }
    return best;
}

uint32_t gemm_small_tile(uint32_t m) {
    return m <= 16 ? 16u : m <= 32 ? 32u : 64u;
}

cudaError_t gemm_q8t(int epi, const TmaMap& hi, const TmaMap& lo, const GemmParams& p, cudaStream_t s) {
    switch (epi) {
    case kGemmStore: return gemm_launch_t<kGemmStore>(hi, lo, p, s);
    case kGemmGeluSplit: return gemm_launch_t<kGemmGeluSplit>(hi, lo, p, s);
    case kGemmArgmax: return gemm_launch_t<kGemmArgmax>(hi, lo, p, s);
    default: return cudaErrorInvalidValue;
    }
}

// Split fp32 rows into fp16 hi/lo operands (x = hi + lo to ~2^-22 relative).
__global__ void split_f16_kernel(const float* __restrict__ x, uint64_t n, __half* __restrict__ hi,
                                 __half* __restrict__ lo) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        __half h, l;
        split_f16(x[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

cudaError_t split_f16(const float* x, uint64_t n, __half* hi, __half* lo, cudaStream_t s) {
    const uint64_t blocks = (n + 255) / 256;
    split_f16_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(x, n, hi, lo);
    return cudaGetLastError();
}

// Context scratch of at least `bytes` (grown by reallocation; not shared
// between concurrent calls on one context).
static int ctx_workspace(vrt_ctx* ctx, size_t bytes, void** out) {
    std::lock_guard<std::mutex> g(ctx->mu);
    if (ctx->ws_bytes < bytes) {
        if (ctx->ws) {
            VRT_CUDA(cudaStreamSynchronize(ctx->stream));
            VRT_CUDA(cudaFree(ctx->ws));
            ctx->ws = nullptr;
            ctx->ws_bytes = 0;
        }
        VRT_CUDA(cudaMalloc(&ctx->ws, bytes));
        ctx->ws_bytes = bytes;
    }
    *out = ctx->ws;
    return VRT_OK;
}

static int gemm_common(vrt_ctx* ctx, int epi, const void* d_packed, uint32_t rows, uint32_t cols, const float* d_x,
                       uint32_t m, float* d_out, void* stream) {
    if (!ctx || !d_packed || !d_x || !d_out) return fail(VRT_E_INVALID, "null argument");
    if (!m || !rows || rows % kGemmBN || !cols || cols % kTileCols) {
        return fail(VRT_E_INVALID, "tensor-core GEMM needs rows %% 128 == 0, cols %% 128 == 0, m > 0");
    }
    if (reinterpret_cast<uintptr_t>(d_packed) % 16) return fail(VRT_E_INVALID, "packed weights must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(d_out) % 16) return fail(VRT_E_INVALID, "output must be 16-byte aligned");
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaSetDevice(ctx->device));
    const uint64_t xn = static_cast<uint64_t>(m) * cols;
    const uint64_t an = epi == kGemmGeluSplit ? static_cast<uint64_t>(m) * (rows / 2) : 0;
    const bool small = m <= 64;  // weight rows on the MMA's 128 lanes, activation rows on N
    const uint32_t nt = small ? gemm_small_tile(m) : 0u;
    const uint32_t ks = small ? gemm_small_ksplit(rows, m, cols, ctx->prop.multiProcessorCount) : 1u;
    const uint64_t ws_f = ks > 1 ? static_cast<uint64_t>(ks) * nt * rows : 0;   // partials (one token tile)
    const uint64_t tk = small ? rows / kGemmBN : 0;
    const uint64_t f16_bytes = ((2 * xn + 2 * an) * sizeof(__half) + 255) / 256 * 256;
    void* ws = nullptr;
    VRT_TRY(ctx_workspace(ctx, f16_bytes + ws_f * 4 + tk * 4 + 256, &ws));
    __half* xh = static_cast<__half*>(ws);
    __half* xl = xh + xn;
    VRT_CUDA(split_f16(d_x, xn, xh, xl, s));
    TmaMap th, tl;
    VRT_TRY(make_f16_tmap(&th, xh, m, cols, small ? 16u : 128u));
    VRT_TRY(make_f16_tmap(&tl, xl, m, cols, small ? 16u : 128u));
    GemmParams p{};
    p.w = static_cast<const uint8_t*>(d_packed);
    p.n = rows;
    p.k = cols;
    p.m = m;
    p.nt = nt;
    p.ksplit = ks;
    p.ws = ks > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + f16_bytes) : nullptr;
    p.tickets = small ? reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + f16_bytes + ws_f * 4) : nullptr;
    if (small) VRT_CUDA(cudaMemsetAsync(p.tickets, 0, tk * 4, s));
    uint32_t* status = reinterpret_cast<uint32_t*>(ctx->d_key + 1);  // word after the argmax key
    p.status = status;
    if (epi == kGemmStore) {
        p.y = d_out;
        p.ldy = rows;
    } else {
        p.act_hi = xl + xn;
        p.act_lo = p.act_hi + an;
        p.act_f32 = d_out;
        p.ld_act = rows / 2;
    }
    VRT_CUDA(cudaMemsetAsync(status, 0, 4, s));
    VRT_CUDA(small ? gemm_q8t_small(epi, th, tl, p, s) : gemm_q8t(epi, th, tl, p, s));
    uint32_t st = 0;
    VRT_CUDA(cudaMemcpyAsync(&st, status, 4, cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaStreamSynchronize(s));
    if (st) return fail(VRT_E_TIMEOUT, "tensor-core GEMM: a bounded device wait timed out");
    return VRT_OK;
}

}  // namespace vrt

using namespace vrt;


extern "C" {

int vrt_q8t_gemm(vrt_ctx* ctx, const void* d_packed, uint32_t rows, uint32_t cols, const float* d_x, uint32_t m,
                 float* d_y, void* stream) {
    clear_error();
    return gemm_common(ctx, kGemmStore, d_packed, rows, cols, d_x, m, d_y, stream);
}

int vrt_q8t_gemm_gelu(vrt_ctx* ctx, const void* d_packed_pair, uint32_t ffn, uint32_t cols, const float* d_x,
                      uint32_t m, float* d_act, void* stream) {
    clear_error();
    if (ffn % 64) return fail(VRT_E_INVALID, "tensor-core gate/up needs ffn %% 64 == 0");
    return gemm_common(ctx, kGemmGeluSplit, d_packed_pair, 2 * ffn, cols, d_x, m, d_act, stream);
}

}  // extern "C"
