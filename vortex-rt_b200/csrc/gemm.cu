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

// x fp32 [rows][ldx] (K columns) -> Q16Out.  One warp per (row, 32-block).
__global__ void quant_rows_kernel(const float* __restrict__ x, uint32_t ldx, uint32_t rows, uint32_t k,
                                  const Q16Out o) {
    const uint32_t warps = (blockDim.x >> 5) * gridDim.x;
    const uint32_t nb = k / 32;
    for (uint32_t w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < rows * nb; w += warps) {
        const uint32_t row = w / nb, kk = (w % nb) * 32 + (threadIdx.x & 31);
        warp_q16_store(o, row, kk, x[static_cast<uint64_t>(row) * ldx + kk]);
    }
}

// Q8T matrix (rows x cols) -> Q8M copy.  One thread per (row, 32-block).
__global__ void q8t_to_q8m_kernel(const uint8_t* __restrict__ src, uint32_t rows, uint32_t cols,
                                  uint8_t* __restrict__ dst) {
    const uint64_t nb = cols / 32, total = static_cast<uint64_t>(rows) * nb;
    const uint32_t kts = cols / kQ8mCols;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t row = static_cast<uint32_t>(i / nb), blk = static_cast<uint32_t>(i % nb);
        uint8_t* tile = dst + q8m_tile(row / kQ8mRows, blk / 4, kts);
        const uint32_t r = row % kQ8mRows, c0 = (blk % 4) * 32;
        // both layouts keep 16 consecutive columns of a row in one aligned 16-byte chunk
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
            *reinterpret_cast<uint4*>(tile + q8m_q_offset(r, c0 + 16 * h)) =
                *reinterpret_cast<const uint4*>(src + q8t_weight_offset(row, blk * 32 + 16 * h, cols));
        }
        const uint64_t so = q8t_scale_offset(row, blk, cols);
        tile[q8m_s_offset(r, blk % 4)] = src[so];
        tile[q8m_s_offset(r, blk % 4) + 1] = src[so + 1];
    }
}

int make_i8_tmap(TmaMap* out, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(VRT_E_UNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
    if (cols % kQ8mCols || reinterpret_cast<uintptr_t>(base) % 16) return fail(VRT_E_INVALID, "int8 operand layout");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols};
    const cuuint32_t box[2] = {kQ8mCols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VRT_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return VRT_OK;
}

template <int EPI>
static cudaError_t gemm_i8_launch_t(const TmaMap& hi, const TmaMap& lo, const GemmI8Params& p, cudaStream_t s) {
    static uint64_t done = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !(done & (1ull << dev))) {
        e = cudaFuncSetAttribute(q8m_gemm_i8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kI8Smem);
        if (e != cudaSuccess) return e;
        done |= 1ull << dev;
    }
    const dim3 grid(p.n / kQ8mRows, (p.m + p.nt - 1) / p.nt, p.ksplit);
    return launch(q8m_gemm_i8_kernel<EPI>, grid, dim3(kI8Threads), kI8Smem, s, false, hi, lo, p);
}

cudaError_t gemm_q8m_i8(int epi, const TmaMap& hi, const TmaMap& lo, const GemmI8Params& p, cudaStream_t s) {
    if ((p.nt != 16 && p.nt != 32) || p.n % kQ8mRows || p.k % kQ8mCols || p.sx_ld % 4) return cudaErrorInvalidValue;
    if (p.ksplit == 0 || (p.ksplit > 1 && (!p.ws || !p.tickets)) || p.k / kQ8mCols < p.ksplit) return cudaErrorInvalidValue;
    switch (epi) {
    case kGemmStore: return gemm_i8_launch_t<kGemmStore>(hi, lo, p, s);
    case kGemmGeluSplit: return gemm_i8_launch_t<kGemmGeluSplit>(hi, lo, p, s);
    case kGemmArgmax: return gemm_i8_launch_t<kGemmArgmax>(hi, lo, p, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t q8t_to_q8m(const uint8_t* src, uint32_t rows, uint32_t cols, uint8_t* dst, cudaStream_t s) {
    if (rows % kQ8mRows || cols % kQ8mCols) return cudaErrorInvalidValue;
    const uint64_t work = static_cast<uint64_t>(rows) * (cols / 32);
    const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>((work + 255) / 256, 65535u));
    return launch(q8t_to_q8m_kernel, dim3(blocks), dim3(256), 0, s, false, src, rows, cols, dst);
}

cudaError_t quant_rows(const float* x, uint32_t ldx, uint32_t rows, uint32_t k, const Q16Out& o, cudaStream_t s) {
    if (k % 32) return cudaErrorInvalidValue;
    const uint64_t warps = static_cast<uint64_t>(rows) * (k / 32);
    const unsigned blocks = static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>((warps + 7) / 8, 4096u)));
    return launch(quant_rows_kernel, dim3(blocks), dim3(256), 0, s, false, x, ldx, rows, k, o);
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
    const dim3 grid((p.m + kGemmBM - 1) / kGemmBM, p.n / kGemmBN);  // M tiles fastest (see q8t_gemm_kernel)
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

// Few-row form on the integer tensor cores (vrt_q8m_gemm*): the activation
// rows are quantised to int16 split halves in the context scratch.
static int gemm_i8_common(vrt_ctx* ctx, int epi, const void* d_q8m, uint32_t rows, uint32_t cols, const float* d_x,
                          uint32_t m, float* d_out, void* stream) {
    if (!ctx || !d_q8m || !d_x || !d_out) return fail(VRT_E_INVALID, "null argument");
    if (m == 0 || m > 32 || !rows || rows % kQ8mRows || !cols || cols % kQ8mCols) {
        return fail(VRT_E_INVALID, "integer tensor-core GEMM needs rows %% 128 == 0, cols %% 128 == 0, 1 <= m <= 32");
    }
    if (reinterpret_cast<uintptr_t>(d_q8m) % 16) return fail(VRT_E_INVALID, "Q8M weights must be 16-byte aligned");
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaSetDevice(ctx->device));
    const uint32_t nt = gemm_small_tile(m), mp = (m + nt - 1) / nt * nt;
    const uint32_t ks = gemm_small_ksplit(rows, m, cols, ctx->prop.multiProcessorCount);
    const uint64_t qb = (static_cast<uint64_t>(mp) * cols + 255) / 256 * 256;
    const uint64_t sxb = (static_cast<uint64_t>(cols / 32) * mp * 4 + 255) / 256 * 256;
    const uint64_t ws_f = ks > 1 ? static_cast<uint64_t>(ks) * mp * rows : 0;
    const uint64_t tk = static_cast<uint64_t>(rows / kQ8mRows) * (mp / nt);
    void* ws = nullptr;
    VRT_TRY(ctx_workspace(ctx, 2 * qb + sxb + ws_f * 4 + tk * 4 + 256, &ws));
    uint8_t* base = static_cast<uint8_t*>(ws);
    Q16Out o{reinterpret_cast<int8_t*>(base), reinterpret_cast<int8_t*>(base + qb), reinterpret_cast<float*>(base + 2 * qb),
             cols, mp};
    VRT_CUDA(quant_rows(d_x, cols, m, cols, o, s));
    TmaMap th, tl;
    VRT_TRY(make_i8_tmap(&th, o.hi, mp, cols, 16u));
    VRT_TRY(make_i8_tmap(&tl, o.lo, mp, cols, 16u));
    GemmI8Params p{};
    p.w = static_cast<const uint8_t*>(d_q8m);
    p.n = rows;
    p.k = cols;
    p.m = m;
    p.sx = o.sx;
    p.sx_ld = mp;
    p.nt = nt;
    p.ksplit = ks;
    p.ws = ks > 1 ? reinterpret_cast<float*>(base + 2 * qb + sxb) : nullptr;
    p.tickets = reinterpret_cast<uint32_t*>(base + 2 * qb + sxb + ws_f * 4);
    VRT_CUDA(cudaMemsetAsync(p.tickets, 0, tk * 4, s));
    uint32_t* status = reinterpret_cast<uint32_t*>(ctx->d_key + 1);
    p.status = status;
    if (epi == kGemmStore) {
        p.y = d_out;
        p.ldy = rows;
    } else {
        p.act = d_out;
        p.ld_act = rows / 2;
    }
    VRT_CUDA(cudaMemsetAsync(status, 0, 4, s));
    VRT_CUDA(gemm_q8m_i8(epi, th, tl, p, s));
    uint32_t st = 0;
    VRT_CUDA(cudaMemcpyAsync(&st, status, 4, cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaStreamSynchronize(s));
    if (st) return fail(VRT_E_TIMEOUT, "integer tensor-core GEMM: a bounded device wait timed out");
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

int vrt_q8t_to_q8m(vrt_ctx* ctx, const void* d_packed, uint32_t rows, uint32_t cols, void* d_out, void* stream) {
    clear_error();
    if (!ctx || !d_packed || !d_out) return fail(VRT_E_INVALID, "null argument");
    if (!rows || rows % kQ8mRows || !cols || cols % kQ8mCols) return fail(VRT_E_INVALID, "Q8M needs rows, cols %% 128 == 0");
    VRT_CUDA(cudaSetDevice(ctx->device));
    VRT_CUDA(q8t_to_q8m(static_cast<const uint8_t*>(d_packed), rows, cols, static_cast<uint8_t*>(d_out),
                        as_stream(ctx, stream)));
    return VRT_OK;
}

int vrt_q8m_gemm(vrt_ctx* ctx, const void* d_q8m, uint32_t rows, uint32_t cols, const float* d_x, uint32_t m,
                 float* d_y, void* stream) {
    clear_error();
    return gemm_i8_common(ctx, kGemmStore, d_q8m, rows, cols, d_x, m, d_y, stream);
}

int vrt_q8m_gemm_gelu(vrt_ctx* ctx, const void* d_q8m_pair, uint32_t ffn, uint32_t cols, const float* d_x, uint32_t m,
                      float* d_act, void* stream) {
    clear_error();
    if (ffn % 64) return fail(VRT_E_INVALID, "tensor-core gate/up needs ffn %% 64 == 0");
    return gemm_i8_common(ctx, kGemmGeluSplit, d_q8m_pair, 2 * ffn, cols, d_x, m, d_act, stream);
}

}  // extern "C"
