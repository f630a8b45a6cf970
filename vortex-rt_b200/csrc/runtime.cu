// Runtime layer of the C ABI: device context, allocation and copies (the
// role of the reference's VulkanContext/Buffer, src/vulkan_context.cpp and
// src/buffer.cpp), the Q8_0 pipeline entry points over raw GGUF rows (the
// role of Q8MatVecPipeline / ArgmaxPipeline), the packed (Q8T) fast path,
// and the kernel dispatch tables used by the model.

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "attention.cuh"
#include "gemv_q8t.cuh"
#include "pipeline_kernels.cuh"
#include "vrt_internal.hpp"
#include "vrt_kernels.hpp"

namespace vrt {

static thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

void clear_error() { g_last_error.clear(); }

int cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
    const char* base = strrchr(file, '/');
    return fail(e == cudaErrorMemoryAllocation ? VRT_E_NOMEM : VRT_E_CUDA, "%s failed: %s (%s:%d)", what,
                cudaGetErrorString(e), base ? base + 1 : file, line);
}

int check_device_ptr(vrt_ctx* ctx, const void* p, const char* what) {
    if (!p) return fail(VRT_E_INVALID, "%s is null", what);
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return fail(VRT_E_INVALID, "%s is not a CUDA pointer", what);
    }
    if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) {
        return fail(VRT_E_INVALID, "%s is not device memory", what);
    }
    if (a.device != ctx->device) return fail(VRT_E_INVALID, "%s lives on another device", what);
    return VRT_OK;
}

// ----------------------------------------------------------- dispatch

template <int PRO, int EPI>
static cudaError_t gemv_launch_t(const GemvParams& p_in, int grid, cudaStream_t s, bool pdl) {
    GemvParams p = p_in;
    if (p.stage_cap == 0) {
        // ring slots: enough for the largest CTA span, 2..8
        const uint64_t kt = p.cols / kTileCols;
        const uint64_t groups = (p.rows + kTileRows - 1) / kTileRows;
        const uint64_t span = (groups * kt + grid - 1) / grid + kt;
        const uint64_t st = (span + kStageTiles - 1) / kStageTiles;
        p.stage_cap = static_cast<uint32_t>(st < 2 ? 2 : (st > kMaxStages ? kMaxStages : st));
    }
    const uint32_t smem = gemv_smem_layout(p.cols, PRO, p.stage_cap).total;
    return launch(q8t_gemv_kernel<PRO, EPI>, dim3(grid), dim3(kGemvThreads), smem, s, pdl, p);
}

// Largest dynamic shared memory a kernel may request: the device's opt-in
// per-block limit minus the kernel's static shared memory.
template <typename K>
static cudaError_t raise_smem_limit(K kernel) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa{};
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                optin - static_cast<int>(fa.sharedSizeBytes));
}

template <int PRO, int EPI>
static cudaError_t gemv_attr_t() {
    return raise_smem_limit(q8t_gemv_kernel<PRO, EPI>);
}

// Raise the dynamic shared-memory limit of every instantiation once, before
// any stream capture.
cudaError_t gemv_init_attributes() {
    cudaError_t e = cudaSuccess;
#define VRT_GA(P, E) if (e == cudaSuccess) e = gemv_attr_t<P, E>();
    VRT_GA(kProPlain, kEpiAtomic)
    VRT_GA(kProRmsInto, kEpiAtomic)
    VRT_GA(kProEmbed, kEpiAtomic)
    VRT_GA(kProResid, kEpiAtomic)
    VRT_GA(kProResid, kEpiGeluPair)
    VRT_GA(kProPlain, kEpiGeluPair)
    VRT_GA(kProRmsInto, kEpiGeluPair)
    VRT_GA(kProResidFinal, kEpiArgmax)
    VRT_GA(kProPlain, kEpiArgmax)
    VRT_GA(kProRmsInto, kEpiArgmax)
#undef VRT_GA
    return e;
}

cudaError_t gemv_q8t(int pro, int epi, const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
#define VRT_G(P, E)                                 \
    if (pro == P && epi == E) return gemv_launch_t<P, E>(p, grid, s, pdl);
    VRT_G(kProPlain, kEpiAtomic)
    VRT_G(kProRmsInto, kEpiAtomic)
    VRT_G(kProEmbed, kEpiAtomic)
    VRT_G(kProResid, kEpiAtomic)
    VRT_G(kProResid, kEpiGeluPair)
    VRT_G(kProPlain, kEpiGeluPair)
    VRT_G(kProRmsInto, kEpiGeluPair)
    VRT_G(kProResidFinal, kEpiArgmax)
    VRT_G(kProPlain, kEpiArgmax)
    VRT_G(kProRmsInto, kEpiArgmax)
#undef VRT_G
    return cudaErrorInvalidValue;
}

uint32_t gemv_smem_bytes(int pro, uint32_t cols) { return gemv_smem_layout(cols, pro, 0).total; }

cudaError_t argmax_unkey_launch(const unsigned long long* key, uint32_t* out, cudaStream_t s) {
    return launch(argmax_unkey_kernel, dim3(1), dim3(1), 0, s, false, key, out);
}

cudaError_t attention_launch(const AttnParams& p, dim3 grid, cudaStream_t s, bool pdl) {
    const uint32_t M = p.hd / 32, R = p.H / p.KV;
    const int rg = R <= 1 ? 1 : R <= 2 ? 2 : R <= 4 ? 4 : 8;
    const bool batch = grid.z > 1;
#define VRT_A(MM, RR)                                                                                          \
    if (M == MM && rg == RR)                                                                                   \
        return batch ? launch(attention_decode_kernel<MM, RR, true>, grid, dim3(kAttnThreads), 0, s, pdl, p)  \
                     : launch(attention_decode_kernel<MM, RR, false>, grid, dim3(kAttnThreads), 0, s, pdl, p);
    VRT_A(2, 1) VRT_A(2, 2) VRT_A(2, 4) VRT_A(2, 8)
    VRT_A(4, 1) VRT_A(4, 2) VRT_A(4, 4) VRT_A(4, 8)
    VRT_A(8, 1) VRT_A(8, 2) VRT_A(8, 4) VRT_A(8, 8)
#undef VRT_A
    return cudaErrorInvalidValue;
}

// The staged kernel for rows of up to kRawStagedMaxBlocks blocks; the
// row-wise kernel serves wider rows, or every call under VRT_RAW_ROWWISE=1
// (which the tests use to cover both kernels).
using RawStagedFn = void (*)(const RawStagedParams);
template <int U>
static RawStagedFn raw_staged_kernel_u(uint32_t lpr) {
    switch (lpr) {
        case 8: return raw_gemv_staged_kernel<8, 1, U>;
        case 16: return raw_gemv_staged_kernel<16, 1, U>;
        case 32: return raw_gemv_staged_kernel<32, 1, U>;
        case 64: return raw_gemv_staged_kernel<64, 1, U>;
        case 128: return raw_gemv_staged_kernel<128, 1, U>;
        case 256: return raw_gemv_staged_kernel<256, 1, U>;
        case 512: return raw_gemv_staged_kernel<512, 1, U>;
        default: return nullptr;
    }
}
static RawStagedFn raw_staged_kernel_for(uint32_t lpr, uint32_t nb, uint32_t u) {
    if (nb == 2) return lpr == 512 && u == 1 ? raw_gemv_staged_kernel<512, 2, 1> : nullptr;
    return u == 2 ? raw_staged_kernel_u<2>(lpr) : raw_staged_kernel_u<1>(lpr);
}

static bool raw_rowwise_forced() {
    static const bool forced = [] {
        const char* e = getenv("VRT_RAW_ROWWISE");
        return e && e[0] == '1';
    }();
    return forced;
}

// Staged launch: lanes per row LPR = the power of two >= each thread's share
// of a row (one block per thread, two above 512 blocks), 512 / LPR row slots,
// two rows per slot and iteration when one pass over the slots is under
// 16 KB; ring slots of one iteration's 128-byte aligned window (plus 4 bytes
// of read slack), as many slots as ~200 KB of shared memory holds (3..10),
// all in flight.  CTAs are split over the matrices in proportion to their
// rows.  Returns VRT_OK when it launched, VRT_E_UNSUPPORTED when the row-wise
// kernel must run.
static int raw_gemv_staged(int sms, const RawGemvParams& p, uint32_t* status, cudaStream_t s) {
    const uint32_t nblk = p.cols / 32;
    if (nblk == 0 || nblk > kRawStagedMaxBlocks || raw_rowwise_forced()) return VRT_E_UNSUPPORTED;
    const uint32_t nb = nblk <= 512 ? 1 : 2;
    const uint32_t per = (nblk + nb - 1) / nb;
    uint32_t lpr = 8;
    while (lpr < per) lpr *= 2;
    const uint32_t rpi0 = kRawStagedThreads / lpr;
    const uint64_t pass = static_cast<uint64_t>(rpi0) * nblk * 34u;
    const uint32_t u = (nb == 1 && pass <= 16u * 1024u) ? 2 : 1;
    const uint32_t rpi = u * rpi0;
    const uint64_t slot =
        ((pass * u + 2 * (kRawWindowAlign - 1) + 4 + kRawWindowAlign - 1) / kRawWindowAlign) * kRawWindowAlign;
    const uint64_t budget = 200u * 1024u;
    if (slot * 3 > budget) return VRT_E_UNSUPPORTED;
    const uint32_t slots = static_cast<uint32_t>(std::min<uint64_t>(kRawStagedMaxSlots, budget / slot));
    RawStagedParams q{};
    q.w = p.w;
    q.count = p.count;
    q.cols = p.cols;
    q.x = p.x;
    q.y = p.y;
    q.amax = p.amax;
    q.status = status;
    q.slot_bytes = static_cast<uint32_t>(slot);
    q.slots = slots;
    const uint64_t total = p.row_start[p.count];
    if (total == 0) return VRT_OK;
    uint32_t ctas = 0;
    for (uint32_t m = 0; m < p.count; ++m) {
        const uint32_t rows = p.row_start[m + 1] - p.row_start[m];
        uint32_t c = static_cast<uint32_t>(static_cast<uint64_t>(sms) * rows / total);
        c = std::max(c, rows ? 1u : 0u);
        c = std::min(c, (rows + rpi - 1) / rpi);  // no CTA without a full iteration's worth of rows
        q.offsets[m] = p.offsets[m];
        q.row_start[m] = p.row_start[m];
        q.cta_start[m] = ctas;
        ctas += c;
    }
    q.row_start[p.count] = p.row_start[p.count];
    q.cta_start[p.count] = ctas;
    RawStagedFn k = raw_staged_kernel_for(lpr, nb, u);
    if (!k) return VRT_E_UNSUPPORTED;
    static std::mutex mu;
    static uint64_t attr_done[16] = {};  // per kernel, bit d: set on device d
    const int ai = nb == 2 ? 15 : (__builtin_ctz(lpr) - 3) + (u == 2 ? 7 : 0);
    int dev = 0;
    VRT_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> g(mu);
        const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
        if (!(attr_done[ai] & bit)) {
            VRT_CUDA(raise_smem_limit(k));
            attr_done[ai] |= bit;
        }
    }
    VRT_CUDA(launch(k, dim3(ctas), dim3(kRawStagedThreads + 32), slots * q.slot_bytes, s, false, q));
    return VRT_OK;
}

static int raw_gemv_sms(int sms, const RawGemvParams& p, cudaStream_t s, uint32_t* status) {
    {
        const int rc = raw_gemv_staged(sms, p, status, s);
        if (rc != VRT_E_UNSUPPORTED) return rc;
        clear_error();
    }
    const uint32_t nblk = p.cols / 32;
    const uint32_t smem = ((nblk * 4 + 15) / 16) * 16 + p.cols * 4;
    const uint32_t rows = p.row_start[p.count];
    const int G = nblk <= 32 ? 8 : (nblk <= 64 ? 16 : 32);
    const uint32_t rows_per_cta = (kRawThreads / 32) * (32 / G);
    int occ = 2;
    const uint32_t max_grid = static_cast<uint32_t>(sms) * occ;
    const uint32_t grid = std::max(1u, std::min(max_grid, (rows + rows_per_cta - 1) / rows_per_cta));
    // the shared-memory limit is a per-device function attribute
    static std::mutex mu;
    static uint64_t attr_done[3] = {0, 0, 0};  // bit d: set on device d
    void (*k)(const RawGemvParams) = G == 8 ? raw_gemv_kernel<8> : (G == 16 ? raw_gemv_kernel<16> : raw_gemv_kernel<32>);
    const int ai = G == 8 ? 0 : (G == 16 ? 1 : 2);
    int dev = 0;
    VRT_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> g(mu);
        const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
        if (!(attr_done[ai] & bit)) {
            VRT_CUDA(raise_smem_limit(k));
            attr_done[ai] |= bit;
        }
    }
    if (smem > 200u * 1024u) return fail(VRT_E_UNSUPPORTED, "input_dim %u too large for one CTA", p.cols);
    VRT_CUDA(launch(k, dim3(grid), dim3(kRawThreads), smem, s, false, p));
    return VRT_OK;
}

// The pipeline status word of a context: the third 32-bit word of its
// 64-byte device scratch (the first two hold the argmax key).
static uint32_t* ctx_status_word(vrt_ctx* ctx) { return reinterpret_cast<uint32_t*>(ctx->d_key) + 2; }

static int raw_gemv(vrt_ctx* ctx, const RawGemvParams& p, cudaStream_t s) {
    return raw_gemv_sms(ctx->prop.multiProcessorCount, p, s, ctx_status_word(ctx));
}

static int check_q8_matrix(uint64_t weights_bytes, uint64_t off, uint32_t in, uint32_t out, const char* what) {
    if (in == 0 || out == 0) return fail(VRT_E_INVALID, "%s dimensions must be non-zero", what);
    if (in % 32) return fail(VRT_E_INVALID, "%s input_dim must be divisible by 32", what);
    if (off & 3u) return fail(VRT_E_INVALID, "%s weight byte offset must be 4-byte aligned", what);
    const uint64_t bytes = static_cast<uint64_t>(in) / 32 * 34 * out;
    if (off > weights_bytes || bytes > weights_bytes - off) return fail(VRT_E_INVALID, "%s weight buffer is too small", what);
    return VRT_OK;
}

}  // namespace vrt

using namespace vrt;

extern "C" {

const char* vrt_last_error(void) { return g_last_error.c_str(); }
const char* vrt_version(void) { return "vortexrt_b200 0.1 (sm_100a)"; }

int vrt_ctx_create(int device, vrt_ctx** out) {
    clear_error();
    if (!out) return fail(VRT_E_INVALID, "out is null");
    if (device < 0) {
        const char* env = getenv("VORTEXRT_DEVICE");
        device = env ? atoi(env) : 0;
    }
    int n = 0;
    VRT_CUDA(cudaGetDeviceCount(&n));
    if (device >= n) return fail(VRT_E_INVALID, "device %d not present (%d devices)", device, n);
    auto* c = new vrt_ctx();
    c->device = device;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaGetDeviceProperties(&c->prop, device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_key, 64);
    if (e == cudaSuccess) e = cudaMemset(c->d_key, 0, 64);  // argmax key + pipeline status word
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "vrt_ctx_create", __FILE__, __LINE__);
    }
    if (c->prop.major < 10) {
        const int rc = fail(VRT_E_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device,
                            c->prop.major, c->prop.minor);
        cudaFree(c->d_key);
        cudaStreamDestroy(c->stream);
        delete c;
        return rc;
    }
    *out = c;
    return VRT_OK;
}

int vrt_ctx_destroy(vrt_ctx* ctx) {
    if (!ctx) return VRT_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto& kv : ctx->allocs) cudaFree(kv.first);
    cudaFree(ctx->d_key);
    cudaFree(ctx->ws);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return VRT_OK;
}

int vrt_ctx_info(vrt_ctx* ctx, vrt_device_info* out) {
    if (!ctx || !out) return fail(VRT_E_INVALID, "null argument");
    memset(out, 0, sizeof *out);
    strncpy(out->name, ctx->prop.name, sizeof out->name - 1);
    out->device = ctx->device;
    out->sm_count = ctx->prop.multiProcessorCount;
    out->cc_major = ctx->prop.major;
    out->cc_minor = ctx->prop.minor;
    out->warp_size = static_cast<uint32_t>(ctx->prop.warpSize);
    out->global_mem_bytes = ctx->prop.totalGlobalMem;
    out->l2_bytes = static_cast<uint64_t>(ctx->prop.l2CacheSize);
    return VRT_OK;
}

int vrt_ctx_synchronize(vrt_ctx* ctx) {
    if (!ctx) return fail(VRT_E_INVALID, "null context");
    VRT_CUDA(cudaSetDevice(ctx->device));
    VRT_CUDA(cudaStreamSynchronize(ctx->stream));
    return VRT_OK;
}

void* vrt_ctx_stream(vrt_ctx* ctx) { return ctx ? ctx->stream : nullptr; }

int vrt_alloc(vrt_ctx* ctx, size_t bytes, void** d_out) {
    if (!ctx || !d_out) return fail(VRT_E_INVALID, "null argument");
    if (bytes == 0) return fail(VRT_E_INVALID, "allocation size must be non-zero");
    VRT_CUDA(cudaSetDevice(ctx->device));
    void* p = nullptr;
    VRT_CUDA(cudaMalloc(&p, bytes + 256));
    VRT_CUDA(cudaMemsetAsync(p, 0, bytes + 256, ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(ctx->stream));
    std::lock_guard<std::mutex> g(ctx->mu);
    ctx->allocs[p] = bytes;
    *d_out = p;
    return VRT_OK;
}

int vrt_free(vrt_ctx* ctx, void* d_ptr) {
    if (!ctx) return fail(VRT_E_INVALID, "null context");
    if (!d_ptr) return VRT_OK;
    {
        std::lock_guard<std::mutex> g(ctx->mu);
        auto it = ctx->allocs.find(d_ptr);
        if (it == ctx->allocs.end()) return fail(VRT_E_INVALID, "pointer was not allocated by vrt_alloc");
        ctx->allocs.erase(it);
    }
    VRT_CUDA(cudaSetDevice(ctx->device));
    VRT_CUDA(cudaStreamSynchronize(ctx->stream));
    VRT_CUDA(cudaFree(d_ptr));
    return VRT_OK;
}

int vrt_upload(vrt_ctx* ctx, void* d_dst, const void* h_src, size_t bytes) {
    if (!ctx || (!d_dst && bytes) || (!h_src && bytes)) return fail(VRT_E_INVALID, "null argument");
    if (!bytes) return VRT_OK;
    VRT_CUDA(cudaSetDevice(ctx->device));
    VRT_CUDA(cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(ctx->stream));
    return VRT_OK;
}

int vrt_download(vrt_ctx* ctx, void* h_dst, const void* d_src, size_t bytes) {
    if (!ctx || (!d_src && bytes) || (!h_dst && bytes)) return fail(VRT_E_INVALID, "null argument");
    if (!bytes) return VRT_OK;
    VRT_CUDA(cudaSetDevice(ctx->device));
    VRT_CUDA(cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(ctx->stream));
    return VRT_OK;
}

int vrt_upload_async(vrt_ctx* ctx, void* d_dst, const void* h_src, size_t bytes, void* stream) {
    if (!ctx) return fail(VRT_E_INVALID, "null context");
    VRT_CUDA(cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, as_stream(ctx, stream)));
    return VRT_OK;
}

int vrt_download_async(vrt_ctx* ctx, void* h_dst, const void* d_src, size_t bytes, void* stream) {
    if (!ctx) return fail(VRT_E_INVALID, "null context");
    VRT_CUDA(cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, as_stream(ctx, stream)));
    return VRT_OK;
}

int vrt_host_alloc_pinned(size_t bytes, void** h_out) {
    if (!h_out || !bytes) return fail(VRT_E_INVALID, "bad argument");
    VRT_CUDA(cudaMallocHost(h_out, bytes));
    return VRT_OK;
}

int vrt_host_free_pinned(void* h_ptr) {
    if (h_ptr) VRT_CUDA(cudaFreeHost(h_ptr));
    return VRT_OK;
}

int vrt_q8_gemv(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes, uint64_t off, const float* d_x,
                float* d_y, uint32_t input_dim, uint32_t output_dim, void* stream) {
    clear_error();
    if (!ctx || !d_weights || !d_x || !d_y) return fail(VRT_E_INVALID, "Q8MatVecPipeline: null argument");
    VRT_TRY(check_q8_matrix(weights_bytes, off, input_dim, output_dim, "Q8MatVecPipeline"));
    RawGemvParams p{};
    p.w = static_cast<const uint8_t*>(d_weights);
    p.offsets[0] = off;
    p.row_start[0] = 0;
    p.row_start[1] = output_dim;
    p.count = 1;
    p.cols = input_dim;
    p.x = d_x;
    p.y = d_y;
    return raw_gemv(ctx, p, as_stream(ctx, stream));
}

int vrt_q8_gemv_multi(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes, const uint64_t* offs,
                      const uint32_t* dims, uint32_t count, const float* d_x, float* d_y, uint32_t input_dim,
                      void* stream) {
    clear_error();
    if (!ctx || !d_weights || !d_x || !d_y || !offs || !dims) return fail(VRT_E_INVALID, "Q8 multi: null argument");
    if (count == 0 || count > kMaxMulti) return fail(VRT_E_INVALID, "Q8 multi: count must be 1..%d", kMaxMulti);
    RawGemvParams p{};
    p.w = static_cast<const uint8_t*>(d_weights);
    p.count = count;
    p.cols = input_dim;
    p.x = d_x;
    p.y = d_y;
    uint64_t total = 0;
    for (uint32_t i = 0; i < count; ++i) {
        VRT_TRY(check_q8_matrix(weights_bytes, offs[i], input_dim, dims[i], "Q8 multi"));
        p.offsets[i] = offs[i];
        p.row_start[i] = static_cast<uint32_t>(total);
        total += dims[i];
        if (total > 0xffffffffull) return fail(VRT_E_INVALID, "Q8 multi: packed output size overflow");
    }
    p.row_start[count] = static_cast<uint32_t>(total);
    return raw_gemv(ctx, p, as_stream(ctx, stream));
}

int vrt_gelu_mul(vrt_ctx* ctx, float* d_gate, const float* d_up, uint32_t count, void* stream) {
    clear_error();
    if (!ctx || !d_gate || !d_up) return fail(VRT_E_INVALID, "gelu_mul: null argument");
    if (!count) return VRT_OK;
    VRT_CUDA(launch(gelu_mul_kernel, dim3((count + 255) / 256), dim3(256), 0, as_stream(ctx, stream), false,
                    d_gate, d_up, count));
    return VRT_OK;
}

int vrt_q8_ffn(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes, uint64_t gate_off, uint64_t up_off,
               uint64_t down_off, const float* d_x, float* d_ws, float* d_y, uint32_t input_dim, uint32_t ffn_dim,
               uint32_t output_dim, void* stream) {
    clear_error();
    if (!ctx || !d_weights || !d_x || !d_ws || !d_y) return fail(VRT_E_INVALID, "Q8 fused FFN: null argument");
    if (!input_dim || !ffn_dim || !output_dim || input_dim % 32 || ffn_dim % 32) {
        return fail(VRT_E_INVALID, "Q8 fused FFN dimensions must be non-zero and Q8 aligned");
    }
    VRT_TRY(check_q8_matrix(weights_bytes, gate_off, input_dim, ffn_dim, "Q8 fused FFN gate"));
    VRT_TRY(check_q8_matrix(weights_bytes, up_off, input_dim, ffn_dim, "Q8 fused FFN up"));
    VRT_TRY(check_q8_matrix(weights_bytes, down_off, ffn_dim, output_dim, "Q8 fused FFN down"));
    const uint64_t offs[2] = {gate_off, up_off};
    const uint32_t dims[2] = {ffn_dim, ffn_dim};
    VRT_TRY(vrt_q8_gemv_multi(ctx, d_weights, weights_bytes, offs, dims, 2, d_x, d_ws, input_dim, stream));
    VRT_TRY(vrt_gelu_mul(ctx, d_ws, d_ws + ffn_dim, ffn_dim, stream));
    return vrt_q8_gemv(ctx, d_weights, weights_bytes, down_off, d_ws, d_y, ffn_dim, output_dim, stream);
}

// ------------------------------------------------------------------------
// Fused FFN for callers that cannot allocate device memory.
//
// vrt_q8_ffn needs a context (whose creation allocates) and a caller-owned
// workspace for the gate and up projections.  Some callers cannot do either:
// code that runs where device allocation is forbidden or unavailable -- inside
// another framework's memory pool that must not grow, in an embedded host
// that has pre-reserved all device memory, or in a tool that may only launch
// work.  For them the gate/up intermediate lives in this file-scope device
// array, which every GPU that loads the library holds until the process exits.
constexpr uint32_t kStaticFfnMax = 32768;  // largest ffn_dim accepted
static __device__ __align__(256) float g_ffn_scratch[2 * kStaticFfnMax];
// pipeline status word of the static entry point (kStatusWaitTimeout bits)
static __device__ uint32_t g_static_status;

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
float* g_static_ptr[kMaxDevices] = {};
uint32_t* g_static_status_ptr[kMaxDevices] = {};
int g_static_sms[kMaxDevices] = {};
}  // namespace

}  // extern "C": reopened after the set-up helper

// Device address of g_ffn_scratch on the current device.  In host code the
// array's name only stands in for the device symbol, so the address must come
// from cudaGetSymbolAddress, once per device, with that device current.
static int static_ffn_setup(float** ptr, int* sms, uint32_t** status) {
    int dev = 0;
    VRT_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(VRT_E_UNSUPPORTED, "device %d beyond %d", dev, kMaxDevices);
    std::lock_guard<std::mutex> g(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* p = nullptr;
        void* st = nullptr;
        VRT_CUDA(cudaGetSymbolAddress(&p, g_ffn_scratch));
        VRT_CUDA(cudaGetSymbolAddress(&st, g_static_status));
        int n = 0;
        VRT_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        g_static_ptr[dev] = static_cast<float*>(p);
        g_static_status_ptr[dev] = static_cast<uint32_t*>(st);
        g_static_sms[dev] = n;
    }
    *ptr = g_static_ptr[dev];
    *sms = g_static_sms[dev];
    if (status) *status = g_static_status_ptr[dev];
    return VRT_OK;
}

extern "C" {

int vrt_q8_ffn_static(const void* d_weights, uint64_t weights_bytes, uint64_t gate_off, uint64_t up_off,
                      uint64_t down_off, const float* d_x, float* d_y, uint32_t input_dim, uint32_t ffn_dim,
                      uint32_t output_dim, void* stream) {
    clear_error();
    if (!d_weights || !d_x || !d_y) return fail(VRT_E_INVALID, "Q8 fused FFN: null argument");
    if (!input_dim || !ffn_dim || !output_dim || input_dim % 32 || ffn_dim % 32) {
        return fail(VRT_E_INVALID, "Q8 fused FFN dimensions must be non-zero and Q8 aligned");
    }
    if (ffn_dim > kStaticFfnMax) {
        return fail(VRT_E_INVALID, "vrt_q8_ffn_static: ffn_dim %u exceeds the static scratch limit of %u", ffn_dim,
                    kStaticFfnMax);
    }
    VRT_TRY(check_q8_matrix(weights_bytes, gate_off, input_dim, ffn_dim, "Q8 fused FFN gate"));
    VRT_TRY(check_q8_matrix(weights_bytes, up_off, input_dim, ffn_dim, "Q8 fused FFN up"));
    VRT_TRY(check_q8_matrix(weights_bytes, down_off, ffn_dim, output_dim, "Q8 fused FFN down"));
    float* ws = nullptr;
    uint32_t* status = nullptr;
    int sms = 0;
    VRT_TRY(static_ffn_setup(&ws, &sms, &status));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // gate and up are written in full before gelu_mul reads them: the scratch
    // needs no clearing between calls
    RawGemvParams p{};
    p.w = static_cast<const uint8_t*>(d_weights);
    p.offsets[0] = gate_off;
    p.offsets[1] = up_off;
    p.row_start[1] = ffn_dim;
    p.row_start[2] = 2 * ffn_dim;
    p.count = 2;
    p.cols = input_dim;
    p.x = d_x;
    p.y = ws;
    VRT_TRY(raw_gemv_sms(sms, p, s, status));
    VRT_CUDA(launch(gelu_mul_kernel, dim3((ffn_dim + 255) / 256), dim3(256), 0, s, false, ws, (const float*)(ws + ffn_dim),
                    ffn_dim));
    RawGemvParams d{};
    d.w = static_cast<const uint8_t*>(d_weights);
    d.offsets[0] = down_off;
    d.row_start[1] = output_dim;
    d.count = 1;
    d.cols = ffn_dim;
    d.x = ws;
    d.y = d_y;
    return raw_gemv_sms(sms, d, s, status);
}

#ifdef VRT_CHAIN_STAMPS
// Timing builds only: copy the first n launch slots of the decode-step stamps
// ([n][6] globaltimer values, see chain_stamp) to the host and reset them.
__attribute__((visibility("default"))) int vrt_chain_stamps(unsigned long long* h_out, uint32_t n) {
    if (n > kChainStampSlots) n = kChainStampSlots;
    VRT_CUDA(cudaDeviceSynchronize());
    VRT_CUDA(cudaMemcpyFromSymbol(h_out, g_chain_stamps, sizeof(unsigned long long) * kChainStampFields * n));
    static unsigned long long init[kChainStampSlots][kChainStampFields];
    for (uint32_t i = 0; i < kChainStampSlots; ++i)
        for (int f = 0; f < kChainStampFields; ++f) init[i][f] = f <= 1 ? ~0ull : 0ull;
    VRT_CUDA(cudaMemcpyToSymbol(g_chain_stamps, init, sizeof(init)));
    return VRT_OK;
}
#endif

int vrt_pipeline_status(vrt_ctx* ctx, uint32_t* h_status) {
    clear_error();
    if (!h_status) return fail(VRT_E_INVALID, "vrt_pipeline_status: null output");
    uint32_t* word = nullptr;
    if (ctx) {
        VRT_CUDA(cudaSetDevice(ctx->device));
        VRT_CUDA(cudaStreamSynchronize(ctx->stream));
        word = ctx_status_word(ctx);
    } else {
        float* ws = nullptr;
        int sms = 0;
        VRT_TRY(static_ffn_setup(&ws, &sms, &word));
    }
    VRT_CUDA(cudaMemcpy(h_status, word, 4, cudaMemcpyDeviceToHost));
    VRT_CUDA(cudaMemset(word, 0, 4));
    return VRT_OK;
}

int vrt_argmax(vrt_ctx* ctx, const float* d_x, uint32_t count, vrt_argmax_result* d_out, void* stream) {
    clear_error();
    if (!ctx || !d_x || !d_out) return fail(VRT_E_INVALID, "ArgmaxPipeline: null argument");
    if (count == 0) return fail(VRT_E_INVALID, "ArgmaxPipeline requires non-zero input");
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaMemsetAsync(ctx->d_key, 0, 8, s));
    const uint32_t grid = std::max(1u, std::min((count + 1023) / 1024, static_cast<uint32_t>(ctx->prop.multiProcessorCount) * 4));
    VRT_CUDA(launch(argmax_kernel, dim3(grid), dim3(1024), 0, s, false, d_x, count, ctx->d_key));
    VRT_CUDA(launch(argmax_unkey_kernel, dim3(1), dim3(1), 0, s, false, (const unsigned long long*)ctx->d_key,
                    reinterpret_cast<uint32_t*>(d_out)));
    return VRT_OK;
}

int vrt_lm_head_argmax(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes, uint64_t off, const float* d_x,
                       uint32_t input_dim, uint32_t vocab, float* d_logits, vrt_argmax_result* d_out, void* stream) {
    clear_error();
    if (!ctx || !d_weights || !d_x || !d_out) return fail(VRT_E_INVALID, "LM head: null argument");
    VRT_TRY(check_q8_matrix(weights_bytes, off, input_dim, vocab, "LM head"));
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaMemsetAsync(ctx->d_key, 0, 8, s));
    RawGemvParams p{};
    p.w = static_cast<const uint8_t*>(d_weights);
    p.offsets[0] = off;
    p.row_start[1] = vocab;
    p.count = 1;
    p.cols = input_dim;
    p.x = d_x;
    p.y = d_logits;
    p.amax = ctx->d_key;
    VRT_TRY(raw_gemv(ctx, p, s));
    VRT_CUDA(launch(argmax_unkey_kernel, dim3(1), dim3(1), 0, s, false, (const unsigned long long*)ctx->d_key,
                    reinterpret_cast<uint32_t*>(d_out)));
    return VRT_OK;
}

}  // extern "C"
