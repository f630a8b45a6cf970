// Device helpers shared by the sm_100a kernels: PTX wrappers for mbarriers,
// bulk (TMA) copies and programmatic dependent launch; bounded waits; the
// Q8_0 tiled weight layout; int16 activation quantisation; argmax keys.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace vrt {

// ----------------------------------------------------------------- layout
//
// "Q8T" tiled Q8_0 layout used by the model path.  A [rows][K] Q8_0 matrix
// (K % 128 == 0) is cut into row groups of 16 rows (zero-padded) and K tiles
// of 128 columns.  Tile (g, j) sits at byte ((g * K/128) + j) * 2176, so a
// row group -- and any run of row groups -- is one contiguous byte span that
// one bulk copy can move.  Inside a tile the bytes are in the order one warp
// consumes them, which makes every shared-memory read a conflict-free
// 16-byte access:
//   bytes [0, 2048): chunk ci = s*32 + lane (s = 0..3) at ci*16 holds the 16
//       int8 weights of row 2*(lane/4) + s/2, columns 32*(lane%4) + 16*(s%2)
//       + [0, 16) of the tile;
//   bytes [2048, 2176): 32-bit word `lane` = fp16 scale of (row 2*(lane/4),
//       block lane%4) in the low half, of row 2*(lane/4)+1 in the high half.
// Bytes per weight are the same as GGUF's 34 per 32.
constexpr int kTileCols = 128;
constexpr int kTileRows = 16;
constexpr int kTileQBytes = 2048;
constexpr int kTileBytes = 2176;

__host__ __device__ inline uint64_t q8t_bytes(uint64_t rows, uint64_t cols) {
    return (rows + kTileRows - 1) / kTileRows * (cols / kTileCols) * kTileBytes;
}

// Byte offset (within the tiled matrix) of weight (row, col) and of its scale.
__host__ __device__ inline uint64_t q8t_weight_offset(uint64_t row, uint64_t col, uint64_t cols) {
    const uint64_t g = row / kTileRows, r = row % kTileRows, j = col / kTileCols, cc = col % kTileCols;
    const uint64_t lane = (r / 2) * 4 + cc / 32;
    const uint64_t s = (r % 2) * 2 + (cc % 32) / 16;
    return (g * (cols / kTileCols) + j) * kTileBytes + (s * 32 + lane) * 16 + (cc % 16);
}
__host__ __device__ inline uint64_t q8t_scale_offset(uint64_t row, uint64_t block, uint64_t cols) {
    const uint64_t g = row / kTileRows, r = row % kTileRows, j = block / 4, b = block % 4;
    const uint64_t lane = (r / 2) * 4 + b;
    return (g * (cols / kTileCols) + j) * kTileBytes + kTileQBytes + lane * 4 + (r % 2) * 2;
}

// Index (in int16 elements) of activation column k in the permuted
// per-tile order of the quantised activation vector (x16p): within each
// 128-column tile, part p = (k%32)/8 of lane-quad c = (k%128)/32 sits at
// p*32 + c*8, so the four lanes of a quad read four adjacent 16-byte words.
__host__ __device__ inline uint32_t x16p_index(uint32_t k) {
    const uint32_t j = k / 128, kk = k % 128, c = kk / 32, b = kk % 32;
    return j * 128 + (b / 8) * 32 + c * 8 + (b % 8);
}

// ------------------------------------------------------------------- PTX

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// A wait that gives up after ~1 s of SM clock (2^31 cycles) instead of
// spinning forever; the caller records the failure in the device status word.
constexpr long long kWaitLimitCycles = 1ll << 31;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
    return true;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes and
// both addresses 16-byte aligned).  No cluster multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Same copy with an L2 cache-policy hint (used with an evict-first policy for
// weights that are streamed once per token).
__device__ __forceinline__ void bulk_copy_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                   uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Bring [src, src + bytes) into L2 without waiting (16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's results /
// allow the next grid to start its prologue.  Both are no-ops when the
// kernel was launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------- timing builds
// An instrumented build (`make stamps`: -DVRT_CHAIN_STAMPS, never the
// default) records per decode-step launch `slot` the globaltimer at phase
// boundaries, reduced over the launch's CTAs: [0] first CTA start (min),
// [1] first wait release (min), [2] last wait release (max), [3] last CTA past
// the tensor-parallel exchange (max), [4] last CTA past its prologue (max),
// [5] last CTA end (max).  One thread per CTA stamps.  In the default build
// every call compiles to nothing.
constexpr uint32_t kChainStampSlots = 2048;
constexpr int kChainStampFields = 6;
#ifdef VRT_CHAIN_STAMPS
static __device__ unsigned long long g_chain_stamps[kChainStampSlots][kChainStampFields];
#endif
__device__ __forceinline__ void chain_stamp(uint32_t slot, int field) {
#ifdef VRT_CHAIN_STAMPS
    if (slot >= kChainStampSlots) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (field <= 1) {
        atomicMin(&g_chain_stamps[slot][field], t);
    } else {
        atomicMax(&g_chain_stamps[slot][field], t);
    }
#else
    (void)slot;
    (void)field;
#endif
}
// Stamps field 5 (end) when the CTA's stamping thread leaves the kernel, on
// every return path.
struct ChainStampEnd {
    uint32_t slot;
    bool on;
    __device__ ~ChainStampEnd() {
        if (on) chain_stamp(slot, 5);
    }
};

// ------------------------------------------------------------- numerics

// Device status bits (vrt_model_device_status).
constexpr uint32_t kStatusWaitTimeout = 1u << 0;
constexpr uint32_t kStatusBadToken = 1u << 1;
constexpr uint32_t kStatusNonFinite = 1u << 2;

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// Block of 32 activations -> int16 with one fp32 scale: s = amax / 32767,
// q = rint(x / s).  Integer block dot products with int8 weights are then
// exact; the activation carries a relative error <= 2^-16 of the block max.
__device__ __forceinline__ float quant_scale(float amax) { return amax / 32767.0f; }
__device__ __forceinline__ int quant_one(float x, float inv) {
    int q = __float2int_rn(x * inv);
    return q > 32767 ? 32767 : (q < -32767 ? -32767 : q);
}

__device__ __forceinline__ float gelu_tanh(float x) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))): shaders/gelu_mul.comp:23-29
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    const float x3 = __fmul_rn(__fmul_rn(x, x), x);
    const float inner = __fmul_rn(k0, __fadd_rn(x, __fmul_rn(k1, x3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// Argmax as one 64-bit key: order-preserving float bits in the high word,
// ~index in the low word, so atomicMax keeps the largest value and, among
// equal values, the lowest index (shaders/argmax.comp:30-43).  NaN is never
// offered.  Key 0 = "no element".
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned long long>(0xffffffffu - index);
}
__host__ __device__ inline void argmax_unkey(unsigned long long key, uint32_t* index, float* value) {
    if (key == 0ull) {
        *index = 0xffffffffu;
        uint32_t ninf = 0xff800000u;
        float f;
        memcpy(&f, &ninf, 4);
        *value = f;
        return;
    }
    uint32_t u = static_cast<uint32_t>(key >> 32);
    u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
    float f;
    memcpy(&f, &u, 4);
    *value = f;
    *index = 0xffffffffu - static_cast<uint32_t>(key & 0xffffffffu);
}

// w = hi + lo with both terms fp16 (to ~2^-22 relative): the tensor-core
// operand form of an fp32 value.
__device__ __forceinline__ void split_f16(float w, __half& hi, __half& lo) {
    hi = __float2half_rn(w);
    lo = __float2half_rn(__fsub_rn(w, __half2float(hi)));
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace vrt
