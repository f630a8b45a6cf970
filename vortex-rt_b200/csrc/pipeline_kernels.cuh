// Kernels behind the reference's pipeline entry points, reading raw GGUF
// Q8_0 rows (34-byte blocks) straight from a caller's buffer at a 4-byte
// aligned offset, the layout Q8MatVecPipeline::run consumes
// (src/q8_matvec.cpp:801-930).
//
// Row mapping: G lanes per row (G = 8/16/32 by row width), rows grid-strided.
// A lane reads each of its blocks with aligned 32-bit loads and realigns
// the quants with funnel shifts (a block starts 2 bytes off a word boundary
// in every other position); no read leaves the block's own bytes and the
// two bytes before it.  The activation vector is quantised once per CTA,
// per 32-block, into two int16 digits in shared memory: x ~= s * (hi +
// lo / 65536), s = amax / 32767, which carries about 31 bits of the block
// maximum -- as fine as the fp32 input -- so the pipeline entry points meet
// the reference test programs' absolute tolerances even on large outputs.
// Block sums are exact dp2a integer sums per digit; lanes combine in a
// fixed shuffle tree, so results replay bit for bit.
#pragma once

#include "vrt_device.cuh"

namespace vrt {

constexpr int kRawThreads = 512;
constexpr int kMaxMulti = 8;

struct RawGemvParams {
    const uint8_t* w;            // weights buffer base
    uint64_t offsets[kMaxMulti]; // byte offset of each matrix
    uint32_t row_start[kMaxMulti + 1]; // prefix sums of output dims
    uint32_t count;
    uint32_t cols;
    const float* x;
    float* y;                    // packed outputs (may be null for argmax-only)
    unsigned long long* amax;    // non-null: fold rows into the argmax key
};

// natural-order int16 activations: block b at b*32, 4-way rotated 16-byte parts
__device__ __forceinline__ uint32_t raw_x16_index(uint32_t blk, uint32_t part) {
    return blk * 32 + ((part + blk) & 3) * 8;
}

template <int G>
__global__ void __launch_bounds__(kRawThreads) raw_gemv_kernel(const RawGemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nblk = p.cols / 32;
    float* sx = reinterpret_cast<float*>(smem);
    int16_t* x16 = reinterpret_cast<int16_t*>(smem + ((nblk * 4 + 15) / 16) * 16);
    int16_t* x16lo = x16 + p.cols;
    __shared__ unsigned long long warp_best[kRawThreads / 32];

    pdl_wait();
    for (uint32_t blk = threadIdx.x; blk < nblk; blk += blockDim.x) {
        float v[32];
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            v[e] = p.x[blk * 32 + e];
            amax = fmaxf(amax, fabsf(v[e]));
        }
        const float sc = quant_scale(amax);
        sx[blk] = sc;
        const float inv = amax > 0.0f ? 32767.0f / amax : 0.0f;
        const float inv_lo = inv * 65536.0f;
#pragma unroll
        for (int part = 0; part < 4; ++part) {
            uint32_t wv[4], wl[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                int q[2], r[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float xv = v[part * 8 + 2 * e + h];
                    q[h] = quant_one(xv, inv);
                    r[h] = quant_one(fmaf(-static_cast<float>(q[h]), sc, xv), inv_lo);
                }
                wv[e] = (static_cast<uint32_t>(q[0]) & 0xffffu) | (static_cast<uint32_t>(q[1]) << 16);
                wl[e] = (static_cast<uint32_t>(r[0]) & 0xffffu) | (static_cast<uint32_t>(r[1]) << 16);
            }
            *reinterpret_cast<uint4*>(x16 + raw_x16_index(blk, part)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            *reinterpret_cast<uint4*>(x16lo + raw_x16_index(blk, part)) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
        }
    }
    __syncthreads();
    pdl_trigger();

    const uint32_t total_rows = p.row_start[p.count];
    const uint32_t lane = threadIdx.x & 31, sub = lane % G;
    const uint32_t rows_per_warp = 32 / G;
    const uint32_t warp_global = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const uint32_t n_warps = gridDim.x * blockDim.x / 32;
    const uint64_t row_bytes = static_cast<uint64_t>(nblk) * 34u;
    unsigned long long best = 0ull;

    for (uint32_t base = warp_global * rows_per_warp; base < total_rows; base += n_warps * rows_per_warp) {
        const uint32_t row = base + lane / G;
        float acc = 0.0f;
        if (row < total_rows) {
            uint32_t m = 0;
            while (row >= p.row_start[m + 1]) ++m;
            const uint8_t* rp = p.w + p.offsets[m] + (row - p.row_start[m]) * row_bytes;
            for (uint32_t b = sub; b < nblk; b += G) {
                const uint8_t* a = rp + static_cast<uint64_t>(b) * 34u;
                // Every read stays inside [a - 2, a + 34): the block itself, or
                // the tail of the previous block of the same matrix (odd case;
                // a matrix starts 4-byte aligned, so its first block is even).
                const bool odd = (reinterpret_cast<uintptr_t>(a) & 3u) != 0u;
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(a - (odd ? 2 : 0));
                uint32_t W[9];
#pragma unroll
                for (int i = 0; i < 8; ++i) W[i] = __ldg(wp + i);
                W[8] = odd ? __ldg(wp + 8) : static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(a + 32)));
                uint32_t q[8];
                uint32_t scale_bits;
                if (odd) {
                    scale_bits = W[0] >> 16;
#pragma unroll
                    for (int i = 0; i < 8; ++i) q[i] = W[i + 1];
                } else {
                    scale_bits = W[0] & 0xffffu;
#pragma unroll
                    for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(W[i], W[i + 1], 16);
                }
                int s = 0, sl = 0;
#pragma unroll
                for (int part = 0; part < 4; ++part) {
                    const uint4 xv = *reinterpret_cast<const uint4*>(x16 + raw_x16_index(b, part));
                    const uint4 xl = *reinterpret_cast<const uint4*>(x16lo + raw_x16_index(b, part));
                    s = __dp2a_lo(static_cast<int>(xv.x), static_cast<int>(q[2 * part]), s);
                    s = __dp2a_hi(static_cast<int>(xv.y), static_cast<int>(q[2 * part]), s);
                    s = __dp2a_lo(static_cast<int>(xv.z), static_cast<int>(q[2 * part + 1]), s);
                    s = __dp2a_hi(static_cast<int>(xv.w), static_cast<int>(q[2 * part + 1]), s);
                    sl = __dp2a_lo(static_cast<int>(xl.x), static_cast<int>(q[2 * part]), sl);
                    sl = __dp2a_hi(static_cast<int>(xl.y), static_cast<int>(q[2 * part]), sl);
                    sl = __dp2a_lo(static_cast<int>(xl.z), static_cast<int>(q[2 * part + 1]), sl);
                    sl = __dp2a_hi(static_cast<int>(xl.w), static_cast<int>(q[2 * part + 1]), sl);
                }
                const float blockv = fmaf(static_cast<float>(sl), 1.0f / 65536.0f, static_cast<float>(s));
                acc += __fmul_rn(half_bits_to_float(scale_bits), sx[b]) * blockv;
            }
        }
#pragma unroll
        for (int o = G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (sub == 0 && row < total_rows) {
            if (p.y) p.y[row] = acc;
            if (p.amax && !isnan(acc)) {
                const unsigned long long k = argmax_key(acc, row);
                best = k > best ? k : best;
            }
        }
    }
    if (p.amax) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) warp_best[threadIdx.x / 32] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long b = 0ull;
            for (uint32_t w = 0; w < blockDim.x / 32; ++w) b = warp_best[w] > b ? warp_best[w] : b;
            if (b) atomicMax(p.amax, b);
        }
    }
}

__global__ void gelu_mul_kernel(float* gate, const float* up, uint32_t n) {
    pdl_wait();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) gate[i] = __fmul_rn(gelu_tanh(gate[i]), up[i]);
}

__global__ void argmax_kernel(const float* x, uint32_t n, unsigned long long* key) {
    pdl_wait();
    unsigned long long best = 0ull;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = x[i];
        if (!isnan(v)) {
            const unsigned long long k = argmax_key(v, i);
            best = k > best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    __shared__ unsigned long long wb[32];
    if ((threadIdx.x & 31) == 0) wb[threadIdx.x / 32] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (uint32_t w = 0; w < blockDim.x / 32; ++w) b = wb[w] > b ? wb[w] : b;
        if (b) atomicMax(key, b);
    }
}

__global__ void argmax_unkey_kernel(const unsigned long long* key, uint32_t* out_index_value) {
    pdl_wait();
    uint32_t idx;
    float val;
    argmax_unkey(*key, &idx, &val);
    out_index_value[0] = idx;
    out_index_value[1] = __float_as_uint(val);
}

}  // namespace vrt
