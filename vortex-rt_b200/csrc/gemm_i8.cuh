// Q8_0 x activation GEMM for few activation rows (batched decode) on the
// integer tensor cores (tcgen05.mma kind::i8), sm_100a.
//
// The fp16 form (gemm_q8t.cuh) dequantises every weight into two fp16 terms
// in shared memory before its MMAs read them back: ~90 KB of shared-memory
// traffic per 8 KB of Q8_0 weights, which bounds it far below HBM speed when
// the activation rows are few.  Here the MMA reads the int8 quants as they
// arrive and the block scales are applied after it:
//
//   * weights: a second copy in the Q8M layout -- 128-row x 128-column tiles,
//     the quants of each tile in the canonical K-major 128B-swizzled operand
//     layout (16 KB), followed by the tile's fp16 block scales [128 rows][4
//     blocks] (1 KB); one 17,408-byte bulk copy per stage, the size of the
//     Q8_0 data it holds;
//   * activations: each 32-block quantised to int16 with the block scale
//     amax / 32512 and split into two signed int8 halves, q = 256 hi + lo
//     (both in [-128, 127]); the B operand is [hi rows | lo rows];
//   * one MMA per Q8_0 block (K = 32): signed int8 x signed int8 into its own
//     int32 TMEM accumulator, exact;
//   * epilogue: per block, y += (w_scale * x_scale) * float(256 acc_hi +
//     acc_lo) in fp32 -- the same per-block arithmetic as the mat-vec
//     (gemv_q8t.cuh), whose block sums are exact int32 too.
//
// One CTA computes 128 weight rows x NT (16 or 32) activation rows over its
// K range.  Warp roles: 0 weight stream (bulk copies, L2 prefetch ahead), 1
// TMEM allocation + MMA issue (one thread), 2 activation stream (2-D TMA,
// 128B swizzle), 4-19 epilogue (warp w reads TMEM lanes 32 (w % 4) ..; four
// warps per lane quarter split the activation rows).  Two accumulator
// buffers of four blocks each ping-pong between the MMA and the epilogue.
// Every mbarrier wait is bounded; TMEM is always freed before exit.
#pragma once

#include "gemm_q8t.cuh"

namespace vrt {

constexpr uint32_t kQ8mRows = 128, kQ8mCols = 128;
constexpr uint32_t kQ8mQBytes = kQ8mRows * kQ8mCols;        // 16,384
constexpr uint32_t kQ8mTileBytes = kQ8mQBytes + kQ8mRows * 8;  // + scales: 17,408
constexpr float kQ16Levels = 32512.0f;                       // 127 * 256: hi stays in [-127, 127]

// Byte of quant (r, c) of a tile (r, c < 128): 8-row swizzle atoms of 1024
// bytes, 16-byte chunk index XOR row % 8.
__host__ __device__ inline uint32_t q8m_q_offset(uint32_t r, uint32_t c) {
    return (r >> 3) * 1024u + (r & 7u) * 128u + ((((c >> 4) ^ r) & 7u) << 4) + (c & 15u);
}
__host__ __device__ inline uint32_t q8m_s_offset(uint32_t r, uint32_t b) { return kQ8mQBytes + r * 8u + b * 2u; }
__host__ __device__ inline uint64_t q8m_tile(uint64_t rt, uint64_t kt, uint64_t kts) {
    return (rt * kts + kt) * kQ8mTileBytes;
}

// Signed int8 halves of a 32-block's int16 quantisation (see above).
struct Q16Out {
    int8_t* hi;        // [rows][ld]
    int8_t* lo;
    float* sx;         // [K / 32][sx_ld] block scales
    uint32_t ld, sx_ld;
};

// Called by all 32 lanes of a warp holding one 32-block (lane = element k
// of row `row`, k % 32 == lane): warp maximum, then each lane its value.
__device__ __forceinline__ void warp_q16_store(const Q16Out& o, uint32_t row, uint32_t k, float v) {
    float am = fabsf(v);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, s));
    am = fmaxf(am, 0.0f);
    const float inv = am > 0.0f ? kQ16Levels / am : 0.0f;
    int q = __float2int_rn(v * inv);
    q = q > 32512 ? 32512 : (q < -32512 ? -32512 : q);
    const int hi = (q + 128) >> 8;
    const int lo = q - hi * 256;
    o.hi[static_cast<uint64_t>(row) * o.ld + k] = static_cast<int8_t>(hi);
    o.lo[static_cast<uint64_t>(row) * o.ld + k] = static_cast<int8_t>(lo);
    if ((k & 31u) == 0) o.sx[static_cast<uint64_t>(k / 32) * o.sx_ld + row] = am / kQ16Levels;
}

struct GemmI8Params {
    const uint8_t* w;          // Q8M copy of an N x K matrix
    uint32_t n, k, m;          // N % 128 == 0, K % 128 == 0, 1 <= M
    const float* sx;           // activation block scales [K / 32][sx_ld]
    uint32_t sx_ld;            // multiple of 4
    float* y;                  // Store / Argmax (optional): y[m * ldy + n]
    uint32_t ldy;
    float* act;                // GeluSplit: act[m * ld_act + n / 2], fp32
    uint32_t ld_act;
    unsigned long long* keys;  // Argmax: [M], zero before the launch
    uint32_t row_base;         // Argmax: global index of weight row 0
    uint32_t nt;               // activation rows per CTA: 16 or 32
    uint32_t ksplit;           // CTAs along K per tile (partials in ws, the last CTA reduces)
    float* ws;                 // [ksplit][t_tiles * nt][n]
    uint32_t* tickets;         // [n / 128 * t_tiles], zero; reset by the reducing CTA
    uint32_t* status;
};

constexpr int kI8EpiWarps = 16;           // 4 TMEM lane quarters x 4 quarters of the activation rows
constexpr int kI8Threads = (4 + kI8EpiWarps) * 32;
constexpr int kI8WStages = 8;             // weight stages in shared memory (139 KB)
constexpr int kI8XStages = 4;
// activation stage: [hi rows | lo rows] x 128 bytes (NT <= 32), then the
// stage's block scales [4 blocks][32 rows] fp32; 1024-byte aligned stages
constexpr uint32_t kI8XOps = 2u * 32u * 128u;
constexpr uint32_t kI8XStage = kI8XOps + 1024u;
constexpr uint32_t kI8Smem = 1024 + kI8WStages * kQ8mTileBytes + kI8XStages * kI8XStage +
                             8 * (2 * kI8WStages + 2 * kI8XStages + 4) + 16;

// D[tmem] = A[smem] * B[smem]^T (no accumulate: every Q8_0 block has its own
// accumulator), M = 128, K = 32, signed int8 inputs, int32 result.
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0u)
        : "memory");
}

// 16 consecutive 32-bit accumulator columns of this warp's 32 TMEM lanes,
// no wait (the caller waits once for several loads).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4_nowait(uint32_t taddr, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int EPI>
__global__ void __launch_bounds__(kI8Threads, 1)
    q8m_gemm_i8_kernel(const __grid_constant__ TmaMap x_hi, const __grid_constant__ TmaMap x_lo, const GemmI8Params p) {
    constexpr int S = kI8WStages, D = kI8XStages;
    extern __shared__ uint8_t gsm_raw[];
    __shared__ uint32_t last_cta;
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* wring = sm;
    uint8_t* xring = wring + S * kQ8mTileBytes;
    uint64_t* w_full = reinterpret_cast<uint64_t*>(xring + D * kI8XStage);
    uint64_t* w_empty = w_full + S;
    uint64_t* x_full = w_empty + S;
    uint64_t* x_empty = x_full + D;
    uint64_t* acc_full = x_empty + D;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t NT = p.nt;  // 16 or 32
    const uint32_t n0 = blockIdx.x * kQ8mRows, t0 = blockIdx.y * NT;
    const uint32_t KTALL = p.k / kQ8mCols;
    const uint32_t kt0 = KTALL * blockIdx.z / p.ksplit, kt1 = KTALL * (blockIdx.z + 1) / p.ksplit;
    const uint32_t KT = kt1 - kt0;
    const uint32_t BC = 2 * NT;         // accumulator columns per block: hi products | lo products
    const uint32_t tcols = 8 * BC;      // two buffers of four blocks: 256 or 512
    // signed int8 A and B, int32 accumulate, both K-major, M = 128, N = 2 NT
    const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((BC >> 3) << 17) | ((kQ8mRows >> 4) << 24);

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], 1 + kI8EpiWarps);  // MMA commit + the epilogue warps (block scales read)
        }
        for (int d = 0; d < D; ++d) {
            mbar_init(&x_full[d], 1);
            mbar_init(&x_empty[d], 1 + kI8EpiWarps);  // MMA commit + the epilogue warps (block scales read)
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], kI8EpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            const uint8_t* wt = p.w + q8m_tile(blockIdx.x, kt0, KTALL);
            for (uint32_t kt = 0; kt < KT && kt < static_cast<uint32_t>(kGemmL2Ahead); ++kt) {
                bulk_prefetch_l2(wt + static_cast<uint64_t>(kt) * kQ8mTileBytes, kQ8mTileBytes);
            }
            for (uint32_t kt = 0; kt < KT; ++kt) {
                if (kt + kGemmL2Ahead < KT) {
                    bulk_prefetch_l2(wt + static_cast<uint64_t>(kt + kGemmL2Ahead) * kQ8mTileBytes, kQ8mTileBytes);
                }
                const uint32_t s = kt % S;
                if (kt >= static_cast<uint32_t>(S)) ok &= mbar_wait_bounded(&w_empty[s], ((kt / S) - 1) & 1);
                mbar_arrive_expect_tx(&w_full[s], kQ8mTileBytes);
                bulk_copy_g2s(wring + s * kQ8mTileBytes, wt + static_cast<uint64_t>(kt) * kQ8mTileBytes, kQ8mTileBytes,
                              &w_full[s]);
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            for (uint32_t kt = 0; kt < KT; ++kt) {
                const uint32_t d = kt % D;
                if (kt >= static_cast<uint32_t>(D)) ok &= mbar_wait_bounded(&x_empty[d], ((kt / D) - 1) & 1);
                uint8_t* st = xring + d * kI8XStage;
                mbar_arrive_expect_tx(&x_full[d], 2 * NT * 128 + 4 * NT * 4);
                const int kx = static_cast<int>((kt0 + kt) * kQ8mCols);  // int8: bytes = columns
                for (uint32_t r0 = 0; r0 < NT; r0 += 16) {
                    tma_load_2d(st + r0 * 128, &x_hi, kx, static_cast<int>(t0 + r0), &x_full[d]);
                    tma_load_2d(st + (NT + r0) * 128, &x_lo, kx, static_cast<int>(t0 + r0), &x_full[d]);
                }
                // this stage's activation block scales (rows t0 .. t0 + NT of blocks 4 kt .. 4 kt + 3)
                for (uint32_t b = 0; b < 4; ++b) {
                    bulk_copy_g2s(st + kI8XOps + b * 128, p.sx + static_cast<uint64_t>((kt0 + kt) * 4 + b) * p.sx_ld + t0,
                                  NT * 4, &x_full[d]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (uint32_t kt = 0; kt < KT; ++kt) {
                const uint32_t a = kt & 1, s = kt % S, d = kt % D;
                if (kt >= 2) ok &= mbar_wait_bounded(&acc_empty[a], ((kt / 2) - 1) & 1);
                ok &= mbar_wait_bounded(&w_full[s], (kt / S) & 1);
                ok &= mbar_wait_bounded(&x_full[d], (kt / D) & 1);
                tc_fence_after();
                const uint32_t wb = smem_addr(wring + s * kQ8mTileBytes), xb = smem_addr(xring + d * kI8XStage);
#pragma unroll
                for (uint32_t b = 0; b < 4; ++b) {  // one Q8_0 block (32 columns = 32 bytes) per MMA
                    umma_i8(tmem + a * 4 * BC + b * BC, sw128_desc(wb + b * 32), sw128_desc(xb + b * 32), idesc);
                }
                umma_commit(&w_empty[s]);
                umma_commit(&x_empty[d]);
                umma_commit(&acc_full[a]);
            }
        }
    } else if (warp >= 4) {
        // epilogue: lanes = weight rows n0 + 32 q + lane; activation rows [t0 + cb, t0 + cb + NT / 2)
        const uint32_t q = warp & 3;
        const uint32_t hc = NT / 4;  // 8 or 4 activation rows per thread
        const uint32_t cb = ((warp - 4) >> 2) * hc;
        const uint32_t r = 32 * q + lane, row = n0 + r;
        float2 acc[4];  // activation rows (2e, 2e + 1) of this thread, paired fp32 arithmetic
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = make_float2(0.0f, 0.0f);
        for (uint32_t kt = 0; kt < KT; ++kt) {
            const uint32_t a = kt & 1, s = kt % S, d = kt % D;
            ok &= mbar_wait_bounded(&acc_full[a], (kt / 2) & 1);
            tc_fence_after();
            const uint2 sw = *reinterpret_cast<const uint2*>(wring + s * kQ8mTileBytes + q8m_s_offset(r, 0));
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_empty[s]);
            const float wsc[4] = {half_bits_to_float(sw.x & 0xffffu), half_bits_to_float(sw.x >> 16),
                                  half_bits_to_float(sw.y & 0xffffu), half_bits_to_float(sw.y >> 16)};
            const float* sxs = reinterpret_cast<const float*>(xring + d * kI8XStage + kI8XOps);
            // per block: this thread's hi and lo columns in two loads, one wait; the
            // int32 block sums of each half are below 2^22 (32 * 127 * 128), so
            // both convert exactly and 256 hi + lo is one rounding, the same
            // as converting the combined int32
#pragma unroll
            for (uint32_t b = 0; b < 4; ++b) {
                const uint32_t col = a * 4 * BC + b * BC + cb;
                uint32_t hv[8], lv[8];
                if (hc == 8) {  // warp-uniform; never reads past this thread's columns of the block
                    tmem_ld8_nowait(tmem + ((32 * q) << 16) + col, hv);
                    tmem_ld8_nowait(tmem + ((32 * q) << 16) + col + NT, lv);
                } else {
                    tmem_ld4_nowait(tmem + ((32 * q) << 16) + col, hv);
                    tmem_ld4_nowait(tmem + ((32 * q) << 16) + col + NT, lv);
#pragma unroll
                    for (int e = 4; e < 8; ++e) hv[e] = lv[e] = 0u;
                }
                float xs[8];
#pragma unroll
                for (uint32_t j0 = 0; j0 < 8; j0 += 4) {
                    const float4 x4 = j0 < hc ? *reinterpret_cast<const float4*>(sxs + b * 32 + cb + j0)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
                    xs[j0] = x4.x;
                    xs[j0 + 1] = x4.y;
                    xs[j0 + 2] = x4.z;
                    xs[j0 + 3] = x4.w;
                }
                tmem_ld_wait();
                // two activation rows per instruction (f32x2).  int -> float is
                // exact for |v| < 2^22: the integer added to the bit pattern of
                // 1.5 * 2^23 lands in the mantissa and subtracting 1.5 * 2^23 is
                // exact (add pipe instead of the quarter-rate conversion unit);
                // then 256 hi + lo, scale, accumulate -- each element rounded as alone
                const float2 magic = make_float2(-12582912.0f, -12582912.0f);
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const float2 h = __fadd2_rn(make_float2(__int_as_float(static_cast<int>(hv[e]) + 0x4B400000),
                                                            __int_as_float(static_cast<int>(hv[e + 1]) + 0x4B400000)),
                                                magic);
                    const float2 l = __fadd2_rn(make_float2(__int_as_float(static_cast<int>(lv[e]) + 0x4B400000),
                                                            __int_as_float(static_cast<int>(lv[e + 1]) + 0x4B400000)),
                                                magic);
                    const float2 v = __ffma2_rn(h, make_float2(256.0f, 256.0f), l);
                    const float2 sc = __fmul2_rn(make_float2(wsc[b], wsc[b]), make_float2(xs[e], xs[e + 1]));
                    acc[e / 2] = __ffma2_rn(sc, v, acc[e / 2]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&x_empty[d]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
        }
        float sum[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sum[2 * j] = acc[j].x;
            sum[2 * j + 1] = acc[j].y;
        }
        bool last = true;
        if (p.ksplit > 1) {
            // partials of this K range out; the last CTA of the tile adds all ranges in split order
            const uint64_t mp = static_cast<uint64_t>(gridDim.y) * NT;
            float* mine = p.ws + static_cast<uint64_t>(blockIdx.z) * mp * p.n;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (static_cast<uint32_t>(j) < hc) mine[(t0 + cb + j) * static_cast<uint64_t>(p.n) + row] = sum[j];
            }
            __threadfence();
            named_bar_sync(2, kI8EpiWarps * 32);
            if (warp == 4 && lane == 0) {
                const uint32_t tk = atomicAdd(p.tickets + blockIdx.y * gridDim.x + blockIdx.x, 1u);
                last_cta = tk == p.ksplit - 1 ? 1u : 0u;
            }
            named_bar_sync(2, kI8EpiWarps * 32);
            last = last_cta != 0;
            if (last) {
                __threadfence();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (static_cast<uint32_t>(j) < hc) {
                        float v = 0.0f;
                        for (uint32_t z = 0; z < p.ksplit; ++z) {
                            const float pz = z == blockIdx.z ? sum[j]
                                                             : __ldcg(p.ws + static_cast<uint64_t>(z) * mp * p.n +
                                                                      (t0 + cb + j) * static_cast<uint64_t>(p.n) + row);
                            v = z == 0 ? pz : __fadd_rn(v, pz);
                        }
                        sum[j] = v;
                    }
                }
                if (warp == 4 && lane == 0) p.tickets[blockIdx.y * gridDim.x + blockIdx.x] = 0u;
            }
        }
        if (last) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (static_cast<uint32_t>(j) >= hc) continue;  // warp-uniform
                const uint32_t tok = t0 + cb + j;
                const float v = sum[j];
                if (EPI == kGemmStore) {
                    if (tok < p.m) p.y[static_cast<uint64_t>(tok) * p.ldy + row] = v;
                } else if (EPI == kGemmGeluSplit) {
                    // rows come as 8 gate + 8 up per 16-row group
                    const float up = __shfl_down_sync(0xffffffffu, v, 8);
                    if (tok < p.m && (lane & 8) == 0) {
                        p.act[static_cast<uint64_t>(tok) * p.ld_act + (row >> 4) * 8 + (lane & 7)] =
                            __fmul_rn(gelu_tanh(v), up);
                    }
                } else {
                    unsigned long long key = isnan(v) ? 0ull : argmax_key(v, p.row_base + row);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                        key = other > key ? other : key;
                    }
                    if (tok < p.m) {
                        if (p.y) p.y[static_cast<uint64_t>(tok) * p.ldy + row] = v;
                        if (lane == 0 && key != 0ull) atomicMax(p.keys + tok, key);
                    }
                }
            }
        }
    }
    __syncwarp();
    if (!ok) atomicOr(p.status, kStatusWaitTimeout);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, tcols);
    }
}

}  // namespace vrt
