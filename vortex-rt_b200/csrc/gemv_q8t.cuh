// Q8_0 x fp32 mat-vec over the tiled (Q8T) weight layout, sm_100a.
//
// One persistent CTA per SM owns a contiguous span of weight tiles.  Warp 8
// (the producer) streams the span through a 4-stage shared-memory ring with
// 1-D bulk copies (cp.async.bulk ... mbarrier::complete_tx), starting before
// griddepcontrol.wait so the weight stream overlaps the previous kernel's
// tail.  Warps 0-7 (consumers) first build the activation vector (the
// prologue: plain copy, RMSNorm, embedding + RMSNorm or residual + two
// RMSNorms, all with fp64 sums of squares like src/gemma3.cpp:948-1104),
// quantise it to int16 per 32-block, then each consumes one tile per stage:
// 16 dp2a per row pair give exact integer block sums, which are scaled by
// the weight's fp16 block scale and the activation block scale and summed in
// fp32.  Row results are reduced across lanes and warps in a fixed order
// (deterministic, replay-identical) and go to one of three epilogues:
//   Atomic   : y[row] += v into a zeroed buffer.  The span is tile-granular,
//              so at most two CTAs touch a row and the sum is order-free.
//   GeluPair : rows come as 8 gate + 8 up per group; act = gelu(g) * u.
//   Argmax   : logits (optional) + a 64-bit atomicMax key (ties -> lower
//              index, NaN skipped), the fused tied LM head + argmax.
#pragma once

#include "tp_exchange.cuh"
#include "vrt_device.cuh"

namespace vrt {

enum Pro : int { kProPlain = 0, kProRmsInto = 1, kProEmbed = 2, kProResid = 3, kProResidFinal = 4 };
enum Epi : int { kEpiAtomic = 0, kEpiGeluPair = 1, kEpiArgmax = 2 };

struct GemvParams {
    const uint8_t* w;      // tiled matrix
    uint32_t rows;         // output rows of the tiled matrix (GeluPair: 2 * ffn)
    uint32_t cols;         // K, multiple of 128
    const float* x;        // Plain: activations; RmsInto: residual; Resid*: block output to post-norm
    const float* h_prev;   // Resid*: residual stream in
    const float* w_post;   // Resid*: post-norm weight
    const float* w_pre;    // RmsInto/Embed/Resid: pre-norm weight; ResidFinal: output norm
    float* h_out;          // Embed/Resid: new residual (CTA 0); ResidFinal: normed hidden (CTA 0)
    float* trace;          // Resid*: optional copy of the new residual (CTA 0)
    const uint8_t* embd;   // Embed: tiled token_embd (cols = K)
    const uint32_t* token; // Embed: device token id
    uint32_t vocab;
    float emb_scale;
    float eps;
    float* y;                    // Atomic: output; GeluPair: act; Argmax: logits or null
    unsigned long long* amax;    // Argmax key
    uint32_t row_base;           // Argmax: global index of local row 0 (vocab shard)
    uint32_t* status;
    float* zero0;                // buffers this launch clears after griddepcontrol.wait
    uint32_t zero0_count;
    float* zero1;
    uint32_t zero1_count;
    uint32_t stage_cap;          // ring slots wanted (0 = as many as fit, up to 8)
    // L2 prefetch of the next mat-vec of the step: after issuing its own
    // copies, CTA b prefetches the first pf_bytes of CTA b's span in the
    // next kernel (same partition rule, next_group: group-granular spans).
    const uint8_t* next_w;
    uint32_t next_rows, next_cols, next_grid, next_group, pf_bytes;
    // Resid*: tensor-parallel exchange of the block output (tp.world > 1);
    // x then points at tp.sum, which this launch fills before its prologue.
    TpParams tp;
    uint32_t stamp;              // timing builds: this launch's stamp slot
};

// First tile of CTA b's span under the partition rule of the kernel below.
__host__ __device__ inline uint64_t gemv_span_start(uint32_t rows, uint32_t cols, uint32_t grid, uint32_t b,
                                                    bool group_granular) {
    const uint64_t kt = cols / kTileCols, groups = (rows + kTileRows - 1) / kTileRows;
    return group_granular ? groups * b / grid * kt : groups * kt * b / grid;
}

__device__ __forceinline__ void prefetch_next_span(const GemvParams& p) {
    if (!p.next_w || blockIdx.x >= p.next_grid) return;
    const uint64_t t0 = gemv_span_start(p.next_rows, p.next_cols, p.next_grid, blockIdx.x, p.next_group != 0);
    const uint64_t t1 = gemv_span_start(p.next_rows, p.next_cols, p.next_grid, blockIdx.x + 1, p.next_group != 0);
    uint64_t bytes = (t1 - t0) * kTileBytes;
    if (bytes > p.pf_bytes) bytes = p.pf_bytes;
    const uint8_t* src = p.next_w + t0 * kTileBytes;
    for (uint64_t off = 0; off < bytes; off += 32768) {
        const uint64_t n = bytes - off < 32768 ? bytes - off : 32768;
        bulk_prefetch_l2(src + off, static_cast<uint32_t>(n));
    }
}

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageTiles = kConsumerWarps;
constexpr int kStageBytes = kStageTiles * kTileBytes;  // 17408
constexpr int kMaxStages = 8;
constexpr uint32_t kSmemBudget = 200u * 1024u;
constexpr int kChunkGroups = 8;                        // rows reduced per chunk barrier = 128
constexpr int kPrologueVec = 6;                        // float4 per consumer thread: d <= 6144 in registers

struct GemvSmem {
    // byte offsets inside dynamic shared memory; `stages` ring slots at 0
    uint32_t n_stages, bars, partial, red, sx, x16, xs, total;
};

// The weight ring takes whatever the activation buffers leave of a 200 KB
// budget, up to 8 stages of 17 KB (139 KB in flight per SM).
__host__ __device__ inline GemvSmem gemv_smem_layout(uint32_t cols, int pro, uint32_t stage_cap = 0) {
    GemvSmem s;
    const uint32_t partial = 2 * kConsumerWarps * kChunkGroups * 16 * 4;
    const uint32_t vec = (cols / 32) * 4 + 16 + cols * 2 + 16 + ((pro == kProPlain) ? 0u : cols * 4u);
    const uint32_t fixed = 2 * kMaxStages * 8 + partial + 64 * 8 + vec;
    uint32_t ns = (kSmemBudget - fixed) / kStageBytes;
    const uint32_t cap = stage_cap ? stage_cap : static_cast<uint32_t>(kMaxStages);
    ns = ns < cap ? ns : cap;
    s.n_stages = ns > static_cast<uint32_t>(kMaxStages) ? static_cast<uint32_t>(kMaxStages) : (ns < 2 ? 2u : ns);
    s.bars = s.n_stages * kStageBytes;
    s.partial = s.bars + 2 * kMaxStages * 8;
    s.red = s.partial + partial;
    s.sx = s.red + 64 * 8;
    s.x16 = (s.sx + (cols / 32) * 4 + 15) / 16 * 16;
    s.xs = (s.x16 + cols * 2 + 15) / 16 * 16;
    s.total = s.xs + ((pro == kProPlain) ? 0u : cols * 4u);
    return s;
}

// 16 int8 weights . 16 int16 activations as two independent dp2a chains.
__device__ __forceinline__ int dot16(const uint4 w, const uint4 xl, const uint4 xh) {
    int a = __dp2a_lo(static_cast<int>(xl.x), static_cast<int>(w.x), 0);
    int b = __dp2a_lo(static_cast<int>(xh.x), static_cast<int>(w.z), 0);
    a = __dp2a_hi(static_cast<int>(xl.y), static_cast<int>(w.x), a);
    b = __dp2a_hi(static_cast<int>(xh.y), static_cast<int>(w.z), b);
    a = __dp2a_lo(static_cast<int>(xl.z), static_cast<int>(w.y), a);
    b = __dp2a_lo(static_cast<int>(xh.z), static_cast<int>(w.w), b);
    a = __dp2a_hi(static_cast<int>(xl.w), static_cast<int>(w.y), a);
    b = __dp2a_hi(static_cast<int>(xh.w), static_cast<int>(w.w), b);
    return a + b;
}

// Sum over the 256 consumer threads in fp64, fixed order; result broadcast.
__device__ __forceinline__ double consumer_sum(double v, double* red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    named_bar_sync(1, kConsumerWarps * 32);
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) s += red[w];
    named_bar_sync(1, kConsumerWarps * 32);
    return s;
}

// Quantise 32 consecutive activations (block `blk`) into the permuted int16
// layout + scale.
__device__ __forceinline__ void quant_block(const float* v, uint32_t blk, int16_t* x16p, float* sx) {
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
    const float s = quant_scale(amax);
    const float inv = amax > 0.0f ? 32767.0f / amax : 0.0f;
    sx[blk] = s;
    const uint32_t base = (blk / 4) * 128 + (blk % 4) * 8;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        uint32_t wv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int q0 = quant_one(v[p * 8 + 2 * e], inv), q1 = quant_one(v[p * 8 + 2 * e + 1], inv);
            wv[e] = (static_cast<uint32_t>(q0) & 0xffffu) | (static_cast<uint32_t>(q1) << 16);
        }
        *reinterpret_cast<uint4*>(x16p + base + p * 32) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
}

// The same quantisation spread over 8 threads per block: thread t8 = 0..7 of
// block blk holds elements 4*t8..4*t8+3 in v.  The block maximum is taken
// with fmaxf from 0 (exact in any order, NaN never wins), so the digits and
// the scale equal quant_block's.  All 32 lanes of the warp must call it
// (shuffles); `valid` is uniform over each aligned group of 8 lanes.
__device__ __forceinline__ void quant_block8(const float4 v, uint32_t blk, uint32_t t8, bool valid, int16_t* x16p,
                                             float* sx) {
    float amax = fmaxf(fmaxf(fmaxf(fmaxf(0.0f, fabsf(v.x)), fabsf(v.y)), fabsf(v.z)), fabsf(v.w));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    if (!valid) return;
    const float s = quant_scale(amax);
    const float inv = amax > 0.0f ? 32767.0f / amax : 0.0f;
    if (t8 == 0) sx[blk] = s;
    const uint32_t base = (blk / 4) * 128 + (blk % 4) * 8 + (t8 / 2) * 32 + (t8 % 2) * 4;
    const int q0 = quant_one(v.x, inv), q1 = quant_one(v.y, inv), q2 = quant_one(v.z, inv), q3 = quant_one(v.w, inv);
    *reinterpret_cast<uint2*>(x16p + base) =
        make_uint2((static_cast<uint32_t>(q0) & 0xffffu) | (static_cast<uint32_t>(q1) << 16),
                   (static_cast<uint32_t>(q2) & 0xffffu) | (static_cast<uint32_t>(q3) << 16));
}

// Prologue helper for the norm modes: every consumer thread holds up to
// kPrologueVec float4 of each input vector in registers, loaded in one round
// trip; returns x (the activation to quantise) in xs[] (shared, fp32).
template <int PRO>
__device__ __forceinline__ void norm_prologue(const GemvParams& p, float* xs, double* red, int ctid) {
    constexpr int NC = kConsumerWarps * 32;
    const uint32_t K = p.cols, n4 = K / 4;
    const float4* x4 = reinterpret_cast<const float4*>(p.x);
    const float4* h4 = reinterpret_cast<const float4*>(p.h_prev);
    const float4* wp4 = reinterpret_cast<const float4*>(p.w_post);
    const float4* wq4 = reinterpret_cast<const float4*>(p.w_pre);
    float4 a[kPrologueVec], b[kPrologueVec], c[kPrologueVec], w[kPrologueVec];
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const bool l2_only = p.tp.world > 1;  // x written by other CTAs of this grid
#pragma unroll
    for (int u = 0; u < kPrologueVec; ++u) {
        const uint32_t i = ctid + u * NC;
        const bool ok = i < n4;
        a[u] = ok ? (l2_only ? __ldcg(x4 + i) : x4[i]) : z;
        w[u] = ok ? wq4[i] : z;
        if (PRO != kProRmsInto) {
            b[u] = ok ? h4[i] : z;
            c[u] = ok ? wp4[i] : z;
        }
    }
    auto sq = [](const float4& v) {
        return static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
               static_cast<double>(v.w) * v.w;
    };
    if (PRO != kProRmsInto) {
        double so = 0.0;
#pragma unroll
        for (int u = 0; u < kPrologueVec; ++u) so += sq(a[u]);
        so = consumer_sum(so, red);
        const float ps = 1.0f / sqrtf(static_cast<float>(so / static_cast<double>(K)) + p.eps);
        bool bad = false;
#pragma unroll
        for (int u = 0; u < kPrologueVec; ++u) {
            // rms_norm_inplace(block output, post norm) then += residual
            float4 h;
            h.x = __fadd_rn(__fmul_rn(a[u].x, __fmul_rn(ps, c[u].x)), b[u].x);
            h.y = __fadd_rn(__fmul_rn(a[u].y, __fmul_rn(ps, c[u].y)), b[u].y);
            h.z = __fadd_rn(__fmul_rn(a[u].z, __fmul_rn(ps, c[u].z)), b[u].z);
            h.w = __fadd_rn(__fmul_rn(a[u].w, __fmul_rn(ps, c[u].w)), b[u].w);
            a[u] = h;
            const uint32_t i = ctid + u * NC;
            if (i < n4) {
                bad |= !(isfinite(h.x) && isfinite(h.y) && isfinite(h.z) && isfinite(h.w));
                if (blockIdx.x == 0) {
                    if (PRO == kProResid) reinterpret_cast<float4*>(p.h_out)[i] = h;
                    if (p.trace) reinterpret_cast<float4*>(p.trace)[i] = h;
                }
            }
        }
        if (bad && blockIdx.x == 0) atomicOr(p.status, kStatusNonFinite);
    }
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < kPrologueVec; ++u) ss += sq(a[u]);
    ss = consumer_sum(ss, red);
    const float sc = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(K)) + p.eps);
#pragma unroll
    for (int u = 0; u < kPrologueVec; ++u) {
        const uint32_t i = ctid + u * NC;
        if (i >= n4) continue;
        float4 v;
        if (PRO == kProResidFinal) {  // rms_norm_inplace: x * (scale * w)
            v.x = __fmul_rn(a[u].x, __fmul_rn(sc, w[u].x));
            v.y = __fmul_rn(a[u].y, __fmul_rn(sc, w[u].y));
            v.z = __fmul_rn(a[u].z, __fmul_rn(sc, w[u].z));
            v.w = __fmul_rn(a[u].w, __fmul_rn(sc, w[u].w));
            if (blockIdx.x == 0) reinterpret_cast<float4*>(p.h_out)[i] = v;
        } else {                       // rms_norm_into: (x * scale) * w
            v.x = __fmul_rn(__fmul_rn(a[u].x, sc), w[u].x);
            v.y = __fmul_rn(__fmul_rn(a[u].y, sc), w[u].y);
            v.z = __fmul_rn(__fmul_rn(a[u].z, sc), w[u].z);
            v.w = __fmul_rn(__fmul_rn(a[u].w, sc), w[u].w);
        }
        reinterpret_cast<float4*>(xs)[i] = v;
    }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) q8t_gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvSmem L = gemv_smem_layout(p.cols, PRO, p.stage_cap);
    const uint32_t NS = L.n_stages;
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + kMaxStages;
    float* partial = reinterpret_cast<float*>(smem + L.partial);
    double* red = reinterpret_cast<double*>(smem + L.red);
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    int16_t* x16p = reinterpret_cast<int16_t*>(smem + L.x16);
    float* xs = reinterpret_cast<float*>(smem + L.xs);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) chain_stamp(p.stamp, 0);
    ChainStampEnd stamp_end{p.stamp, tid == 0};
    const uint32_t kt = p.cols / kTileCols;
    const uint32_t n_groups = (p.rows + kTileRows - 1) / kTileRows;
    uint64_t T0, T1;
    if (EPI == kEpiAtomic) {
        const uint64_t total = static_cast<uint64_t>(n_groups) * kt;
        T0 = total * blockIdx.x / gridDim.x;
        T1 = total * (blockIdx.x + 1) / gridDim.x;
    } else {
        T0 = static_cast<uint64_t>(n_groups) * blockIdx.x / gridDim.x * kt;
        T1 = static_cast<uint64_t>(n_groups) * (blockIdx.x + 1) / gridDim.x * kt;
    }
    const uint32_t n_tiles = static_cast<uint32_t>(T1 - T0);
    const uint32_t n_stages = (n_tiles + kStageTiles - 1) / kStageTiles;

    if (tid == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kConsumerWarps) {
        // ----------------------------------------------------- producer
        if (lane == 0) {
            const uint8_t* src = p.w + T0 * kTileBytes;
            const uint64_t pol = l2_policy_evict_first();
            uint32_t s = 0, r = 0;
            for (uint32_t st = 0; st < n_stages; ++st) {
                if (r > 0 && !mbar_wait_bounded(&empty[s], (r - 1) & 1)) atomicOr(p.status, kStatusWaitTimeout);
                const uint32_t tiles = min(static_cast<uint32_t>(kStageTiles), n_tiles - st * kStageTiles);
                const uint32_t bytes = tiles * kTileBytes;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_copy_g2s_hint(stages + s * kStageBytes, src + static_cast<uint64_t>(st) * kStageBytes, bytes,
                                   &full[s], pol);
                if (++s == NS) {
                    s = 0;
                    ++r;
                }
            }
            prefetch_next_span(p);
        }
        return;
    }

    // --------------------------------------------------------- consumers
    pdl_wait();
    if (tid == 0) {
        chain_stamp(p.stamp, 1);
        chain_stamp(p.stamp, 2);
    }
    const int ctid = tid;  // 0..255
    constexpr int NC = kConsumerWarps * 32;
    if (p.zero0) {
        const uint32_t a = static_cast<uint64_t>(p.zero0_count) * blockIdx.x / gridDim.x;
        const uint32_t b = static_cast<uint64_t>(p.zero0_count) * (blockIdx.x + 1) / gridDim.x;
        for (uint32_t i = a + ctid; i < b; i += NC) p.zero0[i] = 0.0f;
    }
    if (p.zero1) {
        const uint32_t a = static_cast<uint64_t>(p.zero1_count) * blockIdx.x / gridDim.x;
        const uint32_t b = static_cast<uint64_t>(p.zero1_count) * (blockIdx.x + 1) / gridDim.x;
        for (uint32_t i = a + ctid; i < b; i += NC) p.zero1[i] = 0.0f;
    }
    for (int i = ctid; i < 2 * kConsumerWarps * kChunkGroups * 16; i += NC) partial[i] = 0.0f;

    if (PRO == kProResid || PRO == kProResidFinal) {
        if (p.tp.world > 1) {
            // sum the ranks' partials of the block output: this CTA's slice,
            // then a grid barrier so every CTA can read the whole vector
            const uint32_t seq = tp_seq(p.tp);
            const uint32_t a = static_cast<uint64_t>(p.tp.n) * blockIdx.x / gridDim.x;
            const uint32_t e = static_cast<uint64_t>(p.tp.n) * (blockIdx.x + 1) / gridDim.x;
            tp_slice_reduce(p.tp, seq, a, e, ctid, NC, p.status);
            named_bar_sync(1, NC);
            if (ctid == 0) tp_grid_barrier(p.tp, seq, p.status);
            named_bar_sync(1, NC);
            if (ctid == 0) chain_stamp(p.stamp, 3);
        }
    }

    const uint32_t K = p.cols, nblk = K / 32;
    if (PRO == kProPlain && nblk * 8 <= 3 * NC) {
        // short vectors: 8 threads per block, coalesced float4 loads, all in flight at once
        const float4* x4 = reinterpret_cast<const float4*>(p.x);
        float4 f[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const uint32_t i = ctid + r * NC;
            f[r] = i < nblk * 8 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const uint32_t i = ctid + r * NC;
            quant_block8(f[r], i / 8, i % 8, i < nblk * 8, x16p, sx);
        }
    } else if (PRO == kProPlain) {
        // blocks of 32 activations: all loads of a thread issued before use
        for (uint32_t b0 = 0; b0 < nblk; b0 += 3 * NC) {
            float4 f[3][8];
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const uint32_t blk = b0 + ctid + q * NC;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    f[q][e] = blk < nblk ? reinterpret_cast<const float4*>(p.x + blk * 32)[e]
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const uint32_t blk = b0 + ctid + q * NC;
                if (blk < nblk) quant_block(reinterpret_cast<const float*>(f[q]), blk, x16p, sx);
            }
        }
    } else {
        if (PRO == kProEmbed) {
            double ss = 0.0;
            uint32_t tok = *p.token;
            if (tok >= p.vocab) {
                if (ctid == 0 && blockIdx.x == 0) atomicOr(p.status, kStatusBadToken);
                tok = 0;
            }
            for (uint32_t k = ctid; k < K; k += NC) {
                const int8_t q = static_cast<int8_t>(p.embd[q8t_weight_offset(tok, k, K)]);
                const uint64_t so = q8t_scale_offset(tok, k / 32, K);
                const float sc = half_bits_to_float(p.embd[so] | (static_cast<uint32_t>(p.embd[so + 1]) << 8));
                const float h = __fmul_rn(__fmul_rn(sc, static_cast<float>(q)), p.emb_scale);
                xs[k] = h;
                ss += static_cast<double>(h) * static_cast<double>(h);
                if (blockIdx.x == 0) p.h_out[k] = h;
            }
            ss = consumer_sum(ss, red);
            const float scale = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(K)) + p.eps);
            for (uint32_t k = ctid; k < K; k += NC) xs[k] = __fmul_rn(__fmul_rn(xs[k], scale), p.w_pre[k]);
        } else if (K <= kPrologueVec * 4 * NC) {
            norm_prologue<PRO>(p, xs, red, ctid);
        } else {
            // wide vectors (not used by Gemma 3 shapes): looped form
            double so = 0.0;
            float ps = 1.0f;
            if (PRO != kProRmsInto) {
                for (uint32_t k = ctid; k < K; k += NC) so += static_cast<double>(__ldcg(p.x + k)) * __ldcg(p.x + k);
                so = consumer_sum(so, red);
                ps = 1.0f / sqrtf(static_cast<float>(so / static_cast<double>(K)) + p.eps);
            }
            double ss = 0.0;
            for (uint32_t k = ctid; k < K; k += NC) {
                const float xk = __ldcg(p.x + k);
                const float h = PRO == kProRmsInto ? xk : __fadd_rn(__fmul_rn(xk, __fmul_rn(ps, p.w_post[k])), p.h_prev[k]);
                xs[k] = h;
                ss += static_cast<double>(h) * h;
                if (PRO != kProRmsInto && blockIdx.x == 0) {
                    if (PRO == kProResid) p.h_out[k] = h;
                    if (p.trace) p.trace[k] = h;
                }
            }
            ss = consumer_sum(ss, red);
            const float sc = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(K)) + p.eps);
            for (uint32_t k = ctid; k < K; k += NC) {
                const float v = PRO == kProResidFinal ? __fmul_rn(xs[k], __fmul_rn(sc, p.w_pre[k]))
                                                      : __fmul_rn(__fmul_rn(xs[k], sc), p.w_pre[k]);
                xs[k] = v;
                if (PRO == kProResidFinal && blockIdx.x == 0) p.h_out[k] = v;
            }
        }
        named_bar_sync(1, NC);
        if (nblk * 8 <= 2 * NC) {  // short vectors: 8 threads per block
            const float4* xs4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint32_t i = ctid + r * NC;
                const bool ok = i < nblk * 8;
                quant_block8(ok ? xs4[i] : make_float4(0.f, 0.f, 0.f, 0.f), i / 8, i % 8, ok, x16p, sx);
            }
        } else {
            for (uint32_t blk = ctid; blk < nblk; blk += NC) quant_block(xs + blk * 32, blk, x16p, sx);
        }
    }
    named_bar_sync(1, NC);
    if (ctid == 0) chain_stamp(p.stamp, 4);

    // ------------------------------------------------------- main loop
    const uint32_t g_first = static_cast<uint32_t>(T0 / kt);
    const uint32_t n_chunks = n_tiles ? (static_cast<uint32_t>((T1 - 1) / kt) - g_first) / kChunkGroups + 1 : 0;
    const int quad = lane & 3;
    int cur_g = -1;
    float acc0 = 0.0f, acc1 = 0.0f;
    uint32_t chunks_done = 0;
    unsigned long long best = 0ull;  // Argmax: lane 0 of each warp

    auto flush = [&](int g) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        const uint32_t rel = static_cast<uint32_t>(g) - g_first;
        float* part = partial + ((rel / kChunkGroups) & 1) * (kConsumerWarps * kChunkGroups * 16) +
                      warp * (kChunkGroups * 16) + (rel % kChunkGroups) * 16 + 2 * (lane >> 2);
        if (quad == 0) {
            part[0] = acc0;
            part[1] = acc1;
        }
        acc0 = 0.0f;
        acc1 = 0.0f;
    };

    auto chunk_end = [&](uint32_t c) {
        named_bar_sync(1, NC);
        const uint32_t rel = c * kChunkGroups + warp;
        const uint32_t g = g_first + rel;
        const bool live = (static_cast<uint64_t>(g) * kt < T1) && ((static_cast<uint64_t>(g) + 1) * kt > T0);
        if (!live) return;
        float* part = partial + (c & 1) * (kConsumerWarps * kChunkGroups * 16) + warp * 16;
        float v = 0.0f;
        if (lane < 16) {
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                v += part[w * (kChunkGroups * 16) + lane];
                part[w * (kChunkGroups * 16) + lane] = 0.0f;
            }
        }
        const uint32_t row = g * kTileRows + lane;
        if (EPI == kEpiAtomic) {
            if (lane < 16 && row < p.rows) atomicAdd(p.y + row, v);
        } else if (EPI == kEpiGeluPair) {
            const float up = __shfl_down_sync(0xffffffffu, v, 8);
            const uint32_t o = g * 8 + lane;
            if (lane < 8 && o < p.rows / 2) p.y[o] = __fmul_rn(gelu_tanh(v), up);
        } else {
            unsigned long long key = 0ull;
            if (lane < 16 && row < p.rows) {
                if (p.y) p.y[row] = v;
                if (!isnan(v)) key = argmax_key(v, p.row_base + row);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other > key ? other : key;
            }
            best = key > best ? key : best;
        }
    };

    // this warp's tiles are T0 + warp + 8*st; walk (group, column tile) incrementally
    uint32_t g = static_cast<uint32_t>((T0 + warp) / kt), j = static_cast<uint32_t>((T0 + warp) % kt);
    uint32_t s = 0, ph = 0;
    for (uint32_t st = 0; st < n_stages; ++st) {
        if (!mbar_wait_bounded(&full[s], ph) && lane == 0) atomicOr(p.status, kStatusWaitTimeout);
        if (T0 + static_cast<uint64_t>(st) * kStageTiles + warp < T1) {
            if (static_cast<int>(g) != cur_g && cur_g >= 0) flush(cur_g);
            const uint32_t c = (g - g_first) / kChunkGroups;
            while (chunks_done < c) chunk_end(chunks_done++);
            cur_g = static_cast<int>(g);
            const uint8_t* tile = stages + s * kStageBytes + warp * kTileBytes;
            const uint4* tq = reinterpret_cast<const uint4*>(tile);
            const uint4 w0 = tq[lane], w1 = tq[32 + lane], w2 = tq[64 + lane], w3 = tq[96 + lane];
            const uint32_t sc = reinterpret_cast<const uint32_t*>(tile + kTileQBytes)[lane];
            const uint4* xp = reinterpret_cast<const uint4*>(x16p + j * 128);
            const uint4 xa = xp[quad], xb = xp[4 + quad], xc = xp[8 + quad], xd = xp[12 + quad];
            const int s0 = dot16(w0, xa, xb) + dot16(w1, xc, xd);
            const int s1 = dot16(w2, xa, xb) + dot16(w3, xc, xd);
            const float sxb = sx[j * 4 + quad];
            acc0 += __fmul_rn(half_bits_to_float(sc & 0xffffu), sxb) * static_cast<float>(s0);
            acc1 += __fmul_rn(half_bits_to_float(sc >> 16), sxb) * static_cast<float>(s1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        j += kStageTiles;
        while (j >= kt) {
            j -= kt;
            ++g;
        }
        if (++s == NS) {
            s = 0;
            ph ^= 1u;
        }
    }
    if (cur_g >= 0) flush(cur_g);
    while (chunks_done < n_chunks) chunk_end(chunks_done++);

    if (EPI == kEpiArgmax) {
        unsigned long long* keys = reinterpret_cast<unsigned long long*>(red);
        named_bar_sync(1, NC);
        if (lane == 0) keys[warp] = best;
        named_bar_sync(1, NC);
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < kConsumerWarps; ++w) b = keys[w] > b ? keys[w] : b;
            if (b) atomicMax(p.amax, b);
        }
    }
}

}  // namespace vrt
