// Batched prefill of one sequence: a chunk of n prompt tokens at positions
// p0 .. p0+n-1 goes through each layer at once, the projections as
// tensor-core GEMMs (gemm_q8t.cuh) and the rest as the row kernels below.
// The arithmetic of every row kernel is the decode path's, row by row: the
// same fp64 sums of squares and rounding order as the mat-vec prologues
// (gemv_q8t.cuh norm_prologue, src/gemma3.cpp:948-1104), the same per-head
// RMSNorm + NeoX RoPE (attention.cuh head_norm_rope, gemma3.cpp:1309-1424),
// and attention as an fp32 online softmax like the decode kernel.  The
// reference itself prefills token by token through decode_token
// (gemma3.cpp:2080-2149); the results agree within the north-star tolerance.
#pragma once

#include <cuda_fp16.h>

#include "attention.cuh"
#include "gemm_i8.cuh"
#include "vrt_device.cuh"

namespace vrt {

constexpr int kRowThreads = 256;
constexpr int kRowMaxPerThread = 24;  // d <= 6144

__device__ __forceinline__ double block_sum_f64(double v, double* red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    for (int w = 0; w < kRowThreads / 32; ++w) s += red[w];
    return s;
}

__device__ __forceinline__ void store_split(__half* hi, __half* lo, uint64_t i, float v) {
    __half h, l;
    split_f16(v, h, l);
    hi[i] = h;
    lo[i] = l;
}

// The GEMM operand a row kernel writes: fp16 hi / lo terms (x_hi / x_lo,
// when set) and/or the int16 split halves of the integer GEMM (q.hi, when
// set; d % 32 == 0, so each warp holds whole 32-blocks).
// Row m = token m of the chunk: h = token_embd[tok] * sqrt(d) -> h_out;
// x = rms_norm_into(h, w_pre) -> x_hi / x_lo (the embedding prologue).
__global__ void __launch_bounds__(kRowThreads) embed_rows_kernel(const uint8_t* embd, const uint32_t* tokens,
                                                                 uint32_t vocab, uint32_t d, float emb_scale,
                                                                 const float* w_pre, float eps, float* h_out,
                                                                 __half* x_hi, __half* x_lo, const Q16Out q,
                                                                 uint32_t* status) {
    __shared__ double red[kRowThreads / 32];
    const uint32_t m = blockIdx.x;
    uint32_t tok = tokens[m];
    if (tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(status, kStatusBadToken);
        tok = 0;
    }
    float h[kRowMaxPerThread];
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        h[u] = 0.0f;
        if (k < d) {
            const int8_t q = static_cast<int8_t>(embd[q8t_weight_offset(tok, k, d)]);
            const uint64_t so = q8t_scale_offset(tok, k / 32, d);
            const float sc = half_bits_to_float(embd[so] | (static_cast<uint32_t>(embd[so + 1]) << 8));
            h[u] = __fmul_rn(__fmul_rn(sc, static_cast<float>(q)), emb_scale);
            ss += static_cast<double>(h[u]) * static_cast<double>(h[u]);
            h_out[static_cast<uint64_t>(m) * d + k] = h[u];
        }
    }
    ss = block_sum_f64(ss, red);
    const float scale = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(d)) + eps);
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        if (k < d) {
            const float v = __fmul_rn(__fmul_rn(h[u], scale), w_pre[k]);
            if (x_hi) store_split(x_hi, x_lo, static_cast<uint64_t>(m) * d + k, v);
            if (q.hi) warp_q16_store(q, m, k, v);
        }
    }
}

// Row m: h = rms_norm_inplace(y, w_post) + h_prev -> h_out (the residual
// update after a block), x = rms_norm_into(h, w_pre) -> x_hi / x_lo.
__global__ void __launch_bounds__(kRowThreads) resid_rows_kernel(const float* y, const float* h_prev,
                                                                 const float* w_post, const float* w_pre, float eps,
                                                                 uint32_t d, float* h_out, __half* x_hi, __half* x_lo,
                                                                 const Q16Out q, uint32_t* status) {
    __shared__ double red[kRowThreads / 32];
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * d;
    float a[kRowMaxPerThread];
    double so = 0.0;
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        a[u] = k < d ? y[base + k] : 0.0f;
        so += static_cast<double>(a[u]) * static_cast<double>(a[u]);
    }
    so = block_sum_f64(so, red);
    const float ps = 1.0f / sqrtf(static_cast<float>(so / static_cast<double>(d)) + eps);
    double ss = 0.0;
    bool bad = false;
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        if (k < d) {
            const float h = __fadd_rn(__fmul_rn(a[u], __fmul_rn(ps, w_post[k])), h_prev[base + k]);
            a[u] = h;
            bad |= !isfinite(h);
            h_out[base + k] = h;
            ss += static_cast<double>(h) * static_cast<double>(h);
        }
    }
    if (bad) atomicOr(status, kStatusNonFinite);
    ss = block_sum_f64(ss, red);
    const float sc = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(d)) + eps);
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        if (k < d) {
            const float v = __fmul_rn(__fmul_rn(a[u], sc), w_pre[k]);
            if (x_hi) store_split(x_hi, x_lo, base + k, v);
            if (q.hi) warp_q16_store(q, blockIdx.x, k, v);
        }
    }
}

// Row m: h = rms_norm_inplace(y, w_post) + h_prev, then the output norm in
// the rms_norm_inplace form x * (scale * w) (the LM-head prologue) ->
// hidden (fp32) and x_hi / x_lo (the LM-head GEMM operand).
__global__ void __launch_bounds__(kRowThreads) final_rows_kernel(const float* y, const float* h_prev,
                                                                 const float* w_post, const float* w_out, float eps,
                                                                 uint32_t d, float* hidden, __half* x_hi, __half* x_lo,
                                                                 const Q16Out q, uint32_t* status) {
    __shared__ double red[kRowThreads / 32];
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * d;
    float a[kRowMaxPerThread];
    double so = 0.0;
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        a[u] = k < d ? y[base + k] : 0.0f;
        so += static_cast<double>(a[u]) * static_cast<double>(a[u]);
    }
    so = block_sum_f64(so, red);
    const float ps = 1.0f / sqrtf(static_cast<float>(so / static_cast<double>(d)) + eps);
    double ss = 0.0;
    bool bad = false;
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        if (k < d) {
            const float h = __fadd_rn(__fmul_rn(a[u], __fmul_rn(ps, w_post[k])), h_prev[base + k]);
            a[u] = h;
            bad |= !isfinite(h);
            ss += static_cast<double>(h) * static_cast<double>(h);
        }
    }
    if (bad) atomicOr(status, kStatusNonFinite);
    ss = block_sum_f64(ss, red);
    const float sc = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(d)) + eps);
#pragma unroll
    for (int u = 0; u < kRowMaxPerThread; ++u) {
        const uint32_t k = threadIdx.x + u * kRowThreads;
        if (k < d) {
            const float v = __fmul_rn(a[u], __fmul_rn(sc, w_out[k]));
            hidden[base + k] = v;
            if (x_hi) store_split(x_hi, x_lo, base + k, v);
            if (q.hi) warp_q16_store(q, blockIdx.x, k, v);
        }
    }
}

// Batched decode: per sequence s < count, the LM-head argmax key -> next
// token, position + 1, generated id appended (ring of out_cap per sequence).
// With `first` set (after a prefill of n tokens) the position becomes n.
__global__ void batch_finalize_kernel(unsigned long long* keys, uint32_t* tokens, uint32_t* pos, uint32_t* out_ids,
                                      uint32_t* out_count, uint32_t out_cap, uint32_t s0, uint32_t count,
                                      uint32_t vocab, uint32_t first_pos, uint32_t* status) {
    const uint32_t s = s0 + blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= s0 + count) return;
    uint32_t idx;
    float val;
    argmax_unkey(keys[s], &idx, &val);
    keys[s] = 0ull;
    if (idx >= vocab || !isfinite(val)) atomicOr(status, kStatusNonFinite);
    const uint32_t c = first_pos ? 0u : out_count[s];
    if (c < out_cap) out_ids[static_cast<uint64_t>(s) * out_cap + c] = idx;
    out_count[s] = c + 1;
    tokens[s] = idx < vocab ? idx : 0u;
    pos[s] = first_pos ? first_pos : pos[s] + 1;
}

// Token m of the chunk (position p0 + m): q heads and k heads -> per-head
// RMSNorm + RoPE -> q [n][H][hd], k [n][KV][hd]; v copied to v [n][KV][hd].
template <int M>
__global__ void qk_rope_rows_kernel(const float* qkv, uint32_t H, uint32_t KV, const float* q_norm,
                                    const float* k_norm, const float* rope_cos, const float* rope_sin, uint32_t p0,
                                    float eps, float* q, float* k, float* v) {
    constexpr uint32_t HD = M * 32;
    const uint32_t m = blockIdx.x, pos = p0 + m;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const float* row = qkv + static_cast<uint64_t>(m) * (H + 2 * KV) * HD;
    const float* cs = rope_cos + static_cast<uint64_t>(pos) * (HD / 2);
    const float* sn = rope_sin + static_cast<uint64_t>(pos) * (HD / 2);
    for (uint32_t h = warp; h < H + KV; h += nw) {
        float x[M];
#pragma unroll
        for (int i = 0; i < M; ++i) x[i] = row[h * HD + lane + 32 * i];
        head_norm_rope<M>(x, h < H ? q_norm : k_norm, cs, sn, HD, eps, lane);
        float* dst = h < H ? q + (static_cast<uint64_t>(m) * H + h) * HD : k + (static_cast<uint64_t>(m) * KV + (h - H)) * HD;
#pragma unroll
        for (int i = 0; i < M; ++i) dst[lane + 32 * i] = x[i];
        if (h >= H) {
            const float* vs = row + (H + KV + (h - H)) * HD;
            float* vd = v + (static_cast<uint64_t>(m) * KV + (h - H)) * HD;
#pragma unroll
            for (int i = 0; i < M; ++i) vd[lane + 32 * i] = vs[lane + 32 * i];
        }
    }
}

// Chunk K/V -> cache slots (position % cap).  A sliding layer keeps only the
// chunk's last `cap` positions (earlier ones would be overwritten anyway).
__global__ void kv_store_kernel(const float* k, const float* v, float* k_cache, float* v_cache, uint32_t cap,
                                uint32_t KV, uint32_t hd, uint32_t p0, uint32_t n) {
    const uint32_t m = blockIdx.x, g = blockIdx.y, pos = p0 + m;
    if (m + cap < n) return;
    const uint64_t src = (static_cast<uint64_t>(m) * KV + g) * hd;
    const uint64_t dst = (static_cast<uint64_t>(g) * cap + pos % cap) * hd;
    for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
        k_cache[dst + i] = k[src + i];
        v_cache[dst + i] = v[src + i];
    }
}

// ------------------------------------------------------ prefill attention
//
// CTA = (block of QB = 64/G query tokens, KV head g): its 64 rows are
// (token i, head j of the group), row r = i*G + j, query head g*G + j.  Keys
// walk in tiles of 64 positions from the oldest one any row may see; a key at
// position t comes from the cache (slot t % cap) when t < p0 and from the
// chunk's own K/V otherwise (the chunk is written to the cache only after
// this kernel).  Per tile: scores (each thread a 4x4 block of rows x keys
// over head_dim), row max / exp / sums by shuffles among the 16 threads of a
// row group, P through shared memory, then P.V (each thread 4 rows x HD/16
// columns, interleaved at a 64-column stride so a warp's float4 reads of a
// value row are contiguous).  Masked: t > position of the row's token, or t <= position -
// window on sliding layers.
struct PrefillAttnParams {
    const float* q;        // [n][H][hd]
    const float* k;        // [n][KV][hd] chunk keys (normed, roped)
    const float* v;        // [n][KV][hd]
    const float* k_cache;  // [KV][cap][hd]
    const float* v_cache;
    uint32_t cap, window;  // window 0 = global layer
    uint32_t p0, n, H, KV;
    float scale;
    __half* out_hi;        // [n][H*hd] (o-projection operand)
    __half* out_lo;
};

constexpr int kPaRows = 64, kPaKeys = 64, kPaThreads = 256, kPaPad = 4;

template <int HD>
constexpr uint32_t prefill_attn_smem() {
    return (HD * kPaRows + HD * (kPaKeys + kPaPad) + kPaKeys * (HD + kPaPad) + kPaKeys * (kPaRows + kPaPad) +
            3 * kPaRows) * 4;
}

template <int HD, int G>
__global__ void __launch_bounds__(kPaThreads, 1) prefill_attention_kernel(const PrefillAttnParams p) {
    constexpr int QB = kPaRows / G;
    constexpr int CW = HD / 16;  // P.V columns per thread
    extern __shared__ __align__(16) float pa_sm[];
    float* qt = pa_sm;                                  // [HD][64]      q transposed
    float* kt = qt + HD * kPaRows;                      // [HD][64+4]    key tile transposed
    float* vs = kt + HD * (kPaKeys + kPaPad);           // [64][HD+4]    value tile
    float* pt = vs + kPaKeys * (HD + kPaPad);           // [64][64+4]    probabilities, [key][row]
    float* m_s = pt + kPaKeys * (kPaRows + kPaPad);     // [64] running max
    float* l_s = m_s + kPaRows;                         // [64] running sum
    float* c_s = l_s + kPaRows;                         // [64] rescale of this tile

    const int tid = threadIdx.x;
    // heaviest (latest) query blocks first
    const uint32_t nqb = (p.n + QB - 1) / QB;
    const uint32_t qb = nqb - 1 - blockIdx.x, g = blockIdx.y;
    const uint32_t i0 = qb * QB, nq = min(static_cast<uint32_t>(QB), p.n - i0);
    const uint32_t P0 = p.p0 + i0, P1 = p.p0 + i0 + nq - 1;  // first / last query position
    const uint32_t lo = p.window ? (P0 + 1 > p.window ? P0 + 1 - p.window : 0u) : 0u;

    // lanes walk rows: conflict-free transposed stores, one float4 of a row per thread
    for (int idx = tid; idx < kPaRows * (HD / 4); idx += kPaThreads) {
        const int r = idx % kPaRows, d4 = idx / kPaRows;
        const uint32_t i = r / G, j = r % G;
        float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < nq) v4 = reinterpret_cast<const float4*>(p.q + ((static_cast<uint64_t>(i0 + i)) * p.H + g * G + j) * HD)[d4];
        qt[(4 * d4 + 0) * kPaRows + r] = v4.x;
        qt[(4 * d4 + 1) * kPaRows + r] = v4.y;
        qt[(4 * d4 + 2) * kPaRows + r] = v4.z;
        qt[(4 * d4 + 3) * kPaRows + r] = v4.w;
    }
    if (tid < kPaRows) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.0f;
    }
    const int rg = tid >> 4, kg = tid & 15;  // score block: rows 4rg.., keys 4kg..
    float acc[4][CW];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < CW; ++c) acc[a][c] = 0.0f;

    for (uint32_t t0 = lo; t0 <= P1; t0 += kPaKeys) {
        __syncthreads();  // previous tile's K/V/P fully consumed
        for (int idx = tid; idx < kPaKeys * (HD / 4); idx += kPaThreads) {
            const int kk = idx % kPaKeys, d4 = idx / kPaKeys;  // lanes walk keys
            const uint32_t t = t0 + kk;
            float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
            if (t <= P1) {
                const float* ks;
                const float* vsrc;
                if (t < p.p0) {
                    const uint64_t o = (static_cast<uint64_t>(g) * p.cap + t % p.cap) * HD;
                    ks = p.k_cache + o;
                    vsrc = p.v_cache + o;
                } else {
                    const uint64_t o = (static_cast<uint64_t>(t - p.p0) * p.KV + g) * HD;
                    ks = p.k + o;
                    vsrc = p.v + o;
                }
                kv4 = reinterpret_cast<const float4*>(ks)[d4];
                vv4 = reinterpret_cast<const float4*>(vsrc)[d4];
            }
            kt[(4 * d4 + 0) * (kPaKeys + kPaPad) + kk] = kv4.x;
            kt[(4 * d4 + 1) * (kPaKeys + kPaPad) + kk] = kv4.y;
            kt[(4 * d4 + 2) * (kPaKeys + kPaPad) + kk] = kv4.z;
            kt[(4 * d4 + 3) * (kPaKeys + kPaPad) + kk] = kv4.w;
            *reinterpret_cast<float4*>(vs + kk * (HD + kPaPad) + 4 * d4) = vv4;
        }
        __syncthreads();
        // scores
        float s[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) s[a][b] = 0.0f;
#pragma unroll 4
        for (int dd = 0; dd < HD; ++dd) {
            const float4 qv = *reinterpret_cast<const float4*>(qt + dd * kPaRows + 4 * rg);
            const float4 kv = *reinterpret_cast<const float4*>(kt + dd * (kPaKeys + kPaPad) + 4 * kg);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, kb[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) s[a][b] = fmaf(qa[a], kb[b], s[a][b]);
        }
        float tmax[4], mold[4], mnew[4], tsum[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const uint32_t r = 4 * rg + a, i = r / G;
            const uint32_t pos = P0 + i;
            tmax[a] = -INFINITY;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint32_t t = t0 + 4 * kg + b;
                const bool ok = i < nq && t <= pos && (!p.window || t + p.window > pos);
                s[a][b] = ok ? s[a][b] * p.scale : -INFINITY;
                tmax[a] = fmaxf(tmax[a], s[a][b]);
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) tmax[a] = fmaxf(tmax[a], __shfl_xor_sync(0xffffffffu, tmax[a], o));
            mold[a] = m_s[r];
            mnew[a] = fmaxf(mold[a], tmax[a]);
            tsum[a] = 0.0f;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const float pr = s[a][b] == -INFINITY ? 0.0f : expf(s[a][b] - mnew[a]);
                s[a][b] = pr;
                tsum[a] += pr;
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) tsum[a] += __shfl_xor_sync(0xffffffffu, tsum[a], o);
        }
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            *reinterpret_cast<float4*>(pt + (4 * kg + b) * (kPaRows + kPaPad) + 4 * rg) =
                make_float4(s[0][b], s[1][b], s[2][b], s[3][b]);
        }
        if (kg == 0) {
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const uint32_t r = 4 * rg + a;
                const float corr = mnew[a] == -INFINITY ? 1.0f : expf(mold[a] - mnew[a]);
                c_s[r] = corr;
                l_s[r] = l_s[r] * corr + tsum[a];
                m_s[r] = mnew[a];
            }
        }
        __syncthreads();
        // P . V: rows 4*rg .. (same row groups), columns 64*c4 + 4*kg + e
        float cr[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) cr[a] = c_s[4 * rg + a];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < CW; ++c) acc[a][c] *= cr[a];
#pragma unroll 2
        for (int jj = 0; jj < kPaKeys; ++jj) {
            const float4 pv = *reinterpret_cast<const float4*>(pt + jj * (kPaRows + kPaPad) + 4 * rg);
            const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
            for (int c4 = 0; c4 < CW / 4; ++c4) {
                const float4 vv = *reinterpret_cast<const float4*>(vs + jj * (HD + kPaPad) + 64 * c4 + 4 * kg);
                const float vb[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[a][4 * c4 + e] = fmaf(pa[a], vb[e], acc[a][4 * c4 + e]);
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const uint32_t r = 4 * rg + a, i = r / G, j = r % G;
        if (i >= nq) continue;
        const float inv = 1.0f / l_s[r];
        const uint64_t o = (static_cast<uint64_t>(i0 + i) * p.H + g * G + j) * HD + 4 * kg;
#pragma unroll
        for (int c4 = 0; c4 < CW / 4; ++c4)
#pragma unroll
            for (int e = 0; e < 4; ++e) store_split(p.out_hi, p.out_lo, o + 64 * c4 + e, acc[a][4 * c4 + e] * inv);
    }
}

}  // namespace vrt
