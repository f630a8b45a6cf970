// Decode attention for one layer, one token (src/gemma3.cpp:1557-1696 plus
// the KV push of 1590-1600), split over the key history:
//   grid = (splits, kv_heads), 128 threads.  CTA (s, g) serves the R = H/KV
//   query heads of KV head g over its share of the history.
//   1. q heads -> per-head RMSNorm (fp64 sum of squares) -> NeoX RoPE with
//      the position's cos/sin row, in registers (lane l holds dims l + 32m,
//      so both halves of every rotated pair sit in the same lane).
//   2. The CTA holding the newest position builds k (RMSNorm + RoPE) and v
//      for it, writes them to the cache slot (position % capacity: a ring of
//      `window` slots for sliding layers, linear for global ones) and uses
//      them from shared memory; no CTA reads a slot another CTA writes.
//   3. Each warp walks positions with an online softmax; the CTA merges its
//      warps and stores (max, sum, acc) per head to the split scratch.
//   4. The last CTA of the KV head (atomic ticket) merges the splits in split
//      order (deterministic) and writes the attention output, fp32.
#pragma once

#include "vrt_device.cuh"

namespace vrt {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxGroup = 8;   // query heads per KV head handled by one CTA
// Fewest positions one split takes: a short history runs on few CTAs (up to
// this many positions on one CTA, with no split merge at all).
constexpr uint32_t kAttnMinChunk = 32;
// History splits per KV head are capped at kAttnWarps * head_dim (the merge
// keeps one weight per split in the warp-merge buffer).

struct AttnParams {
    const float* qkv;       // q [H*hd] | k [KV*hd] | v [KV*hd]
    const float* q_norm;    // [hd]
    const float* k_norm;    // [hd]
    const float* rope_cos;  // [positions][hd/2]
    const float* rope_sin;
    float* k_cache;         // [KV][cap][hd]
    float* v_cache;
    uint32_t cap;
    uint32_t window;        // 0 for global layers
    const uint32_t* pos;    // device position
    uint32_t H, KV, hd;
    float eps, scale;
    float* part_ml;         // [H][splits][2]
    float* part_acc;        // [H][splits][hd]
    uint32_t* tickets;      // [KV]
    float* out;             // [H*hd]
    uint32_t splits;
    float* zero0;           // buffer this launch clears
    uint32_t zero0_count;
    // batched decode: grid.z = sequence; per-sequence strides in floats (0
    // for one sequence); pos, part_*, tickets are per sequence
    uint64_t seq_qkv, seq_cache, seq_out;
    __half* out_hi;         // when set: output as fp16 hi/lo (the o-projection
    __half* out_lo;         //   GEMM operand) instead of fp32 `out`
    uint32_t stamp;         // timing builds: this launch's stamp slot
};

template <int M>  // M = hd / 32 values per lane
__device__ __forceinline__ void head_norm_rope(float (&v)[M], const float* w, const float* cs, const float* sn,
                                               uint32_t hd, float eps, int lane) {
    double ss = 0.0;
#pragma unroll
    for (int m = 0; m < M; ++m) ss += static_cast<double>(v[m]) * static_cast<double>(v[m]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float scale = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(hd)) + eps);
#pragma unroll
    for (int m = 0; m < M; ++m) v[m] = __fmul_rn(v[m], __fmul_rn(scale, w[lane + 32 * m]));
#pragma unroll
    for (int m = 0; m < M / 2; ++m) {
        const uint32_t i = lane + 32 * m;
        const float c = cs[i], s = sn[i];
        const float a = v[m], b = v[m + M / 2];
        v[m] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        v[m + M / 2] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
}

// Positions a warp loads at once: all their K/V loads are in flight together.
template <int M>
struct AttnBatch {
    static constexpr int P = M >= 8 ? 4 : 8;
};

// K/V of positions tb + i*4 (i < P) of one KV head; positions outside
// [.., t1) and the newest position `pos` (not yet in the cache) read as 0.
template <int M, int P>
__device__ __forceinline__ void load_kv_batch(float (&kb)[P][M], float (&vb)[P][M], const float* kc,
                                              const float* vc, uint32_t tb, uint32_t t1, uint32_t pos,
                                              uint32_t cap, uint32_t hd, int lane) {
#pragma unroll
    for (int i = 0; i < P; ++i) {
        const uint32_t t = tb + i * kAttnWarps;
        const bool ok = t < t1 && t != pos;
        const uint64_t base = static_cast<uint64_t>(ok ? t % cap : 0u) * hd + lane;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            kb[i][m] = ok ? __ldcg(kc + base + 32 * m) : 0.0f;
            vb[i][m] = ok ? __ldcg(vc + base + 32 * m) : 0.0f;
        }
    }
}

// M = head_dim / 32, RG >= H / KV (1, 2, 4 or 8).  BATCH: grid.z walks
// independent sequences (per-sequence strides); the single-sequence
// instantiation keeps z = 0 at compile time and its register budget.
template <int M, int RG, bool BATCH>
__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnParams p) {
    constexpr int HD = M * 32;
    constexpr int P = AttnBatch<M>::P;
    __shared__ float q_s[RG][HD];
    __shared__ float knew[HD], vnew[HD];
    __shared__ float w_ml[kAttnWarps][RG][2];
    __shared__ float w_acc[kAttnWarps][RG][HD];
    __shared__ uint32_t last_flag;

    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) chain_stamp(p.stamp, 0);
    ChainStampEnd stamp_end{p.stamp, tid == 0};
    const uint32_t g = blockIdx.y, s = blockIdx.x, z = BATCH ? blockIdx.z : 0u;
    // this sequence's pointers (z = 0 and zero strides for a single sequence)
    const uint64_t zz = z;
    const float* const qkv = p.qkv + zz * p.seq_qkv;
    float* const k_cache = p.k_cache + zz * p.seq_cache;
    float* const v_cache = p.v_cache + zz * p.seq_cache;
    float* const part_ml = p.part_ml + zz * p.H * p.splits * 2;
    float* const part_acc = p.part_acc + zz * p.H * p.splits * p.hd;
    uint32_t* const tickets = p.tickets + zz * p.KV;
    float* const out = p.out ? p.out + zz * p.seq_out : nullptr;
    __half* const out_hi = p.out_hi ? p.out_hi + zz * p.seq_out : nullptr;
    __half* const out_lo = p.out_lo ? p.out_lo + zz * p.seq_out : nullptr;
    const uint32_t R = p.H / p.KV, hd = p.hd;

    // Nothing the step chain writes is read before griddepcontrol.wait --
    // not even the position: under programmatic launch the previous step's
    // finalize may still be in flight when this grid starts.
    pdl_wait();
    if (tid == 0) {
        chain_stamp(p.stamp, 1);
        chain_stamp(p.stamp, 2);
    }
    // Loads that do not depend on the position go out with it, in one round:
    // this warp's first query row and, for the last warp (which handles the
    // newest key/value), this KV head's new k and v.
    constexpr uint32_t kKvWarp = kAttnWarps - 1;
    float q_first[M], k_new[M], v_new[M];
    if (static_cast<uint32_t>(warp) < R) {
        const float* src = qkv + static_cast<uint64_t>(g * R + warp) * hd;
#pragma unroll
        for (int m = 0; m < M; ++m) q_first[m] = src[lane + 32 * m];
    }
    if (warp == kKvWarp) {
        const float* ks = qkv + static_cast<uint64_t>(p.H) * hd + static_cast<uint64_t>(g) * hd;
        const float* vs = qkv + static_cast<uint64_t>(p.H + p.KV) * hd + static_cast<uint64_t>(g) * hd;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            k_new[m] = ks[lane + 32 * m];
            v_new[m] = vs[lane + 32 * m];
        }
    }
    const uint32_t pos = p.pos[z];
    const uint32_t n = p.window ? min(pos + 1, p.window) : pos + 1;
    const uint32_t first = pos + 1 - n;  // oldest position attended
    // the grid has `splits` CTAs per KV head (sized for the longest history);
    // the ones past the `used` splits of this position only clear their slice
    uint32_t chunk = (n + p.splits - 1) / p.splits;
    if (chunk < kAttnMinChunk) chunk = kAttnMinChunk;
    const uint32_t used = (n + chunk - 1) / chunk;
    const uint32_t t0 = first + s * chunk;
    const uint32_t t1 = min(first + n, t0 + chunk);
    const float* kc = k_cache + static_cast<uint64_t>(g) * p.cap * hd;
    const float* vc = v_cache + static_cast<uint64_t>(g) * p.cap * hd;

    // the first batch of older positions is in flight during the query prologue
    float kb[P][M], vb[P][M];
    load_kv_batch<M, P>(kb, vb, kc, vc, t0 + warp, t1, pos, p.cap, hd, lane);

    if (p.zero0) {
        const uint32_t nb = gridDim.x * gridDim.y, b = blockIdx.y * gridDim.x + blockIdx.x;
        const uint32_t a0 = static_cast<uint64_t>(p.zero0_count) * b / nb;
        const uint32_t a1 = static_cast<uint64_t>(p.zero0_count) * (b + 1) / nb;
        for (uint32_t i = a0 + tid; i < a1; i += kAttnThreads) p.zero0[i] = 0.0f;
    }
    if (s >= used) return;
    const float* cs = p.rope_cos + static_cast<uint64_t>(pos) * (hd / 2);
    const float* sn = p.rope_sin + static_cast<uint64_t>(pos) * (hd / 2);

    // 1. queries
    for (uint32_t r = warp; r < R; r += kAttnWarps) {
        float v[M];
        if (r == static_cast<uint32_t>(warp)) {
#pragma unroll
            for (int m = 0; m < M; ++m) v[m] = q_first[m];
        } else {
            const float* src = qkv + static_cast<uint64_t>(g * R + r) * hd;
#pragma unroll
            for (int m = 0; m < M; ++m) v[m] = src[lane + 32 * m];
        }
        head_norm_rope<M>(v, p.q_norm, cs, sn, hd, p.eps, lane);
#pragma unroll
        for (int m = 0; m < M; ++m) q_s[r][lane + 32 * m] = v[m];
    }
    // 2. the newest key/value
    const bool has_new = t0 < t1 && t1 == pos + 1;
    if (has_new && warp == kKvWarp) {
        head_norm_rope<M>(k_new, p.k_norm, cs, sn, hd, p.eps, lane);
        const uint32_t slot = pos % p.cap;
        float* kd = k_cache + (static_cast<uint64_t>(g) * p.cap + slot) * hd;
        float* vd = v_cache + (static_cast<uint64_t>(g) * p.cap + slot) * hd;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            knew[lane + 32 * m] = k_new[m];
            vnew[lane + 32 * m] = v_new[m];
            kd[lane + 32 * m] = k_new[m];
            vd[lane + 32 * m] = v_new[m];
        }
    }
    __syncthreads();
    if (tid == 0) chain_stamp(p.stamp, 4);

    // 3. online softmax, P positions per warp step
    float mx[RG], sm[RG], acc[RG][M];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
        mx[r] = -INFINITY;
        sm[r] = 0.0f;
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;
    }
    for (uint32_t tb = t0 + warp; tb < t1; tb += P * kAttnWarps) {
        // the newest position (only ever inside this CTA's range) comes from shared memory
#pragma unroll
        for (int i = 0; i < P; ++i) {
            if (has_new && tb + i * kAttnWarps == pos) {
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    kb[i][m] = knew[lane + 32 * m];
                    vb[i][m] = vnew[lane + 32 * m];
                }
            }
        }
        float kcur[P][M], vcur[P][M];
#pragma unroll
        for (int i = 0; i < P; ++i)
#pragma unroll
            for (int m = 0; m < M; ++m) {
                kcur[i][m] = kb[i][m];
                vcur[i][m] = vb[i][m];
            }
        if (tb + P * kAttnWarps < t1) {  // next batch in flight
            load_kv_batch<M, P>(kb, vb, kc, vc, tb + P * kAttnWarps, t1, pos, p.cap, hd, lane);
        }
#pragma unroll
        for (int r = 0; r < RG; ++r) {
            if (r < static_cast<int>(R)) {
                float sc[P];
                float bm = -INFINITY;
#pragma unroll
                for (int i = 0; i < P; ++i) {
                    float d = 0.0f;
#pragma unroll
                    for (int m = 0; m < M; ++m) d = fmaf(q_s[r][lane + 32 * m], kcur[i][m], d);
                    d = warp_sum(d);
                    sc[i] = (tb + i * kAttnWarps < t1) ? d * p.scale : -INFINITY;
                    bm = fmaxf(bm, sc[i]);
                }
                const float nm = fmaxf(mx[r], bm);
                const float corr = expf(mx[r] - nm);
                sm[r] *= corr;
#pragma unroll
                for (int m = 0; m < M; ++m) acc[r][m] *= corr;
#pragma unroll
                for (int i = 0; i < P; ++i) {
                    const float pr = expf(sc[i] - nm);
                    sm[r] += pr;
#pragma unroll
                    for (int m = 0; m < M; ++m) acc[r][m] = fmaf(pr, vcur[i][m], acc[r][m]);
                }
                mx[r] = nm;
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RG; ++r) {
        if (r < static_cast<int>(R)) {
            if (lane == 0) {
                w_ml[warp][r][0] = mx[r];
                w_ml[warp][r][1] = sm[r];
            }
#pragma unroll
            for (int m = 0; m < M; ++m) w_acc[warp][r][lane + 32 * m] = acc[r][m];
        }
    }
    __syncthreads();
    // merge warps -> split partial
    for (uint32_t r = warp; r < R; r += kAttnWarps) {
        float M_ = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M_ = fmaxf(M_, w_ml[w][r][0]);
        float L_ = 0.0f;
        float a[M];
#pragma unroll
        for (int m = 0; m < M; ++m) a[m] = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = (M_ == -INFINITY) ? 0.0f : expf(w_ml[w][r][0] - M_);
            L_ += w_ml[w][r][1] * f;
#pragma unroll
            for (int m = 0; m < M; ++m) a[m] = fmaf(w_acc[w][r][lane + 32 * m], f, a[m]);
        }
        const uint32_t h = g * R + r;
        if (used == 1) {  // the whole history in this CTA: the output directly
            const float inv = 1.0f / L_;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float v = a[m] * inv;
                const uint64_t o = static_cast<uint64_t>(h) * hd + lane + 32 * m;
                if (out_hi) {
                    __half hh, ll;
                    split_f16(v, hh, ll);
                    out_hi[o] = hh;
                    out_lo[o] = ll;
                } else {
                    out[o] = v;
                }
            }
            continue;
        }
        float* pa = part_acc + (static_cast<uint64_t>(h) * p.splits + s) * hd;
#pragma unroll
        for (int m = 0; m < M; ++m) pa[lane + 32 * m] = a[m];
        if (lane == 0) {
            part_ml[(static_cast<uint64_t>(h) * p.splits + s) * 2] = M_;
            part_ml[(static_cast<uint64_t>(h) * p.splits + s) * 2 + 1] = L_;
        }
    }
    if (used == 1) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const uint32_t ticket = atomicAdd(tickets + g, 1u);
        last_flag = (ticket == used - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    // 4. merge the splits that saw positions, in split order: split maxima
    //    and weights one split per lane, then the accumulators with eight
    //    splits' loads in flight per lane
    for (uint32_t r = warp; r < R; r += kAttnWarps) {
        const uint32_t h = g * R + r;
        const float* ml = part_ml + static_cast<uint64_t>(h) * p.splits * 2;
        const float* pa = part_acc + static_cast<uint64_t>(h) * p.splits * hd;
        // split weights reuse the warp-merge buffer (free once this CTA's partial is out)
        float* fw = &w_acc[0][0][0] + r * (kAttnWarps * HD);
        float M_ = -INFINITY;
        for (uint32_t q = lane; q < used; q += 32) M_ = fmaxf(M_, __ldcg(ml + 2 * q));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M_ = fmaxf(M_, __shfl_xor_sync(0xffffffffu, M_, o));
        float L_ = 0.0f;
        for (uint32_t q = lane; q < used; q += 32) {
            const float mq = __ldcg(ml + 2 * q);
            const float f = mq == -INFINITY ? 0.0f : expf(mq - M_);
            fw[q] = f;
            L_ += __ldcg(ml + 2 * q + 1) * f;
        }
        L_ = warp_sum(L_);
        __syncwarp();
        float a[M];
#pragma unroll
        for (int m = 0; m < M; ++m) a[m] = 0.0f;
        for (uint32_t q0 = 0; q0 < used; q0 += 8) {
            float v[8][M];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t q = q0 + u;
#pragma unroll
                for (int m = 0; m < M; ++m) v[u][m] = q < used ? __ldcg(pa + q * hd + lane + 32 * m) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float f = q0 + u < used ? fw[q0 + u] : 0.0f;
#pragma unroll
                for (int m = 0; m < M; ++m) a[m] = fmaf(v[u][m], f, a[m]);
            }
        }
        const float inv = 1.0f / L_;
        if (out_hi) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                __half hh, ll;
                split_f16(a[m] * inv, hh, ll);
                out_hi[static_cast<uint64_t>(h) * hd + lane + 32 * m] = hh;
                out_lo[static_cast<uint64_t>(h) * hd + lane + 32 * m] = ll;
            }
        } else {
#pragma unroll
            for (int m = 0; m < M; ++m) out[static_cast<uint64_t>(h) * hd + lane + 32 * m] = a[m] * inv;
        }
    }
    if (tid == 0) tickets[g] = 0u;
}

}  // namespace vrt
