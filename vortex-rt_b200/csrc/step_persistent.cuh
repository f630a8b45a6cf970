// Persistent decode step for one sequence (bs = 1), sm_100a.
//
// One cooperative launch runs a whole token -- every layer's QKV projection,
// attention, o-projection, gate/up (gelu * up) and down, then the tied LM
// head with greedy argmax and the step's finalize (the work of
// Gemma3Model::decode_token, src/gemma3.cpp:1462-1882, and of one iteration
// of generate_greedy_tokens, 2080-2149).  One CTA per SM, eight consumer
// warps and one producer warp.
//
// Weight stream.  The producer warp walks the step's matrices in execution
// order and streams this CTA's share of each -- a contiguous run of Q8T tiles,
// tile-granular for QKV, o-projection and down, whole row groups for gate/up
// (the gelu needs a row's whole sum) and the LM head -- through a shared-memory
// ring with 1-D bulk copies.  Weights do not depend on activations, so the
// producer never waits for data: it runs ahead of the consumers by as many
// stages as the ring holds, and the HBM stream does not stop at op
// boundaries.  While the layers run it also prefetches the start of this
// CTA's LM-head rows into L2.
//
// Dataflow instead of grid barriers.  Every op output element is published as
// one 64-bit word, (sequence number << 32) | float bits.  A naturally aligned
// 64-bit store is single-copy atomic, so a reader sees either the old word or
// the new one: the word is its own ready flag and needs no fence.  Consumers
// poll exactly the words they need, with all loads in flight at once.  The
// sequence number is epoch * (5 L + 2) + op + 1; the epoch is advanced by the
// step's finalize and never reset, so a stale word never matches.  Output
// buffers alternate between even and odd layers.
//
// Partial sums.  A tile-granular span can begin or end inside a row group, so
// a few CTAs may each hold part of one output row.  CTA b writes its part of
// row group g to plane (b - first CTA of g); readers add the planes in plane
// order (under tensor parallelism rank by rank, in rank order), so the sums are
// deterministic and identical on every CTA and every rank.
//
// Residual stream.  Every CTA keeps its own copy of the residual h (d floats)
// in shared memory and updates it from the gathered o-projection and down
// outputs with the same arithmetic in the same order, so all copies stay
// bit-identical and the RMSNorms (fp64 sums of squares, the reference's
// rounding order, src/gemma3.cpp:948-1104) need no exchange.
//
// Attention.  Items (KV head g, history split s) are spread over the grid; the
// number of splits follows the attended length at run time.  With one split
// an item writes the attention-output words itself; otherwise each split
// stores (max, sum, accumulator) and the last split of the KV head (atomic
// ticket) merges them in split order.
//
// Tensor parallelism.  The o-projection and down outputs are partial sums over
// this rank's K columns; their words go to every rank's receive area over
// NVLink (plain 64-bit stores to peer memory), and readers add ranks in rank
// order.  The argmax keys of the vocabulary shards are exchanged the same way.
//
// Every wait is bounded: data words by globaltimer (`wait_ns`), ring slots by
// clock cycles.  An expired wait sets a status bit; the kernel then stops
// waiting and runs to its end.  No cluster multicast, no grid barrier.
#pragma once

#include "attention.cuh"
#include "gemv_q8t.cuh"
#include "step_state.cuh"
#include "tp_exchange.cuh"

namespace vrt {

constexpr int kPsWarps = 8;                     // consumer warps
constexpr int kPsConsumers = kPsWarps * 32;     // consumer threads
constexpr int kPsThreads = kPsConsumers + 32;   // + the producer warp
constexpr int kPsMaxStages = 12;
constexpr int kPsMaxSlots = 16;                 // ranks x planes added per element
constexpr uint32_t kStatusStepTimeout = 1u << 4;
constexpr uint32_t kPsWordsPerLayer = 5;        // qkv, attention, o, gelu*up, down
constexpr int kPsVec4 = 6;                      // float4 per consumer thread in the norms: d <= 6144

enum PsWord : uint32_t { kPsWQkv = 0, kPsWAtt = 1, kPsWO = 2, kPsWAct = 3, kPsWDn = 4 };

struct PsLayer {
    const uint8_t* qkv;   // Q8T [(H + 2 KV) hd][d] (q | k | v)
    const uint8_t* o;     // Q8T [d][H hd]
    const uint8_t* gu;    // Q8T [2 ff][d], 8 gate + 8 up rows per group
    const uint8_t* down;  // Q8T [d][ff]
    const float *n_attn, *n_q, *n_k, *n_post_attn, *n_ffn, *n_post_ffw;
    float* k_cache;       // [KV][cap][hd]
    float* v_cache;
    const float* rope_cos;  // [positions][hd / 2]
    const float* rope_sin;
    uint32_t cap;
    uint32_t window;      // 0 for global layers
};

struct PsParams {
    const PsLayer* layers;
    uint32_t L, d, H, KV, hd, qw, kw, ff;  // this rank's head counts and widths
    uint32_t vocab, vl, row_base;          // full vocabulary; this rank's LM-head rows and their first id
    const uint8_t* embd;                   // Q8T token_embd (all rows)
    const uint8_t* lm;                     // Q8T LM-head rows of this rank
    const float* out_norm;
    float eps, emb_scale, att_scale;
    StepState* st;
    uint32_t* out_ids;
    uint32_t out_cap;
    const uint32_t* prompt;                // no-head steps: the prompt (next token)
    float* hidden;                         // final normed hidden state (d)
    float* logits;                         // this rank's logits (vl) or null
    float* trace;                          // per-layer residual (L x d) or null
    uint32_t head;                         // 1: LM head + argmax + decode finalize; 0: prefill finalize
    uint32_t rg;                           // query heads per KV head rounded up (template RG)
    // exchange words (local)
    unsigned long long* x_qkv;             // [2][planes_qkv][qw + 2 kw]
    unsigned long long* x_att;             // [2][qw]
    unsigned long long* x_act;             // [2][ff]
    // receive areas of every rank (own included): o-projection / down partials
    // [2 parity][2 kind][world src][planes_rx][d], then argmax keys [world][2]
    unsigned long long* const* rx;
    uint32_t planes_qkv, planes_rx;
    // attention splits
    float* part_ml;                        // [H][s_max][2]
    float* part_acc;                       // [H][s_max][hd]
    uint32_t* att_tickets;                 // [KV]
    uint32_t s_max, min_split;
    uint32_t* fin_ticket;
    uint32_t head_pf_bytes;                // LM-head bytes per CTA prefetched into L2 ...
    uint32_t head_pf_layer;                // ... when the producer reaches this layer
    uint32_t ns;                           // ring stages
    uint64_t wait_ns;
    uint32_t rank, world;
    unsigned long long* stamps;            // timing builds only (VRT_PS_STAMPS): [grid][kPsStamps(L)]
};

// Timing builds (-DVRT_PS_STAMPS): consumer thread 0 of every CTA records
// globaltimer at each phase boundary; 16 stamps per layer, then the head's.
__host__ __device__ inline uint32_t ps_stamp_count(uint32_t L) { return 16 * L + 16; }
#ifdef VRT_PS_STAMPS
// cycles consumer thread 0 spends in ring waits [0] and data waits [1]
__shared__ long long ps_dbg_cycles[2];
#define VRT_PS_DBG_ADD(i, c) \
    do {                     \
        if (threadIdx.x == 0) ps_dbg_cycles[i] += (c); \
    } while (0)
#define VRT_PS_STAMP(k)                                                                       \
    do {                                                                                      \
        if (threadIdx.x == 0 && p.stamps) p.stamps[blockIdx.x * ps_stamp_count(p.L) + (k)] = global_ns(); \
    } while (0)
#else
#define VRT_PS_DBG_ADD(i, c) \
    do {                     \
    } while (0)
#define VRT_PS_STAMP(k) \
    do {                \
    } while (0)
#endif

// Partitions of an op's tiles over the G CTAs.  The host checks that
// (tiles + 1) * G < 2^32 for every op, so all of this stays in 32-bit
// arithmetic on the device (a 64-bit division is a long software routine).
__host__ __device__ inline uint32_t ps_cta_of_tile(uint32_t t, uint32_t total, uint32_t G) {
    return ((t + 1) * G - 1) / total;
}

// Tile span [T0, T1) of CTA b: tile-granular or whole row groups.
__host__ __device__ inline void ps_span(uint32_t rows, uint32_t cols, bool group, uint32_t G, uint32_t b,
                                        uint32_t& T0, uint32_t& T1) {
    const uint32_t kt = cols / kTileCols, groups = (rows + kTileRows - 1) / kTileRows;
    if (group) {
        T0 = groups * b / G * kt;
        T1 = groups * (b + 1) / G * kt;
    } else {
        const uint32_t total = groups * kt;
        T0 = total * b / G;
        T1 = total * (b + 1) / G;
    }
}

// Planes (CTAs holding a part) of row group g of a tile-granular op.
__host__ __device__ inline uint32_t ps_planes_of(uint32_t g, uint32_t kt, uint32_t total, uint32_t G,
                                                 uint32_t* first) {
    const uint32_t bf = ps_cta_of_tile(g * kt, total, G), bl = ps_cta_of_tile(g * kt + kt - 1, total, G);
    if (first) *first = bf;
    return bl - bf + 1;
}

__host__ __device__ inline uint32_t ps_rg_of(uint32_t H, uint32_t KV) {
    const uint32_t R = H / KV;
    return R <= 1 ? 1u : R <= 2 ? 2u : R <= 4 ? 4u : 8u;
}

__host__ __device__ inline uint32_t ps_align16(uint32_t x) { return (x + 15u) & ~15u; }

struct PsSmem {
    uint32_t ns, bars, h, v, x16p, sx, att, part, red, total;
};

// Shared-memory plan for `ns` ring stages: the ring at 0, then barriers,
// residual, gather buffer, the quantised input (aliased by the attention
// scratch), stage sums, reductions.  ps_ring_stages picks the deepest ring
// that fits a byte budget.
__host__ __device__ inline PsSmem ps_smem_layout(const PsParams& p, uint32_t ns) {
    PsSmem s{};
    const uint32_t kmax = p.d > p.qw ? (p.d > p.ff ? p.d : p.ff) : (p.qw > p.ff ? p.qw : p.ff);
    const uint32_t R = p.H / p.KV, HD = p.hd, RG = p.rg;
    const uint32_t vlen = p.d > (R + 2) * HD ? p.d : (R + 2) * HD;
    const uint32_t quant = ps_align16(kmax * 2) + ps_align16(kmax / 32 * 4);
    const uint32_t att = (RG * HD + 2 * HD + kPsWarps * RG * 2 + kPsWarps * RG * HD) * 4;
    const uint32_t uni = ps_align16(quant > att ? quant : att);
    s.ns = ns;
    s.bars = s.ns * kStageBytes;
    s.h = s.bars + 2 * kPsMaxStages * 8;
    s.v = s.h + ps_align16(p.d * 4);
    s.x16p = s.v + ps_align16(vlen * 4);
    s.sx = s.x16p + ps_align16(kmax * 2);
    s.att = s.x16p;
    s.part = s.x16p + uni;
    s.red = s.part + 2 * kPsWarps * 8 * 16 * 4;
    s.total = s.red + 64 * 8;
    return s;
}

__host__ __device__ inline uint32_t ps_ring_stages(const PsParams& p, uint32_t budget) {
    const uint32_t fixed = ps_smem_layout(p, 0).total;
    const uint32_t ns = budget > fixed ? (budget - fixed) / kStageBytes : 0u;
    return ns > static_cast<uint32_t>(kPsMaxStages) ? static_cast<uint32_t>(kPsMaxStages) : ns;
}

__host__ __device__ inline uint64_t ps_rx_index(uint32_t par, uint32_t kind, uint32_t src, uint32_t plane,
                                                uint32_t row, uint32_t world, uint32_t planes, uint32_t d) {
    return ((((static_cast<uint64_t>(par) * 2 + kind) * world + src) * planes + plane) * d) + row;
}
__host__ __device__ inline uint64_t ps_rx_key_index(uint32_t src, uint32_t half, uint32_t world, uint32_t planes,
                                                    uint32_t d) {
    return 4ull * world * planes * d + 2ull * src + half;
}
__host__ __device__ inline uint64_t ps_rx_words(uint32_t world, uint32_t planes, uint32_t d) {
    return 4ull * world * planes * d + 2ull * world;
}

// ------------------------------------------------------------ word access

__device__ __forceinline__ unsigned long long ps_ld(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ps_st(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
template <bool SYS>
__device__ __forceinline__ unsigned long long ps_ld_s(const unsigned long long* p) {
    return SYS ? ld_sys_u64(p) : ps_ld(p);
}

__device__ __forceinline__ bool ps_failed(const uint32_t* status) {
    return (*reinterpret_cast<const volatile uint32_t*>(status) &
            (kStatusStepTimeout | kStatusPeerTimeout | kStatusWaitTimeout)) != 0u;
}

// Ring-slot wait: bounded by ~0.5 s of SM clock, and once any wait of the
// step has expired (status bit) it no longer waits at all, so a failed step
// ends after one time-out instead of one per stage.
static __device__ __noinline__ bool ps_ring_wait_slow(uint64_t* bar, uint32_t parity, uint32_t* status) {
    if (ps_failed(status)) return false;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > (1ll << 30)) {
            atomicOr(status, kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool ps_ring_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
#ifdef VRT_PS_STAMPS
    const long long c0 = clock64();
    const bool r = mbar_try_wait(bar, parity) || ps_ring_wait_slow(bar, parity, status);
    if (threadIdx.x < kPsConsumers) VRT_PS_DBG_ADD(0, clock64() - c0);
    return r;
#else
    return mbar_try_wait(bar, parity) || ps_ring_wait_slow(bar, parity, status);
#endif
}

// Re-read *p until it carries `seq` or the wait expires; returns the word.
template <bool SYS>
__device__ __noinline__ unsigned long long ps_wait_slow(const unsigned long long* p, unsigned long long w,
                                                        uint32_t seq, uint64_t wait_ns, uint32_t* status) {
    if (ps_failed(status)) return w;
    const uint64_t t0 = global_ns();
    for (;;) {
#ifdef VRT_PS_BACKOFF_NS
        __nanosleep(VRT_PS_BACKOFF_NS);
#endif
        w = ps_ld_s<SYS>(p);
        if (static_cast<uint32_t>(w >> 32) == seq) return w;
        if (global_ns() - t0 > wait_ns) {
            atomicOr(status, kStatusStepTimeout);
            return w;
        }
    }
}
template <bool SYS>
__device__ __forceinline__ unsigned long long ps_wait(const unsigned long long* p, unsigned long long w, uint32_t seq,
                                                      uint64_t wait_ns, uint32_t* status) {
    return static_cast<uint32_t>(w >> 32) == seq ? w : ps_wait_slow<SYS>(p, w, seq, wait_ns, status);
}

__device__ __forceinline__ float ps_val(unsigned long long w) { return __uint_as_float(static_cast<uint32_t>(w)); }

// One thread of the CTA polls one word of the round until it is current
// while the others wait at a barrier; then all threads load their words.
// Polling by a single thread per CTA keeps the load traffic on the
// producers' cache lines low (148 pollers instead of 38k), so their stores
// land without queueing behind the polls.
template <bool SYS>
__device__ __forceinline__ void ps_cta_wait(const unsigned long long* w, uint32_t seq, uint64_t wait_ns,
                                            uint32_t* status) {
#ifdef VRT_PS_STAMPS
    const long long c0 = clock64();
#endif
    if (threadIdx.x == 0) {
        const unsigned long long x = ps_ld_s<SYS>(w);
        if (static_cast<uint32_t>(x >> 32) != seq) ps_wait_slow<SYS>(w, x, seq, wait_ns, status);
    }
    named_bar_sync(1, kPsConsumers);
#ifdef VRT_PS_STAMPS
    VRT_PS_DBG_ADD(1, clock64() - c0);
#endif
}

__device__ __forceinline__ double ps_sq4(const float4& v) {
    return static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
           static_cast<double>(v.w) * v.w;
}

// Sum of the 256 consumer threads' doubles in a fixed order, broadcast.
__device__ __forceinline__ double ps_sum(double v, double* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    named_bar_sync(1, kPsConsumers);
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < kPsWarps; ++w) s += red[w];
    named_bar_sync(1, kPsConsumers);
    return s;
}

// dst[i] = sum of the parts of row row_of(i), i < n: ranks in rank order, each
// rank's planes in plane order.  Word of rank r, plane q, row x at
// base + r * src_stride + q * plane_stride + x.  Planes follow the
// tile-granular partition of the producing op (rows_op rows, kt column tiles,
// G CTAs).  EB elements per thread per round with all their (at most MAXQ)
// words in flight: one L2 round trip per round once the words are ready.
template <bool SYS, int MAXQ, int EB, typename RowOf>
__device__ void ps_gather_t(const unsigned long long* base, uint32_t src_stride, uint32_t plane_stride,
                            uint32_t world, uint32_t rows_op, uint32_t kt, uint32_t G, uint32_t n, RowOf row_of,
                            uint32_t seq, float* dst, uint64_t wait_ns, uint32_t* status) {
    const uint32_t total = (rows_op + kTileRows - 1) / kTileRows * kt;
    for (uint32_t r0 = 0; r0 < n; r0 += EB * kPsConsumers) {  // same rounds in every thread (barrier below)
        if (r0 == 0) ps_cta_wait<SYS>(base + row_of(0), seq, wait_ns, status);
        const uint32_t i0 = r0 + threadIdx.x;
        unsigned long long w[EB][MAXQ];
        const unsigned long long* a[EB][MAXQ];
        uint32_t nq[EB];
#pragma unroll
        for (int e = 0; e < EB; ++e) {
            const uint32_t i = i0 + e * kPsConsumers;
            const uint32_t row = i < n ? row_of(i) : 0u;
            const uint32_t np = i < n ? ps_planes_of(row / kTileRows, kt, total, G, nullptr) : 1u;
            nq[e] = i < n ? np * world : 0u;
            uint32_t r = 0, pl = 0;
#pragma unroll
            for (int q = 0; q < MAXQ; ++q) {
                a[e][q] = base + r * src_stride + pl * plane_stride + row;
                if (++pl == np) {
                    pl = 0;
                    ++r;
                }
            }
        }
        // all words of the round in flight at once; while some are stale, spin on
        // the first stale one alone (one load in flight keeps the polling
        // traffic low), then re-read the others together
#pragma unroll
        for (int e = 0; e < EB; ++e)
#pragma unroll
            for (int q = 0; q < MAXQ; ++q) w[e][q] = static_cast<uint32_t>(q) < nq[e] ? ps_ld_s<SYS>(a[e][q]) : 0ull;
        for (;;) {
            bool all = true, spun = false;
#pragma unroll
            for (int e = 0; e < EB; ++e)
#pragma unroll
                for (int q = 0; q < MAXQ; ++q) {
                    if (static_cast<uint32_t>(q) < nq[e] && static_cast<uint32_t>(w[e][q] >> 32) != seq) {
                        if (!spun) {
                            spun = true;
                            w[e][q] = ps_wait<SYS>(a[e][q], w[e][q], seq, wait_ns, status);
                        } else {
                            w[e][q] = ps_ld_s<SYS>(a[e][q]);
                        }
                        all = false;
                    }
                }
            if (all || ps_failed(status)) break;
        }
#pragma unroll
        for (int e = 0; e < EB; ++e) {
            const uint32_t i = i0 + e * kPsConsumers;
            float acc = 0.0f;
#pragma unroll
            for (int q = 0; q < MAXQ; ++q) {
                if (static_cast<uint32_t>(q) < nq[e]) acc = q == 0 ? ps_val(w[e][q]) : __fadd_rn(acc, ps_val(w[e][q]));
            }
            if (i < n) dst[i] = acc;
        }
    }
}

// The gather above with the widest round its slot count allows (16 words in
// flight per thread); maxq = the most words any element has (ranks x planes).
template <bool SYS, typename RowOf>
__device__ __forceinline__ void ps_gather(const unsigned long long* base, uint32_t src_stride, uint32_t plane_stride,
                                          uint32_t world, uint32_t rows_op, uint32_t kt, uint32_t G, uint32_t n,
                                          RowOf row_of, uint32_t seq, float* dst, uint64_t wait_ns, uint32_t* status,
                                          uint32_t maxq) {
    if (maxq <= 2) {
        ps_gather_t<SYS, 2, 8>(base, src_stride, plane_stride, world, rows_op, kt, G, n, row_of, seq, dst, wait_ns, status);
    } else if (maxq <= 4) {
        ps_gather_t<SYS, 4, 4>(base, src_stride, plane_stride, world, rows_op, kt, G, n, row_of, seq, dst, wait_ns, status);
    } else if (maxq <= 8) {
        ps_gather_t<SYS, 8, 2>(base, src_stride, plane_stride, world, rows_op, kt, G, n, row_of, seq, dst, wait_ns, status);
    } else {
        ps_gather_t<SYS, 16, 1>(base, src_stride, plane_stride, world, rows_op, kt, G, n, row_of, seq, dst, wait_ns,
                                status);
    }
}

// Poll the n words base[0, n) (one plane, tag seq) and quantise them per
// 32-block into x16p / sx exactly as quant_block does: eight threads per block,
// four elements each, four blocks per thread in flight.
__device__ inline void ps_poll_quant(const unsigned long long* base, uint32_t n, uint32_t seq, int16_t* x16p, float* sx,
                                     uint64_t wait_ns, uint32_t* status) {
    const int tid = threadIdx.x, sub = tid & 7;
    constexpr int U = 6, GROUPS = kPsConsumers / 8;
    const uint32_t nblk = n / 32;
    for (uint32_t r0 = 0; r0 < nblk; r0 += U * GROUPS) {  // same trip count in every lane (shuffles below)
        if (r0 == 0) ps_cta_wait<false>(base, seq, wait_ns, status);
        const uint32_t b0 = r0 + (tid >> 3);
        unsigned long long w[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int e = 0; e < 4; ++e) w[u][e] = b0 + u * GROUPS < nblk ? ps_ld(base + (b0 + u * GROUPS) * 32 + sub * 4 + e) : 0ull;
        for (;;) {  // spin on the first stale word alone, then re-read the others together
            bool all = true, spun = false;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t blk = b0 + u * GROUPS;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (blk < nblk && static_cast<uint32_t>(w[u][e] >> 32) != seq) {
                        const unsigned long long* ad = base + blk * 32 + sub * 4 + e;
                        if (!spun) {
                            spun = true;
                            w[u][e] = ps_wait<false>(ad, w[u][e], seq, wait_ns, status);
                        } else {
                            w[u][e] = ps_ld(ad);
                        }
                        all = false;
                    }
                }
            }
            if (all || ps_failed(status)) break;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t blk = b0 + u * GROUPS;
            const bool ok = blk < nblk;  // uniform over the 8 threads of a block
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = ok ? ps_val(w[u][e]) : 0.0f;
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
            if (!ok) continue;
            const float s = quant_scale(amax);
            const float inv = amax > 0.0f ? 32767.0f / amax : 0.0f;
            if (sub == 0) sx[blk] = s;
            const int q0 = quant_one(v[0], inv), q1 = quant_one(v[1], inv), q2 = quant_one(v[2], inv),
                      q3 = quant_one(v[3], inv);
            const uint32_t k = blk * 32 + sub * 4;
            *reinterpret_cast<uint2*>(x16p + x16p_index(k)) =
                make_uint2((static_cast<uint32_t>(q0) & 0xffffu) | (static_cast<uint32_t>(q1) << 16),
                           (static_cast<uint32_t>(q2) & 0xffffu) | (static_cast<uint32_t>(q3) << 16));
        }
    }
}

// Quantise xs[0, K) (fp32 in shared memory) into x16p / sx exactly as
// quant_block does: eight threads per 32-block, four elements each.
__device__ __forceinline__ void ps_quant_smem(const float* xs, uint32_t K, int16_t* x16p, float* sx) {
    const int tid = threadIdx.x, sub = tid & 7;
    const uint32_t nblk = K / 32;
    for (uint32_t r0 = 0; r0 < nblk; r0 += kPsConsumers / 8) {  // same trip count in every lane (shuffles)
        const uint32_t blk = r0 + (tid >> 3);
        const bool ok = blk < nblk;
        const float4 x = ok ? reinterpret_cast<const float4*>(xs)[blk * 8 + sub] : make_float4(0.f, 0.f, 0.f, 0.f);
        float amax = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        if (!ok) continue;
        const float sc = quant_scale(amax);
        const float inv = amax > 0.0f ? 32767.0f / amax : 0.0f;
        if (sub == 0) sx[blk] = sc;
        const int q0 = quant_one(x.x, inv), q1 = quant_one(x.y, inv), q2 = quant_one(x.z, inv), q3 = quant_one(x.w, inv);
        *reinterpret_cast<uint2*>(x16p + x16p_index(blk * 32 + sub * 4)) =
            make_uint2((static_cast<uint32_t>(q0) & 0xffffu) | (static_cast<uint32_t>(q1) << 16),
                       (static_cast<uint32_t>(q2) & 0xffffu) | (static_cast<uint32_t>(q3) << 16));
    }
}

// ------------------------------------------------------------ the ring

struct PsRing {
    uint8_t* stages;
    uint64_t* full;
    uint64_t* empty;
    uint32_t ns, s, ph;
};

enum PsEpi : int { kPsEpiParts = 0, kPsEpiGelu = 1, kPsEpiArgmax = 2 };

// Destination of an op's output words.
struct PsOut {
    unsigned long long* const* rx;  // kPsEpiParts to receive areas (TP ops), else null
    unsigned long long* local;      // kPsEpiParts local planes / kPsEpiGelu words
    uint64_t plane_stride;          // words between planes
    uint32_t kind, par, world, rank, planes_rx, d;
    uint32_t seq;
    float* logits;                  // argmax
    uint32_t row_base;
};

// Consume this CTA's span [T0, T1) of one matrix from the ring.  Per stage
// each consumer warp takes one tile (warp w: tile T0 + 8 st + w): 16 dp2a per
// row pair give exact integer block sums, scaled by the weight and activation
// block scales and added in fp32 per warp across its tiles of a row group.  A
// warp flushes a group's two-row-per-lane sums into the chunk buffer when it
// moves on; every 8 row groups (a chunk) the warps meet at a barrier and warp
// w adds the 8 warps' parts of the chunk's group w in warp order and
// publishes the result.  The per-row summation order is fixed, so results are
// replay-identical.  Returns the best argmax key (kPsEpiArgmax, lane 0).
template <int EPI>
__device__ unsigned long long ps_matvec(PsRing& R, uint32_t rows, uint32_t cols, uint32_t T0, uint32_t T1,
                                        uint32_t G, const int16_t* x16p, const float* sx, float* partial,
                                        const PsOut& o, uint32_t* status) {
    constexpr int CG = 8;                              // row groups per chunk
    constexpr int CHUNK_FLOATS = kPsWarps * CG * 16;   // one chunk's partial sums
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quad = lane & 3;
    const uint32_t kt = cols / kTileCols;
    const uint32_t total = (rows + kTileRows - 1) / kTileRows * kt;
    const uint32_t n_tiles = T1 - T0;
    const uint32_t n_st = (n_tiles + kStageTiles - 1) / kStageTiles;
    const uint32_t g_first = T0 / kt;
    const uint32_t n_chunks = n_tiles ? ((T1 - 1) / kt - g_first) / CG + 1 : 0u;
    int cur_g = -1;
    float acc0 = 0.0f, acc1 = 0.0f;
    uint32_t chunks_done = 0;
    unsigned long long best = 0ull;

    auto flush = [&](int g) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        const uint32_t rel = static_cast<uint32_t>(g) - g_first;
        float* part = partial + ((rel / CG) & 1) * CHUNK_FLOATS + warp * (CG * 16) + (rel % CG) * 16 + 2 * (lane >> 2);
        if (quad == 0) {
            part[0] = acc0;
            part[1] = acc1;
        }
        acc0 = 0.0f;
        acc1 = 0.0f;
    };

    auto chunk_end = [&](uint32_t c) {
        named_bar_sync(1, kPsConsumers);
        const uint32_t g = g_first + c * CG + warp;
        const bool live = (g * kt < T1) && ((g + 1) * kt > T0);
        if (!live) return;
        float* part = partial + (c & 1) * CHUNK_FLOATS + warp * 16;
        float v = 0.0f;
        if (lane < 16) {
#pragma unroll
            for (int w = 0; w < kPsWarps; ++w) {
                v += part[w * (CG * 16) + lane];
                part[w * (CG * 16) + lane] = 0.0f;
            }
        }
        if (EPI == kPsEpiParts) {
            const uint32_t row = g * kTileRows + lane;
            uint32_t bf = 0;
            ps_planes_of(g, kt, total, G, &bf);
            const uint32_t plane = blockIdx.x - bf;
            if (lane < kTileRows && row < rows) {
                const unsigned long long word = tp_word(o.seq, __float_as_uint(v));
                if (o.rx) {
                    for (uint32_t r = 0; r < o.world; ++r) {
                        st_sys_u64(o.rx[r] + ps_rx_index(o.par, o.kind, o.rank, plane, row, o.world, o.planes_rx, o.d),
                                   word);
                    }
                } else {
                    ps_st(o.local + plane * o.plane_stride + row, word);
                }
            }
        } else if (EPI == kPsEpiGelu) {
            const float up = __shfl_down_sync(0xffffffffu, v, 8);
            const uint32_t a = g * 8 + lane;
            if (lane < 8 && a < rows / 2) {
                ps_st(o.local + a, tp_word(o.seq, __float_as_uint(__fmul_rn(gelu_tanh(v), up))));
            }
        } else {
            const uint32_t row = g * kTileRows + lane;
            unsigned long long key = 0ull;
            if (lane < kTileRows && row < rows) {
                if (o.logits) o.logits[row] = v;
                if (!isnan(v)) key = argmax_key(v, o.row_base + row);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, off);
                key = other > key ? other : key;
            }
            best = key > best ? key : best;
        }
    };

    // this warp's tiles are T0 + warp + 8 st; walk (group, column tile) incrementally
    uint32_t g = (T0 + warp) / kt, j = (T0 + warp) % kt;
    for (uint32_t st = 0; st < n_st; ++st) {
        const uint32_t s = R.s;
        ps_ring_wait(&R.full[s], R.ph, status);
        if (T0 + st * kStageTiles + warp < T1) {
            if (static_cast<int>(g) != cur_g && cur_g >= 0) flush(cur_g);
            const uint32_t c = (g - g_first) / CG;
            while (chunks_done < c) chunk_end(chunks_done++);
            cur_g = static_cast<int>(g);
            const uint8_t* tile = R.stages + s * kStageBytes + warp * kTileBytes;
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
        if (lane == 0) mbar_arrive(&R.empty[s]);
        if (++R.s == R.ns) {
            R.s = 0;
            R.ph ^= 1u;
        }
        j += kStageTiles;
        while (j >= kt) {
            j -= kt;
            ++g;
        }
    }
    if (cur_g >= 0) flush(cur_g);
    while (chunks_done < n_chunks) chunk_end(chunks_done++);
    if (EPI == kPsEpiArgmax) {
        // each warp emitted its own row groups: maximise over the warps (the
        // reduction scratch that follows the chunk buffer holds the keys)
        unsigned long long* keys = reinterpret_cast<unsigned long long*>(partial + 2 * CHUNK_FLOATS);
        named_bar_sync(1, kPsConsumers);
        if (lane == 0) keys[warp] = best;
        named_bar_sync(1, kPsConsumers);
        if (tid == 0) {
            for (int w = 0; w < kPsWarps; ++w) best = keys[w] > best ? keys[w] : best;
        }
        named_bar_sync(1, kPsConsumers);
    }
    return best;
}

// ------------------------------------------------------------ attention

// K/V of positions tb + i * 8 (i < P) of one KV head; positions outside
// [.., t1) and the newest position (not yet in the cache) read as 0.
template <int M, int P>
__device__ __forceinline__ void ps_load_kv(float (&kb)[P][M], float (&vb)[P][M], const float* kc, const float* vc,
                                           uint32_t tb, uint32_t t1, uint32_t pos, uint32_t cap, uint32_t hd,
                                           int lane) {
#pragma unroll
    for (int i = 0; i < P; ++i) {
        const uint32_t t = tb + i * kPsWarps;
        const bool ok = t < t1 && t != pos;
        const uint64_t base = static_cast<uint64_t>(ok ? t % cap : 0u) * hd + lane;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            kb[i][m] = ok ? __ldcg(kc + base + 32 * m) : 0.0f;
            vb[i][m] = ok ? __ldcg(vc + base + 32 * m) : 0.0f;
        }
    }
}

// Per-head RMSNorm (fp64 sum of squares) + NeoX RoPE of one head held in a
// warp (lane l: dims l + 32 m), weights and rope row already in registers;
// the arithmetic of head_norm_rope (src/gemma3.cpp:1045-1104, 1371-1424).
template <int M>
__device__ __forceinline__ void ps_norm_rope(float (&v)[M], const float (&w)[M], const float (&rc)[M / 2],
                                             const float (&rs)[M / 2], uint32_t hd, float eps) {
    double ss = 0.0;
#pragma unroll
    for (int m = 0; m < M; ++m) ss += static_cast<double>(v[m]) * static_cast<double>(v[m]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float scale = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(hd)) + eps);
#pragma unroll
    for (int m = 0; m < M; ++m) v[m] = __fmul_rn(v[m], __fmul_rn(scale, w[m]));
#pragma unroll
    for (int m = 0; m < M / 2; ++m) {
        const float a = v[m], b = v[m + M / 2];
        v[m] = __fsub_rn(__fmul_rn(a, rc[m]), __fmul_rn(b, rs[m]));
        v[m + M / 2] = __fadd_rn(__fmul_rn(b, rc[m]), __fmul_rn(a, rs[m]));
    }
}

// One attention item: KV head g, history split s of `used`, positions
// [t0, t1).  gather() fills qkv_s with the q rows of the group's R heads,
// then k, then v (fp32); the result goes to the attention-output words (seq).
template <int M, int RG, typename Gather>
__device__ void ps_attention_item(const PsParams& p, const PsLayer& Ly, uint32_t g, uint32_t s, uint32_t used,
                                  uint32_t t0, uint32_t t1, uint32_t pos, float* qkv_s, Gather gather,
                                  float* att_smem, unsigned long long* att_words, uint32_t seq, uint32_t* status) {
    constexpr int HD = M * 32;
    constexpr int P = M >= 8 ? 2 : 4;  // positions per warp step (eight warps; register budget of 168)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t R = p.H / p.KV, hd = p.hd;
    float* q_s = att_smem;                       // [RG][HD]
    float* knew = q_s + RG * HD;                 // [HD]
    float* vnew = knew + HD;                     // [HD]
    float* w_ml = vnew + HD;                     // [8][RG][2]
    float* w_acc = w_ml + kPsWarps * RG * 2;     // [8][RG][HD]
    __shared__ uint32_t ps_last_flag;

    const float* cs = Ly.rope_cos + static_cast<uint64_t>(pos) * (hd / 2);
    const float* sn = Ly.rope_sin + static_cast<uint64_t>(pos) * (hd / 2);
    const float* kc = Ly.k_cache + static_cast<uint64_t>(g) * Ly.cap * hd;
    const float* vc = Ly.v_cache + static_cast<uint64_t>(g) * Ly.cap * hd;
    const bool has_new = t0 < t1 && t1 == pos + 1;

    // Everything that does not depend on this step's projections goes out
    // before the wait for q / k / v: the first batch of cached positions, the
    // RoPE row of this position and both head-norm weights.
    float kb[P][M], vb[P][M];
    ps_load_kv<M, P>(kb, vb, kc, vc, t0 + warp, t1, pos, Ly.cap, hd, lane);
    float wq[M], wk[M], rc[M / 2], rs[M / 2];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        wq[m] = __ldg(Ly.n_q + lane + 32 * m);
        wk[m] = __ldg(Ly.n_k + lane + 32 * m);
    }
#pragma unroll
    for (int m = 0; m < M / 2; ++m) {
        rc[m] = __ldg(cs + lane + 32 * m);
        rs[m] = __ldg(sn + lane + 32 * m);
    }
    gather();  // q rows of the group's heads, then k, then v -> qkv_s
    named_bar_sync(1, kPsConsumers);

    for (uint32_t r = warp; r <= R; r += kPsWarps) {
        float v[M];
#pragma unroll
        for (int m = 0; m < M; ++m) v[m] = qkv_s[r * hd + lane + 32 * m];
        ps_norm_rope<M>(v, r < R ? wq : wk, rc, rs, hd, p.eps);
        if (r < R) {
#pragma unroll
            for (int m = 0; m < M; ++m) q_s[r * HD + lane + 32 * m] = v[m];
        } else {
            const uint32_t slot = pos % Ly.cap;
            float* kd = Ly.k_cache + (static_cast<uint64_t>(g) * Ly.cap + slot) * hd;
            float* vd = Ly.v_cache + (static_cast<uint64_t>(g) * Ly.cap + slot) * hd;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float vv = qkv_s[(R + 1) * hd + lane + 32 * m];
                knew[lane + 32 * m] = v[m];
                vnew[lane + 32 * m] = vv;
                if (has_new) {
                    kd[lane + 32 * m] = v[m];
                    vd[lane + 32 * m] = vv;
                }
            }
        }
    }
    named_bar_sync(1, kPsConsumers);

    float mx[RG], sm[RG], acc[RG][M];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
        mx[r] = -INFINITY;
        sm[r] = 0.0f;
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;
    }
    for (uint32_t tb = t0 + warp; tb < t1; tb += P * kPsWarps) {
#pragma unroll
        for (int i = 0; i < P; ++i) {
            if (has_new && tb + i * kPsWarps == pos) {
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
        if (tb + P * kPsWarps < t1) ps_load_kv<M, P>(kb, vb, kc, vc, tb + P * kPsWarps, t1, pos, Ly.cap, hd, lane);
#pragma unroll
        for (int r = 0; r < RG; ++r) {
            if (r < static_cast<int>(R)) {
                float sc[P];
                float bm = -INFINITY;
#pragma unroll
                for (int i = 0; i < P; ++i) {
                    float dd = 0.0f;
#pragma unroll
                    for (int m = 0; m < M; ++m) dd = fmaf(q_s[r * HD + lane + 32 * m], kcur[i][m], dd);
                    dd = warp_sum(dd);
                    sc[i] = (tb + i * kPsWarps < t1) ? dd * p.att_scale : -INFINITY;
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
                w_ml[(warp * RG + r) * 2] = mx[r];
                w_ml[(warp * RG + r) * 2 + 1] = sm[r];
            }
#pragma unroll
            for (int m = 0; m < M; ++m) w_acc[(warp * RG + r) * HD + lane + 32 * m] = acc[r][m];
        }
    }
    named_bar_sync(1, kPsConsumers);
    // merge the warps: the item's (max, sum, accumulator) per head
    for (uint32_t r = warp; r < R; r += kPsWarps) {
        float M_ = -INFINITY;
        for (int w = 0; w < kPsWarps; ++w) M_ = fmaxf(M_, w_ml[(w * RG + r) * 2]);
        float L_ = 0.0f;
        float a[M];
#pragma unroll
        for (int m = 0; m < M; ++m) a[m] = 0.0f;
        for (int w = 0; w < kPsWarps; ++w) {
            const float f = (M_ == -INFINITY) ? 0.0f : expf(w_ml[(w * RG + r) * 2] - M_);
            L_ += w_ml[(w * RG + r) * 2 + 1] * f;
#pragma unroll
            for (int m = 0; m < M; ++m) a[m] = fmaf(w_acc[(w * RG + r) * HD + lane + 32 * m], f, a[m]);
        }
        const uint32_t h = g * R + r;
        if (used == 1) {
            const float inv = 1.0f / L_;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                ps_st(att_words + static_cast<uint64_t>(h) * hd + lane + 32 * m,
                      tp_word(seq, __float_as_uint(a[m] * inv)));
            }
        } else {
            float* pa = p.part_acc + (static_cast<uint64_t>(h) * p.s_max + s) * hd;
#pragma unroll
            for (int m = 0; m < M; ++m) pa[lane + 32 * m] = a[m];
            if (lane == 0) {
                p.part_ml[(static_cast<uint64_t>(h) * p.s_max + s) * 2] = M_;
                p.part_ml[(static_cast<uint64_t>(h) * p.s_max + s) * 2 + 1] = L_;
            }
        }
    }
    if (used == 1) return;
    __threadfence();
    named_bar_sync(1, kPsConsumers);
    if (tid == 0) {
        const uint32_t ticket = atomicAdd(p.att_tickets + g, 1u);
        ps_last_flag = (ticket == used - 1) ? 1u : 0u;
    }
    named_bar_sync(1, kPsConsumers);
    if (!ps_last_flag) return;
    __threadfence();
    if (tid == 0) {
        // reset before the output is published: the next layer's splits of
        // this KV head only start after they have read it
        p.att_tickets[g] = 0u;
        __threadfence();
    }
    // last split of this KV head: merge the splits in split order
    for (uint32_t r = warp; r < R; r += kPsWarps) {
        const uint32_t h = g * R + r;
        const float* ml = p.part_ml + static_cast<uint64_t>(h) * p.s_max * 2;
        const float* pa = p.part_acc + static_cast<uint64_t>(h) * p.s_max * hd;
        float M_ = -INFINITY;
        for (uint32_t q = lane; q < used; q += 32) M_ = fmaxf(M_, __ldcg(ml + 2 * q));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M_ = fmaxf(M_, __shfl_xor_sync(0xffffffffu, M_, off));
        float L_ = 0.0f;
        float a[M];
#pragma unroll
        for (int m = 0; m < M; ++m) a[m] = 0.0f;
        for (uint32_t q0 = 0; q0 < used; q0 += 8) {
            float mq[8], lq[8], va[8][M];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t q = q0 + k;
                mq[k] = q < used ? __ldcg(ml + 2 * q) : -INFINITY;
                lq[k] = q < used ? __ldcg(ml + 2 * q + 1) : 0.0f;
#pragma unroll
                for (int m = 0; m < M; ++m) va[k][m] = q < used ? __ldcg(pa + q * hd + lane + 32 * m) : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float f = mq[k] == -INFINITY ? 0.0f : expf(mq[k] - M_);
                L_ += lq[k] * f;
#pragma unroll
                for (int m = 0; m < M; ++m) a[m] = fmaf(va[k][m], f, a[m]);
            }
        }
        const float inv = 1.0f / L_;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            ps_st(att_words + static_cast<uint64_t>(h) * hd + lane + 32 * m, tp_word(seq, __float_as_uint(a[m] * inv)));
        }
    }
}

// ------------------------------------------------------------ the kernel

template <int M, int RG>
__global__ void __launch_bounds__(kPsThreads, 1) ps_step_kernel(const PsParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, b = blockIdx.x;
    uint32_t* status = &p.st->status;

    const PsSmem S = ps_smem_layout(p, p.ns);
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S.bars);
    uint64_t* empty = full + kPsMaxStages;
    float* h = reinterpret_cast<float*>(smem + S.h);
    float* v = reinterpret_cast<float*>(smem + S.v);
    int16_t* x16p = reinterpret_cast<int16_t*>(smem + S.x16p);
    float* sx = reinterpret_cast<float*>(smem + S.sx);
    float* att_smem = reinterpret_cast<float*>(smem + S.att);
    float* partial = reinterpret_cast<float*>(smem + S.part);
    double* red = reinterpret_cast<double*>(smem + S.red);

    if (tid == 0) {
        for (uint32_t i = 0; i < S.ns; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kPsWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    const uint32_t L = p.L, d = p.d;
    const uint32_t qkv_rows = p.qw + 2 * p.kw;

    if (warp == kPsWarps) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            uint32_t s = 0, r = 0;
            auto issue = [&](const uint8_t* w, uint32_t rows, uint32_t cols, bool group) {
                uint32_t T0, T1;
                ps_span(rows, cols, group, G, b, T0, T1);
                for (uint32_t t = T0; t < T1; t += kStageTiles) {
                    const uint32_t tiles = T1 - t < static_cast<uint32_t>(kStageTiles) ? T1 - t : kStageTiles;
                    if (r > 0) ps_ring_wait(&empty[s], (r - 1) & 1, status);
                    mbar_arrive_expect_tx(&full[s], tiles * kTileBytes);
                    bulk_copy_g2s_hint(stages + s * kStageBytes, w + static_cast<uint64_t>(t) * kTileBytes,
                                       tiles * kTileBytes, &full[s], pol);
                    if (++s == S.ns) {
                        s = 0;
                        ++r;
                    }
                }
            };
            auto prefetch = [&](const uint8_t* w, uint32_t rows, uint32_t cols, bool group, uint64_t cap) {
                uint32_t T0, T1;
                ps_span(rows, cols, group, G, b, T0, T1);
                uint64_t bytes = static_cast<uint64_t>(T1 - T0) * kTileBytes;
                if (bytes > cap) bytes = cap;
                const uint8_t* src = w + static_cast<uint64_t>(T0) * kTileBytes;
                for (uint64_t off = 0; off < bytes; off += 32768) {
                    const uint64_t nb = bytes - off < 32768 ? bytes - off : 32768;
                    bulk_prefetch_l2(src + off, static_cast<uint32_t>(nb));
                }
            };
            for (uint32_t l = 0; l < L; ++l) {
                const PsLayer& Ly = p.layers[l];
                issue(Ly.qkv, qkv_rows, d, false);
                issue(Ly.o, d, p.qw, false);
                if (l == p.head_pf_layer && p.head && p.head_pf_bytes) prefetch(p.lm, p.vl, d, true, p.head_pf_bytes);
                issue(Ly.gu, 2 * p.ff, d, true);
                issue(Ly.down, d, p.ff, false);
            }
            if (p.head) issue(p.lm, p.vl, d, true);
            prefetch(p.layers[0].qkv, qkv_rows, d, false, 32768);  // the next step starts here
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    VRT_PS_STAMP(16 * L + 2);
#ifdef VRT_PS_STAMPS
    const long long ps_c_start = clock64();
    if (tid == 0) ps_dbg_cycles[0] = ps_dbg_cycles[1] = 0;
#endif
    for (int i = tid; i < 2 * kPsWarps * 8 * 16; i += kPsConsumers) partial[i] = 0.0f;
    const uint32_t epoch = p.st->epoch;
    const uint32_t pos = p.st->pos;
    uint32_t token = p.st->token;
    const uint32_t ops = kPsWordsPerLayer * L + 2;
    auto SEQ = [&](uint32_t l, uint32_t w) { return epoch * ops + l * kPsWordsPerLayer + w + 1; };
    PsRing R{stages, full, empty, S.ns, 0u, 0u};
    const uint32_t R_heads = p.H / p.KV, hd = p.hd;
    const uint32_t qkv_plane = qkv_rows;

    // residual update from gathered partials (already in v): h = v * (s * w_post) + h,
    // then x = rms_norm_into(h, w_pre) (or the final rms_norm_inplace) into v
    auto residual = [&](const float* w_post, const float* w_pre, float* trace_row, bool final_norm) {
        if (d <= 4u * kPsVec4 * kPsConsumers) {
            // every load of the thread (smem vectors, both norm weights) in flight at once
            const uint32_t n4 = d / 4;
            float4* v4 = reinterpret_cast<float4*>(v);
            float4* h4 = reinterpret_cast<float4*>(h);
            const float4* wp4 = reinterpret_cast<const float4*>(w_post);
            const float4* wq4 = reinterpret_cast<const float4*>(w_pre);
            float4 a[kPsVec4], hh[kPsVec4], wp[kPsVec4], wq[kPsVec4];
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < kPsVec4; ++u) {
                const uint32_t i = tid + u * kPsConsumers;
                const bool ok = i < n4;
                wp[u] = ok ? __ldg(wp4 + i) : z;
                wq[u] = ok ? __ldg(wq4 + i) : z;
                a[u] = ok ? v4[i] : z;
                hh[u] = ok ? h4[i] : z;
            }
            double so = 0.0;
#pragma unroll
            for (int u = 0; u < kPsVec4; ++u) so += ps_sq4(a[u]);
            so = ps_sum(so, red);
            const float ps = 1.0f / sqrtf(static_cast<float>(so / static_cast<double>(d)) + p.eps);
            double ss = 0.0;
            bool bad = false;
#pragma unroll
            for (int u = 0; u < kPsVec4; ++u) {
                const uint32_t i = tid + u * kPsConsumers;
                float4 x;
                x.x = __fadd_rn(__fmul_rn(a[u].x, __fmul_rn(ps, wp[u].x)), hh[u].x);
                x.y = __fadd_rn(__fmul_rn(a[u].y, __fmul_rn(ps, wp[u].y)), hh[u].y);
                x.z = __fadd_rn(__fmul_rn(a[u].z, __fmul_rn(ps, wp[u].z)), hh[u].z);
                x.w = __fadd_rn(__fmul_rn(a[u].w, __fmul_rn(ps, wp[u].w)), hh[u].w);
                hh[u] = x;
                if (i < n4) {
                    h4[i] = x;
                    bad |= !(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w));
                    if (b == 0 && trace_row) reinterpret_cast<float4*>(trace_row)[i] = x;
                }
                ss += ps_sq4(x);
            }
            if (bad && b == 0) atomicOr(status, kStatusNonFinite);
            ss = ps_sum(ss, red);
            const float sc = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(d)) + p.eps);
#pragma unroll
            for (int u = 0; u < kPsVec4; ++u) {
                const uint32_t i = tid + u * kPsConsumers;
                if (i >= n4) continue;
                float4 x;
                if (final_norm) {  // rms_norm_inplace: h * (scale * w)
                    x.x = __fmul_rn(hh[u].x, __fmul_rn(sc, wq[u].x));
                    x.y = __fmul_rn(hh[u].y, __fmul_rn(sc, wq[u].y));
                    x.z = __fmul_rn(hh[u].z, __fmul_rn(sc, wq[u].z));
                    x.w = __fmul_rn(hh[u].w, __fmul_rn(sc, wq[u].w));
                    if (b == 0) reinterpret_cast<float4*>(p.hidden)[i] = x;
                } else {           // rms_norm_into: (h * scale) * w
                    x.x = __fmul_rn(__fmul_rn(hh[u].x, sc), wq[u].x);
                    x.y = __fmul_rn(__fmul_rn(hh[u].y, sc), wq[u].y);
                    x.z = __fmul_rn(__fmul_rn(hh[u].z, sc), wq[u].z);
                    x.w = __fmul_rn(__fmul_rn(hh[u].w, sc), wq[u].w);
                }
                v4[i] = x;
            }
        } else {
            // wider than any Gemma 3 model: looped form
            double so = 0.0;
            for (uint32_t k = tid; k < d; k += kPsConsumers) so += static_cast<double>(v[k]) * v[k];
            so = ps_sum(so, red);
            const float ps = 1.0f / sqrtf(static_cast<float>(so / static_cast<double>(d)) + p.eps);
            double ss = 0.0;
            bool bad = false;
            for (uint32_t k = tid; k < d; k += kPsConsumers) {
                const float hk = __fadd_rn(__fmul_rn(v[k], __fmul_rn(ps, w_post[k])), h[k]);
                h[k] = hk;
                bad |= !isfinite(hk);
                if (b == 0 && trace_row) trace_row[k] = hk;
                ss += static_cast<double>(hk) * hk;
            }
            if (bad && b == 0) atomicOr(status, kStatusNonFinite);
            ss = ps_sum(ss, red);
            const float sc = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(d)) + p.eps);
            for (uint32_t k = tid; k < d; k += kPsConsumers) {
                const float x = final_norm ? __fmul_rn(h[k], __fmul_rn(sc, w_pre[k])) : __fmul_rn(__fmul_rn(h[k], sc), w_pre[k]);
                v[k] = x;
                if (final_norm && b == 0) p.hidden[k] = x;
            }
        }
        named_bar_sync(1, kPsConsumers);
    };
    // peers write the receive area over NVLink: system-scope loads under
    // tensor parallelism, GPU scope on one GPU
    auto gather_rx = [&](uint32_t kind, uint32_t par, uint32_t cols, uint32_t seq) {
        const unsigned long long* base = p.rx[p.rank] + ps_rx_index(par, kind, 0, 0, 0, p.world, p.planes_rx, d);
        if (p.world > 1) {
            ps_gather<true>(base, p.planes_rx * d, d, p.world, d, cols / kTileCols, G, d, [](uint32_t i) { return i; },
                            seq, v, p.wait_ns, status, p.planes_rx * p.world);
        } else {
            ps_gather<false>(base, p.planes_rx * d, d, 1, d, cols / kTileCols, G, d, [](uint32_t i) { return i; }, seq,
                             v, p.wait_ns, status, p.planes_rx);
        }
        named_bar_sync(1, kPsConsumers);
    };

    for (uint32_t l = 0; l < L; ++l) {
        const PsLayer& Ly = p.layers[l];
        const uint32_t par = l & 1u;
        // ---- QKV: input = rms_norm_into(residual, attn_norm)
        if (l == 0) {
            if (token >= p.vocab) {
                if (tid == 0 && b == 0) atomicOr(status, kStatusBadToken);
                token = 0;
            }
            double ss = 0.0;
            for (uint32_t k0 = 0; k0 < d; k0 += 8 * kPsConsumers) {  // eight elements per thread in flight
                int8_t q[8];
                uint32_t sb[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint32_t k = k0 + tid + u * kPsConsumers;
                    const uint64_t so = q8t_scale_offset(token, k / 32, d);
                    q[u] = k < d ? static_cast<int8_t>(p.embd[q8t_weight_offset(token, k, d)]) : int8_t(0);
                    sb[u] = k < d ? (p.embd[so] | (static_cast<uint32_t>(p.embd[so + 1]) << 8)) : 0u;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint32_t k = k0 + tid + u * kPsConsumers;
                    if (k >= d) continue;
                    const float hk = __fmul_rn(__fmul_rn(half_bits_to_float(sb[u]), static_cast<float>(q[u])), p.emb_scale);
                    h[k] = hk;
                    ss += static_cast<double>(hk) * hk;
                }
            }
            ss = ps_sum(ss, red);
            const float sc = 1.0f / sqrtf(static_cast<float>(ss / static_cast<double>(d)) + p.eps);
            for (uint32_t k0 = 0; k0 < d; k0 += 8 * kPsConsumers) {
                float w[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint32_t k = k0 + tid + u * kPsConsumers;
                    w[u] = k < d ? __ldg(Ly.n_attn + k) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint32_t k = k0 + tid + u * kPsConsumers;
                    if (k < d) v[k] = __fmul_rn(__fmul_rn(h[k], sc), w[u]);
                }
            }
            named_bar_sync(1, kPsConsumers);
        } else {
            gather_rx(1, par ^ 1u, p.ff, SEQ(l - 1, kPsWDn));
            VRT_PS_STAMP(16 * l + 0);
            residual(p.layers[l - 1].n_post_ffw, Ly.n_attn, p.trace ? p.trace + static_cast<uint64_t>(l - 1) * d : nullptr,
                     false);
        }
        VRT_PS_STAMP(16 * l + 1);
        ps_quant_smem(v, d, x16p, sx);
        named_bar_sync(1, kPsConsumers);
        {
            uint32_t T0, T1;
            ps_span(qkv_rows, d, false, G, b, T0, T1);
            PsOut o{};
            o.local = p.x_qkv + par * p.planes_qkv * qkv_plane;
            o.plane_stride = qkv_plane;
            o.seq = SEQ(l, kPsWQkv);
            ps_matvec<kPsEpiParts>(R, qkv_rows, d, T0, T1, G, x16p, sx, partial, o, status);
        }
        VRT_PS_STAMP(16 * l + 2);
        // ---- attention items of this CTA
        {
            const uint32_t n_att = Ly.window ? min(pos + 1, Ly.window) : pos + 1;
            const uint32_t first = pos + 1 - n_att;
            uint32_t S_ = (n_att + p.min_split - 1) / p.min_split;
            S_ = S_ < 1u ? 1u : (S_ > p.s_max ? p.s_max : S_);
            const uint32_t chunk = (n_att + S_ - 1) / S_;
            const uint32_t used = (n_att + chunk - 1) / chunk;
            // items it with it * G / items == b: [ceil(b items / G), ceil((b + 1) items / G))
            const uint32_t items = p.KV * p.s_max;
            const uint32_t it0 = (b * items + G - 1) / G, it1 = ((b + 1) * items + G - 1) / G;
            for (uint32_t it = it0; it < it1; ++it) {
                const uint32_t g = it / p.s_max, s = it % p.s_max;
                if (s >= used) continue;
                const uint32_t t0 = first + s * chunk;
                const uint32_t t1 = min(first + n_att, t0 + chunk);
                // q rows of the R heads of KV head g, its k row and v row
                const uint32_t qw = p.qw, kw = p.kw;
                auto row_of = [=](uint32_t i) -> uint32_t {
                    const uint32_t qn = R_heads * hd;
                    return i < qn ? g * qn + i : (i < qn + hd ? qw + g * hd + (i - qn) : qw + kw + g * hd + (i - qn - hd));
                };
                auto gather = [&]() {
                    ps_gather<false>(p.x_qkv + par * p.planes_qkv * qkv_plane, 0, qkv_plane, 1, qkv_rows, d / kTileCols,
                                     G, (R_heads + 2) * hd, row_of, SEQ(l, kPsWQkv), v, p.wait_ns, status, p.planes_qkv);
                    VRT_PS_STAMP(16 * l + 3);
                };
                ps_attention_item<M, RG>(p, Ly, g, s, used, t0, t1, pos, v, gather, att_smem, p.x_att + par * p.qw,
                                         SEQ(l, kPsWAtt), status);
                named_bar_sync(1, kPsConsumers);
            }
        }
        VRT_PS_STAMP(16 * l + 4);
        // ---- o-projection: input = the attention output words
        ps_poll_quant(p.x_att + par * p.qw, p.qw, SEQ(l, kPsWAtt), x16p, sx, p.wait_ns, status);
        named_bar_sync(1, kPsConsumers);
        VRT_PS_STAMP(16 * l + 5);
        {
            uint32_t T0, T1;
            ps_span(d, p.qw, false, G, b, T0, T1);
            PsOut o{};
            o.rx = p.rx;
            o.kind = 0;
            o.par = par;
            o.world = p.world;
            o.rank = p.rank;
            o.planes_rx = p.planes_rx;
            o.d = d;
            o.seq = SEQ(l, kPsWO);
            ps_matvec<kPsEpiParts>(R, d, p.qw, T0, T1, G, x16p, sx, partial, o, status);
        }
        VRT_PS_STAMP(16 * l + 6);
        // ---- gate/up: residual + post-attention norm, ffn norm; gelu(gate) * up
        gather_rx(0, par, p.qw, SEQ(l, kPsWO));
        VRT_PS_STAMP(16 * l + 7);
        residual(Ly.n_post_attn, Ly.n_ffn, nullptr, false);
        VRT_PS_STAMP(16 * l + 8);
        ps_quant_smem(v, d, x16p, sx);
        named_bar_sync(1, kPsConsumers);
        {
            uint32_t T0, T1;
            ps_span(2 * p.ff, d, true, G, b, T0, T1);
            PsOut o{};
            o.local = p.x_act + par * p.ff;
            o.seq = SEQ(l, kPsWAct);
            ps_matvec<kPsEpiGelu>(R, 2 * p.ff, d, T0, T1, G, x16p, sx, partial, o, status);
        }
        VRT_PS_STAMP(16 * l + 9);
        // ---- down: input = gelu(gate) * up words
        ps_poll_quant(p.x_act + par * p.ff, p.ff, SEQ(l, kPsWAct), x16p, sx, p.wait_ns, status);
        named_bar_sync(1, kPsConsumers);
        VRT_PS_STAMP(16 * l + 10);
        {
            uint32_t T0, T1;
            ps_span(d, p.ff, false, G, b, T0, T1);
            PsOut o{};
            o.rx = p.rx;
            o.kind = 1;
            o.par = par;
            o.world = p.world;
            o.rank = p.rank;
            o.planes_rx = p.planes_rx;
            o.d = d;
            o.seq = SEQ(l, kPsWDn);
            ps_matvec<kPsEpiParts>(R, d, p.ff, T0, T1, G, x16p, sx, partial, o, status);
        }
        VRT_PS_STAMP(16 * l + 11);
    }

    // ---- final residual and output norm; LM head + argmax
    gather_rx(1, (L - 1) & 1u, p.ff, SEQ(L - 1, kPsWDn));
    residual(p.layers[L - 1].n_post_ffw, p.out_norm, p.trace ? p.trace + static_cast<uint64_t>(L - 1) * d : nullptr,
             true);
    VRT_PS_STAMP(16 * L + 0);
    if (p.head) {
        ps_quant_smem(v, d, x16p, sx);
        named_bar_sync(1, kPsConsumers);
        uint32_t T0, T1;
        ps_span(p.vl, d, true, G, b, T0, T1);
        PsOut o{};
        o.logits = p.logits;
        o.row_base = p.row_base;
        const unsigned long long best = ps_matvec<kPsEpiArgmax>(R, p.vl, d, T0, T1, G, x16p, sx, partial, o, status);
        if (tid == 0 && best) atomicMax(&p.st->key, best);
    }
    VRT_PS_STAMP(16 * L + 1);
#ifdef VRT_PS_STAMPS
    if (tid == 0 && p.stamps) {
        unsigned long long* st_ = p.stamps + blockIdx.x * ps_stamp_count(p.L) + 16 * L;
        st_[4] = ps_dbg_cycles[0];
        st_[5] = ps_dbg_cycles[1];
        st_[6] = clock64() - ps_c_start;
    }
#endif

    // ---- finalize: the last CTA to get here
    __shared__ uint32_t ps_fin_last;
    named_bar_sync(1, kPsConsumers);
    if (tid == 0) {
        __threadfence();
        ps_fin_last = atomicAdd(p.fin_ticket, 1u) == G - 1 ? 1u : 0u;
    }
    named_bar_sync(1, kPsConsumers);
    if (!ps_fin_last || tid != 0) return;
    __threadfence();
    *p.fin_ticket = 0u;
    StepState* st = p.st;
    if (p.head) {
        unsigned long long key = *reinterpret_cast<volatile unsigned long long*>(&st->key);
        if (p.world > 1) {
            // argmax keys of the vocabulary shards: (seq, half) words to every peer
            const uint32_t seq = epoch * ops + kPsWordsPerLayer * L + 1;
            for (uint32_t r = 0; r < p.world; ++r) {
                if (r == p.rank) continue;
                st_sys_u64(p.rx[r] + ps_rx_key_index(p.rank, 0, p.world, p.planes_rx, d),
                           tp_word(seq, static_cast<uint32_t>(key >> 32)));
                st_sys_u64(p.rx[r] + ps_rx_key_index(p.rank, 1, p.world, p.planes_rx, d),
                           tp_word(seq, static_cast<uint32_t>(key)));
            }
            for (uint32_t r = 0; r < p.world; ++r) {
                if (r == p.rank) continue;
                const unsigned long long* kb = p.rx[p.rank] + ps_rx_key_index(r, 0, p.world, p.planes_rx, d);
                const unsigned long long hi = ps_wait<true>(kb, ld_sys_u64(kb), seq, p.wait_ns, status);
                const unsigned long long lo = ps_wait<true>(kb + 1, ld_sys_u64(kb + 1), seq, p.wait_ns, status);
                const unsigned long long k = (static_cast<unsigned long long>(static_cast<uint32_t>(hi)) << 32) |
                                             static_cast<uint32_t>(lo);
                key = k > key ? k : key;
            }
        }
        uint32_t idx;
        float val;
        argmax_unkey(key, &idx, &val);
        st->result_index = idx;
        st->result_value = val;
        if (idx >= p.vocab || !isfinite(val)) st->status |= kStatusNonFinite;
        const uint32_t c = st->out_count;
        if (p.out_ids && c < p.out_cap) p.out_ids[c] = idx;
        st->out_count = c + 1;
        st->token = idx < p.vocab ? idx : 0u;
        st->pos = pos + 1;
        st->key = 0ull;
    } else {
        const uint32_t np = pos + 1;
        st->pos = np;
        if (np < st->prompt_count) st->token = p.prompt[np];
    }
    st->epoch = epoch + 1;
}

}  // namespace vrt
