// Gemma 3 Q8_0 model on one B200 (or one tensor-parallel rank): the device
// arena, weight loading/repacking, the decode step as a chain of kernels
// captured in a CUDA graph, and the C ABI of the model (the role of the
// reference's Gemma3Model, src/gemma3.cpp).
//
// Arena (256-byte aligned pieces):
//   token_embd       Q8T [vocab][d]          (embedding rows + tied LM head)
//   per layer        Q8T qkv   [(Hl+2KVl)*hd][d]   q | k | v rows stacked
//                    Q8T o     [d][Hl*hd]
//                    Q8T gu    [2*ffl][d]          8 gate + 8 up rows per group
//                    Q8T down  [d][ffl]
//                    fp32 norms attn, q, k, post_attn, ffn, post_ffw
//   output_norm      fp32 [d]
// plus RoPE tables (host-computed cos/sin per position, as the reference's
// build_rope_table), the KV cache (fp32, [KVl][cap][hd] per layer; cap =
// window for sliding layers, positions for global ones) and activations.
//
// One decode step = per layer: QKV (embedding or residual + RMSNorm prologue)
// -> attention -> o-proj -> gate/up (residual + 2 RMSNorm prologue, gelu*up
// epilogue) -> down; then the LM head (residual + output norm prologue,
// argmax epilogue) and a 1-thread finalize.  Each kernel clears, after its
// griddepcontrol.wait, a buffer that a later kernel accumulates into and no
// running kernel reads, so the graph needs no memset nodes and the PDL chain
// is unbroken.  With tensor parallelism an NCCL all-reduce follows o-proj and
// down, and an NCCL max-reduce merges the per-shard argmax keys.

#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "prefill.cuh"
#include "step_state.cuh"
#include "vortexrt/gguf.hpp"
#include "vrt_device.cuh"
#include "vrt_internal.hpp"
#include "vrt_kernels.hpp"

namespace vrt {

// ---------------------------------------------------------------- kernels

struct RepackParams {
    const uint8_t* src;      // raw Q8_0 rows
    uint64_t src_row_bytes;
    uint32_t src_blk0;       // first block of each source row to take
    uint32_t rows;
    uint32_t nblk;           // blocks per destination row
    uint8_t* dst;            // Q8T matrix
    uint32_t dst_cols;
    uint32_t dst_row0;
    int mode;                // 0: dst row = row0 + r; 1/2: gate/up interleave
};

__device__ __forceinline__ uint32_t dst_row_of(uint32_t r, uint32_t row0, int mode) {
    if (mode == 0) return row0 + r;
    return (r / 8) * 16 + (mode == 2 ? 8 : 0) + (r % 8);
}

__device__ __forceinline__ void store_q8t_block(uint8_t* dst, uint32_t cols, uint32_t row, uint32_t blk,
                                                const uint8_t q[32], uint16_t scale_bits) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w[i] = q[4 * i] | (static_cast<uint32_t>(q[4 * i + 1]) << 8) | (static_cast<uint32_t>(q[4 * i + 2]) << 16) |
               (static_cast<uint32_t>(q[4 * i + 3]) << 24);
    }
    *reinterpret_cast<uint4*>(dst + q8t_weight_offset(row, blk * 32, cols)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(dst + q8t_weight_offset(row, blk * 32 + 16, cols)) = make_uint4(w[4], w[5], w[6], w[7]);
    *reinterpret_cast<uint16_t*>(dst + q8t_scale_offset(row, blk, cols)) = scale_bits;
}

__global__ void repack_kernel(const RepackParams p) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<uint64_t>(p.rows) * p.nblk) return;
    const uint32_t r = static_cast<uint32_t>(i / p.nblk), b = static_cast<uint32_t>(i % p.nblk);
    const uint8_t* s = p.src + r * p.src_row_bytes + static_cast<uint64_t>(p.src_blk0 + b) * 34u;
    uint8_t q[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) q[k] = s[2 + k];
    store_q8t_block(p.dst, p.dst_cols, dst_row_of(r, p.dst_row0, p.mode), b, q,
                    static_cast<uint16_t>(s[0] | (s[1] << 8)));
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ int32_t irwin_hall4(uint64_t key, uint64_t idx) {
    const uint64_t h = splitmix64(key + idx);
    const int64_t s = static_cast<int64_t>(h & 0xffff) + static_cast<int64_t>((h >> 16) & 0xffff) +
                      static_cast<int64_t>((h >> 32) & 0xffff) + static_cast<int64_t>(h >> 48);
    return static_cast<int32_t>(s - 131070);
}

struct SynthParams {
    uint64_t key;
    uint32_t cols_full;  // columns of the logical (unsharded) matrix
    uint32_t r0, nr;     // source rows to generate
    uint32_t b0, nb;     // source blocks per row to generate
    float mult;
    uint8_t* dst;
    uint32_t dst_cols;
    uint32_t dst_row0;
    int mode;
};

// Same values and quantisation as synth_gguf.q8_matrix_bytes.
__global__ void synth_q8_kernel(const SynthParams p) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<uint64_t>(p.nr) * p.nb) return;
    const uint32_t r = static_cast<uint32_t>(i / p.nb), b = static_cast<uint32_t>(i % p.nb);
    const uint64_t base = static_cast<uint64_t>(p.r0 + r) * p.cols_full + static_cast<uint64_t>(p.b0 + b) * 32u;
    float v[32];
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        v[k] = __fmul_rn(static_cast<float>(irwin_hall4(p.key, base + k)), p.mult);
        amax = fmaxf(amax, fabsf(v[k]));
    }
    const float scale = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
    const __half hs = __float2half_rn(scale);
    const float dq = __half2float(hs);
    uint8_t q[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        float t = rintf(__fdiv_rn(v[k], dq));
        t = fminf(127.0f, fmaxf(-127.0f, t));
        q[k] = static_cast<uint8_t>(static_cast<int8_t>(t));
    }
    store_q8t_block(p.dst, p.dst_cols, dst_row_of(r, p.dst_row0, p.mode), b, q, __half_as_ushort(hs));
}

__global__ void synth_norm_kernel(uint64_t key, uint32_t n, float mult, float* out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fadd_rn(1.0f, __fmul_rn(static_cast<float>(irwin_hall4(key, i)), mult));
}


__global__ void finalize_decode_kernel(StepState* st, uint32_t vocab, uint32_t* out_ids, uint32_t out_cap,
                                       const TpParams tp) {
    pdl_wait();
    uint32_t idx;
    float val;
    const unsigned long long key = tp.world > 1 ? tp_key_max(tp, st->key, &st->status) : st->key;
    argmax_unkey(key, &idx, &val);
    st->result_index = idx;
    st->result_value = val;
    if (idx >= vocab || !isfinite(val)) st->status |= kStatusNonFinite;
    const uint32_t c = st->out_count;
    if (out_ids && c < out_cap) out_ids[c] = idx;
    st->out_count = c + 1;
    st->token = idx < vocab ? idx : 0u;
    st->pos += 1;
    st->key = 0ull;
    st->epoch += 1;
}

__global__ void finalize_prefill_kernel(StepState* st, const uint32_t* prompt) {
    pdl_wait();
    const uint32_t p = st->pos + 1;
    st->pos = p;
    if (p < st->prompt_count) st->token = prompt[p];
    st->epoch += 1;
}

// Final residual + output norm without the LM head (top_k == 0 steps).
__global__ void final_hidden_kernel(const float* dn, const float* h_prev, const float* w_post, const float* w_out,
                                    float* hidden, float* trace, uint32_t d, float eps, uint32_t* status,
                                    const TpParams tp) {
    pdl_wait();
    if (tp.world > 1) {  // tensor parallel: sum the ranks' partials of the last FFN output first
        tp_slice_reduce(tp, tp_seq(tp), 0, d, threadIdx.x, blockDim.x, status);
        __syncthreads();
        dn = tp.sum;
    }
    __shared__ double red[32];
    __shared__ float scale_s;
    extern __shared__ float hs[];
    const int tid = threadIdx.x;
    double so = 0.0;
    for (uint32_t k = tid; k < d; k += blockDim.x) {
        const double v = __ldcg(dn + k);
        so += v * v;
    }
    so = warp_sum(so);
    if ((tid & 31) == 0) red[tid / 32] = so;
    __syncthreads();
    if (tid == 0) {
        double s = 0.0;
        for (uint32_t w = 0; w < blockDim.x / 32; ++w) s += red[w];
        scale_s = 1.0f / sqrtf(static_cast<float>(s / static_cast<double>(d)) + eps);
    }
    __syncthreads();
    const float ps = scale_s;
    double ss = 0.0;
    bool bad = false;
    for (uint32_t k = tid; k < d; k += blockDim.x) {
        const float h = __fadd_rn(__fmul_rn(__ldcg(dn + k), __fmul_rn(ps, w_post[k])), h_prev[k]);
        hs[k] = h;
        bad |= !isfinite(h);
        if (trace) trace[k] = h;
        ss += static_cast<double>(h) * static_cast<double>(h);
    }
    if (bad) atomicOr(status, kStatusNonFinite);
    __syncthreads();
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid / 32] = ss;
    __syncthreads();
    if (tid == 0) {
        double s = 0.0;
        for (uint32_t w = 0; w < blockDim.x / 32; ++w) s += red[w];
        scale_s = 1.0f / sqrtf(static_cast<float>(s / static_cast<double>(d)) + eps);
    }
    __syncthreads();
    const float sc = scale_s;
    for (uint32_t k = tid; k < d; k += blockDim.x) hidden[k] = __fmul_rn(hs[k], __fmul_rn(sc, w_out[k]));
}

// ------------------------------------------------------------------ host

constexpr uint32_t kMaxSteps = 1u << 16;  // capacity of the generated-id ring

struct LayerW {
    uint64_t qkv, o, gu, down;
    uint64_t n_attn, n_q, n_k, n_post_attn, n_ffn, n_post_ffw;
    float* k_cache;
    float* v_cache;
    uint32_t cap;
    bool global;
    uint32_t splits;
};

// minimal NCCL surface, resolved at run time so single-GPU use needs no NCCL
struct Nccl {
    void* lib = nullptr;
    int (*CommInitRank)(void**, int, const void*, int) = nullptr;  // ncclUniqueId passed by value -> by pointer shim
    int (*AllReduce)(const void*, void*, size_t, int, int, void*, cudaStream_t) = nullptr;
    int (*CommDestroy)(void*) = nullptr;
    int (*GetUniqueId)(void*) = nullptr;
    const char* (*GetErrorString)(int) = nullptr;
    int (*AllGather)(const void*, void*, size_t, int, void*, cudaStream_t) = nullptr;
};

}  // namespace vrt

struct vrt_model {
    vrt_ctx* ctx = nullptr;
    vrt_gemma3_config cfg{};
    vrt_model_options opt{};
    uint64_t eos = 1;
    int rank = 0, world = 1;
    uint32_t Hl = 0, KVl = 0, qwl = 0, kwl = 0, ffl = 0, vocab_lo = 0, vocab_hi = 0;
    uint8_t* arena = nullptr;
    uint64_t arena_bytes = 0;
    uint64_t embd = 0, out_norm = 0;
    std::vector<vrt::LayerW> layers;
    uint32_t P = 0;  // positions (rope/KV capacity)
    float *rope_cos_l = nullptr, *rope_sin_l = nullptr, *rope_cos_g = nullptr, *rope_sin_g = nullptr;
    float* kv_mem = nullptr;
    float* act_mem = nullptr;
    float *h0, *h1, *qkv, *att, *o, *act, *dn, *hidden, *logits, *trace, *part_ml, *part_acc;
    uint32_t* tickets = nullptr;
    uint32_t* out_ids = nullptr;
    uint32_t* prompt = nullptr;
    vrt::StepState* st = nullptr;      // device
    vrt::StepState* st_host = nullptr; // pinned mirror
    float* hidden_host = nullptr;      // pinned
    uint32_t next_pos = 0;
    uint32_t generated = 0;  // ids in out_ids since the last prefill
    bool trace_on = false;
    cudaGraphExec_t g_head = nullptr, g_nohead = nullptr;
    uint32_t kernels_per_step = 0;
    void* comm = nullptr;
    unsigned long long* key_tmp = nullptr;
    vrt::Nccl nccl;
    // peer-memory exchange (tp_exchange == VRT_TP_PEER, world > 1)
    bool tp_peer = false;
    unsigned long long* tp_slots = nullptr;             // own receive slots (exported by CUDA IPC)
    std::vector<unsigned long long*> tp_peer_slots;     // every rank's slots, mapped here (own included)
    unsigned long long** tp_peers_dev = nullptr;        // the same table on the device
    float* tp_sum = nullptr;                            // reduced vectors, [2][d]
    uint32_t* tp_bar = nullptr;                         // grid barrier counter, generation
    float* logits_full = nullptr;                       // tensor parallel: all ranks' logits shards, [vocab]
    // persistent decode step (one cooperative kernel per token)
    bool ps_on = false;
    vrt::PsParams ps{};             // launch parameters; head, trace set per launch
    uint32_t ps_grid = 0, ps_smem = 0;
    void* ps_mem = nullptr;         // layer table, exchange words, split scratch, tickets
    unsigned long long** ps_rx_dev = nullptr;  // [world] receive-area bases
    uint64_t ps_rx_offset = 0;      // words from the start of a rank's peer slots to its receive area
    // Q8M copies of the projections and the LM-head rows (integer tensor-core
    // GEMM of batched decode), built at the first batch: per layer qkv, o, gu,
    // down offsets, then the head
    uint8_t* q8m = nullptr;
    std::vector<uint64_t> q8m_off;
    // batched prefill buffers, [chunk][...] rows (allocated at the first batched prefill)
    struct Prefill {
        uint32_t cap = 0;
        void* mem = nullptr;
        float *h0 = nullptr, *h1 = nullptr, *qkv = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr,
              *dn = nullptr;
        __half *xh = nullptr, *xl = nullptr, *ah = nullptr, *al = nullptr;
        vrt::TmaMap xd_hi, xd_lo, xq_hi, xq_lo, xf_hi, xf_lo;  // operands with K = d, q width, ffn width
    } pf;
};

// Independent sequences decoded together on one model: per-sequence KV
// caches, device-resident tokens / positions, one step = one token for each
// of the first `count` sequences, projections as tensor-core GEMMs with M =
// count rows, the LM head as a GEMM with a fused per-row argmax.
struct vrt_batch {
    vrt_model* m = nullptr;
    uint32_t S = 0, P = 0, out_cap = 0;
    bool keep_logits = false;
    void* mem = nullptr;                       // caches + step buffers
    std::vector<float*> kc, vc;                // per layer: sequence 0's K / V cache, [S][KV][cap][hd]
    std::vector<uint32_t> cap;
    uint32_t* tokens = nullptr;                // [S]
    uint32_t* pos = nullptr;                   // [S]
    uint32_t* out_ids = nullptr;               // [S][out_cap]
    uint32_t* out_count = nullptr;             // [S]
    uint32_t* prompt = nullptr;                // [P] prefill staging
    unsigned long long* keys = nullptr;        // [S]
    uint32_t* tickets = nullptr;               // [S][KV]
    float *h0, *h1, *qkv, *o, *dn, *hidden, *logits, *part_ml, *part_acc;
    __half *xh, *xl, *ah, *al;
    vrt::TmaMap xd_hi, xd_lo, xq_hi, xq_lo, xf_hi, xf_lo;        // 16-row boxes: small-M GEMM (<= 128 sequences)
    vrt::TmaMap Xd_hi, Xd_lo, Xq_hi, Xq_lo, Xf_hi, Xf_lo;        // 128-row boxes: large-M GEMM
    uint32_t max_splits = 0;
    float* gws = nullptr;                      // small-M GEMM split-K partials
    uint32_t* gtickets = nullptr;              // small-M GEMM reduction tickets (zero between launches)
    uint64_t gws_floats = 0, gtickets_n = 0;
    std::vector<uint32_t> host_pos;            // positions as the host last set them
    cudaGraphExec_t graph = nullptr;
    uint32_t graph_count = 0;
    // integer tensor-core GEMMs (count <= 32): int16 split operands [Sp][K]
    // (row stride K of the GEMM at hand), block scales [K / 32][Sp], fp32
    // attention output and gelu(gate) * up for their quantisation
    bool i8 = false;
    uint32_t Sp = 0;
    int8_t *q_hi = nullptr, *q_lo = nullptr;
    float *q_sx = nullptr, *att32 = nullptr, *act32 = nullptr;
    vrt::TmaMap Qd_hi, Qd_lo, Qq_hi, Qq_lo, Qf_hi, Qf_lo;
};

namespace vrt {

static int nccl_load(Nccl& n) {
    if (n.lib) return VRT_OK;
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char* nm : names) {
        n.lib = dlopen(nm, RTLD_NOW | RTLD_GLOBAL);
        if (n.lib) break;
    }
    if (!n.lib) return fail(VRT_E_UNSUPPORTED, "tensor parallelism needs libnccl.so.2: %s", dlerror());
    n.AllReduce = reinterpret_cast<decltype(n.AllReduce)>(dlsym(n.lib, "ncclAllReduce"));
    n.CommDestroy = reinterpret_cast<decltype(n.CommDestroy)>(dlsym(n.lib, "ncclCommDestroy"));
    n.GetUniqueId = reinterpret_cast<decltype(n.GetUniqueId)>(dlsym(n.lib, "ncclGetUniqueId"));
    n.GetErrorString = reinterpret_cast<decltype(n.GetErrorString)>(dlsym(n.lib, "ncclGetErrorString"));
    n.AllGather = reinterpret_cast<decltype(n.AllGather)>(dlsym(n.lib, "ncclAllGather"));
    if (!n.AllReduce || !n.CommDestroy || !n.GetUniqueId || !n.GetErrorString || !n.AllGather) {
        return fail(VRT_E_UNSUPPORTED, "libnccl.so.2 lacks the expected symbols");
    }
    return VRT_OK;
}

// ncclCommInitRank takes ncclUniqueId (128 bytes) by value.
struct NcclId {
    char b[128];
};
using CommInitRankFn = int (*)(void**, int, NcclId, int);

static uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

static uint64_t fnv1a64(const std::string& s) {
    uint64_t h = 0xCBF29CE484222325ull;
    for (unsigned char c : s) {
        h ^= c;
        h *= 0x100000001B3ull;
    }
    return h;
}
static uint64_t splitmix64_h(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static uint64_t stream_key(uint64_t seed, const std::string& name) {
    return splitmix64_h(seed ^ ((fnv1a64(name) + 1ull) * 0xD1B54A32D192ED03ull));
}

static std::string lname(uint32_t l, const char* suffix) { return "blk." + std::to_string(l) + "." + suffix; }

static int validate_config(const vrt_gemma3_config& c) {
    if (!c.embedding_length || !c.block_count || !c.feed_forward_length || !c.head_count || !c.head_count_kv ||
        !c.head_dim || !c.value_dim || !c.vocab_size) {
        return fail(VRT_E_INVALID, "Gemma 3 configuration contains zero dimensions");
    }
    if (c.head_count % c.head_count_kv) return fail(VRT_E_INVALID, "Gemma 3 head_count must be divisible by head_count_kv");
    if (c.value_dim != c.head_dim) return fail(VRT_E_UNSUPPORTED, "key and value head dimensions must be equal");
    if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256) {
        return fail(VRT_E_UNSUPPORTED, "head_dim %u unsupported (64, 128 or 256)", c.head_dim);
    }
    if (c.head_count / c.head_count_kv > 8) return fail(VRT_E_UNSUPPORTED, "more than 8 query heads per KV head");
    if (c.embedding_length % 128 || c.feed_forward_length % 128 || (c.head_count * c.head_dim) % 128) {
        return fail(VRT_E_UNSUPPORTED, "model widths must be multiples of 128");
    }
    return VRT_OK;
}

// Tensor-parallel shard of one rank: heads, FFN rows and vocab rows split in
// equal contiguous ranges; every piece keeps whole 128-column tiles.
static int tp_plan(const vrt_gemma3_config& c, int W, int rank, vrt_tp_shard& s) {
    if (W < 1 || rank < 0 || rank >= W) return fail(VRT_E_INVALID, "bad tensor-parallel rank %d of %d", rank, W);
    if (c.head_count_kv % W || c.head_count % W || c.feed_forward_length % (W * 128) || c.vocab_size % (W * 16)) {
        return fail(VRT_E_UNSUPPORTED, "model does not split evenly over %d ranks", W);
    }
    if ((c.head_count / W) * c.head_dim % 128) {
        return fail(VRT_E_UNSUPPORTED, "per-rank attention width must be a multiple of 128");
    }
    s.q_heads = c.head_count / W;
    s.q_head0 = s.q_heads * rank;
    s.kv_heads = c.head_count_kv / W;
    s.kv_head0 = s.kv_heads * rank;
    s.ffn = c.feed_forward_length / W;
    s.ffn0 = s.ffn * rank;
    s.vocab = c.vocab_size / W;
    s.vocab0 = s.vocab * rank;
    return VRT_OK;
}

// Shard sizes and the arena plan.
static int plan(vrt_model* m) {
    const auto& c = m->cfg;
    vrt_tp_shard sh{};
    VRT_TRY(tp_plan(c, m->world, m->rank, sh));
    m->Hl = sh.q_heads;
    m->KVl = sh.kv_heads;
    m->qwl = m->Hl * c.head_dim;
    m->kwl = m->KVl * c.head_dim;
    m->ffl = sh.ffn;
    m->vocab_lo = sh.vocab0;
    m->vocab_hi = sh.vocab0 + sh.vocab;
    const uint32_t d = c.embedding_length;
    uint64_t at = 0;
    m->embd = at;
    at = align256(at + q8t_bytes(c.vocab_size, d));
    m->layers.resize(c.block_count);
    for (uint32_t l = 0; l < c.block_count; ++l) {
        auto& L = m->layers[l];
        L.qkv = at;
        at = align256(at + q8t_bytes(m->qwl + 2 * m->kwl, d));
        L.o = at;
        at = align256(at + q8t_bytes(d, m->qwl));
        L.gu = at;
        at = align256(at + q8t_bytes(2 * m->ffl, d));
        L.down = at;
        at = align256(at + q8t_bytes(d, m->ffl));
        L.n_attn = at;
        at = align256(at + 4ull * d);
        L.n_q = at;
        at = align256(at + 4ull * c.head_dim);
        L.n_k = at;
        at = align256(at + 4ull * c.head_dim);
        L.n_post_attn = at;
        at = align256(at + 4ull * d);
        L.n_ffn = at;
        at = align256(at + 4ull * d);
        L.n_post_ffw = at;
        at = align256(at + 4ull * d);
        L.global = ((l + 1u) % 6u) == 0u;  // gemma3.cpp:1301-1307
    }
    m->out_norm = at;
    at = align256(at + 4ull * d);
    m->arena_bytes = at + 4096;
    return VRT_OK;
}

static void host_rope_table(uint32_t hd, float theta, uint32_t P, std::vector<float>& cs, std::vector<float>& sn) {
    // build_rope_inverse_frequencies + build_rope_table (src/gemma3.cpp:1309-1369)
    const uint32_t half = hd / 2;
    std::vector<float> inv(half);
    for (uint32_t i = 0; i < half; ++i) {
        const float e = (2.0f * static_cast<float>(i)) / static_cast<float>(hd);
        inv[i] = 1.0f / std::pow(theta, e);
    }
    cs.resize(static_cast<size_t>(P) * half);
    sn.resize(static_cast<size_t>(P) * half);
    for (uint32_t p = 0; p < P; ++p) {
        const float pf = static_cast<float>(p);
        for (uint32_t i = 0; i < half; ++i) {
            const float a = pf * inv[i];
            cs[static_cast<size_t>(p) * half + i] = std::cos(a);
            sn[static_cast<size_t>(p) * half + i] = std::sin(a);
        }
    }
}

static int alloc_runtime(vrt_model* m) {
    const auto& c = m->cfg;
    vrt_ctx* ctx = m->ctx;
    const uint32_t d = c.embedding_length, hd = c.head_dim;
    uint32_t P = m->opt.max_positions ? m->opt.max_positions : std::min<uint32_t>(c.context_length, 8192u);
    if (c.context_length && P > c.context_length) P = c.context_length;
    if (P == 0) return fail(VRT_E_INVALID, "no positions available");
    m->P = P;
    VRT_CUDA(cudaMalloc(&m->arena, m->arena_bytes));
    VRT_CUDA(cudaMemsetAsync(m->arena, 0, m->arena_bytes, ctx->stream));
    // KV cache
    uint64_t kv_floats = 0;
    const int sms = ctx->prop.multiProcessorCount;
    uint32_t max_splits = 1;
    for (auto& L : m->layers) {
        L.cap = (!L.global && c.sliding_window) ? std::min(c.sliding_window, P) : P;
        kv_floats += 2ull * m->KVl * L.cap * hd;
        const uint32_t by_len = std::max(1u, (L.cap + 15) / 16);
        const uint32_t by_sm = std::max(1u, static_cast<uint32_t>(3 * sms) / m->KVl);
        L.splits = std::min(std::min(by_len, by_sm), static_cast<uint32_t>(kAttnWarps) * hd);
        max_splits = std::max(max_splits, L.splits);
    }
    VRT_CUDA(cudaMalloc(&m->kv_mem, kv_floats * 4));
    VRT_CUDA(cudaMemsetAsync(m->kv_mem, 0, kv_floats * 4, ctx->stream));
    float* kp = m->kv_mem;
    for (auto& L : m->layers) {
        L.k_cache = kp;
        kp += static_cast<uint64_t>(m->KVl) * L.cap * hd;
        L.v_cache = kp;
        kp += static_cast<uint64_t>(m->KVl) * L.cap * hd;
    }
    // RoPE tables
    std::vector<float> cs, sn;
    const uint64_t tab = static_cast<uint64_t>(P) * (hd / 2) * 4;
    float* rope = nullptr;
    VRT_CUDA(cudaMalloc(&rope, 4 * tab));
    m->rope_cos_l = rope;
    m->rope_sin_l = rope + tab / 4;
    m->rope_cos_g = rope + 2 * (tab / 4);
    m->rope_sin_g = rope + 3 * (tab / 4);
    host_rope_table(hd, c.local_rope_base, P, cs, sn);
    VRT_CUDA(cudaMemcpy(m->rope_cos_l, cs.data(), tab, cudaMemcpyHostToDevice));
    VRT_CUDA(cudaMemcpy(m->rope_sin_l, sn.data(), tab, cudaMemcpyHostToDevice));
    host_rope_table(hd, c.global_rope_base, P, cs, sn);
    VRT_CUDA(cudaMemcpy(m->rope_cos_g, cs.data(), tab, cudaMemcpyHostToDevice));
    VRT_CUDA(cudaMemcpy(m->rope_sin_g, sn.data(), tab, cudaMemcpyHostToDevice));
    // activations
    const uint32_t vl = m->vocab_hi - m->vocab_lo;
    const uint64_t sizes[] = {d, d, m->qwl + 2ull * m->kwl, m->qwl, d, m->ffl, d, d, vl,
                              static_cast<uint64_t>(c.block_count) * d,
                              static_cast<uint64_t>(m->Hl) * max_splits * 2,
                              static_cast<uint64_t>(m->Hl) * max_splits * hd};
    uint64_t total = 0;
    for (auto s : sizes) total += align256(s * 4) / 4;
    VRT_CUDA(cudaMalloc(&m->act_mem, total * 4));
    VRT_CUDA(cudaMemsetAsync(m->act_mem, 0, total * 4, ctx->stream));
    float* ap = m->act_mem;
    float** dst[] = {&m->h0, &m->h1, &m->qkv, &m->att, &m->o, &m->act, &m->dn, &m->hidden, &m->logits, &m->trace,
                     &m->part_ml, &m->part_acc};
    for (size_t i = 0; i < 12; ++i) {
        *dst[i] = ap;
        ap += align256(sizes[i] * 4) / 4;
    }
    VRT_CUDA(cudaMalloc(&m->tickets, 4ull * std::max(1u, m->KVl)));
    VRT_CUDA(cudaMemsetAsync(m->tickets, 0, 4ull * std::max(1u, m->KVl), ctx->stream));
    VRT_CUDA(cudaMalloc(&m->out_ids, 4ull * kMaxSteps));
    VRT_CUDA(cudaMalloc(&m->prompt, 4ull * P));
    VRT_CUDA(cudaMalloc(&m->st, sizeof(StepState)));
    VRT_CUDA(cudaMemsetAsync(m->st, 0, sizeof(StepState), ctx->stream));
    VRT_CUDA(cudaMalloc(&m->key_tmp, 8));
    VRT_CUDA(cudaMallocHost(&m->st_host, sizeof(StepState)));
    VRT_CUDA(cudaMallocHost(&m->hidden_host, 4ull * d));
    VRT_CUDA(cudaStreamSynchronize(ctx->stream));
    return VRT_OK;
}

// ------------------------------------------------------- weight loading

// Streaming Q8_0 upload: the GGUF file is memory-mapped; row runs are copied
// into one of kLoadBufs pinned staging buffers by host worker threads, then
// uploaded and repacked into the Q8T layout on the device stream.  A buffer
// is refilled only after the CUDA event recorded behind its repack has
// completed, so the host copy of chunk k+1 overlaps the upload and repack of
// chunk k (the reference uploads 32 MiB chunks synchronously,
// src/gemma3.cpp:571-600).
struct Loader {
    static constexpr int kLoadBufs = 3;
    vrt_model* m;
    uint8_t* h_stage[kLoadBufs] = {};  // pinned
    uint8_t* d_stage[kLoadBufs] = {};
    cudaEvent_t done[kLoadBufs] = {};
    bool used[kLoadBufs] = {};
    int next = 0;
    uint64_t cap = 32ull << 20;
    unsigned workers = 1;
    ~Loader() {
        if (m) cudaStreamSynchronize(m->ctx->stream);
        for (int i = 0; i < kLoadBufs; ++i) {
            if (h_stage[i]) cudaFreeHost(h_stage[i]);
            if (d_stage[i]) cudaFree(d_stage[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
    }
    int init() {
        for (int i = 0; i < kLoadBufs; ++i) {
            VRT_CUDA(cudaMallocHost(&h_stage[i], cap));
            VRT_CUDA(cudaMalloc(&d_stage[i], cap));
            VRT_CUDA(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        }
        workers = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
        return VRT_OK;
    }
    // all queued uploads and repacks finished
    int finish() {
        VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
        return VRT_OK;
    }
    // rows [r0, r0+nr) x blocks [b0, b0+nb) of a raw Q8_0 tensor -> Q8T destination
    int q8(const uint8_t* src, uint32_t src_cols, uint32_t r0, uint32_t nr, uint32_t b0, uint32_t nb, uint8_t* dst,
           uint32_t dst_cols, uint32_t dst_row0, int mode) {
        const uint64_t src_row_bytes = static_cast<uint64_t>(src_cols) / 32 * 34;
        const uint64_t take = static_cast<uint64_t>(nb) * 34;
        // chunks of whole 8-row groups keep the gate/up interleave aligned
        const uint32_t rows_per = static_cast<uint32_t>(std::max<uint64_t>(8, cap / take / 8 * 8));
        cudaStream_t s = m->ctx->stream;
        for (uint32_t r = 0; r < nr; r += rows_per) {
            const uint32_t n = std::min(rows_per, nr - r);
            const int k = next;
            next = (next + 1) % kLoadBufs;
            if (used[k]) VRT_CUDA(cudaEventSynchronize(done[k]));  // its previous upload + repack are done
            used[k] = true;
            uint8_t* hs = h_stage[k];
            auto copy_rows = [&](uint32_t i0, uint32_t i1) {
                for (uint32_t i = i0; i < i1; ++i) {
                    memcpy(hs + i * take, src + (static_cast<uint64_t>(r0 + r + i)) * src_row_bytes + b0 * 34ull, take);
                }
            };
            const unsigned T = static_cast<uint64_t>(n) * take >= (4ull << 20) ? workers : 1u;
            if (T > 1) {
                std::vector<std::thread> pool;
                for (unsigned t = 1; t < T; ++t) pool.emplace_back(copy_rows, n * t / T, n * (t + 1) / T);
                copy_rows(0, n / T);
                for (auto& th : pool) th.join();
            } else {
                copy_rows(0, n);
            }
            VRT_CUDA(cudaMemcpyAsync(d_stage[k], hs, n * take, cudaMemcpyHostToDevice, s));
            RepackParams p{d_stage[k], take, 0, n, nb, dst, dst_cols, 0, mode};
            if (mode == 0) {
                p.dst_row0 = dst_row0 + r;
            } else {
                // interleave keeps source-row numbering: offset the destination by whole groups
                p.dst = dst + static_cast<uint64_t>(r / 8) * (dst_cols / kTileCols) * kTileBytes;
                if (r % 8) return fail(VRT_E_INVALID, "interleaved repack chunk not group aligned");
            }
            const uint64_t work = static_cast<uint64_t>(n) * nb;
            VRT_CUDA(launch(repack_kernel, dim3(static_cast<unsigned>((work + 255) / 256)), dim3(256), 0, s, false, p));
            VRT_CUDA(cudaEventRecord(done[k], s));
        }
        return VRT_OK;
    }
};

static int read_config(const vortexrt::GgufFile& g, vrt_gemma3_config& c, uint64_t& eos) {
    // Gemma3Model::Gemma3Model config section (src/gemma3.cpp:174-257)
    if (g.metadata_string("general.architecture") != std::optional<std::string>{"gemma3"}) {
        return fail(VRT_E_INVALID, "Gemma3Model requires general.architecture=gemma3");
    }
    auto u32 = [&](const char* key, uint32_t& out) -> int {
        const auto v = g.metadata_u64(key);
        if (!v || *v > 0xffffffffull) return fail(VRT_E_INVALID, "Missing/invalid Gemma 3 metadata: %s", key);
        out = static_cast<uint32_t>(*v);
        return VRT_OK;
    };
    VRT_TRY(u32("gemma3.context_length", c.context_length));
    VRT_TRY(u32("gemma3.embedding_length", c.embedding_length));
    VRT_TRY(u32("gemma3.block_count", c.block_count));
    VRT_TRY(u32("gemma3.feed_forward_length", c.feed_forward_length));
    VRT_TRY(u32("gemma3.attention.head_count", c.head_count));
    VRT_TRY(u32("gemma3.attention.head_count_kv", c.head_count_kv));
    VRT_TRY(u32("gemma3.attention.key_length", c.head_dim));
    VRT_TRY(u32("gemma3.attention.value_length", c.value_dim));
    const auto* eps = g.find_metadata("gemma3.attention.layer_norm_rms_epsilon");
    if (!eps) return fail(VRT_E_INVALID, "Missing Gemma 3 metadata: gemma3.attention.layer_norm_rms_epsilon");
    const auto ev = eps->as_f64();
    if (!ev || !std::isfinite(*ev)) return fail(VRT_E_INVALID, "Invalid Gemma 3 floating metadata: gemma3.attention.layer_norm_rms_epsilon");
    c.rms_epsilon = static_cast<float>(*ev);
    c.sliding_window = 0;
    if (const auto sw = g.metadata_u64("gemma3.attention.sliding_window"); sw && *sw <= 0xffffffffull) {
        c.sliding_window = static_cast<uint32_t>(*sw);
    }
    c.global_rope_base = 1.0e6f;
    c.local_rope_base = 1.0e4f;
    if (const auto* r = g.find_metadata("gemma3.rope.freq_base")) {
        if (const auto v = r->as_f64(); v && std::isfinite(*v) && *v > 0.0) c.global_rope_base = static_cast<float>(*v);
    }
    const auto* emb = g.find_tensor("token_embd.weight");
    if (!emb) return fail(VRT_E_INVALID, "Missing Gemma 3 tensor: token_embd.weight");
    if (emb->type != 8 || emb->dimensions.size() != 2 || emb->dimensions[0] != c.embedding_length ||
        emb->dimensions[1] > 0xffffffffull) {
        return fail(VRT_E_INVALID, "Unsupported token_embd.weight layout");
    }
    c.vocab_size = static_cast<uint32_t>(emb->dimensions[1]);
    eos = g.metadata_u64("tokenizer.ggml.eos_token_id").value_or(1);
    return validate_config(c);
}

static int load_weights(vrt_model* m, const vortexrt::GgufFile& g) {
    const auto& c = m->cfg;
    const uint32_t d = c.embedding_length, hd = c.head_dim;
    Loader ld{m};
    VRT_TRY(ld.init());
    auto q8 = [&](const std::string& name, uint64_t cols, uint64_t rows) -> const uint8_t* {
        const auto* t = g.find_tensor(name);
        if (!t || t->type != 8 || t->dimensions.size() != 2 || t->dimensions[0] != cols || t->dimensions[1] != rows) {
            return nullptr;
        }
        return g.tensor_data(*t);
    };
    // norm vectors: checked now, copied after the Q8_0 stream (a synchronous
    // copy in between would drain the upload pipeline)
    std::vector<std::pair<uint64_t, std::pair<const uint8_t*, uint64_t>>> norms;
    auto f32 = [&](const std::string& name, uint64_t n, uint64_t dst) -> int {
        const auto* t = g.find_tensor(name);
        if (!t || t->type != 0 || t->dimensions.size() != 1 || t->dimensions[0] != n) {
            return fail(VRT_E_INVALID, "Missing or mis-shaped Gemma 3 tensor: %s", name.c_str());
        }
        norms.push_back({dst, {g.tensor_data(*t), n * 4}});
        return VRT_OK;
    };
    const uint8_t* emb = q8("token_embd.weight", d, c.vocab_size);
    if (!emb) return fail(VRT_E_INVALID, "Unsupported token_embd.weight layout");
    VRT_TRY(ld.q8(emb, d, 0, c.vocab_size, 0, d / 32, m->arena + m->embd, d, 0, 0));
    const uint32_t h0 = m->Hl * m->rank, g0 = m->KVl * m->rank, f0 = m->ffl * m->rank;
    for (uint32_t l = 0; l < c.block_count; ++l) {
        const auto& L = m->layers[l];
        const uint8_t* wq = q8(lname(l, "attn_q.weight"), d, static_cast<uint64_t>(c.head_count) * hd);
        const uint8_t* wk = q8(lname(l, "attn_k.weight"), d, static_cast<uint64_t>(c.head_count_kv) * hd);
        const uint8_t* wv = q8(lname(l, "attn_v.weight"), d, static_cast<uint64_t>(c.head_count_kv) * hd);
        const uint8_t* wo = q8(lname(l, "attn_output.weight"), static_cast<uint64_t>(c.head_count) * hd, d);
        const uint8_t* wg = q8(lname(l, "ffn_gate.weight"), d, c.feed_forward_length);
        const uint8_t* wu = q8(lname(l, "ffn_up.weight"), d, c.feed_forward_length);
        const uint8_t* wd = q8(lname(l, "ffn_down.weight"), c.feed_forward_length, d);
        if (!wq || !wk || !wv || !wo || !wg || !wu || !wd) {
            return fail(VRT_E_INVALID, "Missing or mis-shaped Q8_0 projection in layer %u", l);
        }
        uint8_t* qkv = m->arena + L.qkv;
        VRT_TRY(ld.q8(wq, d, h0 * hd, m->qwl, 0, d / 32, qkv, d, 0, 0));
        VRT_TRY(ld.q8(wk, d, g0 * hd, m->kwl, 0, d / 32, qkv, d, m->qwl, 0));
        VRT_TRY(ld.q8(wv, d, g0 * hd, m->kwl, 0, d / 32, qkv, d, m->qwl + m->kwl, 0));
        VRT_TRY(ld.q8(wo, c.head_count * hd, 0, d, h0 * hd / 32, m->qwl / 32, m->arena + L.o, m->qwl, 0, 0));
        VRT_TRY(ld.q8(wg, d, f0, m->ffl, 0, d / 32, m->arena + L.gu, d, 0, 1));
        VRT_TRY(ld.q8(wu, d, f0, m->ffl, 0, d / 32, m->arena + L.gu, d, 0, 2));
        VRT_TRY(ld.q8(wd, c.feed_forward_length, 0, d, f0 / 32, m->ffl / 32, m->arena + L.down, m->ffl, 0, 0));
        VRT_TRY(f32(lname(l, "attn_norm.weight"), d, L.n_attn));
        VRT_TRY(f32(lname(l, "attn_q_norm.weight"), hd, L.n_q));
        VRT_TRY(f32(lname(l, "attn_k_norm.weight"), hd, L.n_k));
        VRT_TRY(f32(lname(l, "post_attention_norm.weight"), d, L.n_post_attn));
        VRT_TRY(f32(lname(l, "ffn_norm.weight"), d, L.n_ffn));
        VRT_TRY(f32(lname(l, "post_ffw_norm.weight"), d, L.n_post_ffw));
    }
    VRT_TRY(f32("output_norm.weight", d, m->out_norm));
    VRT_TRY(ld.finish());
    for (const auto& nv : norms) {
        VRT_CUDA(cudaMemcpy(m->arena + nv.first, nv.second.first, nv.second.second, cudaMemcpyHostToDevice));
    }
    return VRT_OK;
}

static int synth_weights(vrt_model* m, uint64_t seed) {
    const auto& c = m->cfg;
    const uint32_t d = c.embedding_length, hd = c.head_dim;
    cudaStream_t s = m->ctx->stream;
    const float mult_w = static_cast<float>(0.02 / 37837.2265);
    const float mult_n = static_cast<float>(0.1 / 37837.2265);
    auto gen = [&](const std::string& name, uint32_t cols_full, uint32_t r0, uint32_t nr, uint32_t b0, uint32_t nb,
                   uint64_t dst, uint32_t dst_cols, uint32_t dst_row0, int mode) -> int {
        SynthParams p{stream_key(seed, name), cols_full, r0, nr, b0, nb, mult_w, m->arena + dst, dst_cols, dst_row0, mode};
        const uint64_t work = static_cast<uint64_t>(nr) * nb;
        VRT_CUDA(launch(synth_q8_kernel, dim3(static_cast<unsigned>((work + 255) / 256)), dim3(256), 0, s, false, p));
        return VRT_OK;
    };
    auto norm = [&](const std::string& name, uint32_t n, uint64_t dst) -> int {
        VRT_CUDA(launch(synth_norm_kernel, dim3((n + 255) / 256), dim3(256), 0, s, false, stream_key(seed, name), n,
                        mult_n, reinterpret_cast<float*>(m->arena + dst)));
        return VRT_OK;
    };
    VRT_TRY(gen("token_embd.weight", d, 0, c.vocab_size, 0, d / 32, m->embd, d, 0, 0));
    const uint32_t h0 = m->Hl * m->rank, g0 = m->KVl * m->rank, f0 = m->ffl * m->rank;
    for (uint32_t l = 0; l < c.block_count; ++l) {
        const auto& L = m->layers[l];
        VRT_TRY(gen(lname(l, "attn_q.weight"), d, h0 * hd, m->qwl, 0, d / 32, L.qkv, d, 0, 0));
        VRT_TRY(gen(lname(l, "attn_k.weight"), d, g0 * hd, m->kwl, 0, d / 32, L.qkv, d, m->qwl, 0));
        VRT_TRY(gen(lname(l, "attn_v.weight"), d, g0 * hd, m->kwl, 0, d / 32, L.qkv, d, m->qwl + m->kwl, 0));
        VRT_TRY(gen(lname(l, "attn_output.weight"), c.head_count * hd, 0, d, h0 * hd / 32, m->qwl / 32, L.o, m->qwl, 0, 0));
        VRT_TRY(gen(lname(l, "ffn_gate.weight"), d, f0, m->ffl, 0, d / 32, L.gu, d, 0, 1));
        VRT_TRY(gen(lname(l, "ffn_up.weight"), d, f0, m->ffl, 0, d / 32, L.gu, d, 0, 2));
        VRT_TRY(gen(lname(l, "ffn_down.weight"), c.feed_forward_length, 0, d, f0 / 32, m->ffl / 32, L.down, m->ffl, 0, 0));
        VRT_TRY(norm(lname(l, "attn_norm.weight"), d, L.n_attn));
        VRT_TRY(norm(lname(l, "attn_q_norm.weight"), hd, L.n_q));
        VRT_TRY(norm(lname(l, "attn_k_norm.weight"), hd, L.n_k));
        VRT_TRY(norm(lname(l, "post_attention_norm.weight"), d, L.n_post_attn));
        VRT_TRY(norm(lname(l, "ffn_norm.weight"), d, L.n_ffn));
        VRT_TRY(norm(lname(l, "post_ffw_norm.weight"), d, L.n_post_ffw));
    }
    VRT_TRY(norm("output_norm.weight", d, m->out_norm));
    VRT_CUDA(cudaStreamSynchronize(s));
    return VRT_OK;
}

// ------------------------------------------------------------ the step

static int nccl_sum(vrt_model* m, float* buf, size_t n, cudaStream_t s) {
    if (m->world <= 1) return VRT_OK;
    const int r = m->nccl.AllReduce(buf, buf, n, /*ncclFloat32*/ 7, /*ncclSum*/ 0, m->comm, s);
    if (r) return fail(VRT_E_CUDA, "ncclAllReduce failed: %s", m->nccl.GetErrorString(r));
    return VRT_OK;
}

// Tensor parallelism, batched paths: the per-row argmax keys (64-bit,
// value-ordered) maximised over the ranks' vocabulary shards.
static int nccl_key_max(vrt_model* m, unsigned long long* keys, size_t n, cudaStream_t s) {
    if (m->world <= 1) return VRT_OK;
    const int r = m->nccl.AllReduce(keys, keys, n, /*ncclUint64*/ 5, /*ncclMax*/ 2, m->comm, s);
    if (r) return fail(VRT_E_CUDA, "ncclAllReduce(max) failed: %s", m->nccl.GetErrorString(r));
    return VRT_OK;
}

// Exchange parameters of one consumer of row-parallel partial sums.  Ops are
// numbered per step: 2l = attention output of layer l (slot set 0), 2l+1 =
// FFN down of layer l (set 1), 2L = the argmax key.
static TpParams tp_params(vrt_model* m, uint32_t set, uint32_t op, const float* local) {
    TpParams t{};
    if (!m->tp_peer) return t;
    const uint32_t d = m->cfg.embedding_length;
    t.peers = m->tp_peers_dev;
    t.slots = m->tp_slots;
    t.local = local;
    t.sum = m->tp_sum + static_cast<uint64_t>(set) * d;
    t.bar_count = m->tp_bar;
    t.bar_gen = m->tp_bar + 1;
    t.epoch = &m->st->epoch;
    t.wait_ns = static_cast<uint64_t>(m->opt.tp_wait_ms ? m->opt.tp_wait_ms : 10000u) * 1000000ull;
    t.rank = static_cast<uint32_t>(m->rank);
    t.world = static_cast<uint32_t>(m->world);
    t.set = set;
    t.op = op;
    t.ops_per_step = 2 * m->cfg.block_count + 1;
    t.n = d;
    return t;
}

// The mat-vecs of one decode step, in launch order: weight base, rows, cols,
// and whether the epilogue partitions by whole row groups.
struct StepGemv {
    const uint8_t* w;
    uint32_t rows, cols;
    bool group;
};

static std::vector<StepGemv> step_gemvs(vrt_model* m, bool head) {
    const auto& c = m->cfg;
    const uint32_t d = c.embedding_length;
    std::vector<StepGemv> v;
    for (uint32_t l = 0; l < c.block_count; ++l) {
        const auto& L = m->layers[l];
        v.push_back({m->arena + L.qkv, m->qwl + 2 * m->kwl, d, false});
        v.push_back({m->arena + L.o, d, m->qwl, false});
        v.push_back({m->arena + L.gu, 2 * m->ffl, d, true});
        v.push_back({m->arena + L.down, d, m->ffl, false});
    }
    if (head) {
        const uint32_t kt = d / kTileCols;
        v.push_back({m->arena + m->embd + static_cast<uint64_t>(m->vocab_lo / kTileRows) * kt * kTileBytes,
                     m->vocab_hi - m->vocab_lo, d, true});
    }
    return v;
}

// ------------------------------------------------ persistent decode step

// Most planes (CTAs holding a part of one row group) of a tile-granular span
// of a rows x cols matrix over G CTAs.
static uint32_t ps_max_planes(uint32_t rows, uint32_t cols, uint32_t G) {
    const uint32_t kt = cols / kTileCols, groups = (rows + kTileRows - 1) / kTileRows, total = groups * kt;
    uint32_t mx = 1;
    for (uint32_t g = 0; g < groups; ++g) mx = std::max(mx, ps_planes_of(g, kt, total, G, nullptr));
    return mx;
}

// Whether the step runs as one persistent kernel, and its sizes (grid, ring,
// exchange planes, attention splits).  Host arithmetic plus kernel attribute
// queries; runs before the tensor-parallel slots are allocated, since those
// hold the kernel's receive areas.  Every CTA must own part of every
// projection (the grid is capped by the smallest one): the order in which
// exchange buffers are reused relies on each CTA publishing words in every op.
static int ps_plan(vrt_model* m) {
    m->ps_on = false;
    if (m->opt.step_mode != VRT_STEP_PERSISTENT) return VRT_OK;
    if (m->world > 1 && m->opt.tp_exchange != VRT_TP_PEER) return VRT_OK;
    const auto& c = m->cfg;
    const uint32_t d = c.embedding_length, hd = c.head_dim;
    if (m->KVl == 0 || m->Hl % m->KVl != 0 || m->Hl / m->KVl > 8) return VRT_OK;
    if (hd != 64 && hd != 128 && hd != 256) return VRT_OK;
    auto tiles = [](uint64_t r, uint64_t k) { return (r + kTileRows - 1) / kTileRows * (k / kTileCols); };
    const uint32_t qkv_rows = m->qwl + 2 * m->kwl;
    uint64_t G = static_cast<uint64_t>(m->ctx->prop.multiProcessorCount);
    G = std::min<uint64_t>(G, tiles(qkv_rows, d));
    G = std::min<uint64_t>(G, tiles(d, m->qwl));
    G = std::min<uint64_t>(G, (2ull * m->ffl + kTileRows - 1) / kTileRows);
    G = std::min<uint64_t>(G, tiles(d, m->ffl));
    if (G < 1) return VRT_OK;
    // the device partition arithmetic is 32-bit: (tiles + 1) * G must fit
    const uint64_t most = std::max({tiles(qkv_rows, d), tiles(d, m->qwl), tiles(2ull * m->ffl, d), tiles(d, m->ffl),
                                    tiles(m->vocab_hi - m->vocab_lo, d)});
    if ((most + 1) * G >= (1ull << 32)) return VRT_OK;
    const uint32_t g32 = static_cast<uint32_t>(G);
    PsParams p{};
    p.L = c.block_count;
    p.d = d;
    p.H = m->Hl;
    p.KV = m->KVl;
    p.hd = hd;
    p.qw = m->qwl;
    p.kw = m->kwl;
    p.ff = m->ffl;
    p.vocab = c.vocab_size;
    p.vl = m->vocab_hi - m->vocab_lo;
    p.row_base = m->vocab_lo;
    p.eps = c.rms_epsilon;
    p.emb_scale = std::sqrt(static_cast<float>(d));
    p.att_scale = 1.0f / std::sqrt(static_cast<float>(hd));
    p.rg = ps_rg_of(p.H, p.KV);
    p.planes_qkv = ps_max_planes(qkv_rows, d, g32);
    p.planes_rx = std::max(ps_max_planes(d, m->qwl, g32), ps_max_planes(d, m->ffl, g32));
    if (p.planes_qkv > static_cast<uint32_t>(kPsMaxSlots) ||
        p.planes_rx * static_cast<uint32_t>(m->world) > static_cast<uint32_t>(kPsMaxSlots)) {
        return VRT_OK;
    }
    p.s_max = std::max(1u, std::min(64u, g32 / p.KV));
    p.min_split = 64;
    // tuning overrides (attention split size and count)
    if (const char* e = getenv("VRT_PS_MIN_SPLIT")) p.min_split = std::max(1u, static_cast<uint32_t>(atoi(e)));
    if (const char* e = getenv("VRT_PS_SPLITS")) p.s_max = std::max(1u, std::min(p.s_max, static_cast<uint32_t>(atoi(e))));
    // LM-head rows prefetched into L2 while the last layers run: up to half of
    // L2 over the grid, issued from the first layer after which the remaining
    // layer weights fit in the other half.
    const uint64_t l2 = static_cast<uint64_t>(m->ctx->prop.l2CacheSize);
    const uint64_t layer_bytes = q8t_bytes(qkv_rows, d) + q8t_bytes(d, m->qwl) + q8t_bytes(2ull * m->ffl, d) +
                                 q8t_bytes(d, m->ffl);
    uint32_t pf_layer = p.L - 1;
    while (pf_layer > 0 && layer_bytes * (p.L - pf_layer + 1) <= l2 / 2) --pf_layer;
    p.head_pf_layer = pf_layer;
    p.head_pf_bytes = static_cast<uint32_t>(std::min<uint64_t>(l2 / 2 / G, 1u << 30) & ~uint64_t(15));
    if (const char* e = getenv("VRT_PS_HEAD_PF")) p.head_pf_bytes = static_cast<uint32_t>(atoi(e)) & ~15u;  // tuning
    const uint32_t wait_ms = m->opt.tp_wait_ms ? m->opt.tp_wait_ms : (m->world > 1 ? 10000u : 2000u);
    p.wait_ns = static_cast<uint64_t>(wait_ms) * 1000000ull;
    p.rank = static_cast<uint32_t>(m->rank);
    p.world = static_cast<uint32_t>(m->world);
    uint32_t max_dyn = 0;
    int blocks = 0;
    VRT_CUDA(ps_limits(hd, p.rg, 0, &max_dyn, nullptr));
    p.ns = ps_ring_stages(p, max_dyn);
    if (p.ns < 2) return VRT_OK;
    const uint32_t smem = ps_smem_layout(p, p.ns).total;
    VRT_CUDA(ps_limits(hd, p.rg, smem, &max_dyn, &blocks));
    if (blocks < 1) return VRT_OK;
    m->ps = p;
    m->ps_smem = smem;
    m->ps_grid = g32;
    m->ps_on = true;
    return VRT_OK;
}

// Device memory of the persistent step: layer table, exchange words (zero:
// tag 0 never matches a sequence number), split scratch, tickets, and the
// receive-area table (single GPU: a local area; tensor parallel: every rank's
// area inside its mapped peer slots).
static int ps_alloc(vrt_model* m) {
    if (!m->ps_on) return VRT_OK;
    PsParams& p = m->ps;
    const auto& c = m->cfg;
    const uint32_t L = p.L, d = p.d, W = p.world;
    const uint64_t qkv_rows = p.qw + 2ull * p.kw;
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t o = off;
        off = align256(off + bytes);
        return o;
    };
    const uint64_t o_layers = take(sizeof(PsLayer) * L);
    const uint64_t o_qkv = take(8ull * 2 * p.planes_qkv * qkv_rows);
    const uint64_t o_att = take(8ull * 2 * p.qw);
    const uint64_t o_act = take(8ull * 2 * p.ff);
    const uint64_t o_ml = take(4ull * p.H * p.s_max * 2);
    const uint64_t o_acc = take(4ull * p.H * p.s_max * p.hd);
    const uint64_t o_tk = take(4ull * (p.KV + 1));
    const uint64_t o_rxt = take(8ull * W);
    const uint64_t o_rx = W > 1 ? 0 : take(8ull * ps_rx_words(1, p.planes_rx, d));
    VRT_CUDA(cudaMalloc(&m->ps_mem, off));
    VRT_CUDA(cudaMemsetAsync(m->ps_mem, 0, off, m->ctx->stream));
    uint8_t* base = static_cast<uint8_t*>(m->ps_mem);
    auto F = [&](uint64_t o) { return reinterpret_cast<const float*>(m->arena + o); };
    std::vector<PsLayer> ly(L);
    for (uint32_t l = 0; l < L; ++l) {
        const auto& S = m->layers[l];
        PsLayer& t = ly[l];
        t.qkv = m->arena + S.qkv;
        t.o = m->arena + S.o;
        t.gu = m->arena + S.gu;
        t.down = m->arena + S.down;
        t.n_attn = F(S.n_attn);
        t.n_q = F(S.n_q);
        t.n_k = F(S.n_k);
        t.n_post_attn = F(S.n_post_attn);
        t.n_ffn = F(S.n_ffn);
        t.n_post_ffw = F(S.n_post_ffw);
        t.k_cache = S.k_cache;
        t.v_cache = S.v_cache;
        t.rope_cos = S.global ? m->rope_cos_g : m->rope_cos_l;
        t.rope_sin = S.global ? m->rope_sin_g : m->rope_sin_l;
        t.cap = S.cap;
        t.window = S.global ? 0u : c.sliding_window;
    }
    std::vector<unsigned long long*> rx(W);
    for (uint32_t r = 0; r < W; ++r) {
        rx[r] = W > 1 ? m->tp_peer_slots[r] + m->ps_rx_offset : reinterpret_cast<unsigned long long*>(base + o_rx);
    }
    VRT_CUDA(cudaMemcpyAsync(base + o_layers, ly.data(), sizeof(PsLayer) * L, cudaMemcpyHostToDevice, m->ctx->stream));
    VRT_CUDA(cudaMemcpyAsync(base + o_rxt, rx.data(), 8ull * W, cudaMemcpyHostToDevice, m->ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    p.layers = reinterpret_cast<const PsLayer*>(base + o_layers);
    p.x_qkv = reinterpret_cast<unsigned long long*>(base + o_qkv);
    p.x_att = reinterpret_cast<unsigned long long*>(base + o_att);
    p.x_act = reinterpret_cast<unsigned long long*>(base + o_act);
    p.part_ml = reinterpret_cast<float*>(base + o_ml);
    p.part_acc = reinterpret_cast<float*>(base + o_acc);
    p.att_tickets = reinterpret_cast<uint32_t*>(base + o_tk);
    p.fin_ticket = p.att_tickets + p.KV;
    p.rx = reinterpret_cast<unsigned long long* const*>(base + o_rxt);
    const uint32_t kt = d / kTileCols;
    p.embd = m->arena + m->embd;
    p.lm = m->arena + m->embd + static_cast<uint64_t>(m->vocab_lo / kTileRows) * kt * kTileBytes;
    p.out_norm = F(m->out_norm);
    p.st = m->st;
    p.out_ids = m->out_ids;
    p.out_cap = kMaxSteps;
    p.prompt = m->prompt;
    p.hidden = m->hidden;
    p.logits = m->logits;
    p.trace = nullptr;
#ifdef VRT_PS_STAMPS
    VRT_CUDA(cudaMalloc(&p.stamps, 8ull * m->ps_grid * ps_stamp_count(L)));
    VRT_CUDA(cudaMemset(p.stamps, 0, 8ull * m->ps_grid * ps_stamp_count(L)));
#endif
    return VRT_OK;
}

static int record_step(vrt_model* m, cudaStream_t s, bool head, uint32_t* kernels) {
    if (m->ps_on) {
        PsParams p = m->ps;
        p.head = head ? 1u : 0u;
        p.trace = m->trace_on ? m->trace : nullptr;
        VRT_CUDA(ps_launch(p, m->ps_grid, m->ps_smem, s));
        if (kernels) *kernels = 1;
        return VRT_OK;
    }
    const auto& c = m->cfg;
    const bool pdl = m->opt.use_pdl != 0;
    const int sms = m->ctx->prop.multiProcessorCount;
    const uint32_t d = c.embedding_length, hd = c.head_dim;
    uint32_t nk = 0;
    uint32_t* status = &m->st->status;
    float* trace = m->trace_on ? m->trace : nullptr;
    auto F = [&](uint64_t off) { return reinterpret_cast<const float*>(m->arena + off); };
    // next-kernel L2 prefetch chain; the step's last mat-vec points at the
    // first one (the next step starts with it)
    const std::vector<StepGemv> seq = step_gemvs(m, head);
    size_t gi = 0;
    auto gemv = [&](int pro, int epi, GemvParams p) -> int {
        p.status = status;
        p.eps = c.rms_epsilon;
        const StepGemv& nx = seq[(gi + 1) % seq.size()];
        p.next_w = nx.w;
        p.next_rows = nx.rows;
        p.next_cols = nx.cols;
        p.next_grid = static_cast<uint32_t>(gemv_grid(sms, nx.rows));
        p.next_group = nx.group ? 1u : 0u;
        p.pf_bytes = 64u * 1024u;
        p.stamp = nk;
        ++gi;
        VRT_CUDA(gemv_q8t(pro, epi, p, gemv_grid(sms, p.rows), s, pdl));
        ++nk;
        return VRT_OK;
    };
    for (uint32_t l = 0; l < c.block_count; ++l) {
        const auto& L = m->layers[l];
        // QKV
        {
            GemvParams p{};
            p.w = m->arena + L.qkv;
            p.rows = m->qwl + 2 * m->kwl;
            p.cols = d;
            p.w_pre = F(L.n_attn);
            p.h_out = m->h0;
            p.y = m->qkv;
            if (l == 0) {
                p.embd = m->arena + m->embd;
                p.token = &m->st->token;
                p.vocab = c.vocab_size;
                p.emb_scale = std::sqrt(static_cast<float>(d));
                VRT_TRY(gemv(kProEmbed, kEpiAtomic, p));
            } else {
                p.x = m->tp_peer ? m->tp_sum + d : m->dn;
                p.tp = tp_params(m, 1, 2 * (l - 1) + 1, m->dn);
                p.h_prev = m->h1;
                p.w_post = F(m->layers[l - 1].n_post_ffw);
                p.trace = trace ? trace + static_cast<uint64_t>(l - 1) * d : nullptr;
                VRT_TRY(gemv(kProResid, kEpiAtomic, p));
            }
        }
        // attention (clears dn for this layer's down projection)
        {
            AttnParams a{};
            a.qkv = m->qkv;
            a.q_norm = F(L.n_q);
            a.k_norm = F(L.n_k);
            a.rope_cos = L.global ? m->rope_cos_g : m->rope_cos_l;
            a.rope_sin = L.global ? m->rope_sin_g : m->rope_sin_l;
            a.k_cache = L.k_cache;
            a.v_cache = L.v_cache;
            a.cap = L.cap;
            a.window = L.global ? 0u : c.sliding_window;
            a.pos = &m->st->pos;
            a.H = m->Hl;
            a.KV = m->KVl;
            a.hd = hd;
            a.eps = c.rms_epsilon;
            a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
            a.part_ml = m->part_ml;
            a.part_acc = m->part_acc;
            a.tickets = m->tickets;
            a.out = m->att;
            a.splits = L.splits;
            a.zero0 = m->dn;
            a.zero0_count = d;
            a.stamp = nk;
            VRT_CUDA(attention_launch(a, dim3(L.splits, m->KVl), s, pdl));
            ++nk;
        }
        // o-proj (clears qkv for the next QKV)
        {
            GemvParams p{};
            p.w = m->arena + L.o;
            p.rows = d;
            p.cols = m->qwl;
            p.x = m->att;
            p.y = m->o;
            p.zero0 = m->qkv;
            p.zero0_count = m->qwl + 2 * m->kwl;
            VRT_TRY(gemv(kProPlain, kEpiAtomic, p));
            if (!m->tp_peer) VRT_TRY(nccl_sum(m, m->o, d, s));
        }
        // gate/up with residual + post-attention norm + ffn norm
        {
            GemvParams p{};
            p.w = m->arena + L.gu;
            p.rows = 2 * m->ffl;
            p.cols = d;
            p.x = m->tp_peer ? m->tp_sum : m->o;
            p.tp = tp_params(m, 0, 2 * l, m->o);
            p.h_prev = m->h0;
            p.w_post = F(L.n_post_attn);
            p.w_pre = F(L.n_ffn);
            p.h_out = m->h1;
            p.y = m->act;
            VRT_TRY(gemv(kProResid, kEpiGeluPair, p));
        }
        // down (clears o for the next o-proj)
        {
            GemvParams p{};
            p.w = m->arena + L.down;
            p.rows = d;
            p.cols = m->ffl;
            p.x = m->act;
            p.y = m->dn;
            p.zero0 = m->o;
            p.zero0_count = d;
            VRT_TRY(gemv(kProPlain, kEpiAtomic, p));
            if (!m->tp_peer) VRT_TRY(nccl_sum(m, m->dn, d, s));
        }
    }
    const auto& last = m->layers[c.block_count - 1];
    float* tlast = trace ? trace + static_cast<uint64_t>(c.block_count - 1) * d : nullptr;
    if (head) {
        GemvParams p{};
        const uint32_t kt = d / kTileCols;
        p.w = m->arena + m->embd + static_cast<uint64_t>(m->vocab_lo / kTileRows) * kt * kTileBytes;
        p.rows = m->vocab_hi - m->vocab_lo;
        p.cols = d;
        p.x = m->tp_peer ? m->tp_sum + d : m->dn;
        p.tp = tp_params(m, 1, 2 * c.block_count - 1, m->dn);
        p.h_prev = m->h1;
        p.w_post = F(last.n_post_ffw);
        p.w_pre = F(m->out_norm);
        p.h_out = m->hidden;
        p.trace = tlast;
        p.y = m->logits;
        p.amax = &m->st->key;
        p.row_base = m->vocab_lo;
        VRT_TRY(gemv(kProResidFinal, kEpiArgmax, p));
        if (m->world > 1 && !m->tp_peer) {
            const int r = m->nccl.AllReduce(&m->st->key, &m->st->key, 1, /*ncclUint64*/ 5, /*ncclMax*/ 2, m->comm, s);
            if (r) return fail(VRT_E_CUDA, "ncclAllReduce(max) failed: %s", m->nccl.GetErrorString(r));
        }
        VRT_CUDA(launch(finalize_decode_kernel, dim3(1), dim3(1), 0, s, pdl && (m->world <= 1 || m->tp_peer), m->st,
                        c.vocab_size, m->out_ids, kMaxSteps, tp_params(m, 0, 2 * c.block_count, nullptr)));
        nk += 1;
    } else {
        VRT_CUDA(launch(final_hidden_kernel, dim3(1), dim3(1024), d * 4, s, pdl, (const float*)m->dn,
                        (const float*)m->h1, F(last.n_post_ffw), F(m->out_norm), m->hidden, tlast, d, c.rms_epsilon,
                        status, tp_params(m, 1, 2 * c.block_count - 1, m->dn)));
        VRT_CUDA(launch(finalize_prefill_kernel, dim3(1), dim3(1), 0, s, pdl, m->st, (const uint32_t*)m->prompt));
        nk += 2;
    }
    if (kernels) *kernels = nk;
    return VRT_OK;
}

static int build_graphs(vrt_model* m) {
    if (!m->opt.use_graph) return VRT_OK;
    for (int head = 0; head < 2; ++head) {
        cudaGraph_t g = nullptr;
        cudaStream_t s = m->ctx->stream;
        VRT_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        uint32_t nk = 0;
        const int rc = record_step(m, s, head != 0, &nk);
        const cudaError_t e = cudaStreamEndCapture(s, &g);
        if (rc != VRT_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture", __FILE__, __LINE__);
        cudaGraphExec_t ex = nullptr;
        const cudaError_t ei = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (ei != cudaSuccess) return cuda_fail(ei, "cudaGraphInstantiate", __FILE__, __LINE__);
        (head ? m->g_head : m->g_nohead) = ex;
        if (head) m->kernels_per_step = nk;
    }
    return VRT_OK;
}

static int run_step(vrt_model* m, bool head) {
    cudaStream_t s = m->ctx->stream;
    cudaGraphExec_t ex = head ? m->g_head : m->g_nohead;
    if (ex) {
        VRT_CUDA(cudaGraphLaunch(ex, s));
        return VRT_OK;
    }
    return record_step(m, s, head, nullptr);
}

// Peer-memory exchange set-up: allocate and export this rank's receive
// slots, gather every rank's CUDA IPC handle with one NCCL all-gather, map
// the peers' slots (NVLink peer access).
static int tp_peer_setup(vrt_model* m) {
    const uint32_t d = m->cfg.embedding_length, W = static_cast<uint32_t>(m->world);
    cudaStream_t s = m->ctx->stream;
    // the persistent step's receive area follows the exchange slots
    m->ps_rx_offset = tp_slot_words(W, d);
    const uint64_t bytes = (tp_slot_words(W, d) + (m->ps_on ? ps_rx_words(W, m->ps.planes_rx, d) : 0)) * 8;
    VRT_CUDA(cudaMalloc(&m->tp_slots, bytes));
    VRT_CUDA(cudaMemsetAsync(m->tp_slots, 0, bytes, s));
    VRT_CUDA(cudaMalloc(&m->tp_sum, 2ull * d * 4 + 256));
    VRT_CUDA(cudaMemsetAsync(m->tp_sum, 0, 2ull * d * 4 + 256, s));
    m->tp_bar = reinterpret_cast<uint32_t*>(m->tp_sum + 2ull * d);
    cudaIpcMemHandle_t h;
    VRT_CUDA(cudaIpcGetMemHandle(&h, m->tp_slots));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    uint8_t* dh = nullptr;
    VRT_CUDA(cudaMalloc(&dh, 64ull * W));
    std::vector<cudaIpcMemHandle_t> hs(W);
    cudaError_t e = cudaMemcpyAsync(dh + 64ull * m->rank, &h, 64, cudaMemcpyHostToDevice, s);
    const int r = e == cudaSuccess ? m->nccl.AllGather(dh + 64ull * m->rank, dh, 64, /*ncclUint8*/ 1, m->comm, s) : 0;
    if (e == cudaSuccess && !r) e = cudaMemcpyAsync(hs.data(), dh, 64ull * W, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && !r) e = cudaStreamSynchronize(s);
    cudaFree(dh);
    if (r) return fail(VRT_E_CUDA, "ncclAllGather failed: %s", m->nccl.GetErrorString(r));
    if (e != cudaSuccess) return cuda_fail(e, "IPC handle exchange", __FILE__, __LINE__);
    m->tp_peer_slots.assign(W, nullptr);
    for (uint32_t q = 0; q < W; ++q) {
        if (q == static_cast<uint32_t>(m->rank)) {
            m->tp_peer_slots[q] = m->tp_slots;
            continue;
        }
        void* ptr = nullptr;
        e = cudaIpcOpenMemHandle(&ptr, hs[q], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            return fail(VRT_E_UNSUPPORTED, "tensor parallelism: cannot map rank %u's memory (%s); tp_exchange = VRT_TP_NCCL "
                        "works without peer access", q, cudaGetErrorString(e));
        }
        m->tp_peer_slots[q] = static_cast<unsigned long long*>(ptr);
    }
    VRT_CUDA(cudaMalloc(&m->tp_peers_dev, 8ull * W));
    VRT_CUDA(cudaMemcpy(m->tp_peers_dev, m->tp_peer_slots.data(), 8ull * W, cudaMemcpyHostToDevice));
    m->tp_peer = true;
    return VRT_OK;
}

// All ranks stop touching each other's slots before any rank unmaps or
// frees them (an NCCL all-reduce of one float on each side).
static void tp_peer_teardown(vrt_model* m) {
    cudaStream_t s = m->ctx->stream;
    auto barrier = [&] {
        if (m->tp_peer && m->comm && m->tp_sum) {
            m->nccl.AllReduce(m->tp_sum, m->tp_sum, 1, /*ncclFloat32*/ 7, /*ncclSum*/ 0, m->comm, s);
            cudaStreamSynchronize(s);
        }
    };
    barrier();
    for (size_t q = 0; q < m->tp_peer_slots.size(); ++q) {
        if (m->tp_peer_slots[q] && m->tp_peer_slots[q] != m->tp_slots) cudaIpcCloseMemHandle(m->tp_peer_slots[q]);
    }
    barrier();
    m->tp_peer_slots.clear();
    m->tp_peer = false;
    cudaFree(m->tp_peers_dev);
    cudaFree(m->tp_sum);
    cudaFree(m->tp_slots);
}

static int finish_create(vrt_model* m) {
    VRT_TRY(ps_plan(m));
    if (m->world > 1) {
        VRT_TRY(nccl_load(m->nccl));
        auto init = reinterpret_cast<CommInitRankFn>(dlsym(m->nccl.lib, "ncclCommInitRank"));
        if (!init) return fail(VRT_E_UNSUPPORTED, "ncclCommInitRank missing");
        NcclId id;
        memcpy(id.b, m->opt.nccl_id, 128);
        const int r = init(&m->comm, m->world, id, m->rank);
        if (r) return fail(VRT_E_CUDA, "ncclCommInitRank failed: %s", m->nccl.GetErrorString(r));
        if (m->opt.tp_exchange == VRT_TP_PEER) VRT_TRY(tp_peer_setup(m));
    }
    VRT_TRY(ps_alloc(m));
    VRT_TRY(build_graphs(m));
    return VRT_OK;
}

static void destroy_model(vrt_model* m) {
    if (!m) return;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->g_head) cudaGraphExecDestroy(m->g_head);
    if (m->g_nohead) cudaGraphExecDestroy(m->g_nohead);
    tp_peer_teardown(m);
    if (m->comm && m->nccl.CommDestroy) m->nccl.CommDestroy(m->comm);
    cudaFree(m->arena);
    cudaFree(m->kv_mem);
    cudaFree(m->rope_cos_l);
    cudaFree(m->act_mem);
    cudaFree(m->tickets);
    cudaFree(m->out_ids);
    cudaFree(m->prompt);
    cudaFree(m->st);
    cudaFree(m->key_tmp);
    cudaFree(m->logits_full);
    cudaFree(m->q8m);
    cudaFree(m->pf.mem);
    cudaFree(m->ps_mem);
    if (m->st_host) cudaFreeHost(m->st_host);
    if (m->hidden_host) cudaFreeHost(m->hidden_host);
    delete m;
}

static int begin_model(vrt_ctx* ctx, const vrt_model_options* opts, vrt_model** out, std::unique_ptr<vrt_model>& m) {
    if (!ctx || !out) return fail(VRT_E_INVALID, "null argument");
    m.reset(new vrt_model());
    m->ctx = ctx;
    vrt_model_options_default(&m->opt);
    if (opts) m->opt = *opts;
    m->world = m->opt.tp_world > 1 ? m->opt.tp_world : 1;
    m->rank = m->world > 1 ? m->opt.tp_rank : 0;
    if (m->world > 1 && (m->rank < 0 || m->rank >= m->world || !m->opt.nccl_id)) {
        return fail(VRT_E_INVALID, "tensor-parallel rank/world/nccl_id invalid");
    }
    if (m->opt.tp_exchange != VRT_TP_PEER && m->opt.tp_exchange != VRT_TP_NCCL) {
        return fail(VRT_E_INVALID, "tp_exchange must be VRT_TP_PEER or VRT_TP_NCCL");
    }
    VRT_CUDA(cudaSetDevice(ctx->device));
    VRT_CUDA(gemv_init_attributes());
    return VRT_OK;
}

// ------------------------------------------------------- batched prefill

static int prefill_alloc(vrt_model* m, uint32_t cap) {
    auto& B = m->pf;
    if (B.cap >= cap) return VRT_OK;
    if (B.mem) {
        VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
        cudaFree(B.mem);
        B = vrt_model::Prefill{};
    }
    const auto& c = m->cfg;
    const uint64_t d = c.embedding_length, hd = c.head_dim, C = cap;
    const uint64_t xw = std::max<uint64_t>(d, m->qwl);
    const uint64_t f32[] = {C * d, C * d, C * (m->qwl + 2ull * m->kwl), C * m->Hl * hd, C * m->KVl * hd,
                            C * m->KVl * hd, C * d, C * d};
    const uint64_t f16[] = {C * xw, C * xw, C * m->ffl, C * m->ffl};
    uint64_t total = 0;
    for (auto n : f32) total += align256(n * 4);
    for (auto n : f16) total += align256(n * 2);
    VRT_CUDA(cudaMalloc(&B.mem, total));
    uint8_t* p = static_cast<uint8_t*>(B.mem);
    float** fd[] = {&B.h0, &B.h1, &B.qkv, &B.q, &B.k, &B.v, &B.o, &B.dn};
    for (int i = 0; i < 8; ++i) {
        *fd[i] = reinterpret_cast<float*>(p);
        p += align256(f32[i] * 4);
    }
    __half** hd16[] = {&B.xh, &B.xl, &B.ah, &B.al};
    for (int i = 0; i < 4; ++i) {
        *hd16[i] = reinterpret_cast<__half*>(p);
        p += align256(f16[i] * 2);
    }
    VRT_CUDA(cudaMemsetAsync(B.mem, 0, total, m->ctx->stream));
    VRT_TRY(make_f16_tmap(&B.xd_hi, B.xh, C, d, 128));
    VRT_TRY(make_f16_tmap(&B.xd_lo, B.xl, C, d, 128));
    VRT_TRY(make_f16_tmap(&B.xq_hi, B.xh, C, m->qwl, 128));
    VRT_TRY(make_f16_tmap(&B.xq_lo, B.xl, C, m->qwl, 128));
    VRT_TRY(make_f16_tmap(&B.xf_hi, B.ah, C, m->ffl, 128));
    VRT_TRY(make_f16_tmap(&B.xf_lo, B.al, C, m->ffl, 128));
    B.cap = cap;
    return VRT_OK;
}

template <int HD, int G>
static cudaError_t prefill_attn_launch_t(const PrefillAttnParams& a, cudaStream_t s) {
    static uint64_t done = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    constexpr uint32_t smem = prefill_attn_smem<HD>();
    if (dev < 64 && !(done & (1ull << dev))) {
        e = cudaFuncSetAttribute(prefill_attention_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        done |= 1ull << dev;
    }
    constexpr uint32_t QB = kPaRows / G;
    const dim3 grid((a.n + QB - 1) / QB, a.KV);
    prefill_attention_kernel<HD, G><<<grid, kPaThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <int HD>
static cudaError_t prefill_attn_launch_hd(const PrefillAttnParams& a, uint32_t G, cudaStream_t s) {
    switch (G) {
    case 1: return prefill_attn_launch_t<HD, 1>(a, s);
    case 2: return prefill_attn_launch_t<HD, 2>(a, s);
    case 4: return prefill_attn_launch_t<HD, 4>(a, s);
    case 8: return prefill_attn_launch_t<HD, 8>(a, s);
    default: return cudaErrorInvalidValue;
    }
}

static cudaError_t prefill_attn_launch(const PrefillAttnParams& a, uint32_t hd, uint32_t G, cudaStream_t s) {
    switch (hd) {
    case 64: return prefill_attn_launch_hd<64>(a, G, s);
    case 128: return prefill_attn_launch_hd<128>(a, G, s);
    case 256: return prefill_attn_launch_hd<256>(a, G, s);
    default: return cudaErrorInvalidValue;
    }
}

static cudaError_t qk_rope_launch(const float* qkv, vrt_model* m, const LayerW& L, uint32_t p0, uint32_t n, float* q,
                                  float* k, float* v, cudaStream_t s) {
    const auto& c = m->cfg;
    auto F = [&](uint64_t off) { return reinterpret_cast<const float*>(m->arena + off); };
    const float* cs = L.global ? m->rope_cos_g : m->rope_cos_l;
    const float* sn = L.global ? m->rope_sin_g : m->rope_sin_l;
    switch (c.head_dim) {
    case 64: qk_rope_rows_kernel<2><<<n, 256, 0, s>>>(qkv, m->Hl, m->KVl, F(L.n_q), F(L.n_k), cs, sn, p0, c.rms_epsilon, q, k, v); break;
    case 128: qk_rope_rows_kernel<4><<<n, 256, 0, s>>>(qkv, m->Hl, m->KVl, F(L.n_q), F(L.n_k), cs, sn, p0, c.rms_epsilon, q, k, v); break;
    case 256: qk_rope_rows_kernel<8><<<n, 256, 0, s>>>(qkv, m->Hl, m->KVl, F(L.n_q), F(L.n_k), cs, sn, p0, c.rms_epsilon, q, k, v); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// Shapes the tensor-core GEMM tiles (128-row weight tiles) and the prefill
// attention is instantiated for (query heads per KV head 1, 2, 4 or 8).
static bool prefill_supported(const vrt_model* m) {
    const uint32_t d = m->cfg.embedding_length, G = m->KVl ? m->Hl / m->KVl : 0;
    return (m->qwl + 2 * m->kwl) % kGemmBN == 0 && d % kGemmBN == 0 && m->qwl % kTileCols == 0 &&
           (2 * m->ffl) % kGemmBN == 0 && m->ffl % kTileCols == 0 && (G == 1 || G == 2 || G == 4 || G == 8);
}

// Where a prefill writes: the sequence's KV caches (per layer base and
// capacity, [KV][cap][hd]), its prompt ids on the device, and the last
// prompt token's LM-head outputs.
struct SeqTarget {
    const uint32_t* prompt = nullptr;
    std::vector<float*> kc, vc;
    std::vector<uint32_t> cap;
    uint32_t positions = 0;              // capacity the caches were sized for
    unsigned long long* key = nullptr;   // argmax key (zero on entry)
    float* hidden = nullptr;             // normed hidden of the last token
    float* logits = nullptr;             // optional full logits of the last token
};

static SeqTarget model_target(vrt_model* m) {
    SeqTarget t;
    t.prompt = m->prompt;
    for (const auto& L : m->layers) {
        t.kc.push_back(L.k_cache);
        t.vc.push_back(L.v_cache);
        t.cap.push_back(L.cap);
    }
    t.positions = m->P;
    t.key = &m->st->key;
    t.hidden = m->hidden;
    t.logits = m->logits;
    return t;
}

// The prompt (t.prompt, n tokens) through every layer in chunks of pf.cap
// tokens, then the fused LM head + argmax on the last token.
static int prefill_layers(vrt_model* m, const SeqTarget& t, uint32_t n) {
    const auto& c = m->cfg;
    const uint32_t want = m->opt.prefill_chunk ? m->opt.prefill_chunk : 2048u;
    VRT_TRY(prefill_alloc(m, std::min(want, t.positions)));
    auto& B = m->pf;
    cudaStream_t s = m->ctx->stream;
    const uint32_t d = c.embedding_length, hd = c.head_dim, G = m->Hl / m->KVl;
    uint32_t* status = &m->st->status;
    auto F = [&](uint64_t off) { return reinterpret_cast<const float*>(m->arena + off); };
    auto gemm = [&](int epi, const TmaMap& hi, const TmaMap& lo, const uint8_t* w, uint32_t rows, uint32_t k,
                    uint32_t mrows, float* y, __half* ah, __half* al) -> int {
        GemmParams p{};
        p.w = w;
        p.n = rows;
        p.k = k;
        p.m = mrows;
        p.status = status;
        p.y = y;
        p.ldy = rows;
        p.act_hi = ah;
        p.act_lo = al;
        p.ld_act = rows / 2;
        VRT_CUDA(gemm_q8t(epi, hi, lo, p, s));
        return VRT_OK;
    };
    uint32_t last = 0;
    for (uint32_t p0 = 0; p0 < n; p0 += B.cap) {
        const uint32_t nc = std::min(B.cap, n - p0);
        last = nc;
        embed_rows_kernel<<<nc, kRowThreads, 0, s>>>(m->arena + m->embd, t.prompt + p0, c.vocab_size, d,
                                                    std::sqrt(static_cast<float>(d)), F(m->layers[0].n_attn),
                                                    c.rms_epsilon, B.h0, B.xh, B.xl, Q16Out{}, status);
        VRT_CUDA(cudaGetLastError());
        for (uint32_t l = 0; l < c.block_count; ++l) {
            const auto& L = m->layers[l];
            if (l > 0) {
                resid_rows_kernel<<<nc, kRowThreads, 0, s>>>(B.dn, B.h1, F(m->layers[l - 1].n_post_ffw), F(L.n_attn),
                                                            c.rms_epsilon, d, B.h0, B.xh, B.xl, Q16Out{}, status);
                VRT_CUDA(cudaGetLastError());
            }
            VRT_TRY(gemm(kGemmStore, B.xd_hi, B.xd_lo, m->arena + L.qkv, m->qwl + 2 * m->kwl, d, nc, B.qkv, nullptr,
                         nullptr));
            VRT_CUDA(qk_rope_launch(B.qkv, m, L, p0, nc, B.q, B.k, B.v, s));
            PrefillAttnParams a{};
            a.q = B.q;
            a.k = B.k;
            a.v = B.v;
            a.k_cache = t.kc[l];
            a.v_cache = t.vc[l];
            a.cap = t.cap[l];
            a.window = L.global ? 0u : c.sliding_window;
            a.p0 = p0;
            a.n = nc;
            a.H = m->Hl;
            a.KV = m->KVl;
            a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
            a.out_hi = B.xh;
            a.out_lo = B.xl;
            VRT_CUDA(prefill_attn_launch(a, hd, G, s));
            kv_store_kernel<<<dim3(nc, m->KVl), 128, 0, s>>>(B.k, B.v, t.kc[l], t.vc[l], t.cap[l], m->KVl, hd, p0, nc);
            VRT_CUDA(cudaGetLastError());
            VRT_TRY(gemm(kGemmStore, B.xq_hi, B.xq_lo, m->arena + L.o, d, m->qwl, nc, B.o, nullptr, nullptr));
            VRT_TRY(nccl_sum(m, B.o, static_cast<size_t>(nc) * d, s));  // row-parallel partials (tensor parallel)
            resid_rows_kernel<<<nc, kRowThreads, 0, s>>>(B.o, B.h0, F(L.n_post_attn), F(L.n_ffn), c.rms_epsilon, d,
                                                        B.h1, B.xh, B.xl, Q16Out{}, status);
            VRT_CUDA(cudaGetLastError());
            VRT_TRY(gemm(kGemmGeluSplit, B.xd_hi, B.xd_lo, m->arena + L.gu, 2 * m->ffl, d, nc, nullptr, B.ah, B.al));
            VRT_TRY(gemm(kGemmStore, B.xf_hi, B.xf_lo, m->arena + L.down, d, m->ffl, nc, B.dn, nullptr, nullptr));
            VRT_TRY(nccl_sum(m, B.dn, static_cast<size_t>(nc) * d, s));
        }
    }
    // last prompt token: final residual + output norm -> tied LM head + argmax
    const auto& lastL = m->layers[c.block_count - 1];
    GemvParams p{};
    const uint32_t kt = d / kTileCols;
    p.w = m->arena + m->embd + static_cast<uint64_t>(m->vocab_lo / kTileRows) * kt * kTileBytes;
    p.rows = m->vocab_hi - m->vocab_lo;
    p.cols = d;
    p.x = B.dn + static_cast<uint64_t>(last - 1) * d;
    p.h_prev = B.h1 + static_cast<uint64_t>(last - 1) * d;
    p.w_post = F(lastL.n_post_ffw);
    p.w_pre = F(m->out_norm);
    p.h_out = t.hidden;
    p.y = t.logits;
    p.amax = t.key;
    p.row_base = m->vocab_lo;
    p.status = status;
    p.eps = c.rms_epsilon;
    VRT_CUDA(gemv_q8t(kProResidFinal, kEpiArgmax, p, gemv_grid(m->ctx->prop.multiProcessorCount, p.rows), s, false));
    VRT_TRY(nccl_key_max(m, t.key, 1, s));
    return VRT_OK;
}

// The model's own sequence: the step state ends exactly as after a
// token-by-token prefill (position n, first generated id emitted).
static int prefill_batched(vrt_model* m, uint32_t n) {
    VRT_TRY(prefill_layers(m, model_target(m), n));
    VRT_CUDA(launch(finalize_decode_kernel, dim3(1), dim3(1), 0, m->ctx->stream, false, m->st, m->cfg.vocab_size,
                    m->out_ids, kMaxSteps, TpParams{}));
    return VRT_OK;
}

// --------------------------------------------------------- batched decode

static bool batch_supported(const vrt_model* m) {
    return prefill_supported(m) && (m->vocab_hi - m->vocab_lo) % kGemmBN == 0;
}

static uint32_t batch_splits(const vrt_batch* b, uint32_t count, uint32_t cap) {
    const vrt_model* m = b->m;
    const uint32_t ctas = count * m->KVl;
    const uint32_t want = (2u * m->ctx->prop.multiProcessorCount + ctas - 1) / ctas;
    return std::max(1u, std::min({want, (cap + 15) / 16, b->max_splits}));
}

// Split-K workspace and tickets for the step's small-M GEMMs at `count` rows.
// The Q8M copies of every projection and of this rank's LM-head rows, made
// once per model from the Q8T arena (same byte count: 28.7 GB more for the
// 27B shape).  Returns VRT_E_NOMEM, with nothing allocated, when they do not fit.
static int model_q8m(vrt_model* m) {
    if (m->q8m) return VRT_OK;
    const auto& c = m->cfg;
    const uint32_t d = c.embedding_length, kt = d / kTileCols, vl = m->vocab_hi - m->vocab_lo;
    struct Mat { const uint8_t* src; uint32_t rows, cols; };
    std::vector<Mat> mats;
    for (const auto& L : m->layers) {
        mats.push_back({m->arena + L.qkv, m->qwl + 2 * m->kwl, d});
        mats.push_back({m->arena + L.o, d, m->qwl});
        mats.push_back({m->arena + L.gu, 2 * m->ffl, d});
        mats.push_back({m->arena + L.down, d, m->ffl});
    }
    mats.push_back({m->arena + m->embd + static_cast<uint64_t>(m->vocab_lo / kTileRows) * kt * kTileBytes, vl, d});
    std::vector<uint64_t> off;
    uint64_t total = 0;
    for (const auto& x : mats) {
        if (x.rows % kQ8mRows || x.cols % kQ8mCols) return fail(VRT_E_UNSUPPORTED, "Q8M needs 128-multiple shapes");
        off.push_back(total);
        total += align256(static_cast<uint64_t>(x.rows) * x.cols / 32 * 34);
    }
    uint8_t* mem = nullptr;
    if (cudaMalloc(&mem, total) != cudaSuccess) {
        cudaGetLastError();
        return fail(VRT_E_NOMEM, "no room for the Q8M weight copy (%.1f GB)", total / 1e9);
    }
    cudaStream_t s = m->ctx->stream;
    for (size_t i = 0; i < mats.size(); ++i) {
        const cudaError_t e = q8t_to_q8m(mats[i].src, mats[i].rows, mats[i].cols, mem + off[i], s);
        if (e != cudaSuccess) {
            cudaStreamSynchronize(s);
            cudaFree(mem);
            return cuda_fail(e, "q8t_to_q8m", __FILE__, __LINE__);
        }
    }
    m->q8m = mem;
    m->q8m_off = off;
    return VRT_OK;
}

static int batch_gemm_workspace(vrt_batch* b, uint32_t count) {
    vrt_model* m = b->m;
    const auto& c = m->cfg;
    const int sms = m->ctx->prop.multiProcessorCount;
    const uint32_t d = c.embedding_length;
    const uint32_t shapes[][2] = {{m->qwl + 2 * m->kwl, d}, {d, m->qwl}, {2 * m->ffl, d}, {d, m->ffl},
                                  {m->vocab_hi - m->vocab_lo, d}};
    if (count > 64) return VRT_OK;  // large-M kernel: no split-K workspace
    const uint32_t nt = gemm_small_tile(count), tt = (count + nt - 1) / nt;
    uint64_t wsf = 0, tk = 0;
    for (const auto& sh : shapes) {
        const uint32_t ks = gemm_small_ksplit(sh[0], count, sh[1], sms);
        if (ks > 1) wsf = std::max<uint64_t>(wsf, static_cast<uint64_t>(ks) * tt * nt * sh[0]);
        tk = std::max<uint64_t>(tk, static_cast<uint64_t>(sh[0] / kGemmBN) * tt);
    }
    cudaStream_t s = m->ctx->stream;
    if (wsf > b->gws_floats || tk > b->gtickets_n) {
        VRT_CUDA(cudaStreamSynchronize(s));
        if (wsf > b->gws_floats) {
            cudaFree(b->gws);
            b->gws = nullptr;
            VRT_CUDA(cudaMalloc(&b->gws, std::max<uint64_t>(wsf, 1) * 4));
            b->gws_floats = wsf;
        }
        if (tk > b->gtickets_n) {
            cudaFree(b->gtickets);
            b->gtickets = nullptr;
            VRT_CUDA(cudaMalloc(&b->gtickets, tk * 4));
            VRT_CUDA(cudaMemsetAsync(b->gtickets, 0, tk * 4, s));
            b->gtickets_n = tk;
        }
    }
    return VRT_OK;
}

// One decode step for sequences [0, count) on the model stream.
static int batch_record_step(vrt_batch* b, uint32_t count) {
    vrt_model* m = b->m;
    const auto& c = m->cfg;
    cudaStream_t s = m->ctx->stream;
    const uint32_t d = c.embedding_length, hd = c.head_dim, qkvw = m->qwl + 2 * m->kwl;
    uint32_t* status = &m->st->status;
    auto F = [&](uint64_t off) { return reinterpret_cast<const float*>(m->arena + off); };
    auto gemm = [&](int epi, const TmaMap& hi, const TmaMap& lo, const uint8_t* w, uint32_t rows, uint32_t k,
                    float* y, __half* ah, __half* al) -> int {
        GemmParams p{};
        p.w = w;
        p.n = rows;
        p.k = k;
        p.m = count;
        p.status = status;
        p.y = y;
        p.ldy = epi == kGemmArgmax ? c.vocab_size : rows;
        p.act_hi = ah;
        p.act_lo = al;
        p.ld_act = rows / 2;
        p.keys = b->keys;
        p.row_base = epi == kGemmArgmax ? m->vocab_lo : 0u;
        if (count > 64) {  // large-M kernel: 128-row token tiles, operands through the 128-row-box maps
            const TmaMap& H = &hi == &b->xd_hi ? b->Xd_hi : &hi == &b->xq_hi ? b->Xq_hi : b->Xf_hi;
            const TmaMap& Lo = &lo == &b->xd_lo ? b->Xd_lo : &lo == &b->xq_lo ? b->Xq_lo : b->Xf_lo;
            VRT_CUDA(gemm_q8t(epi, H, Lo, p, s));
            return VRT_OK;
        }
        p.nt = gemm_small_tile(count);
        p.ksplit = gemm_small_ksplit(rows, count, k, m->ctx->prop.multiProcessorCount);
        p.ws = b->gws;
        p.tickets = b->gtickets;
        VRT_CUDA(gemm_q8t_small(epi, hi, lo, p, s));
        return VRT_OK;
    };
    // up to 32 sequences: integer tensor-core GEMMs on the Q8M copies, operands
    // as int16 split halves (the row kernels and quant_rows write them)
    const bool i8 = b->i8 && count <= 32;
    auto q16 = [&](uint32_t K) { return i8 ? Q16Out{b->q_hi, b->q_lo, b->q_sx, K, b->Sp} : Q16Out{}; };
    __half* oxh = i8 ? nullptr : b->xh;
    __half* oxl = i8 ? nullptr : b->xl;
    size_t wi = 0;  // next Q8M matrix: per layer qkv, o, gu, down, then the head
    auto gemm8 = [&](int epi, const TmaMap& hi, const TmaMap& lo, uint32_t rows, uint32_t k, float* y,
                     float* act) -> int {
        GemmI8Params p{};
        p.w = m->q8m + m->q8m_off[wi++];
        p.n = rows;
        p.k = k;
        p.m = count;
        p.sx = b->q_sx;
        p.sx_ld = b->Sp;
        p.y = y;
        p.ldy = epi == kGemmArgmax ? c.vocab_size : rows;
        p.act = act;
        p.ld_act = rows / 2;
        p.keys = b->keys;
        p.row_base = epi == kGemmArgmax ? m->vocab_lo : 0u;
        p.nt = gemm_small_tile(count);
        p.ksplit = gemm_small_ksplit(rows, count, k, m->ctx->prop.multiProcessorCount);
        p.ws = b->gws;
        p.tickets = b->gtickets;
        p.status = status;
        VRT_CUDA(gemm_q8m_i8(epi, hi, lo, p, s));
        return VRT_OK;
    };
    embed_rows_kernel<<<count, kRowThreads, 0, s>>>(m->arena + m->embd, b->tokens, c.vocab_size, d,
                                                   std::sqrt(static_cast<float>(d)), F(m->layers[0].n_attn),
                                                   c.rms_epsilon, b->h0, oxh, oxl, q16(d), status);
    VRT_CUDA(cudaGetLastError());
    for (uint32_t l = 0; l < c.block_count; ++l) {
        const auto& L = m->layers[l];
        if (l > 0) {
            resid_rows_kernel<<<count, kRowThreads, 0, s>>>(b->dn, b->h1, F(m->layers[l - 1].n_post_ffw), F(L.n_attn),
                                                           c.rms_epsilon, d, b->h0, oxh, oxl, q16(d), status);
            VRT_CUDA(cudaGetLastError());
        }
        wi = 4 * static_cast<size_t>(l);
        if (i8) {
            VRT_TRY(gemm8(kGemmStore, b->Qd_hi, b->Qd_lo, qkvw, d, b->qkv, nullptr));
        } else {
            VRT_TRY(gemm(kGemmStore, b->xd_hi, b->xd_lo, m->arena + L.qkv, qkvw, d, b->qkv, nullptr, nullptr));
        }
        AttnParams a{};
        a.qkv = b->qkv;
        a.q_norm = F(L.n_q);
        a.k_norm = F(L.n_k);
        a.rope_cos = L.global ? m->rope_cos_g : m->rope_cos_l;
        a.rope_sin = L.global ? m->rope_sin_g : m->rope_sin_l;
        a.k_cache = b->kc[l];
        a.v_cache = b->vc[l];
        a.cap = b->cap[l];
        a.window = L.global ? 0u : c.sliding_window;
        a.pos = b->pos;
        a.H = m->Hl;
        a.KV = m->KVl;
        a.hd = hd;
        a.eps = c.rms_epsilon;
        a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
        a.part_ml = b->part_ml;
        a.part_acc = b->part_acc;
        a.tickets = b->tickets;
        a.splits = batch_splits(b, count, b->cap[l]);
        a.seq_qkv = qkvw;
        a.seq_cache = static_cast<uint64_t>(m->KVl) * b->cap[l] * hd;
        a.seq_out = m->qwl;
        if (i8) {
            a.out = b->att32;
        } else {
            a.out_hi = b->xh;
            a.out_lo = b->xl;
        }
        VRT_CUDA(attention_launch(a, dim3(a.splits, m->KVl, count), s, false));
        if (i8) {
            VRT_CUDA(quant_rows(b->att32, m->qwl, count, m->qwl, q16(m->qwl), s));
            VRT_TRY(gemm8(kGemmStore, b->Qq_hi, b->Qq_lo, d, m->qwl, b->o, nullptr));
        } else {
            VRT_TRY(gemm(kGemmStore, b->xq_hi, b->xq_lo, m->arena + L.o, d, m->qwl, b->o, nullptr, nullptr));
        }
        VRT_TRY(nccl_sum(m, b->o, static_cast<size_t>(count) * d, s));  // row-parallel partials (tensor parallel)
        resid_rows_kernel<<<count, kRowThreads, 0, s>>>(b->o, b->h0, F(L.n_post_attn), F(L.n_ffn), c.rms_epsilon, d,
                                                       b->h1, oxh, oxl, q16(d), status);
        VRT_CUDA(cudaGetLastError());
        if (i8) {
            VRT_TRY(gemm8(kGemmGeluSplit, b->Qd_hi, b->Qd_lo, 2 * m->ffl, d, nullptr, b->act32));
            VRT_CUDA(quant_rows(b->act32, m->ffl, count, m->ffl, q16(m->ffl), s));
            VRT_TRY(gemm8(kGemmStore, b->Qf_hi, b->Qf_lo, d, m->ffl, b->dn, nullptr));
        } else {
            VRT_TRY(gemm(kGemmGeluSplit, b->xd_hi, b->xd_lo, m->arena + L.gu, 2 * m->ffl, d, nullptr, b->ah, b->al));
            VRT_TRY(gemm(kGemmStore, b->xf_hi, b->xf_lo, m->arena + L.down, d, m->ffl, b->dn, nullptr, nullptr));
        }
        VRT_TRY(nccl_sum(m, b->dn, static_cast<size_t>(count) * d, s));
    }
    const auto& lastL = m->layers[c.block_count - 1];
    final_rows_kernel<<<count, kRowThreads, 0, s>>>(b->dn, b->h1, F(lastL.n_post_ffw), F(m->out_norm), c.rms_epsilon, d,
                                                   b->hidden, oxh, oxl, q16(d), status);
    VRT_CUDA(cudaGetLastError());
    // tied LM head over this rank's vocabulary rows; logits rows keep the
    // full-vocabulary stride (this rank's columns at vocab_lo)
    const uint32_t kt = d / kTileCols, vl = m->vocab_hi - m->vocab_lo;
    if (i8) {
        wi = 4 * static_cast<size_t>(c.block_count);
        VRT_TRY(gemm8(kGemmArgmax, b->Qd_hi, b->Qd_lo, vl, d, b->keep_logits ? b->logits + m->vocab_lo : nullptr, nullptr));
    } else {
        VRT_TRY(gemm(kGemmArgmax, b->xd_hi, b->xd_lo,
                     m->arena + m->embd + static_cast<uint64_t>(m->vocab_lo / kTileRows) * kt * kTileBytes, vl, d,
                     b->keep_logits ? b->logits + m->vocab_lo : nullptr, nullptr, nullptr));
    }
    VRT_TRY(nccl_key_max(m, b->keys, count, s));
    batch_finalize_kernel<<<(count + 127) / 128, 128, 0, s>>>(b->keys, b->tokens, b->pos, b->out_ids, b->out_count,
                                                             b->out_cap, 0, count, c.vocab_size, 0, status);
    VRT_CUDA(cudaGetLastError());
    return VRT_OK;
}

static void batch_free(vrt_batch* b) {
    if (!b) return;
    if (b->m) {
        cudaSetDevice(b->m->ctx->device);
        cudaStreamSynchronize(b->m->ctx->stream);
    }
    if (b->graph) cudaGraphExecDestroy(b->graph);
    cudaFree(b->gws);
    cudaFree(b->gtickets);
    cudaFree(b->mem);
    delete b;
}

static int device_status(vrt_model* m, uint32_t& status) {
    status = m->st_host->status;
    if (!status) return VRT_OK;
    const bool timeout = (status & (kStatusWaitTimeout | kStatusPeerTimeout | kStatusStepTimeout)) != 0u;
    const char* what = (status & kStatusPeerTimeout)   ? "a tensor-parallel peer did not answer in time"
                       : (status & kStatusStepTimeout) ? "a persistent-step data wait timed out"
                       : (status & kStatusWaitTimeout) ? "a bounded device wait timed out"
                       : (status & kStatusBadToken)    ? "Token id is outside Gemma 3 vocabulary"
                                                       : "Non-finite value in the Gemma 3 hidden state or logits";
    return fail(timeout ? VRT_E_TIMEOUT : VRT_E_NUMERIC, "%s (device status 0x%x)", what, status);
}

}  // namespace vrt

using namespace vrt;

extern "C" {

void vrt_model_options_default(vrt_model_options* o) {
    if (!o) return;
    memset(o, 0, sizeof *o);
    o->use_graph = 1;
    o->use_pdl = 1;
    o->step_mode = VRT_STEP_LAUNCHES;
}

int vrt_model_load(vrt_ctx* ctx, const char* path, const vrt_model_options* opts, vrt_model** out) {
    clear_error();
    std::unique_ptr<vrt_model> m;
    VRT_TRY(begin_model(ctx, opts, out, m));
    if (!path) return fail(VRT_E_INVALID, "null path");
    try {
        vortexrt::GgufFile g(path);
        VRT_TRY(read_config(g, m->cfg, m->eos));
        VRT_TRY(plan(m.get()));
        VRT_TRY(alloc_runtime(m.get()));
        const int rc = load_weights(m.get(), g);
        if (rc != VRT_OK) {
            destroy_model(m.release());
            return rc;
        }
    } catch (const std::exception& e) {
        vrt_model* raw = m.release();
        if (raw && raw->arena) destroy_model(raw); else delete raw;
        return fail(VRT_E_IO, "%s", e.what());
    }
    const int rc = finish_create(m.get());
    if (rc != VRT_OK) {
        destroy_model(m.release());
        return rc;
    }
    *out = m.release();
    return VRT_OK;
}

int vrt_model_create_synthetic(vrt_ctx* ctx, const vrt_gemma3_config* cfg, uint64_t seed,
                               const vrt_model_options* opts, vrt_model** out) {
    clear_error();
    std::unique_ptr<vrt_model> m;
    VRT_TRY(begin_model(ctx, opts, out, m));
    if (!cfg) return fail(VRT_E_INVALID, "null config");
    m->cfg = *cfg;
    m->cfg.value_dim = m->cfg.value_dim ? m->cfg.value_dim : m->cfg.head_dim;
    if (m->cfg.local_rope_base == 0.0f) m->cfg.local_rope_base = 1.0e4f;
    if (m->cfg.global_rope_base == 0.0f) m->cfg.global_rope_base = 1.0e6f;
    if (m->cfg.rms_epsilon == 0.0f) m->cfg.rms_epsilon = 1e-6f;
    VRT_TRY(validate_config(m->cfg));
    VRT_TRY(plan(m.get()));
    int rc = alloc_runtime(m.get());
    if (rc == VRT_OK) rc = synth_weights(m.get(), seed);
    if (rc == VRT_OK) rc = finish_create(m.get());
    if (rc != VRT_OK) {
        destroy_model(m.release());
        return rc;
    }
    *out = m.release();
    return VRT_OK;
}

int vrt_model_destroy(vrt_model* m) {
    destroy_model(m);
    return VRT_OK;
}

int vrt_model_config(vrt_model* m, vrt_gemma3_config* out) {
    if (!m || !out) return fail(VRT_E_INVALID, "null argument");
    *out = m->cfg;
    return VRT_OK;
}

int vrt_model_reset(vrt_model* m) {
    if (!m) return fail(VRT_E_INVALID, "null model");
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    memset(m->st_host, 0, kStepStateHostBytes);
    VRT_CUDA(cudaMemcpyAsync(m->st, m->st_host, kStepStateHostBytes, cudaMemcpyHostToDevice, m->ctx->stream));
    if (m->tp_bar) VRT_CUDA(cudaMemsetAsync(m->tp_bar, 0, 8, m->ctx->stream));
    if (m->ps_on) VRT_CUDA(cudaMemsetAsync(m->ps.att_tickets, 0, 4ull * (m->ps.KV + 1), m->ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    m->next_pos = 0;
    m->generated = 0;
    return VRT_OK;
}

// Tensor parallelism: every rank's logits shard into m->logits_full (the
// vocabulary in order; shards are equal and contiguous) by one in-place NCCL
// all-gather on the model's communicator.  Collective: every rank calls it.
static int gather_logits(vrt_model* m, cudaStream_t s) {
    const uint32_t vl = m->vocab_hi - m->vocab_lo;
    if (!m->logits_full) VRT_CUDA(cudaMalloc(&m->logits_full, 4ull * m->cfg.vocab_size));
    float* mine = m->logits_full + m->vocab_lo;
    VRT_CUDA(cudaMemcpyAsync(mine, m->logits, 4ull * vl, cudaMemcpyDeviceToDevice, s));
    const int r = m->nccl.AllGather(mine, m->logits_full, vl, /*ncclFloat32*/ 7, m->comm, s);
    if (r) return fail(VRT_E_CUDA, "ncclAllGather(logits) failed: %s", m->nccl.GetErrorString(r));
    return VRT_OK;
}

int vrt_decode_step(vrt_model* m, uint32_t token, uint32_t position, uint32_t top_k, float* h_hidden,
                    uint32_t* h_ids, float* h_logits) {
    clear_error();
    if (!m) return fail(VRT_E_INVALID, "null model");
    const auto& c = m->cfg;
    if (position != m->next_pos) return fail(VRT_E_STATE, "Gemma 3 decode positions must be contiguous");
    if (position >= c.context_length) return fail(VRT_E_STATE, "Gemma 3 context length exceeded");
    if (position >= m->P) return fail(VRT_E_STATE, "position %u exceeds the allocated KV capacity %u", position, m->P);
    if (token >= c.vocab_size) {
        vrt_model_reset(m);
        return fail(VRT_E_INVALID, "Token id is outside Gemma 3 vocabulary");
    }
    cudaStream_t s = m->ctx->stream;
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    StepState* sh = m->st_host;
    sh->token = token;
    sh->pos = position;
    sh->status = 0;
    sh->prompt_count = 0;
    VRT_CUDA(cudaMemcpyAsync(m->st, sh, 20, cudaMemcpyHostToDevice, s));
    VRT_TRY(run_step(m, top_k > 0));
    // top_k > 1 under tensor parallelism: gather the logits shards (every
    // rank makes the same call, as for the step itself)
    if (top_k > 1 && m->world > 1) VRT_TRY(gather_logits(m, s));
    VRT_CUDA(cudaMemcpyAsync(sh, m->st, kStepStateHostBytes, cudaMemcpyDeviceToHost, s));
    if (h_hidden) VRT_CUDA(cudaMemcpyAsync(m->hidden_host, m->hidden, 4ull * c.embedding_length, cudaMemcpyDeviceToHost, s));
    std::vector<float> logits;
    if (top_k > 1) {
        logits.resize(c.vocab_size);
        VRT_CUDA(cudaMemcpyAsync(logits.data(), m->world > 1 ? m->logits_full : m->logits, 4ull * c.vocab_size,
                                 cudaMemcpyDeviceToHost, s));
    }
    VRT_CUDA(cudaStreamSynchronize(s));
    uint32_t status;
    if (const int rc = device_status(m, status); rc != VRT_OK) {
        vrt_model_reset(m);
        return rc;
    }
    if (h_hidden) memcpy(h_hidden, m->hidden_host, 4ull * c.embedding_length);
    if (top_k == 1) {
        if (sh->result_index >= c.vocab_size || !std::isfinite(sh->result_value)) {
            vrt_model_reset(m);
            return fail(VRT_E_NUMERIC, "GPU argmax produced invalid result");
        }
        if (h_ids) h_ids[0] = sh->result_index;
        if (h_logits) h_logits[0] = sh->result_value;
    } else if (top_k > 1) {
        const uint32_t k = std::min(top_k, c.vocab_size);
        std::vector<uint32_t> ids(c.vocab_size);
        for (uint32_t i = 0; i < c.vocab_size; ++i) ids[i] = i;
        std::partial_sort(ids.begin(), ids.begin() + k, ids.end(), [&](uint32_t a, uint32_t b) {
            return logits[a] > logits[b] || (logits[a] == logits[b] && a < b);
        });
        for (uint32_t i = 0; i < k; ++i) {
            if (!std::isfinite(logits[ids[i]])) {
                vrt_model_reset(m);
                return fail(VRT_E_NUMERIC, "Non-finite Gemma 3 logit");
            }
            if (h_ids) h_ids[i] = ids[i];
            if (h_logits) h_logits[i] = logits[ids[i]];
        }
    }
    m->next_pos = position + 1;
    if (top_k > 0) m->generated = sh->out_count;  // the step emitted a greedy id: device-resident steps may follow
    return VRT_OK;
}

int vrt_model_logits(vrt_model* m, float* h_logits) {
    clear_error();
    if (!m || !h_logits) return fail(VRT_E_INVALID, "null argument");
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    cudaStream_t s = m->ctx->stream;
    if (m->world > 1) VRT_TRY(gather_logits(m, s));
    VRT_CUDA(cudaMemcpyAsync(h_logits, m->world > 1 ? m->logits_full : m->logits, 4ull * m->cfg.vocab_size,
                             cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaStreamSynchronize(s));
    return VRT_OK;
}

int vrt_prefill(vrt_model* m, const uint32_t* h_prompt, uint32_t n) {
    clear_error();
    if (!m || (!h_prompt && n)) return fail(VRT_E_INVALID, "null argument");
    if (n == 0) return fail(VRT_E_INVALID, "Gemma 3 prompt produced no input tokens");
    const auto& c = m->cfg;
    if (n > m->P || n > c.context_length) return fail(VRT_E_STATE, "prompt of %u tokens exceeds capacity %u", n, m->P);
    for (uint32_t i = 0; i < n; ++i) {
        if (h_prompt[i] >= c.vocab_size) return fail(VRT_E_INVALID, "Token id is outside Gemma 3 vocabulary");
    }
    cudaStream_t s = m->ctx->stream;
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    VRT_CUDA(cudaStreamSynchronize(s));
    VRT_CUDA(cudaMemcpyAsync(m->prompt, h_prompt, 4ull * n, cudaMemcpyHostToDevice, s));
    StepState* sh = m->st_host;
    memset(sh, 0, kStepStateHostBytes);
    const bool batched = !m->trace_on && m->opt.prefill_chunk != 1 && n >= 2 && prefill_supported(m);
    sh->token = batched ? h_prompt[n - 1] : h_prompt[0];
    sh->pos = batched ? n - 1 : 0;  // the batched pass leaves only the last token's LM head + finalize
    sh->prompt_count = n;
    VRT_CUDA(cudaMemcpyAsync(m->st, sh, kStepStateHostBytes, cudaMemcpyHostToDevice, s));
    if (batched) {
        VRT_TRY(prefill_batched(m, n));
    } else {
        for (uint32_t i = 0; i + 1 < n; ++i) VRT_TRY(run_step(m, false));
        VRT_TRY(run_step(m, true));
    }
    VRT_CUDA(cudaMemcpyAsync(sh, m->st, sizeof(StepState), cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaStreamSynchronize(s));
    uint32_t status;
    if (const int rc = device_status(m, status); rc != VRT_OK) {
        vrt_model_reset(m);
        return rc;
    }
    m->next_pos = n;
    m->generated = 1;
    return VRT_OK;
}

int vrt_decode_steps_async(vrt_model* m, uint32_t steps, uint32_t* d_out_ids, void* stream) {
    clear_error();
    if (!m) return fail(VRT_E_INVALID, "null model");
    if (m->generated == 0) return fail(VRT_E_STATE, "decode steps need a prefill (or a decode step) first");
    if (m->next_pos + steps > m->P || m->next_pos + steps > m->cfg.context_length) {
        return fail(VRT_E_STATE, "decode would exceed the KV capacity");
    }
    if (m->generated + steps > kMaxSteps) return fail(VRT_E_STATE, "more than %u generated ids since the prefill", kMaxSteps);
    cudaStream_t s = m->ctx->stream;
    if (stream && stream != s) {
        // order the steps after the caller's stream
        cudaEvent_t ev;
        VRT_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        VRT_CUDA(cudaEventRecord(ev, static_cast<cudaStream_t>(stream)));
        VRT_CUDA(cudaStreamWaitEvent(s, ev, 0));
        VRT_CUDA(cudaEventDestroy(ev));
    }
    for (uint32_t i = 0; i < steps; ++i) VRT_TRY(run_step(m, true));
    const uint32_t first = m->generated;
    m->generated += steps;
    m->next_pos += steps;
    if (d_out_ids) {
        VRT_CUDA(cudaMemcpyAsync(d_out_ids, m->out_ids + first, 4ull * steps, cudaMemcpyDeviceToDevice, s));
    }
    if (stream && stream != s) {
        cudaEvent_t ev;
        VRT_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        VRT_CUDA(cudaEventRecord(ev, s));
        VRT_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), ev, 0));
        VRT_CUDA(cudaEventDestroy(ev));
    }
    return VRT_OK;
}

int vrt_model_next_token(vrt_model* m, uint32_t* h_token, uint32_t* h_position) {
    if (!m) return fail(VRT_E_INVALID, "null model");
    VRT_CUDA(cudaMemcpyAsync(m->st_host, m->st, sizeof(StepState), cudaMemcpyDeviceToHost, m->ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (h_token) *h_token = m->st_host->token;
    if (h_position) *h_position = m->st_host->pos;
    return VRT_OK;
}

int vrt_generate_greedy(vrt_model* m, const uint32_t* h_prompt, uint32_t n, uint32_t max_new, uint32_t* h_out,
                        uint32_t* h_count) {
    clear_error();
    if (!m || !h_count || (max_new && !h_out)) return fail(VRT_E_INVALID, "null argument");
    *h_count = 0;
    VRT_TRY(vrt_model_reset(m));
    if (max_new == 0) return VRT_OK;
    if (max_new > kMaxSteps) return fail(VRT_E_INVALID, "max_new above %u", kMaxSteps);
    if (static_cast<uint64_t>(n) + max_new - 1 > m->P) return fail(VRT_E_STATE, "generation exceeds the KV capacity");
    VRT_TRY(vrt_prefill(m, h_prompt, n));  // emits generated id 0
    if (max_new > 1) VRT_TRY(vrt_decode_steps_async(m, max_new - 1, nullptr, nullptr));
    std::vector<uint32_t> ids(max_new);
    VRT_CUDA(cudaMemcpyAsync(ids.data(), m->out_ids, 4ull * max_new, cudaMemcpyDeviceToHost, m->ctx->stream));
    VRT_CUDA(cudaMemcpyAsync(m->st_host, m->st, sizeof(StepState), cudaMemcpyDeviceToHost, m->ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    uint32_t status;
    if (const int rc = device_status(m, status); rc != VRT_OK) {
        vrt_model_reset(m);
        return rc;
    }
    uint32_t cnt = 0;
    for (uint32_t i = 0; i < max_new; ++i) {
        h_out[cnt++] = ids[i];
        if (ids[i] == m->eos) break;  // gemma3.cpp:2139-2141
    }
    *h_count = cnt;
    return VRT_OK;
}

int vrt_model_step_kernels(vrt_model* m, uint32_t* out) {
    if (!m || !out) return fail(VRT_E_INVALID, "null argument");
    if (!m->kernels_per_step) {
        // count by recording into a throw-away capture
        cudaGraph_t g = nullptr;
        VRT_CUDA(cudaStreamBeginCapture(m->ctx->stream, cudaStreamCaptureModeThreadLocal));
        uint32_t nk = 0;
        record_step(m, m->ctx->stream, true, &nk);
        cudaStreamEndCapture(m->ctx->stream, &g);
        if (g) cudaGraphDestroy(g);
        m->kernels_per_step = nk;
    }
    *out = m->kernels_per_step;
    return VRT_OK;
}

int vrt_model_device_status(vrt_model* m, uint32_t* h_status) {
    if (!m || !h_status) return fail(VRT_E_INVALID, "null argument");
    VRT_CUDA(cudaMemcpyAsync(m->st_host, m->st, sizeof(StepState), cudaMemcpyDeviceToHost, m->ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    *h_status = m->st_host->status;
    return VRT_OK;
}

int vrt_model_set_trace(vrt_model* m, int enabled) {
    if (!m) return fail(VRT_E_INVALID, "null model");
    if ((enabled != 0) == m->trace_on) return VRT_OK;
    m->trace_on = enabled != 0;
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (m->g_head) cudaGraphExecDestroy(m->g_head);
    if (m->g_nohead) cudaGraphExecDestroy(m->g_nohead);
    m->g_head = m->g_nohead = nullptr;
    return build_graphs(m);
}

int vrt_model_trace(vrt_model* m, float* h_out) {
    if (!m || !h_out) return fail(VRT_E_INVALID, "null argument");
    VRT_CUDA(cudaMemcpy(h_out, m->trace, 4ull * m->cfg.block_count * m->cfg.embedding_length, cudaMemcpyDeviceToHost));
    return VRT_OK;
}

// ----------------------------------------------- packed (Q8T) fast path

uint64_t vrt_q8t_bytes(uint32_t rows, uint32_t cols) { return q8t_bytes(rows, cols); }

static int check_packable(vrt_ctx* ctx, uint64_t raw_bytes, uint64_t off, uint32_t rows, uint32_t cols) {
    if (!ctx) return fail(VRT_E_INVALID, "null context");
    if (!rows || !cols || cols % 128) return fail(VRT_E_INVALID, "packed Q8_0 needs rows > 0 and cols %% 128 == 0");
    const uint64_t bytes = static_cast<uint64_t>(rows) * (cols / 32) * 34;
    if (off > raw_bytes || bytes > raw_bytes - off) return fail(VRT_E_INVALID, "raw weight buffer is too small");
    return VRT_OK;
}

int vrt_q8t_pack(vrt_ctx* ctx, const void* d_raw, uint64_t raw_bytes, uint64_t off, uint32_t rows, uint32_t cols,
                 void* d_packed, void* stream) {
    clear_error();
    VRT_TRY(check_packable(ctx, raw_bytes, off, rows, cols));
    if (!d_raw || !d_packed) return fail(VRT_E_INVALID, "null buffer");
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaMemsetAsync(d_packed, 0, q8t_bytes(rows, cols), s));
    RepackParams p{static_cast<const uint8_t*>(d_raw) + off, static_cast<uint64_t>(cols) / 32 * 34, 0, rows,
                   cols / 32, static_cast<uint8_t*>(d_packed), cols, 0, 0};
    const uint64_t work = static_cast<uint64_t>(rows) * (cols / 32);
    VRT_CUDA(launch(repack_kernel, dim3(static_cast<unsigned>((work + 255) / 256)), dim3(256), 0, s, false, p));
    return VRT_OK;
}

int vrt_q8t_pack_pair(vrt_ctx* ctx, const void* d_raw, uint64_t raw_bytes, uint64_t gate_off, uint64_t up_off,
                      uint32_t ffn, uint32_t cols, void* d_packed, void* stream) {
    clear_error();
    VRT_TRY(check_packable(ctx, raw_bytes, gate_off, ffn, cols));
    VRT_TRY(check_packable(ctx, raw_bytes, up_off, ffn, cols));
    if (ffn % 8) return fail(VRT_E_INVALID, "gate/up rows must be a multiple of 8");
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaMemsetAsync(d_packed, 0, q8t_bytes(2ull * ffn, cols), s));
    for (int mode = 1; mode <= 2; ++mode) {
        RepackParams p{static_cast<const uint8_t*>(d_raw) + (mode == 1 ? gate_off : up_off),
                       static_cast<uint64_t>(cols) / 32 * 34, 0, ffn, cols / 32, static_cast<uint8_t*>(d_packed), cols,
                       0, mode};
        const uint64_t work = static_cast<uint64_t>(ffn) * (cols / 32);
        VRT_CUDA(launch(repack_kernel, dim3(static_cast<unsigned>((work + 255) / 256)), dim3(256), 0, s, false, p));
    }
    return VRT_OK;
}

static int packed_gemv(vrt_ctx* ctx, int pro, int epi, GemvParams& p, cudaStream_t s) {
    static uint32_t* status = nullptr;
    if (!status) VRT_CUDA(cudaMalloc(&status, 4));
    p.status = status;
    if (p.eps == 0.0f) p.eps = 1e-6f;
    VRT_CUDA(gemv_init_attributes());
    VRT_CUDA(gemv_q8t(pro, epi, p, gemv_grid(ctx->prop.multiProcessorCount, p.rows), s, false));
    return VRT_OK;
}

int vrt_q8t_gemv(vrt_ctx* ctx, const void* d_packed, uint32_t rows, uint32_t cols, const float* d_x, float* d_y,
                 void* stream) {
    clear_error();
    if (!ctx || !d_packed || !d_x || !d_y) return fail(VRT_E_INVALID, "null argument");
    if (!rows || !cols || cols % 128) return fail(VRT_E_INVALID, "packed Q8_0 needs rows > 0 and cols %% 128 == 0");
    if (reinterpret_cast<uintptr_t>(d_packed) % 16) return fail(VRT_E_INVALID, "packed weights must be 16-byte aligned");
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaMemsetAsync(d_y, 0, 4ull * rows, s));
    GemvParams p{};
    p.w = static_cast<const uint8_t*>(d_packed);
    p.rows = rows;
    p.cols = cols;
    p.x = d_x;
    p.y = d_y;
    return packed_gemv(ctx, kProPlain, kEpiAtomic, p, s);
}

int vrt_q8t_gate_up(vrt_ctx* ctx, const void* d_packed_pair, uint32_t ffn, uint32_t cols, const float* d_x,
                    float* d_act, void* stream) {
    clear_error();
    if (!ctx || !d_packed_pair || !d_x || !d_act) return fail(VRT_E_INVALID, "null argument");
    if (!ffn || ffn % 8 || !cols || cols % 128) return fail(VRT_E_INVALID, "gate/up shape unsupported");
    if (reinterpret_cast<uintptr_t>(d_packed_pair) % 16) return fail(VRT_E_INVALID, "packed weights must be 16-byte aligned");
    GemvParams p{};
    p.w = static_cast<const uint8_t*>(d_packed_pair);
    p.rows = 2 * ffn;
    p.cols = cols;
    p.x = d_x;
    p.y = d_act;
    return packed_gemv(ctx, kProPlain, kEpiGeluPair, p, as_stream(ctx, stream));
}

int vrt_q8t_ffn(vrt_ctx* ctx, const void* d_gate_up, const void* d_down, uint32_t input_dim, uint32_t ffn_dim,
                uint32_t output_dim, const float* d_x, float* d_act, float* d_y, void* stream) {
    VRT_TRY(vrt_q8t_gate_up(ctx, d_gate_up, ffn_dim, input_dim, d_x, d_act, stream));
    return vrt_q8t_gemv(ctx, d_down, output_dim, ffn_dim, d_act, d_y, stream);
}

int vrt_q8t_lm_head_argmax(vrt_ctx* ctx, const void* d_packed, uint32_t vocab, uint32_t cols, const float* d_x,
                           float* d_logits, vrt_argmax_result* d_out, void* stream) {
    clear_error();
    if (!ctx || !d_packed || !d_x || !d_out) return fail(VRT_E_INVALID, "null argument");
    if (!vocab || !cols || cols % 128) return fail(VRT_E_INVALID, "packed Q8_0 needs rows > 0 and cols %% 128 == 0");
    if (reinterpret_cast<uintptr_t>(d_packed) % 16) return fail(VRT_E_INVALID, "packed weights must be 16-byte aligned");
    cudaStream_t s = as_stream(ctx, stream);
    VRT_CUDA(cudaMemsetAsync(ctx->d_key, 0, 8, s));
    GemvParams p{};
    p.w = static_cast<const uint8_t*>(d_packed);
    p.rows = vocab;
    p.cols = cols;
    p.x = d_x;
    p.y = d_logits;
    p.amax = ctx->d_key;
    VRT_TRY(packed_gemv(ctx, kProPlain, kEpiArgmax, p, s));
    VRT_CUDA(argmax_unkey_launch(ctx->d_key, reinterpret_cast<uint32_t*>(d_out), s));
    return VRT_OK;
}

// Time one of the step's mat-vec launches in isolation (same kernel and
// parameters as inside the step, no PDL), on the model stream, between CUDA
// events.  which: 0 qkv, 1 o-proj, 2 gate/up, 3 down, 4 LM head.  Clobbers
// activations: call vrt_model_reset before decoding again.
int vrt_model_time_kernel(vrt_model* m, uint32_t layer, uint32_t which, uint32_t iters, float* ms_per_launch,
                          uint64_t* algorithmic_bytes) {
    clear_error();
    if (!m || !ms_per_launch || which > 4 || layer >= m->cfg.block_count || iters == 0) {
        return fail(VRT_E_INVALID, "bad argument");
    }
    const auto& c = m->cfg;
    const auto& L = m->layers[layer];
    const uint32_t d = c.embedding_length;
    auto F = [&](uint64_t off) { return reinterpret_cast<const float*>(m->arena + off); };
    GemvParams p{};
    int pro = kProPlain, epi = kEpiAtomic;
    uint64_t vec_bytes = 0;
    p.status = &m->st->status;
    p.eps = c.rms_epsilon;
    switch (which) {
    case 0:
        p.w = m->arena + L.qkv; p.rows = m->qwl + 2 * m->kwl; p.cols = d;
        p.x = m->dn; p.h_prev = m->h1; p.w_post = F(L.n_post_ffw); p.w_pre = F(L.n_attn); p.h_out = m->h0; p.y = m->qkv;
        pro = kProResid;
        vec_bytes = 4ull * (5 * d + p.rows);
        break;
    case 1:
        p.w = m->arena + L.o; p.rows = d; p.cols = m->qwl; p.x = m->att; p.y = m->o;
        vec_bytes = 4ull * (p.cols + d);
        break;
    case 2:
        p.w = m->arena + L.gu; p.rows = 2 * m->ffl; p.cols = d;
        p.x = m->o; p.h_prev = m->h0; p.w_post = F(L.n_post_attn); p.w_pre = F(L.n_ffn); p.h_out = m->h1; p.y = m->act;
        pro = kProResid; epi = kEpiGeluPair;
        vec_bytes = 4ull * (5 * d + m->ffl);
        break;
    case 3:
        p.w = m->arena + L.down; p.rows = d; p.cols = m->ffl; p.x = m->act; p.y = m->dn;
        vec_bytes = 4ull * (m->ffl + d);
        break;
    default: {
        const uint32_t kt = d / kTileCols;
        p.w = m->arena + m->embd + static_cast<uint64_t>(m->vocab_lo / kTileRows) * kt * kTileBytes;
        p.rows = m->vocab_hi - m->vocab_lo; p.cols = d;
        p.x = m->dn; p.h_prev = m->h1; p.w_post = F(L.n_post_ffw); p.w_pre = F(m->out_norm); p.h_out = m->hidden;
        p.y = m->logits; p.amax = m->key_tmp; p.row_base = m->vocab_lo;
        pro = kProResidFinal; epi = kEpiArgmax;
        vec_bytes = 4ull * (4 * d + 2 * d + p.rows);
    }
    }
    const uint64_t wbytes = q8t_bytes(p.rows, p.cols);
    if (algorithmic_bytes) *algorithmic_bytes = static_cast<uint64_t>(p.rows) * (p.cols / 32) * 34 + vec_bytes;
    (void)wbytes;
    cudaStream_t s = m->ctx->stream;
    const int grid = gemv_grid(m->ctx->prop.multiProcessorCount, p.rows);
    cudaEvent_t e0, e1;
    VRT_CUDA(cudaEventCreate(&e0));
    VRT_CUDA(cudaEventCreate(&e1));
    VRT_CUDA(gemv_q8t(pro, epi, p, grid, s, false));  // warm
    VRT_CUDA(cudaEventRecord(e0, s));
    for (uint32_t i = 0; i < iters; ++i) VRT_CUDA(gemv_q8t(pro, epi, p, grid, s, false));
    VRT_CUDA(cudaEventRecord(e1, s));
    VRT_CUDA(cudaEventSynchronize(e1));
    float ms = 0.0f;
    VRT_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms_per_launch = ms / static_cast<float>(iters);
    return VRT_OK;
}

#ifdef VRT_PS_STAMPS
// Timing builds only: the persistent step's phase stamps of the last step,
// [grid][10 L + 10] globaltimer values; returns the count through *n.
extern "C" VRT_API int vrt_ps_stamps(vrt_model* m, uint64_t* h_out, size_t cap, size_t* n) {
    if (!m || !m->ps_on || !m->ps.stamps) return fail(VRT_E_STATE, "no stamps");
    const size_t cnt = static_cast<size_t>(m->ps_grid) * ps_stamp_count(m->ps.L);
    *n = cnt;
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    VRT_CUDA(cudaMemcpy(h_out, m->ps.stamps, 8 * std::min(cap, cnt), cudaMemcpyDeviceToHost));
    return VRT_OK;
}
#endif

int vrt_tp_plan(const vrt_gemma3_config* cfg, int world, int rank, vrt_tp_shard* out) {
    clear_error();
    if (!cfg || !out) return fail(VRT_E_INVALID, "null argument");
    VRT_TRY(validate_config(*cfg));
    return tp_plan(*cfg, world, rank, *out);
}

int vrt_tp_unique_id(void* h_out128) {
    clear_error();
    if (!h_out128) return fail(VRT_E_INVALID, "null argument");
    static Nccl n;
    VRT_TRY(nccl_load(n));
    const int r = n.GetUniqueId(h_out128);
    if (r) return fail(VRT_E_CUDA, "ncclGetUniqueId failed: %s", n.GetErrorString(r));
    return VRT_OK;
}

int vrt_batch_create(vrt_model* m, uint32_t max_seqs, uint32_t max_positions, int keep_logits, vrt_batch** out) {
    clear_error();
    if (!m || !out) return fail(VRT_E_INVALID, "null argument");
    *out = nullptr;
    if (!batch_supported(m)) {
        return fail(VRT_E_UNSUPPORTED, "batched decode needs 128-multiple projection widths per rank, "
                                       "1/2/4/8 query heads per KV head and a 128-multiple vocabulary shard");
    }
    if (max_seqs == 0 || max_seqs > 4096) return fail(VRT_E_INVALID, "max_seqs must be 1..4096");
    if (max_positions == 0 || max_positions > m->P) {
        return fail(VRT_E_INVALID, "batch max_positions must be 1..%u (the model's positions)", m->P);
    }
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    // batch_free releases the device memory too when a later step fails
    std::unique_ptr<vrt_batch, void (*)(vrt_batch*)> b(new vrt_batch(), batch_free);
    b->m = m;
    b->S = max_seqs;
    b->P = max_positions;
    b->out_cap = max_positions;
    b->keep_logits = keep_logits != 0;
    const auto& c = m->cfg;
    const uint64_t S = max_seqs, d = c.embedding_length, hd = c.head_dim;
    b->max_splits = std::min<uint32_t>(32u, kAttnWarps * c.head_dim);
    std::vector<uint64_t> sizes;  // bytes, 256-aligned pieces in this order
    for (uint32_t l = 0; l < c.block_count; ++l) {
        const uint32_t cap = m->layers[l].global ? max_positions : std::min(c.sliding_window, max_positions);
        b->cap.push_back(cap);
        sizes.push_back(S * m->KVl * cap * hd * 4);  // K
        sizes.push_back(S * m->KVl * cap * hd * 4);  // V
    }
    const uint64_t xw = std::max<uint64_t>(d, m->qwl);
    const uint64_t Sp = (S + 31) / 32 * 32, kmax = std::max<uint64_t>(xw, m->ffl);
    b->Sp = static_cast<uint32_t>(Sp);
    const uint64_t fixed[] = {S * 4, S * 4, S * b->out_cap * 4, S * 4, uint64_t(max_positions) * 4, S * 8,
                              S * m->KVl * 4,
                              S * d * 4, S * d * 4, S * (m->qwl + 2ull * m->kwl) * 4, S * d * 4, S * d * 4, S * d * 4,
                              b->keep_logits ? S * c.vocab_size * 4 : 0,
                              S * m->Hl * b->max_splits * 2 * 4, S * m->Hl * b->max_splits * hd * 4,
                              S * xw * 2, S * xw * 2, S * m->ffl * 2, S * m->ffl * 2,
                              Sp * kmax, Sp * kmax, kmax / 32 * Sp * 4, S * m->qwl * 4, S * m->ffl * 4};
    for (auto x : fixed) sizes.push_back(x);
    uint64_t total = 0;
    for (auto x : sizes) total += align256(x);
    VRT_CUDA(cudaMalloc(&b->mem, total));
    VRT_CUDA(cudaMemsetAsync(b->mem, 0, total, m->ctx->stream));
    uint8_t* p = static_cast<uint8_t*>(b->mem);
    size_t i = 0;
    auto take = [&]() {
        uint8_t* q = p;
        p += align256(sizes[i++]);
        return q;
    };
    for (uint32_t l = 0; l < c.block_count; ++l) {
        b->kc.push_back(reinterpret_cast<float*>(take()));
        b->vc.push_back(reinterpret_cast<float*>(take()));
    }
    b->tokens = reinterpret_cast<uint32_t*>(take());
    b->pos = reinterpret_cast<uint32_t*>(take());
    b->out_ids = reinterpret_cast<uint32_t*>(take());
    b->out_count = reinterpret_cast<uint32_t*>(take());
    b->prompt = reinterpret_cast<uint32_t*>(take());
    b->keys = reinterpret_cast<unsigned long long*>(take());
    b->tickets = reinterpret_cast<uint32_t*>(take());
    float** fl[] = {&b->h0, &b->h1, &b->qkv, &b->o, &b->dn, &b->hidden, &b->logits, &b->part_ml, &b->part_acc};
    for (auto f : fl) *f = reinterpret_cast<float*>(take());
    if (!b->keep_logits) b->logits = nullptr;
    __half** hl[] = {&b->xh, &b->xl, &b->ah, &b->al};
    for (auto h : hl) *h = reinterpret_cast<__half*>(take());
    b->q_hi = reinterpret_cast<int8_t*>(take());
    b->q_lo = reinterpret_cast<int8_t*>(take());
    b->q_sx = reinterpret_cast<float*>(take());
    b->att32 = reinterpret_cast<float*>(take());
    b->act32 = reinterpret_cast<float*>(take());
    VRT_TRY(make_f16_tmap(&b->xd_hi, b->xh, S, d, 16));
    VRT_TRY(make_f16_tmap(&b->xd_lo, b->xl, S, d, 16));
    VRT_TRY(make_f16_tmap(&b->xq_hi, b->xh, S, m->qwl, 16));
    VRT_TRY(make_f16_tmap(&b->xq_lo, b->xl, S, m->qwl, 16));
    VRT_TRY(make_f16_tmap(&b->xf_hi, b->ah, S, m->ffl, 16));
    VRT_TRY(make_f16_tmap(&b->xf_lo, b->al, S, m->ffl, 16));
    VRT_TRY(make_f16_tmap(&b->Xd_hi, b->xh, S, d, 128));
    VRT_TRY(make_f16_tmap(&b->Xd_lo, b->xl, S, d, 128));
    VRT_TRY(make_f16_tmap(&b->Xq_hi, b->xh, S, m->qwl, 128));
    VRT_TRY(make_f16_tmap(&b->Xq_lo, b->xl, S, m->qwl, 128));
    VRT_TRY(make_f16_tmap(&b->Xf_hi, b->ah, S, m->ffl, 128));
    VRT_TRY(make_f16_tmap(&b->Xf_lo, b->al, S, m->ffl, 128));
    VRT_TRY(make_i8_tmap(&b->Qd_hi, b->q_hi, Sp, d, 16));
    VRT_TRY(make_i8_tmap(&b->Qd_lo, b->q_lo, Sp, d, 16));
    VRT_TRY(make_i8_tmap(&b->Qq_hi, b->q_hi, Sp, m->qwl, 16));
    VRT_TRY(make_i8_tmap(&b->Qq_lo, b->q_lo, Sp, m->qwl, 16));
    VRT_TRY(make_i8_tmap(&b->Qf_hi, b->q_hi, Sp, m->ffl, 16));
    VRT_TRY(make_i8_tmap(&b->Qf_lo, b->q_lo, Sp, m->ffl, 16));
    // steps of up to 32 sequences run the integer tensor-core GEMMs when the
    // Q8M weight copy fits (else the fp16 form)
    b->i8 = model_q8m(m) == VRT_OK;
    if (!b->i8) clear_error();
    b->host_pos.assign(max_seqs, 0);
    VRT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    *out = b.release();
    return VRT_OK;
}

int vrt_batch_destroy(vrt_batch* b) {
    batch_free(b);
    return VRT_OK;
}

int vrt_batch_prefill(vrt_batch* b, uint32_t seq, const uint32_t* h_prompt, uint32_t n) {
    clear_error();
    if (!b || (!h_prompt && n)) return fail(VRT_E_INVALID, "null argument");
    vrt_model* m = b->m;
    const auto& c = m->cfg;
    if (seq >= b->S) return fail(VRT_E_INVALID, "sequence %u outside the batch of %u", seq, b->S);
    if (n == 0) return fail(VRT_E_INVALID, "Gemma 3 prompt produced no input tokens");
    if (n > b->P) return fail(VRT_E_STATE, "prompt of %u tokens exceeds the batch capacity %u", n, b->P);
    for (uint32_t i = 0; i < n; ++i) {
        if (h_prompt[i] >= c.vocab_size) return fail(VRT_E_INVALID, "Token id is outside Gemma 3 vocabulary");
    }
    cudaStream_t s = m->ctx->stream;
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    VRT_CUDA(cudaStreamSynchronize(s));
    VRT_CUDA(cudaMemcpyAsync(b->prompt, h_prompt, 4ull * n, cudaMemcpyHostToDevice, s));
    VRT_CUDA(cudaMemsetAsync(&m->st->status, 0, 4, s));
    SeqTarget t;
    t.prompt = b->prompt;
    for (uint32_t l = 0; l < c.block_count; ++l) {
        const uint64_t off = static_cast<uint64_t>(seq) * m->KVl * b->cap[l] * c.head_dim;
        t.kc.push_back(b->kc[l] + off);
        t.vc.push_back(b->vc[l] + off);
        t.cap.push_back(b->cap[l]);
    }
    t.positions = b->P;
    t.key = b->keys + seq;
    t.hidden = b->hidden + static_cast<uint64_t>(seq) * c.embedding_length;
    t.logits = b->keep_logits ? b->logits + static_cast<uint64_t>(seq) * c.vocab_size + m->vocab_lo : nullptr;
    VRT_CUDA(cudaMemsetAsync(t.key, 0, 8, s));
    VRT_TRY(prefill_layers(m, t, n));
    batch_finalize_kernel<<<1, 1, 0, s>>>(b->keys, b->tokens, b->pos, b->out_ids, b->out_count, b->out_cap, seq, 1,
                                          c.vocab_size, n, &m->st->status);
    VRT_CUDA(cudaGetLastError());
    uint32_t status = 0;
    VRT_CUDA(cudaMemcpyAsync(&status, &m->st->status, 4, cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaStreamSynchronize(s));
    if (status) return fail(status & kStatusWaitTimeout ? VRT_E_TIMEOUT : VRT_E_NUMERIC, "batch prefill: device status 0x%x", status);
    b->host_pos[seq] = n;
    return VRT_OK;
}

int vrt_batch_decode_steps(vrt_batch* b, uint32_t count, uint32_t steps) {
    clear_error();
    if (!b) return fail(VRT_E_INVALID, "null batch");
    if (count == 0 || count > b->S) return fail(VRT_E_INVALID, "count must be 1..%u", b->S);
    for (uint32_t i = 0; i < count; ++i) {
        if (b->host_pos[i] == 0) return fail(VRT_E_STATE, "sequence %u has not been prefilled", i);
        if (b->host_pos[i] + steps > b->P) return fail(VRT_E_STATE, "sequence %u would exceed the batch capacity", i);
    }
    vrt_model* m = b->m;
    cudaStream_t s = m->ctx->stream;
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    VRT_TRY(batch_gemm_workspace(b, count));
    if (m->opt.use_graph && (!b->graph || b->graph_count != count)) {
        if (b->graph) {
            VRT_CUDA(cudaStreamSynchronize(s));
            cudaGraphExecDestroy(b->graph);
            b->graph = nullptr;
        }
        cudaGraph_t g = nullptr;
        VRT_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        const int rc = batch_record_step(b, count);
        const cudaError_t e = cudaStreamEndCapture(s, &g);
        if (rc != VRT_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture", __FILE__, __LINE__);
        const cudaError_t ei = cudaGraphInstantiate(&b->graph, g, 0);
        cudaGraphDestroy(g);
        if (ei != cudaSuccess) return cuda_fail(ei, "cudaGraphInstantiate", __FILE__, __LINE__);
        b->graph_count = count;
    }
    for (uint32_t i = 0; i < steps; ++i) {
        if (b->graph) {
            VRT_CUDA(cudaGraphLaunch(b->graph, s));
        } else {
            VRT_TRY(batch_record_step(b, count));
        }
    }
    for (uint32_t i = 0; i < count; ++i) b->host_pos[i] += steps;
    return VRT_OK;
}

int vrt_batch_read(vrt_batch* b, uint32_t seq, uint32_t* h_ids, uint32_t cap, uint32_t* h_count,
                   uint32_t* h_position) {
    clear_error();
    if (!b || !h_count || (cap && !h_ids)) return fail(VRT_E_INVALID, "null argument");
    if (seq >= b->S) return fail(VRT_E_INVALID, "sequence %u outside the batch of %u", seq, b->S);
    vrt_model* m = b->m;
    cudaStream_t s = m->ctx->stream;
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    uint32_t cnt = 0, pos = 0, status = 0;
    VRT_CUDA(cudaMemcpyAsync(&cnt, b->out_count + seq, 4, cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaMemcpyAsync(&pos, b->pos + seq, 4, cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaMemcpyAsync(&status, &m->st->status, 4, cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaStreamSynchronize(s));
    if (status) return fail(status & kStatusWaitTimeout ? VRT_E_TIMEOUT : VRT_E_NUMERIC, "batch decode: device status 0x%x", status);
    const uint32_t k = std::min({cnt, cap, b->out_cap});
    if (k) {
        VRT_CUDA(cudaMemcpy(h_ids, b->out_ids + static_cast<uint64_t>(seq) * b->out_cap, 4ull * k, cudaMemcpyDeviceToHost));
    }
    *h_count = cnt;
    if (h_position) *h_position = pos;
    return VRT_OK;
}

int vrt_batch_last_ids(vrt_batch* b, uint32_t count, uint32_t* h_ids) {
    clear_error();
    if (!b || !h_ids) return fail(VRT_E_INVALID, "null argument");
    if (count > b->S) return fail(VRT_E_INVALID, "count must be <= %u", b->S);
    VRT_CUDA(cudaSetDevice(b->m->ctx->device));
    VRT_CUDA(cudaMemcpyAsync(h_ids, b->tokens, 4ull * count, cudaMemcpyDeviceToHost, b->m->ctx->stream));
    VRT_CUDA(cudaStreamSynchronize(b->m->ctx->stream));
    return VRT_OK;
}

int vrt_batch_logits(vrt_batch* b, uint32_t seq, float* h_logits) {
    clear_error();
    if (!b || !h_logits) return fail(VRT_E_INVALID, "null argument");
    if (!b->keep_logits) return fail(VRT_E_STATE, "batch created without keep_logits");
    if (seq >= b->S) return fail(VRT_E_INVALID, "sequence %u outside the batch of %u", seq, b->S);
    vrt_model* m = b->m;
    const uint32_t V = m->cfg.vocab_size, vl = m->vocab_hi - m->vocab_lo;
    cudaStream_t s = m->ctx->stream;
    VRT_CUDA(cudaSetDevice(m->ctx->device));
    float* row = b->logits + static_cast<uint64_t>(seq) * V;
    if (m->world > 1) {  // every rank holds its vocabulary columns: gather them (collective)
        const int r = m->nccl.AllGather(row + m->vocab_lo, row, vl, /*ncclFloat32*/ 7, m->comm, s);
        if (r) return fail(VRT_E_CUDA, "ncclAllGather(logits) failed: %s", m->nccl.GetErrorString(r));
    }
    VRT_CUDA(cudaMemcpyAsync(h_logits, row, 4ull * V, cudaMemcpyDeviceToHost, s));
    VRT_CUDA(cudaStreamSynchronize(s));
    return VRT_OK;
}

}  // extern "C"
