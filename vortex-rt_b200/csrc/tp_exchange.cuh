// Tensor-parallel exchange over peer memory (NVLink / NVSwitch), sm_100a.
//
// Row-parallel projections (attention output and FFN down) leave each rank
// with a partial sum of the d-wide block output.  Instead of an all-reduce
// kernel between the producer and the consumer, the consumer kernel (the
// next mat-vec, whose prologue needs the full vector for its RMSNorms) does
// the exchange itself:
//
//   1. push: every CTA takes a slice of the d elements and stores its rank's
//      partials into every peer's receive slots, one 64-bit word per element:
//      (sequence number << 32) | float bits.  A naturally aligned 64-bit
//      store is single-copy atomic, so a reader sees either the old word or
//      the new one, never a mix: the data carries its own ready flag and no
//      fence or separate signal is needed.
//   2. reduce: the same CTA polls its slice of its own receive slots until
//      every peer's word carries this exchange's sequence number, then sums
//      the ranks in rank order 0..world-1 (the same order on every rank, so
//      all ranks hold bit-identical residual streams).
//   3. share: a grid barrier (one arrival counter + a generation word set to
//      the sequence number) publishes the reduced vector to all CTAs.
//
// Sequence numbers are epoch * ops_per_step + op + 1, where the epoch is a
// device counter advanced by the step's finalize kernel and never reset, so a
// slot's stale word can never match.  Slots alternate between two sets (the
// attention-output exchange and the FFN-down exchange): a peer can only
// overwrite a set after this rank has pushed the following exchange, which
// it does only after it finished reading the set.
//
// Every wait is bounded by wall-clock time (globaltimer); on expiry the
// kernel sets kStatusPeerTimeout in the step status and carries on, and every
// later wait returns at once, so a lost peer costs one time-out, not one per
// element.  No multicast and no bulk copies touch peer memory.
#pragma once

#include "vrt_device.cuh"

namespace vrt {

constexpr uint32_t kStatusPeerTimeout = 1u << 3;
constexpr int kTpMaxWorld = 8;

struct TpParams {
    unsigned long long* const* peers;  // [world] receive-slot bases of all ranks (own included), device array
    unsigned long long* slots;         // this rank's receive slots
    const float* local;                // this rank's partial sums (n floats)
    float* sum;                        // reduced vector (n floats), this rank's memory
    uint32_t* bar_count;               // grid barrier arrival counter (starts at 0)
    uint32_t* bar_gen;                 // grid barrier generation word
    const uint32_t* epoch;             // StepState epoch
    uint64_t wait_ns;                  // time limit of one wait
    uint32_t rank, world, set, op, ops_per_step, n;
};

// Receive-slot word index: two sets of [world][n] partials, then [world][2]
// argmax key halves.
__host__ __device__ inline uint64_t tp_slot(uint32_t set, uint32_t src, uint32_t k, uint32_t world, uint32_t n) {
    return (static_cast<uint64_t>(set) * world + src) * n + k;
}
__host__ __device__ inline uint64_t tp_key_slot(uint32_t src, uint32_t half, uint32_t world, uint32_t n) {
    return 2ull * world * n + 2ull * src + half;
}
__host__ __device__ inline uint64_t tp_slot_words(uint32_t world, uint32_t n) { return 2ull * world * n + 2ull * world; }

__device__ __forceinline__ uint32_t tp_seq(const TpParams& t) {
    return *t.epoch * t.ops_per_step + t.op + 1u;
}

__device__ __forceinline__ void st_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool peer_timed_out(const uint32_t* status) {
    return (*reinterpret_cast<const volatile uint32_t*>(status) & kStatusPeerTimeout) != 0u;
}

__device__ __forceinline__ unsigned long long tp_word(uint32_t seq, uint32_t bits) {
    return (static_cast<unsigned long long>(seq) << 32) | bits;
}

// Wait (bounded) until *p carries `seq`; returns its low 32 bits.
__device__ __forceinline__ uint32_t tp_poll(const unsigned long long* p, uint32_t seq, uint64_t wait_ns,
                                            uint32_t* status) {
    unsigned long long w = ld_sys_u64(p);
    if (static_cast<uint32_t>(w >> 32) == seq) return static_cast<uint32_t>(w);
    if (peer_timed_out(status)) return static_cast<uint32_t>(w);
    const uint64_t t0 = global_ns();
    while (static_cast<uint32_t>(w >> 32) != seq) {
        if (global_ns() - t0 > wait_ns) {
            atomicOr(status, kStatusPeerTimeout);
            break;
        }
        w = ld_sys_u64(p);
    }
    return static_cast<uint32_t>(w);
}

// Steps 1 and 2 for elements [a, e): push this rank's partials to every
// peer, then sum all ranks' partials of the slice into t.sum.  Threads
// tid = 0..nthreads-1 of the calling CTA take part.
__device__ __forceinline__ void tp_slice_reduce(const TpParams& t, uint32_t seq, uint32_t a, uint32_t e, int tid,
                                                int nthreads, uint32_t* status) {
    const uint32_t ne = e - a;
    const uint32_t pushes = (t.world - 1) * ne;
    for (uint32_t i = tid; i < pushes; i += nthreads) {
        const uint32_t q = i / ne, k = a + i % ne;
        const uint32_t r = q < t.rank ? q : q + 1;
        const float v = __ldcg(t.local + k);
        st_sys_u64(t.peers[r] + tp_slot(t.set, t.rank, k, t.world, t.n), tp_word(seq, __float_as_uint(v)));
    }
    for (uint32_t k = a + tid; k < e; k += nthreads) {
        float acc = 0.0f;
        for (uint32_t r = 0; r < t.world; ++r) {
            const float v = r == t.rank ? __ldcg(t.local + k)
                                        : __uint_as_float(tp_poll(t.slots + tp_slot(t.set, r, k, t.world, t.n), seq,
                                                                  t.wait_ns, status));
            acc = r == 0 ? v : __fadd_rn(acc, v);
        }
        t.sum[k] = acc;
    }
}

// Step 3: called by one thread per CTA after the CTA's slice is written (and
// a CTA-wide barrier); returns when every CTA of the grid has arrived.
__device__ __forceinline__ void tp_grid_barrier(const TpParams& t, uint32_t seq, uint32_t* status) {
    __threadfence();
    const uint32_t old = atomicAdd(t.bar_count, 1u);
    if (old == gridDim.x - 1) {
        __threadfence();
        atomicExch(t.bar_count, 0u);
        st_release_gpu_u32(t.bar_gen, seq);
        return;
    }
    if (ld_acquire_gpu_u32(t.bar_gen) == seq || peer_timed_out(status)) return;
    const uint64_t t0 = global_ns();
    while (ld_acquire_gpu_u32(t.bar_gen) != seq) {
        if (global_ns() - t0 > t.wait_ns) {
            atomicOr(status, kStatusPeerTimeout);
            break;
        }
    }
    __threadfence();
}

// The argmax key exchange of the LM head (one thread): max over all ranks'
// 64-bit keys, each sent as two (seq, half) words.
__device__ __forceinline__ unsigned long long tp_key_max(const TpParams& t, unsigned long long key, uint32_t* status) {
    const uint32_t seq = tp_seq(t);
    for (uint32_t r = 0; r < t.world; ++r) {
        if (r == t.rank) continue;
        st_sys_u64(t.peers[r] + tp_key_slot(t.rank, 0, t.world, t.n), tp_word(seq, static_cast<uint32_t>(key >> 32)));
        st_sys_u64(t.peers[r] + tp_key_slot(t.rank, 1, t.world, t.n), tp_word(seq, static_cast<uint32_t>(key)));
    }
    unsigned long long best = key;
    for (uint32_t r = 0; r < t.world; ++r) {
        if (r == t.rank) continue;
        const uint32_t hi = tp_poll(t.slots + tp_key_slot(r, 0, t.world, t.n), seq, t.wait_ns, status);
        const uint32_t lo = tp_poll(t.slots + tp_key_slot(r, 1, t.world, t.n), seq, t.wait_ns, status);
        const unsigned long long k = (static_cast<unsigned long long>(hi) << 32) | lo;
        best = k > best ? k : best;
    }
    return best;
}

}  // namespace vrt
