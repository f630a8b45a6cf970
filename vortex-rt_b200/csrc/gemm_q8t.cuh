// Q8_0 x activation GEMM on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// Y[m][n] = sum_k X[m][k] * W[n][k] for M activation rows (prompt tokens or
// batched sequences) against a Q8T-tiled Q8_0 matrix W [N][K].  Q8_0 carries
// one fp16 scale per 32 weights along K for every row, which no tensor-core
// format can apply inside the accumulation, so the weights are dequantised
// on chip: w = scale * q is exact in fp32 (11 + 7 significant bits) and is
// split into two fp16 terms, w = w_hi + w_lo; the activations are split the
// same way.  Three MMAs per K step (x_hi.w_hi + x_lo.w_hi + x_hi.w_lo) into
// one fp32 TMEM accumulator leave a relative error near 1e-7, far inside the
// 1e-3 tolerance the fp32 reference path is held to (a single fp16 product
// would sit near 3e-4).
//
// The tensor core's fp32 accumulation truncates at every MMA, a bias that
// grows linearly with the number of MMAs into one accumulator (4e-4 relative
// at K = 21504 measured on B200).  So the K loop is cut into chunks of 256
// columns: each chunk accumulates into one of two TMEM accumulators (ping-
// pong), and a dedicated epilogue warpgroup drains every finished chunk into
// fp32 registers with round-to-nearest adds while the MMAs fill the other.
//
// One CTA computes a 128 (M) x 128 (N) tile.  Warp roles:
//   warp 0    producer: 2-D TMA loads (128B swizzle) of the x_hi / x_lo tiles
//             (64 K columns x 128 rows each) into the operand ring, and 1-D
//             bulk copies of the Q8T weight tiles (8 row groups x 128 K
//             columns, 17,408 bytes) into the raw ring;
//   warp 1    TMEM allocation; lane 0 issues tcgen05.mma (kind::f16, fp32
//             accumulate, both operands K-major) and tcgen05.commit;
//   warps 2-5 dequantise each raw stage into the w_hi / w_lo operand tiles in
//             the canonical K-major 128B-swizzled layout;
//   warps 6-13 epilogue: tcgen05.ld of each finished chunk accumulator (warp
//             w owns the 32 TMEM lanes = output rows of quarter w % 4 and 64
//             of the 128 columns), running fp32 sums in registers, then the
//             fused output stage.
// Every mbarrier wait is bounded; TMEM is always freed before exit.
#pragma once

#include <cuda_fp16.h>

#include "vrt_device.cuh"

namespace vrt {

enum GemmEpi : int {
    kGemmStore = 0,      // y[m][n] fp32
    kGemmGeluSplit = 1,  // W rows are 8 gate + 8 up per group: act = gelu(gate) * up -> fp16 hi/lo (+ optional fp32)
    kGemmArgmax = 2,     // per-row argmax key (atomicMax into keys[m]; ties -> lower index, NaN skipped) + optional y
};

constexpr int kGemmBM = 128;
constexpr int kGemmBN = 128;
constexpr int kGemmBK = 64;                                   // fp16 columns per operand stage (one 128-byte row)
constexpr int kGemmStages = 2;                                // operand ring
constexpr int kGemmRawStages = 2;                             // Q8T weight ring
constexpr int kGemmOpTile = kGemmBM * kGemmBK * 2;            // 16 KB: one 128 x 64 fp16 operand
constexpr int kGemmStageBytes = 4 * kGemmOpTile;              // x_hi, x_lo, w_hi, w_lo
constexpr int kGemmRawBytes = (kGemmBN / kTileRows) * kTileBytes;  // 17,408
constexpr int kGemmThreads = 448;
constexpr int kGemmEpiCols = 64;                              // accumulator columns per epilogue warp
constexpr int kGemmChunkStages = 4;                           // operand stages (256 K columns) per accumulator chunk
// Weight stages prefetched into L2 ahead of the shared-memory ring: a loaded
// B200 answers a bulk copy from HBM in ~3.5 us, so ~140 KB per SM must be in
// flight to stream at full rate; L2 holds that instead of shared memory.
constexpr int kGemmL2Ahead = 8;

// Prefetch raw stage `kt` (8 row groups' 2176-byte tiles, one 128-column K
// tile) of a Q8T matrix whose row groups start at `wg` (KT tiles per group).
__device__ __forceinline__ void prefetch_raw_stage(const uint8_t* wg, uint32_t KT, uint32_t kt) {
#pragma unroll
    for (int g = 0; g < kGemmBN / kTileRows; ++g) {
        bulk_prefetch_l2(wg + (static_cast<uint64_t>(g) * KT + kt) * kTileBytes, kTileBytes);
    }
}
constexpr uint32_t kGemmSmemBytes =
    1024 + kGemmStages * kGemmStageBytes + kGemmRawStages * kGemmRawBytes + 8 * (2 * kGemmStages + 2 * kGemmRawStages + 4) + 16;

// CUtensorMap storage (the driver's opaque 128-byte tensor map).
struct alignas(64) TmaMap {
    unsigned long long raw[16];
};

struct GemmParams {
    const uint8_t* w;     // Q8T matrix, N rows x K columns
    uint32_t n, k, m;     // N % 128 == 0, K % 128 == 0, M >= 1
    float* y;             // Store: y[m * ldy + n]
    uint32_t ldy;
    __half* act_hi;       // GeluSplit: act_*[m * ld_act + n / 2]
    __half* act_lo;
    float* act_f32;       // GeluSplit: optional fp32 copy
    uint32_t ld_act;
    unsigned long long* keys;  // Argmax: [M] keys, zero before the launch
    uint32_t row_base;         // Argmax: global index of weight row 0 (vocab shard)
    uint32_t nt;               // small-M form: activation rows per CTA (16, 32, 64 or 128)
    uint32_t ksplit;           // small-M form: CTAs along K per tile (partials in ws, last CTA reduces)
    float* ws;                 // [ksplit][t_tiles * nt][n] partial sums (ksplit > 1)
    uint32_t* tickets;         // [n / 128 * t_tiles], zero; reset by the reducing CTA
    uint32_t* status;
};

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ void tma_load_2d(void* dst, const TmaMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, M = 128, N = 128, K = 16, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on `bar` when all tcgen05.mma issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 8 consecutive fp32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive fp32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand of 128-byte rows, 8-row
// swizzle atoms of 1024 bytes stacked contiguously, 128B swizzle (layout 2),
// descriptor version 1, leading-byte offset 1 (unused for swizzled K-major).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptors: fp32 accumulate, fp16 A and B, both K-major, M = 128, N = 128 / 256.
constexpr uint32_t kGemmIdesc = (1u << 4) | (static_cast<uint32_t>(kGemmBN >> 3) << 17) | (static_cast<uint32_t>(kGemmBM >> 4) << 24);
constexpr uint32_t kGemmIdesc2 = (1u << 4) | (static_cast<uint32_t>((2 * kGemmBN) >> 3) << 17) | (static_cast<uint32_t>(kGemmBM >> 4) << 24);

// Byte offset of element (row, col) (col < 64) in a 128-row K-major operand
// tile with 128-byte rows and the 128B swizzle (16-byte chunk index XOR row % 8).
__host__ __device__ inline uint32_t sw128_offset(uint32_t row, uint32_t col) {
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((((col >> 3) ^ (row & 7u)) & 7u) << 4) + (col & 7u) * 2u;
}

// Dequantise one K half (64 columns) of a raw stage (8 Q8T tiles = 128 rows x
// 128 columns) into w_hi / w_lo.  t = 0..127: thread t handles Q8T tile t/16
// and one of the 16 lanes whose 32-column blocks fall into half h.
// Packed fp16 arithmetic, two weights per instruction: a byte permute puts
// each int8 (offset by 128) under the fp16 exponent of 1024, so subtracting
// 1152 gives q exactly; hi = RN(q * s) (one HMUL2 of the exact product) and
// lo = RN(q * s - hi) (one HFMA2) -- bit-identical to computing w = q * s in
// fp32 (exact) and splitting it there.
// PARTS threads share one (tile, lane) unit: thread t takes chunks
// s = (4/PARTS)*(t % PARTS) .. of unit t / PARTS (PARTS = 1: 128 threads,
// 2: 256 threads, each half the work).
template <int PARTS = 1>
__device__ __forceinline__ void dequant_half(const uint8_t* raw, int t, int h, uint8_t* whi, uint8_t* wlo) {
    constexpr int SN = 4 / PARTS;
    const int s0 = SN * (t % PARTS);
    t /= PARTS;
    const int tile = t >> 4, i = t & 15;
    const int ln = 4 * (i >> 1) + 2 * h + (i & 1);  // Q8T lane: rows 2*(ln/4)+{0,1}, block ln % 4
    const uint8_t* src = raw + tile * kTileBytes;
    const uint32_t sw = *reinterpret_cast<const uint32_t*>(src + kTileQBytes + 4 * ln);
    const __half2 s_even = __half2half2(__ushort_as_half(static_cast<unsigned short>(sw & 0xffffu)));
    const __half2 s_odd = __half2half2(__ushort_as_half(static_cast<unsigned short>(sw >> 16)));
    const __half2 bias = __float2half2_rn(1152.0f);
    const int kb = 32 * ((ln & 3) - 2 * h);  // 0 or 32 within the half
#pragma unroll
    for (int ss = 0; ss < SN; ++ss) {
        const int s = s0 + ss;
        const uint4 q = *reinterpret_cast<const uint4*>(src + (s * 32 + ln) * 16);
        const uint32_t row = tile * 16 + 2 * (ln >> 2) + (s >> 1);
        const uint32_t k0 = kb + 16 * (s & 1);
        const __half2 sc = (s >> 1) ? s_odd : s_even;
        const uint32_t qw[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
        for (int c = 0; c < 2; ++c) {  // two 16-byte chunks of 8 halves
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t word = qw[c * 2 + e / 2];
                const uint32_t biased = __byte_perm(word, 0x64646464u, (e & 1) ? 0x4342u : 0x4140u);
                const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&biased), bias);
                const __half2 hi = __hmul2(qv, sc);
                const __half2 lo = __hfma2(qv, sc, __hneg2(hi));
                hw[e] = *reinterpret_cast<const uint32_t*>(&hi);
                lw[e] = *reinterpret_cast<const uint32_t*>(&lo);
            }
            const uint32_t off = sw128_offset(row, k0 + 8 * c);
            *reinterpret_cast<uint4*>(whi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(wlo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    q8t_gemm_kernel(const __grid_constant__ TmaMap x_hi, const __grid_constant__ TmaMap x_lo, const GemmParams p) {
    extern __shared__ uint8_t gsm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = sm;
    uint8_t* raw = sm + kGemmStages * kGemmStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(raw + kGemmRawStages * kGemmRawBytes);
    uint64_t* empty = full + kGemmStages;
    uint64_t* raw_full = empty + kGemmStages;
    uint64_t* raw_empty = raw_full + kGemmRawStages;
    uint64_t* acc_full = raw_empty + kGemmRawStages;  // [2]: chunk accumulator ready
    uint64_t* acc_empty = acc_full + 2;               // [2]: chunk accumulator drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // M tiles vary fastest in launch order: the CTAs that share one weight
    // column run at the same time, so each weight tile leaves HBM once and the
    // other M tiles read it from L2 (the activations, M x K, stay in L2)
    const uint32_t m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * kGemmBN;
    const uint32_t KT = p.k / kTileCols;  // raw stages (128 K columns each)
    const uint32_t NI = 2 * KT;           // operand stages (64 K columns each)
    const uint32_t NC = (NI + kGemmChunkStages - 1) / kGemmChunkStages;  // accumulator chunks

    if (tid == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(&full[s], 1 + 4);
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < kGemmRawStages; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_empty[r], 4);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 8);
        }
        fence_mbar_init();
    }
    // w_lo follows w_hi in the stage, so one B operand of 256 rows covers both:
    // x_hi.[w_hi | w_lo] -> accumulator columns [0, 256), x_lo.w_hi adds into
    // [0, 128); the epilogue adds the two column blocks.  Two accumulators of
    // 256 columns fill TMEM.
    if (warp == 1) tmem_alloc(tmem_slot, 4 * kGemmBN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            const uint8_t* wg = p.w + static_cast<uint64_t>(n0 / kTileRows) * KT * kTileBytes;
            for (uint32_t kt = 0; kt < KT && kt < static_cast<uint32_t>(kGemmL2Ahead); ++kt) prefetch_raw_stage(wg, KT, kt);
            for (uint32_t kt = 0; kt < KT; ++kt) {
                if (kt + kGemmL2Ahead < KT) prefetch_raw_stage(wg, KT, kt + kGemmL2Ahead);
                const uint32_t r = kt % kGemmRawStages;
                if (kt >= kGemmRawStages) ok &= mbar_wait_bounded(&raw_empty[r], ((kt / kGemmRawStages) - 1) & 1);
                mbar_arrive_expect_tx(&raw_full[r], kGemmRawBytes);
                for (int g = 0; g < kGemmBN / kTileRows; ++g) {
                    bulk_copy_g2s(raw + r * kGemmRawBytes + g * kTileBytes,
                                  wg + (static_cast<uint64_t>(g) * KT + kt) * kTileBytes, kTileBytes, &raw_full[r]);
                }
                for (int h = 0; h < 2; ++h) {
                    const uint32_t i = 2 * kt + h, s = i % kGemmStages;
                    if (i >= kGemmStages) ok &= mbar_wait_bounded(&empty[s], ((i / kGemmStages) - 1) & 1);
                    uint8_t* st = ring + s * kGemmStageBytes;
                    mbar_arrive_expect_tx(&full[s], 2 * kGemmOpTile);
                    const int kx = static_cast<int>(kt * kTileCols + h * kGemmBK);
                    tma_load_2d(st, &x_hi, kx, static_cast<int>(m0), &full[s]);
                    tma_load_2d(st + kGemmOpTile, &x_lo, kx, static_cast<int>(m0), &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            for (uint32_t i = 0; i < NI; ++i) {
                const uint32_t c = i / kGemmChunkStages, a = c & 1, first = i % kGemmChunkStages == 0;
                if (first && c >= 2) ok &= mbar_wait_bounded(&acc_empty[a], ((c / 2) - 1) & 1);
                const uint32_t s = i % kGemmStages;
                ok &= mbar_wait_bounded(&full[s], (i / kGemmStages) & 1);
                tc_fence_after();
                const uint32_t base = smem_addr(ring + s * kGemmStageBytes);
                const uint32_t acc = tmem + a * 2 * kGemmBN;
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk) {
                    const uint32_t o = kk * 32;  // 16 fp16 = 32 bytes along K inside the swizzle atom
                    const uint64_t ahi = sw128_desc(base + o), alo = sw128_desc(base + kGemmOpTile + o);
                    const uint64_t bhl = sw128_desc(base + 2 * kGemmOpTile + o);  // w_hi rows then w_lo rows
                    umma_f16(acc, ahi, bhl, kGemmIdesc2, (first && kk == 0) ? 0u : 1u);
                    umma_f16(acc, alo, bhl, kGemmIdesc, 1u);
                }
                umma_commit(&empty[s]);
                if ((i + 1) % kGemmChunkStages == 0 || i + 1 == NI) umma_commit(&acc_full[a]);
            }
        }
    } else if (warp < 6) {
        // ------------------------------------------------------- dequant
        const int t = tid - 64;  // 0..127
        for (uint32_t kt = 0; kt < KT; ++kt) {
            const uint32_t r = kt % kGemmRawStages;
            ok &= mbar_wait_bounded(&raw_full[r], (kt / kGemmRawStages) & 1);
            for (int h = 0; h < 2; ++h) {
                const uint32_t i = 2 * kt + h, s = i % kGemmStages;
                if (i >= kGemmStages) ok &= mbar_wait_bounded(&empty[s], ((i / kGemmStages) - 1) & 1);
                uint8_t* st = ring + s * kGemmStageBytes;
                dequant_half(raw + r * kGemmRawBytes, t, h, st + 2 * kGemmOpTile, st + 3 * kGemmOpTile);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[r]);
        }
    } else {
        // ------------------------------------------------------- epilogue
        const uint32_t q = warp & 3;  // TMEM lane quarter this warp may access
        const uint32_t cb = ((warp - 6) >> 2) * kGemmEpiCols;  // first accumulator column of this warp
        const uint32_t row = m0 + 32 * q + lane;
        float sum[kGemmEpiCols];
#pragma unroll
        for (int j = 0; j < kGemmEpiCols; ++j) sum[j] = 0.0f;
        for (uint32_t c = 0; c < NC; ++c) {
            const uint32_t a = c & 1;
            ok &= mbar_wait_bounded(&acc_full[a], (c / 2) & 1);
            tc_fence_after();
#pragma unroll
            for (int c0 = 0; c0 < kGemmEpiCols; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + ((32 * q) << 16) + a * 2 * kGemmBN + cb + c0, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[c0 + j] = __fadd_rn(sum[c0 + j], __uint_as_float(v[j]));
                tmem_ld32(tmem + ((32 * q) << 16) + a * 2 * kGemmBN + kGemmBN + cb + c0, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[c0 + j] = __fadd_rn(sum[c0 + j], __uint_as_float(v[j]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
        }
        unsigned long long best = 0ull;
#pragma unroll
        for (int cl = 0; cl < kGemmEpiCols; cl += 32) {
            float* v = sum + cl;
            const uint32_t c0 = cb + cl;
            if (row >= p.m) continue;
            if (EPI == kGemmArgmax) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (!isnan(v[j])) {
                        const unsigned long long key = argmax_key(v[j], p.row_base + n0 + c0 + j);
                        best = key > best ? key : best;
                    }
                }
                if (p.y) {
                    float4* dst = reinterpret_cast<float4*>(p.y + static_cast<uint64_t>(row) * p.ldy + n0 + c0);
#pragma unroll
                    for (int e = 0; e < 8; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
                }
            } else if (EPI == kGemmStore) {
                float4* dst = reinterpret_cast<float4*>(p.y + static_cast<uint64_t>(row) * p.ldy + n0 + c0);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
                }
            } else {
                // columns c0..c0+31 = two row groups of 8 gate + 8 up rows
                const uint64_t o = static_cast<uint64_t>(row) * p.ld_act + (n0 + c0) / 2;
                uint32_t hw[8], lw[8];
                float a[16];
#pragma unroll
                for (int gg = 0; gg < 2; ++gg) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        a[8 * gg + j] = __fmul_rn(gelu_tanh(v[16 * gg + j]), v[16 * gg + 8 + j]);
                    }
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    __half h0, l0, h1, l1;
                    split_f16(a[2 * e], h0, l0);
                    split_f16(a[2 * e + 1], h1, l1);
                    hw[e] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
                    lw[e] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
                }
                uint4* dh = reinterpret_cast<uint4*>(p.act_hi + o);
                uint4* dl = reinterpret_cast<uint4*>(p.act_lo + o);
                dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                if (p.act_f32) {
                    float4* df = reinterpret_cast<float4*>(p.act_f32 + o);
#pragma unroll
                    for (int e = 0; e < 4; ++e) df[e] = make_float4(a[4 * e], a[4 * e + 1], a[4 * e + 2], a[4 * e + 3]);
                }
            }
        }
        if (EPI == kGemmArgmax && best != 0ull) atomicMax(p.keys + row, best);
    }
    __syncwarp();  // reconverge each warp (lane 0 of warps 0 and 1 ran alone) before the CTA barrier
    if (!ok) atomicOr(p.status, kStatusWaitTimeout);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 4 * kGemmBN);
    }
}

// --------------------------------------------------------------- small M
//
// Batched decode form: the 128 lanes of the MMA carry weight rows and N
// carries p.nt activation rows (16..128), so 32 sequences issue a quarter of
// the tensor work of a 128-row tile.  The weight stream is the bottleneck at
// small M, so this form keeps more of it in flight (operand stages sized for
// NTMAX activation rows, 5-7 raw Q8T stages) and splits K across grid.z when
// the tiles alone do not fill the SMs: each CTA sums a K range, non-final
// CTAs leave fp32 partials in p.ws, and the last CTA of the tile (atomic
// ticket) adds the splits in split order -- deterministic whichever CTA is
// last -- and runs the epilogue.  Same dequantisation, hi/lo split and
// chunked promotion as the large-M kernel.  Epilogue per token column,
// writes coalesced across lanes: store, gelu(gate) * up (gate row r and up
// row r + 8 of a 16-row group meet through a lane shuffle), or argmax (warp
// max of the 64-bit keys, one atomicMax per token and warp).
template <int NTMAX>
struct SmallGemmLayout {
    static constexpr int kW = NTMAX <= 64 ? 4 : 3;                       // dequantised weight stages (w_hi, w_lo)
    static constexpr int kWStage = 2 * kGemmOpTile;                      // 32 KB
    static constexpr int kX = 2;                                         // activation stages (x_hi, x_lo)
    static constexpr int kXBytes = NTMAX * 128;                          // one activation operand tile
    static constexpr int kXStage = 2 * kXBytes;
    static constexpr int kFree = 232448 - 1024 - 512 - kW * kWStage - kX * kXStage;
    static constexpr int kRaw = kFree / kGemmRawBytes > 8 ? 8 : kFree / kGemmRawBytes;   // Q8T stages in flight
    static constexpr uint32_t kBars = 8 * (2 * kW + 2 * kX + 2 * kRaw + 4);
    static constexpr uint32_t kSmem = 1024 + kW * kWStage + kX * kXStage + kRaw * kGemmRawBytes + kBars + 16;
};

// warps: 0 weight stream, 1 MMA, 2-5 and 14-17 dequantisation, 6-13 epilogue,
// 18 activation stream
constexpr int kGemmSmallThreads = 608;

template <int EPI, int NTMAX>
__global__ void __launch_bounds__(kGemmSmallThreads, 1)
    q8t_gemm_small_kernel(const __grid_constant__ TmaMap x_hi, const __grid_constant__ TmaMap x_lo, const GemmParams p) {
    using LY = SmallGemmLayout<NTMAX>;
    constexpr int S = LY::kW, D = LY::kX, R = LY::kRaw;
    extern __shared__ uint8_t gsm_raw[];
    __shared__ uint32_t last_cta;
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* wring = sm;
    uint8_t* xring = wring + S * LY::kWStage;
    uint8_t* raw = xring + D * LY::kXStage;
    uint64_t* w_full = reinterpret_cast<uint64_t*>(raw + R * kGemmRawBytes);
    uint64_t* w_empty = w_full + S;
    uint64_t* x_full = w_empty + S;
    uint64_t* x_empty = x_full + D;
    uint64_t* raw_full = x_empty + D;
    uint64_t* raw_empty = raw_full + R;
    uint64_t* acc_full = raw_empty + R;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t NT = p.nt;  // 16, 32, 64 or 128 (<= NTMAX)
    const uint32_t n0 = blockIdx.x * kGemmBN, t0 = blockIdx.y * NT;
    const uint32_t KTALL = p.k / kTileCols;
    const uint32_t kt0 = KTALL * blockIdx.z / p.ksplit, kt1 = KTALL * (blockIdx.z + 1) / p.ksplit;
    const uint32_t KT = kt1 - kt0, NI = 2 * KT;
    const uint32_t NC = (NI + kGemmChunkStages - 1) / kGemmChunkStages;
    // x_lo sits right after x_hi's NT rows, so one B operand of 2*NT rows
    // covers both: w_hi.[x_hi | x_lo] -> accumulator columns [0, 2NT), then
    // w_lo.x_hi adds into [0, NT); the epilogue adds the two column blocks.
    // Two MMAs per K step read each weight tile once.
    const uint32_t tcols = 4u * NT;  // two accumulators of 2*NT columns
    const uint32_t idesc2 = (1u << 4) | (((2 * NT) >> 3) << 17) | (static_cast<uint32_t>(kGemmBN >> 4) << 24);
    const uint32_t idesc1 = (1u << 4) | ((NT >> 3) << 17) | (static_cast<uint32_t>(kGemmBN >> 4) << 24);

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&w_full[s], 8);
            mbar_init(&w_empty[s], 1);
        }
        for (int d = 0; d < D; ++d) {
            mbar_init(&x_full[d], 1);
            mbar_init(&x_empty[d], 1);
        }
        for (int r = 0; r < R; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_empty[r], 8);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 8);
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
        // weight stream, up to R stages ahead of the dequantisation
        if (lane == 0) {
            const uint8_t* wg = p.w + static_cast<uint64_t>(n0 / kTileRows) * KTALL * kTileBytes;
            for (uint32_t kt = 0; kt < KT && kt < static_cast<uint32_t>(kGemmL2Ahead); ++kt) {
                prefetch_raw_stage(wg, KTALL, kt0 + kt);
            }
            for (uint32_t kt = 0; kt < KT; ++kt) {
                if (kt + kGemmL2Ahead < KT) prefetch_raw_stage(wg, KTALL, kt0 + kt + kGemmL2Ahead);
                const uint32_t r = kt % R;
                if (kt >= static_cast<uint32_t>(R)) ok &= mbar_wait_bounded(&raw_empty[r], ((kt / R) - 1) & 1);
                mbar_arrive_expect_tx(&raw_full[r], kGemmRawBytes);
                for (int g = 0; g < kGemmBN / kTileRows; ++g) {
                    bulk_copy_g2s(raw + r * kGemmRawBytes + g * kTileBytes,
                                  wg + (static_cast<uint64_t>(g) * KTALL + kt0 + kt) * kTileBytes, kTileBytes,
                                  &raw_full[r]);
                }
            }
        }
    } else if (warp == 18) {
        // activation tiles (16-row TMA boxes), up to D stages ahead of the MMAs
        if (lane == 0) {
            for (uint32_t i = 0; i < NI; ++i) {
                const uint32_t d = i % D;
                if (i >= static_cast<uint32_t>(D)) ok &= mbar_wait_bounded(&x_empty[d], ((i / D) - 1) & 1);
                uint8_t* st = xring + d * LY::kXStage;
                mbar_arrive_expect_tx(&x_full[d], 2 * NT * 128);
                const int kx = static_cast<int>((kt0 + i / 2) * kTileCols + (i & 1) * kGemmBK);
                for (uint32_t r0 = 0; r0 < NT; r0 += 16) {
                    tma_load_2d(st + r0 * 128, &x_hi, kx, static_cast<int>(t0 + r0), &x_full[d]);
                    tma_load_2d(st + (NT + r0) * 128, &x_lo, kx, static_cast<int>(t0 + r0), &x_full[d]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (uint32_t i = 0; i < NI; ++i) {
                const uint32_t c = i / kGemmChunkStages, a = c & 1, first = i % kGemmChunkStages == 0;
                if (first && c >= 2) ok &= mbar_wait_bounded(&acc_empty[a], ((c / 2) - 1) & 1);
                const uint32_t s = i % S, d = i % D;
                ok &= mbar_wait_bounded(&w_full[s], (i / S) & 1);
                ok &= mbar_wait_bounded(&x_full[d], (i / D) & 1);
                tc_fence_after();
                const uint32_t wb = smem_addr(wring + s * LY::kWStage), xb = smem_addr(xring + d * LY::kXStage);
                const uint32_t acc = tmem + a * 2 * NT;
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk) {
                    const uint32_t o = kk * 32;
                    const uint64_t xhl = sw128_desc(xb + o);  // x_hi rows then x_lo rows
                    const uint64_t whi = sw128_desc(wb + o), wlo = sw128_desc(wb + kGemmOpTile + o);
                    umma_f16(acc, whi, xhl, idesc2, (first && kk == 0) ? 0u : 1u);
                    umma_f16(acc, wlo, xhl, idesc1, 1u);
                }
                umma_commit(&w_empty[s]);
                umma_commit(&x_empty[d]);
                if ((i + 1) % kGemmChunkStages == 0 || i + 1 == NI) umma_commit(&acc_full[a]);
            }
        }
    } else if (warp < 6 || warp >= 14) {
        const int t = warp < 6 ? tid - 64 : tid - 448 + 128;  // 0..255
        for (uint32_t kt = 0; kt < KT; ++kt) {
            const uint32_t r = kt % R;
            ok &= mbar_wait_bounded(&raw_full[r], (kt / R) & 1);
            for (int h = 0; h < 2; ++h) {
                const uint32_t i = 2 * kt + h, s = i % S;
                if (i >= static_cast<uint32_t>(S)) ok &= mbar_wait_bounded(&w_empty[s], ((i / S) - 1) & 1);
                uint8_t* st = wring + s * LY::kWStage;
                dequant_half<2>(raw + r * kGemmRawBytes, t, h, st, st + kGemmOpTile);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&w_full[s]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[r]);
        }
    } else {
        // epilogue: lanes = weight rows n0 + 32q + lane; this warp's token columns [cb, cb + NT/2)
        const uint32_t q = warp & 3;
        const uint32_t half_cols = NT / 2;
        const uint32_t cb = ((warp - 6) >> 2) * half_cols;
        const uint32_t row = n0 + 32 * q + lane;
        float sum[NTMAX / 2];
#pragma unroll
        for (int j = 0; j < NTMAX / 2; ++j) sum[j] = 0.0f;
        for (uint32_t c = 0; c < NC; ++c) {
            const uint32_t a = c & 1;
            ok &= mbar_wait_bounded(&acc_full[a], (c / 2) & 1);
            tc_fence_after();
#pragma unroll
            for (int j0 = 0; j0 < NTMAX / 2; j0 += 8) {
                if (static_cast<uint32_t>(j0) < half_cols) {
                    uint32_t v[8], u[8];
                    tmem_ld8(tmem + ((32 * q) << 16) + a * 2 * NT + cb + j0, v);
                    tmem_ld8(tmem + ((32 * q) << 16) + a * 2 * NT + NT + cb + j0, u);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        sum[j0 + e] = __fadd_rn(__fadd_rn(sum[j0 + e], __uint_as_float(v[e])), __uint_as_float(u[e]));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
        }
        bool last = true;
        if (p.ksplit > 1) {
            // partials of this K range out; the last CTA of the tile adds all ranges in split order
            const uint64_t mp = static_cast<uint64_t>(gridDim.y) * NT;  // padded token rows
            float* mine = p.ws + static_cast<uint64_t>(blockIdx.z) * mp * p.n;
#pragma unroll
            for (int j = 0; j < NTMAX / 2; ++j) {
                if (static_cast<uint32_t>(j) < half_cols) mine[(t0 + cb + j) * static_cast<uint64_t>(p.n) + row] = sum[j];
            }
            __threadfence();
            named_bar_sync(2, 256);
            if (warp == 6 && lane == 0) {
                const uint32_t tk = atomicAdd(p.tickets + blockIdx.y * gridDim.x + blockIdx.x, 1u);
                last_cta = tk == p.ksplit - 1 ? 1u : 0u;
            }
            named_bar_sync(2, 256);
            last = last_cta != 0;
            if (last) {
                __threadfence();
#pragma unroll
                for (int j = 0; j < NTMAX / 2; ++j) {
                    if (static_cast<uint32_t>(j) < half_cols) {
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
                if (warp == 6 && lane == 0) p.tickets[blockIdx.y * gridDim.x + blockIdx.x] = 0u;
            }
        }
        if (last) {
#pragma unroll
            for (int j = 0; j < NTMAX / 2; ++j) {
                if (static_cast<uint32_t>(j) >= half_cols) continue;  // warp-uniform
                const uint32_t tok = t0 + cb + j;
                const float v = sum[j];
                if (EPI == kGemmStore) {
                    if (tok < p.m) p.y[static_cast<uint64_t>(tok) * p.ldy + row] = v;
                } else if (EPI == kGemmGeluSplit) {
                    const float up = __shfl_down_sync(0xffffffffu, v, 8);
                    if (tok < p.m && (lane & 8) == 0) {
                        const float act = __fmul_rn(gelu_tanh(v), up);
                        const uint64_t o = static_cast<uint64_t>(tok) * p.ld_act + (row >> 4) * 8 + (lane & 7);
                        __half hh, ll;
                        split_f16(act, hh, ll);
                        p.act_hi[o] = hh;
                        p.act_lo[o] = ll;
                        if (p.act_f32) p.act_f32[o] = act;
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
