// Launch entry points shared between runtime.cu and model.cu.
#pragma once

#include <cuda_runtime.h>

#include "attention.cuh"
#include "gemm_i8.cuh"
#include "gemm_q8t.cuh"
#include "gemv_q8t.cuh"
#include "step_persistent.cuh"

namespace vrt {

// Q8T mat-vec with prologue `pro` (Pro) and epilogue `epi` (Epi).
cudaError_t gemv_q8t(int pro, int epi, const GemvParams& p, int grid, cudaStream_t s, bool pdl);
uint32_t gemv_smem_bytes(int pro, uint32_t cols);
cudaError_t gemv_init_attributes();
cudaError_t argmax_unkey_launch(const unsigned long long* key, uint32_t* out, cudaStream_t s);
cudaError_t attention_launch(const AttnParams& p, dim3 grid, cudaStream_t s, bool pdl);

// Tensor-core Q8T GEMM (gemm.cu): epilogue `epi` (GemmEpi); operands from
// make_f16_tmap over fp16 hi / lo activation matrices of at least p.m rows.
cudaError_t gemm_q8t(int epi, const TmaMap& hi, const TmaMap& lo, const GemmParams& p, cudaStream_t s);
// Small-M form (p.m rows in tiles of p.nt = gemm_small_tile(...); operand maps with 16-row boxes).
cudaError_t gemm_q8t_small(int epi, const TmaMap& hi, const TmaMap& lo, const GemmParams& p, cudaStream_t s);
uint32_t gemm_small_tile(uint32_t m);
uint32_t gemm_small_ksplit(uint32_t n, uint32_t m, uint32_t k, int sms);
int make_f16_tmap(TmaMap* out, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
cudaError_t split_f16(const float* x, uint64_t n, __half* hi, __half* lo, cudaStream_t s);

// Integer tensor-core GEMM for few activation rows (gemm_i8.cuh): Q8M copy
// of a Q8T matrix, int16 split activations (operand maps over the int8
// hi / lo arrays with 16-row boxes), p.nt = 16 or 32.
cudaError_t q8t_to_q8m(const uint8_t* src, uint32_t rows, uint32_t cols, uint8_t* dst, cudaStream_t s);
cudaError_t quant_rows(const float* x, uint32_t ldx, uint32_t rows, uint32_t k, const Q16Out& o, cudaStream_t s);
cudaError_t gemm_q8m_i8(int epi, const TmaMap& hi, const TmaMap& lo, const GemmI8Params& p, cudaStream_t s);
int make_i8_tmap(TmaMap* out, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);

// Persistent decode step (step.cu): raise the kernel's dynamic shared-memory
// limit and report it (and, for `smem` bytes, the resident CTAs per SM);
// cooperative launch of one step.
cudaError_t ps_limits(uint32_t hd, uint32_t rg, uint32_t smem, uint32_t* max_dynamic, int* blocks_per_sm);
cudaError_t ps_launch(const PsParams& p, uint32_t grid, uint32_t smem, cudaStream_t s);

// CTAs for a Q8T mat-vec: one per SM, at most one per row group.
inline int gemv_grid(int sms, uint32_t rows) {
    const uint32_t groups = (rows + kTileRows - 1) / kTileRows;
    return static_cast<int>(groups < static_cast<uint32_t>(sms) ? groups : static_cast<uint32_t>(sms));
}

}  // namespace vrt
