// Launch entry points shared between runtime.cu and model.cu.
#pragma once

#include <cuda_runtime.h>

#include "attention.cuh"
#include "gemm_q8t.cuh"
#include "gemv_q8t.cuh"

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

// CTAs for a Q8T mat-vec: one per SM, at most one per row group.
inline int gemv_grid(int sms, uint32_t rows) {
    const uint32_t groups = (rows + kTileRows - 1) / kTileRows;
    return static_cast<int>(groups < static_cast<uint32_t>(sms) ? groups : static_cast<uint32_t>(sms));
}

}  // namespace vrt
