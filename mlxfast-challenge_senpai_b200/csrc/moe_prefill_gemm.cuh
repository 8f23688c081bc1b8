// Prefill grouped GEMMs (tcgen05) and their helpers; see moe_prefill_gemm.cu.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace b2 {
namespace pf {

// Bytes of the prefill bank (the same as the three MLX-layout banks).
size_t prefill_bank_bytes(const b2_moe_block* blk);
// hidden % 256 == 0, ffn % 128 == 0, at most 1024 experts.
bool prefill_gemm_supported(const b2_moe_block* blk);
int prepare_prefill(const b2_moe_block* blk, void* dst, cudaStream_t st);
// f16 copy of `rows` bf16 rows of K values with a per-row power-of-two
// pre-scale (exps[row] = p, values times 2^-p).
int to_f16_rows(const uint16_t* src, int64_t rows, int K, __half* dst, int* exps, cudaStream_t st);
// dst[p] = src[order[p] / k] for p < rows (f16 rows of K values).
int gather_rows(const __half* src, const uint32_t* order, int k, int64_t rows, int K, __half* dst, cudaStream_t st);
// tile_off[e] = first 128-row M-tile of expert e; tile_off[E] = total.
int tile_offsets(const uint32_t* offsets, int E, uint32_t* tile_off, cudaStream_t st);
// mode 0: act[rows][F] = SwiGLU(x16[token(row)] * gate/up^T); mode 1:
// y[rows][H] = act16[row] * down^T (bf16, per sorted row).
// a16: a_rows rows of K f16 values in expert-sorted order (gate/up: the token
// rows gathered by gather_rows; down: the SwiGLU rows).
int grouped_gemm(int mode, const b2_moe_block* blk, const __half* a16, int64_t a_rows, const int* rexp,
                 const uint32_t* order, const uint32_t* offsets, const uint32_t* tile_off, uint16_t* out,
                 cudaStream_t st);

}  // namespace pf
}  // namespace b2
