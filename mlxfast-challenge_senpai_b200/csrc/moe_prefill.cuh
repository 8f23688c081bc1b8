// MoE block entry points shared between the decode and prefill paths.
#pragma once

#include "common.cuh"

namespace b2 {

// Calls with at most this many tokens take the fused gathered-GEMV path.
constexpr int64_t kDecodeMaxTokens = 8;

int validate_block(const b2_moe_block* b, const char* op);
int decode_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits,
                   const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, void* workspace,
                   size_t ws_bytes, cudaStream_t st);
size_t decode_workspace_bytes(const b2_moe_block* blk, int64_t T);
size_t prefill_workspace_bytes(const b2_moe_block* blk, int64_t T);
int prefill_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits,
                    const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, void* workspace,
                    size_t ws_bytes, cudaStream_t st);

}  // namespace b2
