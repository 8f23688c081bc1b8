// Fused decode MoE block (one cooperative launch); see moe_decode.cu.
#pragma once

#include "common.cuh"

namespace b2 {
namespace dec {

// Scratch layout (offsets 256-byte aligned): [cross-launch state:
// kDecodeStateBytes, zero before the first call; activation counters, launch
// epochs and tagged router logits, see moe_decode_common.cuh] [inds T*k u32]
// [weights T*k f32] [activations T*k*F bf16].
size_t scratch_bytes(const b2_moe_block* blk, int64_t T);

int forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits, const uint16_t* residual,
            uint16_t* out, uint32_t* inds, float* weights, void* scratch, size_t scratch_len, cudaStream_t st);

size_t bank_bytes(const b2_moe_block* blk);
int prepare(const b2_moe_block* blk, void* dst, cudaStream_t st);

}  // namespace dec
}  // namespace b2
