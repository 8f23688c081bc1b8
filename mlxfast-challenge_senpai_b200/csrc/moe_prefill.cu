// MoE block, prefill path (many tokens): sorted grouped expert GEMMs.
#include "moe.cuh"
#include "moe_prefill.cuh"

namespace b2 {

size_t prefill_workspace_bytes(const b2_moe_block* blk, int64_t T) { return decode_workspace_bytes(blk, T); }

int prefill_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits,
                    const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, void* workspace,
                    size_t ws_bytes, cudaStream_t st) {
  return decode_forward(blk, x, T, logits, residual, out, inds, weights, workspace, ws_bytes, st);
}

}  // namespace b2
