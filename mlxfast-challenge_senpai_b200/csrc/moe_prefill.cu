// MoE block, prefill path (many tokens).
//
// Interim implementation: the block is processed in chunks of 8 tokens by the
// fused decode kernel.  The sorted grouped-GEMM path replaces it.
#include <algorithm>

#include "moe.cuh"
#include "moe_prefill.cuh"

namespace b2 {

size_t prefill_workspace_bytes(const b2_moe_block* blk, int64_t T) {
  (void)T;
  return decode_workspace_bytes(blk, kDecodeMaxTokens);
}

int prefill_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits,
                    const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, void* workspace,
                    size_t ws_bytes, cudaStream_t st) {
  const int64_t H = blk->hidden, E = blk->n_experts, k = blk->top_k;
  for (int64_t t0 = 0; t0 < T; t0 += kDecodeMaxTokens) {
    const int64_t n = std::min<int64_t>(kDecodeMaxTokens, T - t0);
    const int rc = decode_forward(blk, x + t0 * H, n, logits ? logits + t0 * E : nullptr,
                                  residual ? residual + t0 * H : nullptr, out + t0 * H, inds ? inds + t0 * k : nullptr,
                                  weights ? weights + t0 * k : nullptr, workspace, ws_bytes, st);
    if (rc) return rc;
  }
  return B2_OK;
}

}  // namespace b2
