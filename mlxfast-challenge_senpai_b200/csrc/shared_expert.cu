// Shared expert of the MoE block (the reference runtime's LagunaRuntimeMLP,
// RM:7971-8275): a dense NVFP4 SwiGLU MLP on every token,
//   s = down(silu(gate(x)) * up(x)),
// each projection a quantized_matmul with bf16 output (MLX's
// QuantizedLinear on bf16 x: QuantizedMM output in x's dtype), the SwiGLU
// the reference's bf16 chain (RM:6843-6852).  Its output enters the block's
// combine after the routed scale and before the residual (RM:10170-10186).
#include "moe.cuh"

namespace b2 {

namespace {
size_t a256(size_t v) { return (v + 255) & ~size_t(255); }
}  // namespace

size_t shared_scratch_bytes(const b2_moe_block* blk, int64_t T) {
  if (!blk->shared_gate_codes) return 0;
  const size_t Fs = (size_t)blk->shared_ffn, H = (size_t)blk->hidden;
  return 3 * a256((size_t)T * Fs * 2) + a256((size_t)T * H * 2);
}

int shared_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, void* scratch, const uint16_t** s,
                   cudaStream_t st) {
  *s = nullptr;
  if (!blk->shared_gate_codes) return B2_OK;
  const int64_t Fs = blk->shared_ffn, H = blk->hidden;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  uint16_t* g = reinterpret_cast<uint16_t*>(base);
  uint16_t* u = reinterpret_cast<uint16_t*>(base + a256((size_t)T * Fs * 2));
  uint16_t* a = reinterpret_cast<uint16_t*>(base + 2 * a256((size_t)T * Fs * 2));
  uint16_t* out = reinterpret_cast<uint16_t*>(base + 3 * a256((size_t)T * Fs * 2));
  int rc = qmm_bf16(x, blk->shared_gate_codes, blk->shared_gate_scales, T, Fs, H, g, st);
  if (rc) return rc;
  rc = qmm_bf16(x, blk->shared_up_codes, blk->shared_up_scales, T, Fs, H, u, st);
  if (rc) return rc;
  rc = launch_silu_mul(g, u, T * Fs, a, st);
  if (rc) return rc;
  rc = qmm_bf16(a, blk->shared_down_codes, blk->shared_down_scales, T, H, Fs, out, st);
  if (rc) return rc;
  *s = out;
  return B2_OK;
}

}  // namespace b2
