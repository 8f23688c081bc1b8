// MoE block, prefill path (more than 8 tokens).
//
// With a prepared prefill bank (b2_moe_prepare_prefill_bank) the block runs
// as the reference's sorted prefill branch (RM:9867-10187 prefill side,
// SWL:476-524 with sorted indices):
//   router logits -> top-k -> stable expert sort of the (token, slot) rows
//   -> token tiles per expert -> token rows gathered into expert order (as
//   f16 with a per-row power-of-two pre-scale, exact) ->
//   gate/up grouped GEMM with the SwiGLU epilogue -> down grouped GEMM ->
//   ordered weighted combine (+ scale, + residual).
// Without it (or for shapes the grouped GEMM does not cover) the tokens go
// through the fused decode kernel 8 at a time.
#include <algorithm>

#include "moe.cuh"
#include "moe_prefill.cuh"
#include "moe_prefill_gemm.cuh"
#include "router.cuh"

namespace b2 {

struct PrefillWs {
  float* logits;
  uint32_t* inds;
  float* weights;
  uint32_t *order, *sorted, *inverse, *offsets, *sort_scratch;
  int4* tiles;
  int* ntiles;
  uint16_t *xs, *act, *y;
  int* xexp;  // per gathered row: f16 pre-scale exponent of its token
  uint8_t* shared_scratch;
  size_t bytes;
};

// Carve the workspace (the head, kDecodeStateBytes, is the decode kernels'
// cross-launch state and is left untouched).  base == nullptr only sizes it.
static PrefillWs carve(const b2_moe_block* blk, int64_t T, uint8_t* base) {
  const int64_t E = blk->n_experts, H = blk->hidden, F = blk->ffn, k = blk->top_k, n = T * k;
  PrefillWs w{};
  size_t off = kDecodeStateBytes;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += (bytes + 255) & ~size_t(255);
    return p;
  };
  w.logits = reinterpret_cast<float*>(take((size_t)T * E * 4));
  w.inds = reinterpret_cast<uint32_t*>(take((size_t)n * 4));
  w.weights = reinterpret_cast<float*>(take((size_t)n * 4));
  w.order = reinterpret_cast<uint32_t*>(take((size_t)n * 4));
  w.sorted = reinterpret_cast<uint32_t*>(take((size_t)n * 4));
  w.inverse = reinterpret_cast<uint32_t*>(take((size_t)n * 4));
  w.offsets = reinterpret_cast<uint32_t*>(take((size_t)(E + 1) * 4));
  w.sort_scratch = reinterpret_cast<uint32_t*>(take(gather_sort_scratch_bytes(n, E)));
  w.tiles = reinterpret_cast<int4*>(take((size_t)pf::max_tiles(E, n) * sizeof(int4)));
  w.ntiles = reinterpret_cast<int*>(take(4));
  w.xs = reinterpret_cast<uint16_t*>(take((size_t)n * H * 2));
  w.xexp = reinterpret_cast<int*>(take((size_t)n * 4));
  w.act = reinterpret_cast<uint16_t*>(take((size_t)n * F * 2));
  w.y = reinterpret_cast<uint16_t*>(take((size_t)n * H * 2));
  w.shared_scratch = take(shared_scratch_bytes(blk, T));
  w.bytes = off;
  return w;
}

namespace {

bool use_gemm(const b2_moe_block* blk) { return blk->prefill_bank != nullptr && pf::prefill_gemm_supported(blk); }

}  // namespace

int experts_sorted(const b2_moe_block* blk, const uint16_t* x, int64_t T, const uint32_t* inds, PrefillWs& w,
                   uint16_t* y, cudaStream_t st);

size_t prefill_workspace_bytes(const b2_moe_block* blk, int64_t T) {
  if (use_gemm(blk)) return carve(blk, T, nullptr).bytes;
  return decode_workspace_bytes(blk, kDecodeMaxTokens);
}

int prefill_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits,
                    const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, void* workspace,
                    size_t ws_bytes, cudaStream_t st) {
  const int64_t H = blk->hidden, E = blk->n_experts, k = blk->top_k, F = blk->ffn;
  if (!use_gemm(blk)) {
    for (int64_t t0 = 0; t0 < T; t0 += kDecodeMaxTokens) {
      const int64_t n = std::min<int64_t>(kDecodeMaxTokens, T - t0);
      const int rc = decode_forward(blk, x + t0 * H, n, logits ? logits + t0 * E : nullptr,
                                    residual ? residual + t0 * H : nullptr, out + t0 * H,
                                    inds ? inds + t0 * k : nullptr, weights ? weights + t0 * k : nullptr, workspace,
                                    ws_bytes, st);
      if (rc) return rc;
    }
    return B2_OK;
  }
  PrefillWs w = carve(blk, T, static_cast<uint8_t*>(workspace));
  B2_REQUIRE(ws_bytes >= w.bytes, "[moe_block] workspace too small (%zu < %zu bytes)", ws_bytes, w.bytes);
  B2_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "[moe_block] workspace must be 256-byte aligned");
  B2_REQUIRE(T * k <= (int64_t)INT32_MAX && T * k * (int64_t)std::max(H, F) <= ((int64_t)1 << 40),
             "[moe_block] too many rows");
  uint32_t* ri = inds ? inds : w.inds;
  float* rw = weights ? weights : w.weights;
  int rc;
  if (!logits) {
    rc = launch_router_logits(x, blk->router_w, blk->router_w_dtype, T, E, H, w.logits, st);
    if (rc) return rc;
  }
  rc = launch_router_topk(logits ? logits : w.logits, blk->router_bias, blk->router_mode, T, E, (int)k, blk->renorm,
                          ri, rw, st);
  if (rc) return rc;
  rc = experts_sorted(blk, x, T, ri, w, w.y, st);
  if (rc) return rc;
  const uint16_t* shared = nullptr;
  rc = shared_forward(blk, x, T, w.shared_scratch, &shared, st);
  if (rc) return rc;
  // y is in (token, slot) order: each token's k rows are contiguous
  return launch_combine(w.y, nullptr, rw, T, (int)k, H, blk->routed_scale, shared, residual, out, st);
}

// Expert SwiGLU MLPs of every (token, slot) row in expert-sorted order: sort
// -> token tiles -> gather rows -> gate/up GEMM + SwiGLU -> down GEMM, which
// writes y [T*k][H] in (token, slot) order (row t*k+s).
int experts_sorted(const b2_moe_block* blk, const uint16_t* x, int64_t T, const uint32_t* inds, PrefillWs& w,
                   uint16_t* y, cudaStream_t st) {
  const int64_t H = blk->hidden, E = blk->n_experts, k = blk->top_k, F = blk->ffn;
  int rc = launch_gather_sort_ws(inds, T * k, E, w.order, w.sorted, w.inverse, w.offsets, w.sort_scratch, st);
  if (rc) return rc;
  rc = pf::make_tiles(w.offsets, (int)E, w.tiles, w.ntiles, pf::pair_mode(blk), st);
  if (rc) return rc;
  rc = pf::gather_rows_f16(x, w.order, (int)k, T * k, (int)H, w.xs, w.xexp, st);
  if (rc) return rc;
  rc = pf::expert_gemm(0, blk, w.xs, T * k, w.tiles, w.ntiles, w.act, nullptr, st, nullptr, 0, w.xexp);
  if (rc) return rc;
  return pf::expert_gemm(1, blk, w.act, T * k, w.tiles, w.ntiles, y, w.order, st);
}

}  // namespace b2

extern "C" size_t b2_moe_prefill_bank_size(const b2_moe_block* blk) {
  if (!blk || blk->n_experts <= 0 || blk->hidden <= 0 || blk->ffn <= 0) return 0;
  return b2::pf::prefill_bank_bytes(blk);
}

extern "C" int b2_moe_prepare_prefill_bank(const b2_moe_block* blk, void* bank, size_t bank_bytes,
                                           b2_stream_t stream) {
  int rc = b2::validate_block(blk, "prepare_prefill_bank");
  if (rc) return rc;
  B2_REQUIRE(bank != nullptr, "[prepare_prefill_bank] destination is NULL");
  B2_REQUIRE(b2::pf::prefill_gemm_supported(blk),
             "[prepare_prefill_bank] needs hidden %% 128 == 0 and ffn %% 64 == 0 (got %lld, %lld)",
             (long long)blk->hidden, (long long)blk->ffn);
  B2_REQUIRE(bank_bytes >= b2::pf::prefill_bank_bytes(blk), "[prepare_prefill_bank] destination too small (%zu < %zu)",
             bank_bytes, b2::pf::prefill_bank_bytes(blk));
  B2_REQUIRE(reinterpret_cast<uintptr_t>(bank) % 16 == 0, "[prepare_prefill_bank] destination must be 16-byte aligned");
  return b2::pf::prepare_prefill(blk, bank, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t b2_moe_switch_glu_workspace_size(const b2_moe_block* blk, int64_t tokens, int k) {
  if (!blk || tokens < 0 || k <= 0) return 0;
  b2_moe_block b = *blk;
  b.top_k = k;
  b.shared_gate_codes = nullptr;  // SwitchGLU is the routed experts only
  return b2::carve(&b, tokens, nullptr).bytes;
}

extern "C" int b2_moe_switch_glu(const b2_moe_block* blk, const uint16_t* x, int64_t tokens, const uint32_t* inds,
                                 int k, uint16_t* y, void* workspace, size_t workspace_bytes, b2_stream_t stream) {
  int rc = b2::validate_block(blk, "switch_glu");
  if (rc) return rc;
  B2_REQUIRE(k > 0 && k <= 8, "[switch_glu] indices per token must be in [1, 8] (got %d)", k);
  B2_REQUIRE(tokens >= 0 && tokens * k <= (int64_t)INT32_MAX, "[switch_glu] invalid token count");
  if (tokens == 0) return B2_OK;
  B2_REQUIRE(x && inds && y && workspace, "[switch_glu] null pointer argument");
  B2_REQUIRE(blk->prefill_bank != nullptr && b2::pf::prefill_gemm_supported(blk),
             "[switch_glu] needs a prepared prefill bank (b2_moe_prepare_prefill_bank)");
  B2_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "[switch_glu] workspace must be 256-byte aligned");
  b2_moe_block b = *blk;
  b.top_k = k;
  b.shared_gate_codes = nullptr;  // SwitchGLU is the routed experts only
  b2::PrefillWs w = b2::carve(&b, tokens, static_cast<uint8_t*>(workspace));
  B2_REQUIRE(workspace_bytes >= w.bytes, "[switch_glu] workspace too small (%zu < %zu bytes)", workspace_bytes,
             w.bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the down GEMM writes each row straight to its (token, slot) position in y
  return b2::experts_sorted(&b, x, tokens, inds, w, y, st);
}

extern "C" int b2_gather_rows16(const void* src, const uint32_t* idx, int64_t n, int64_t K, void* dst,
                                b2_stream_t stream) {
  B2_REQUIRE(src && idx && dst, "[gather_rows] null pointer argument");
  B2_REQUIRE(n >= 0 && K > 0 && K % 8 == 0, "[gather_rows] row length must be a positive multiple of 8");
  B2_REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0 && reinterpret_cast<uintptr_t>(dst) % 16 == 0,
             "[gather_rows] rows must be 16-byte aligned");
  return b2::pf::gather_rows(static_cast<const uint16_t*>(src), idx, 1, n, (int)K, static_cast<uint16_t*>(dst),
                             reinterpret_cast<cudaStream_t>(stream));
}
