// MoE expert block entry points.  Decode-shaped calls (<= 8 tokens) run the
// fused cooperative kernel of moe_decode.cu; larger calls the prefill path.
#include <mutex>

#include "moe.cuh"
#include "moe_decode.cuh"
#include "moe_prefill.cuh"

namespace b2 {

int validate_block(const b2_moe_block* b, const char* op) {
  B2_REQUIRE(b != nullptr, "[%s] block descriptor is NULL", op);
  B2_REQUIRE(b->hidden > 0 && b->ffn > 0 && b->n_experts > 0 && b->top_k > 0, "[%s] invalid block sizes", op);
  B2_REQUIRE(b->hidden % 256 == 0 && b->ffn % 256 == 0,
             "[%s] hidden (%lld) and ffn (%lld) must be multiples of 256", op, (long long)b->hidden,
             (long long)b->ffn);
  B2_REQUIRE(b->top_k <= 8, "[%s] top_k must be <= 8 (got %d)", op, b->top_k);
  B2_REQUIRE(b->n_experts <= 1024, "[%s] at most 1024 experts", op);
  B2_REQUIRE(b->router_mode == B2_ROUTER_SOFTMAX || b->router_mode == B2_ROUTER_SIGMOID_BIAS,
             "[%s] unknown router mode", op);
  B2_REQUIRE(b->gate_codes && b->gate_scales && b->up_codes && b->up_scales && b->down_codes && b->down_scales,
             "[%s] expert bank pointer is NULL", op);
  if (b->shared_gate_codes) {
    B2_REQUIRE(b->shared_gate_scales && b->shared_up_codes && b->shared_up_scales && b->shared_down_codes &&
                   b->shared_down_scales,
               "[%s] shared expert pointer is NULL", op);
    B2_REQUIRE(b->shared_ffn > 0 && b->shared_ffn % 16 == 0 && b->shared_ffn <= (int64_t)INT32_MAX,
               "[%s] shared_ffn must be a positive multiple of 16 (got %lld)", op, (long long)b->shared_ffn);
  }
  return B2_OK;
}

int decode_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits,
                   const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, void* workspace,
                   size_t ws_bytes, cudaStream_t st) {
  return dec::forward(blk, x, T, logits, residual, out, inds, weights, workspace, ws_bytes, st);
}

size_t decode_workspace_bytes(const b2_moe_block* blk, int64_t T) { return dec::scratch_bytes(blk, T); }

}  // namespace b2

extern "C" size_t b2_moe_block_workspace_size(const b2_moe_block* blk, int64_t tokens) {
  if (!blk || tokens <= 0) return 0;
  if (tokens <= b2::kDecodeMaxTokens) return b2::decode_workspace_bytes(blk, tokens);
  return b2::prefill_workspace_bytes(blk, tokens);
}

extern "C" int b2_moe_block_forward(const b2_moe_block* blk, const uint16_t* x, int64_t tokens, const float* logits,
                                    const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights,
                                    void* workspace, size_t workspace_bytes, b2_stream_t stream) {
  int rc = b2::validate_block(blk, "moe_block");
  if (rc) return rc;
  B2_REQUIRE(x && out, "[moe_block] null x/out");
  B2_REQUIRE(tokens >= 0 && tokens <= 65535, "[moe_block] token count must be in [0, 65535]");
  if (tokens == 0) return B2_OK;
  B2_REQUIRE(workspace != nullptr, "[moe_block] workspace is NULL");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (tokens <= b2::kDecodeMaxTokens)
    return b2::decode_forward(blk, x, tokens, logits, residual, out, inds, weights, workspace, workspace_bytes, st);
  return b2::prefill_forward(blk, x, tokens, logits, residual, out, inds, weights, workspace, workspace_bytes, st);
}

// ---------------------------------------------------------------------------
// Decode-shaped block forward with library-owned scratch.
//
// For callers that cannot allocate device memory: a custom-op callback running
// inside another framework's runtime (that framework's allocator owns every
// device buffer and the callback only receives the op's inputs and outputs),
// or a process held to a fixed device-memory budget that forbids allocations
// after start-up.  Such callers cannot provide the workspace
// b2_moe_block_forward needs, so this entry point takes its scratch from the
// file-scope array below instead.
namespace b2 {
namespace {

constexpr size_t kStaticScratchBytes = 512 * 1024;
static __device__ __align__(256) uint8_t g_block_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of g_block_scratch on the current device, looked up once per
// device (with that device current).  In host code the symbol is only a host
// stand-in; the kernels must be given this address.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "moe_block_decode_static");
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_UNSUPPORTED, "[moe_block_decode_static] device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_block_scratch);
    if (e != cudaSuccess) return check_cuda(e, "moe_block_decode_static: cudaGetSymbolAddress");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return B2_OK;
}

}  // namespace
}  // namespace b2

extern "C" int b2_moe_block_decode_static(const b2_moe_block* blk, const uint16_t* x, int64_t tokens,
                                          const float* logits, const uint16_t* residual, uint16_t* out,
                                          uint32_t* inds, float* weights, b2_stream_t stream) {
  int rc = b2::validate_block(blk, "moe_block_decode_static");
  if (rc) return rc;
  B2_REQUIRE(x && out, "[moe_block_decode_static] null x/out");
  B2_REQUIRE(tokens >= 0 && tokens <= b2::kDecodeMaxTokens,
             "[moe_block_decode_static] token count %lld is outside [0, %lld]; larger calls need "
             "b2_moe_block_forward with a caller workspace",
             (long long)tokens, (long long)b2::kDecodeMaxTokens);
  if (tokens == 0) return B2_OK;
  const size_t need = b2::decode_workspace_bytes(blk, tokens);
  B2_REQUIRE(need <= b2::kStaticScratchBytes,
             "[moe_block_decode_static] this block needs %zu bytes of scratch but the static scratch holds %zu; "
             "use b2_moe_block_forward with a caller workspace",
             need, b2::kStaticScratchBytes);
  void* scratch = nullptr;
  rc = b2::static_scratch(&scratch);
  if (rc) return rc;
  // The head of the scratch is the kernels' cross-launch state: zero with the
  // module, and every launch (one that gave up on a wait included) leaves it
  // valid for the next one, whatever block that is.  Every other scratch byte
  // is written before it is read within the call, so the call is one launch.
  return b2::decode_forward(blk, x, tokens, logits, residual, out, inds, weights, scratch, b2::kStaticScratchBytes,
                            reinterpret_cast<cudaStream_t>(stream));
}
