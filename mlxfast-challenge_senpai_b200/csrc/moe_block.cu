// MoE expert block: decode path (fused gathered GEMVs) and the block entry
// point.  Decode-shaped calls run four kernels:
//   router logits -> top-k -> gate/up GEMV + SwiGLU -> down GEMV + combine.
#include <mutex>

#include "moe.cuh"
#include "moe_prefill.cuh"
#include "qmv.cuh"

namespace b2 {
namespace {

using namespace qmv;

// Gate/up projection of one (token, slot) pair for 8 features, fused with
// SwiGLU.  CTA tiles: rows [8f, 8f+8) of the gate bank and of the up bank of
// expert inds[pair]; x row = token pair/k.  Output a[pair, 8f .. 8f+8).
__global__ void __launch_bounds__(kThreads)
decode_gateup_kernel(const uint16_t* __restrict__ x, const uint32_t* __restrict__ inds, int k, int E, int H, int F,
                     const uint8_t* __restrict__ gcodes, const uint8_t* __restrict__ gscales,
                     const uint8_t* __restrict__ ucodes, const uint8_t* __restrict__ uscales,
                     uint16_t* __restrict__ a, unsigned* status) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const TileGeom g = make_geom(H);
  const Smem s = carve(smem_raw, g, 16, 1);
  const int pair = blockIdx.y, f0 = blockIdx.x * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t e = inds[pair];
  if (e >= (uint32_t)E) {
    if (threadIdx.x == 0) report_status(status, B2_STATUS_BAD_INDEX);
    if (threadIdx.x < 8 && f0 + threadIdx.x < F) a[(int64_t)pair * F + f0 + threadIdx.x] = 0;
    return;
  }
  const int nvalid = min(8, F - f0);
  if (threadIdx.x == 0) {
    mbar_init(s.bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) mbar_expect_tx(s.bar, 2u * nvalid * (uint32_t)(H / 2 + H / 16));
    __syncwarp();
    const int64_t rowbase = (int64_t)e * F + f0;
    issue_rows(s, g, 16, [&](int r, const uint8_t*& c, const uint8_t*& sc) {
      const int rr = r & 7;
      if (rr >= nvalid) return false;
      const bool up = r >= 8;
      c = (up ? ucodes : gcodes) + (rowbase + rr) * (H / 2);
      sc = (up ? uscales : gscales) + (rowbase + rr) * (H / 16);
      return true;
    });
  }
  const uint16_t* xr = x + (int64_t)(pair / k) * H;
  stage_x(s, g, 1, [&](int) { return xr; });
  if (!mbar_wait_bounded(s.bar, 0, status)) return;

  float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  const int groups = H / 16, c = lane & 3, gi = lane >> 2;
  for (int grp = warp; grp < groups; grp += kWarps) {
    uint32_t af[4];
    load_a_frag(s, g, grp, lane, 0, 1, af);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      uint32_t b[2];
      load_b_frag(s, g, rt * 8 + gi, grp, c, b);
      mma_16816_f16(acc[rt], af, b);
    }
  }
  // only fragment row 0 (token) is meaningful: lanes 0..3 hold c0,c1
  float* red = s.red;  // [warps][2 tiles][8 rows]
  if (lane < 4) {
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      red[(warp * 2 + rt) * 8 + 2 * lane] = acc[rt][0];
      red[(warp * 2 + rt) * 8 + 2 * lane + 1] = acc[rt][1];
    }
  }
  __syncthreads();
  if (threadIdx.x < nvalid) {
    const int r = threadIdx.x;
    float gv = 0.0f, uv = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      gv += red[(w * 2 + 0) * 8 + r];
      uv += red[(w * 2 + 1) * 8 + r];
    }
    const int p = s.xexp[0];
    gv = round_bf16(ldexpf(gv, p));
    uv = round_bf16(ldexpf(uv, p));
    a[(int64_t)pair * F + f0 + r] = f32_to_bf16_bits(swiglu_bf16(gv, uv));
  }
}

constexpr int kMaxSlots = 8;

// Down projection of all k slots of one token for 8 hidden features, fused
// with the weighted combine (+ optional scale / residual).  Tile s holds rows
// [8h, 8h+8) of the down bank of expert inds[t*k+s] and reads staged
// activation row s (= a[t*k+s]).
__global__ void __launch_bounds__(kThreads)
decode_down_kernel(const uint16_t* __restrict__ a, const uint32_t* __restrict__ inds, const float* __restrict__ wts,
                   int k, int E, int H, int F, const uint8_t* __restrict__ dcodes, const uint8_t* __restrict__ dscales,
                   float routed_scale, const uint16_t* __restrict__ residual, uint16_t* __restrict__ out,
                   unsigned* status) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const TileGeom g = make_geom(F);
  const Smem s = carve(smem_raw, g, kMaxSlots * 8, kMaxSlots);
  const int t = blockIdx.y, h0 = blockIdx.x * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ uint32_t ex[kMaxSlots];
  if (threadIdx.x < kMaxSlots) {
    uint32_t e = threadIdx.x < k ? inds[(int64_t)t * k + threadIdx.x] : 0u;
    if (e >= (uint32_t)E) {
      report_status(status, B2_STATUS_BAD_INDEX);
      e = 0xffffffffu;
    }
    ex[threadIdx.x] = e;
  }
  if (threadIdx.x == 0) {
    mbar_init(s.bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  int nslots = 0;
  for (int q = 0; q < k; ++q) nslots += (ex[q] != 0xffffffffu);
  if (warp == 0) {
    if (lane == 0) mbar_expect_tx(s.bar, (uint32_t)nslots * 8u * (uint32_t)(F / 2 + F / 16));
    __syncwarp();
    issue_rows(s, g, kMaxSlots * 8, [&](int r, const uint8_t*& c, const uint8_t*& sc) {
      const int q = r >> 3;
      if (q >= k || ex[q] == 0xffffffffu) return false;
      const int64_t row = (int64_t)ex[q] * H + h0 + (r & 7);
      c = dcodes + row * (F / 2);
      sc = dscales + row * (F / 16);
      return true;
    });
  }
  stage_x(s, g, k, [&](int q) -> const uint16_t* {
    return ex[q] == 0xffffffffu ? nullptr : a + ((int64_t)t * k + q) * F;
  });
  if (!mbar_wait_bounded(s.bar, 0, status)) return;

  float acc[kMaxSlots][4];
#pragma unroll
  for (int q = 0; q < kMaxSlots; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.0f;
  const int groups = F / 16, c = lane & 3, gi = lane >> 2;
  for (int grp = warp; grp < groups; grp += kWarps) {
#pragma unroll
    for (int q = 0; q < kMaxSlots; ++q) {
      if (q < k) {
        uint32_t af[4];
        load_a_frag(s, g, grp, lane, q, 1, af);
        uint32_t b[2];
        load_b_frag(s, g, q * 8 + gi, grp, c, b);
        mma_16816_f16(acc[q], af, b);
      }
    }
  }
  float* red = s.red;  // [warps][slots][8 rows]
  if (lane < 4) {
#pragma unroll
    for (int q = 0; q < kMaxSlots; ++q) {
      red[(warp * kMaxSlots + q) * 8 + 2 * lane] = acc[q][0];
      red[(warp * kMaxSlots + q) * 8 + 2 * lane + 1] = acc[q][1];
    }
  }
  __syncthreads();
  // d[q][r] for the 8 rows, then the combine by one thread per row
  if (threadIdx.x < 8) {
    const int r = threadIdx.x;
    float tot = 0.0f;
    for (int q = 0; q < k; ++q) {
      float d = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) d += red[(w * kMaxSlots + q) * 8 + r];
      d = (ex[q] == 0xffffffffu) ? 0.0f : round_bf16(ldexpf(d, s.xexp[q]));
      const float rw = round_bf16(wts[(int64_t)t * k + q]);
      tot = round_bf16(__fadd_rn(round_bf16(__fmul_rn(d, rw)), tot));
    }
    s.red[kWarps * kMaxSlots * 8 + r] = tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) tot[r] = s.red[kWarps * kMaxSlots * 8 + r];
    finish_combine(tot, t, h0, H, routed_scale, nullptr, residual, out);
  }
}

struct Workspace {
  float* logits;
  uint32_t* inds;
  float* weights;
  uint16_t* a;
  size_t bytes;
};

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

Workspace decode_workspace(const b2_moe_block* blk, int64_t T, uint8_t* base) {
  Workspace w{};
  size_t off = 0;
  w.logits = reinterpret_cast<float*>(base + off);
  off += align256((size_t)T * blk->n_experts * 4);
  w.inds = reinterpret_cast<uint32_t*>(base + off);
  off += align256((size_t)T * blk->top_k * 4);
  w.weights = reinterpret_cast<float*>(base + off);
  off += align256((size_t)T * blk->top_k * 4);
  w.a = reinterpret_cast<uint16_t*>(base + off);
  off += align256((size_t)T * blk->top_k * blk->ffn * 2);
  w.bytes = off;
  return w;
}

}  // namespace

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
  return B2_OK;
}

int decode_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits,
                   const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, void* workspace,
                   size_t ws_bytes, cudaStream_t st) {
  Workspace w = decode_workspace(blk, T, static_cast<uint8_t*>(workspace));
  B2_REQUIRE(ws_bytes >= w.bytes, "[moe_block] workspace too small (%zu < %zu)", ws_bytes, w.bytes);
  const int E = (int)blk->n_experts, k = blk->top_k, H = (int)blk->hidden, F = (int)blk->ffn;
  uint32_t* ind = inds ? inds : w.inds;
  float* wt = weights ? weights : w.weights;
  if (!logits) {
    B2_REQUIRE(blk->router_w != nullptr, "[moe_block] router weight is NULL and no logits were given");
    int rc = launch_router_logits(x, blk->router_w, blk->router_w_dtype, T, E, H, w.logits, st);
    if (rc) return rc;
    logits = w.logits;
  }
  int rc = launch_router_topk(logits, blk->router_bias, blk->router_mode, T, E, k, blk->renorm, ind, wt, st);
  if (rc) return rc;
  unsigned* status = device_status_ptr();
  {
    const TileGeom g = make_geom(H);
    const size_t smem = smem_bytes(g, 16, 1, kWarps * 16);
    int rc2 = ensure_dynamic_smem((const void*)decode_gateup_kernel, smem, "moe_block.gateup");
    if (rc2) return rc2;
    dim3 grid((unsigned)((F + 7) / 8), (unsigned)(T * k));
    decode_gateup_kernel<<<grid, kThreads, smem, st>>>(
        x, ind, k, E, H, F, reinterpret_cast<const uint8_t*>(blk->gate_codes), blk->gate_scales,
        reinterpret_cast<const uint8_t*>(blk->up_codes), blk->up_scales, w.a, status);
    B2_CHECK_LAUNCH("moe_block.gateup");
  }
  {
    const TileGeom g = make_geom(F);
    const size_t smem = smem_bytes(g, kMaxSlots * 8, kMaxSlots, kWarps * kMaxSlots * 8 + 8);
    int rc2 = ensure_dynamic_smem((const void*)decode_down_kernel, smem, "moe_block.down");
    if (rc2) return rc2;
    dim3 grid((unsigned)(H / 8), (unsigned)T);
    decode_down_kernel<<<grid, kThreads, smem, st>>>(w.a, ind, wt, k, E, H, F,
                                                     reinterpret_cast<const uint8_t*>(blk->down_codes),
                                                     blk->down_scales, blk->routed_scale, residual, out, status);
    B2_CHECK_LAUNCH("moe_block.down");
  }
  return B2_OK;
}

size_t decode_workspace_bytes(const b2_moe_block* blk, int64_t T) { return decode_workspace(blk, T, nullptr).bytes; }

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
  // Every scratch byte this path reads is written earlier in the same call
  // (logits, routing, SwiGLU activations), so nothing needs clearing.
  return b2::decode_forward(blk, x, tokens, logits, residual, out, inds, weights, scratch, b2::kStaticScratchBytes,
                            reinterpret_cast<cudaStream_t>(stream));
}
