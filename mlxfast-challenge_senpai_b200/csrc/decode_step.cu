// One-token decode step of a Laguna-shaped decoder stack:
// per layer
//   n  = rms_norm(x, attn_norm)                        (MLXFast.rmsNorm)
//   q, k, v = n . Wqkv^T                               (NVFP4 quantized_matmul)
//   q, k = rope(q, k, pos), theta, half-split pairs    (MLXFast.RoPE, traditional false)
//   k_cache[:, pos] = k, v_cache[:, pos] = v           (KVCache update)
//   a  = softmax(q k^T * hd^-0.5) v over positions 0..pos, kv head = q head / (nq / nkv)
//   h  = x + a . Wo^T                                  (NVFP4 quantized_matmul, residual)
//   x' = h + moe(rms_norm(h, mlp_norm))                (the fused decode MoE block)
// then a final rms_norm.  Reference shapes and semantics: the decoder layer
// and attention of Laguna.swift:22-128 without the checkpoint-specific
// extras BASELINE's config 4 leaves out (per-head q/k norm, the softplus
// output gate, sliding windows, YaRN): full-head RoPE with theta, full
// attention, bf16 KV cache.
//
// Kernels: rms_norm (one CTA, optional residual add fused), rope + cache
// append (one CTA per head), split-K attention over the cache (grid = kv
// heads x splits, flash-decoding partials in f32) and its merge; the
// projections are the quantized_matmul GEMV, the MoE block the fused decode
// kernel with the residual fused in its epilogue.
#include <algorithm>
#include <cmath>

#include "moe.cuh"
#include "moe_prefill.cuh"

namespace b2 {
namespace {

constexpr int kNormThreads = 256;
constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxGroup = 8;  // q heads per kv head handled by one attention CTA
constexpr int kHd = 128;      // head_dim (4 values per lane)

size_t a256(size_t v) { return (v + 255) & ~size_t(255); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// n = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))) with h = x (or bf16(x + add),
// written to h_out): MLX's rms_norm in f32, rounded to bf16 before the
// weight, as its kernels do.  One CTA per row.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const uint16_t* __restrict__ x,
                                                                const uint16_t* __restrict__ add,
                                                                const uint16_t* __restrict__ w, int H, float eps,
                                                                uint16_t* __restrict__ h_out,
                                                                uint16_t* __restrict__ n_out) {
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  x += (int64_t)row * H;
  if (add) add += (int64_t)row * H;
  if (h_out) h_out += (int64_t)row * H;
  n_out += (int64_t)row * H;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < H; i += kNormThreads) {
    float v = bf16_bits_to_f32(x[i]);
    if (add) {
      v = round_bf16(v + bf16_bits_to_f32(add[i]));
      h_out[i] = f32_to_bf16_bits(v);
    }
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += kNormThreads) {
    const float v = add ? bf16_bits_to_f32(h_out[i]) : bf16_bits_to_f32(x[i]);
    n_out[i] = f32_to_bf16_bits(bf16_bits_to_f32(w[i]) * round_bf16(v * inv));
  }
}

// RoPE (half-split pairs i, i + hd/2; angle = pos * theta^(-2i/hd), f32) on
// the q and k heads of the fused projection output, k and v appended to the
// caches at `pos`.  One CTA per head (nq + nkv + nkv), hd/2 threads.
__global__ void rope_cache_kernel(const uint16_t* __restrict__ qkv, int nq, int nkv, int64_t pos,
                                  float log2_theta, int64_t max_seq, uint16_t* __restrict__ q_out,
                                  uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache) {
  const int head = blockIdx.x, i = threadIdx.x;  // i < kHd / 2
  const uint16_t* src = qkv + (int64_t)head * kHd;
  if (head >= nq + nkv) {
    // v head: copy to the cache
    const int hv = head - nq - nkv;
    uint16_t* dst = v_cache + ((int64_t)hv * max_seq + pos) * kHd;
    dst[i] = src[i];
    dst[i + kHd / 2] = src[i + kHd / 2];
    return;
  }
  const float inv_freq = exp2f(-(float)(2 * i) / (float)kHd * log2_theta);
  float s, c;
  sincosf((float)pos * inv_freq, &s, &c);
  const float x1 = bf16_bits_to_f32(src[i]), x2 = bf16_bits_to_f32(src[i + kHd / 2]);
  const uint16_t o1 = f32_to_bf16_bits(x1 * c - x2 * s), o2 = f32_to_bf16_bits(x1 * s + x2 * c);
  if (head < nq) {
    q_out[(int64_t)head * kHd + i] = o1;
    q_out[(int64_t)head * kHd + i + kHd / 2] = o2;
  } else {
    uint16_t* dst = k_cache + ((int64_t)(head - nq) * max_seq + pos) * kHd;
    dst[i] = o1;
    dst[i + kHd / 2] = o2;
  }
}

// Split-K attention partials: CTA (kv head h, split s) runs the online
// softmax of its group's q heads over positions [s*chunk, min(L, (s+1)*chunk)),
// each warp a strided subset, lanes holding 4 of the 128 dims; then the CTA
// merges its warps and writes (max, sum, acc[hd]) per q head in f32.
// Scores are in base 2 (q pre-scaled by hd^-0.5 * log2 e).
__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(const uint16_t* __restrict__ q, int group,
                                                                    const uint16_t* __restrict__ k_cache,
                                                                    const uint16_t* __restrict__ v_cache,
                                                                    int64_t max_seq, int L, int chunk, float qscale,
                                                                    float* __restrict__ part) {
  __shared__ float s_m[kAttnWarps][kMaxGroup], s_l[kAttnWarps][kMaxGroup];
  __shared__ float s_acc[kAttnWarps][kMaxGroup][kHd];
  const int h = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float qv[kMaxGroup][4];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g < group) {
      const uint2 r = *reinterpret_cast<const uint2*>(q + ((int64_t)(h * group + g) * kHd) + 4 * lane);
      qv[g][0] = __uint_as_float(r.x << 16) * qscale;
      qv[g][1] = __uint_as_float(r.x & 0xffff0000u) * qscale;
      qv[g][2] = __uint_as_float(r.y << 16) * qscale;
      qv[g][3] = __uint_as_float(r.y & 0xffff0000u) * qscale;
    }
  }
  float m[kMaxGroup], l[kMaxGroup], acc[kMaxGroup][4];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
    acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0f;
  }
  const int j0 = split * chunk, j1 = min(L, j0 + chunk);
  const uint16_t* kb = k_cache + (int64_t)h * max_seq * kHd + 4 * lane;
  const uint16_t* vb = v_cache + (int64_t)h * max_seq * kHd + 4 * lane;
  for (int j = j0 + warp; j < j1; j += kAttnWarps) {
    const uint2 kr = __ldg(reinterpret_cast<const uint2*>(kb + (int64_t)j * kHd));
    const uint2 vr = __ldg(reinterpret_cast<const uint2*>(vb + (int64_t)j * kHd));
    const float kx[4] = {__uint_as_float(kr.x << 16), __uint_as_float(kr.x & 0xffff0000u),
                         __uint_as_float(kr.y << 16), __uint_as_float(kr.y & 0xffff0000u)};
    const float vx[4] = {__uint_as_float(vr.x << 16), __uint_as_float(vr.x & 0xffff0000u),
                         __uint_as_float(vr.y << 16), __uint_as_float(vr.y & 0xffff0000u)};
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g >= group) break;
      float sc = qv[g][0] * kx[0];
      sc = fmaf(qv[g][1], kx[1], sc);
      sc = fmaf(qv[g][2], kx[2], sc);
      sc = fmaf(qv[g][3], kx[3], sc);
      sc = warp_sum(sc);
      const float mn = fmaxf(m[g], sc);
      const float corr = exp2f(m[g] - mn), p = exp2f(sc - mn);
      l[g] = fmaf(l[g], corr, p);
#pragma unroll
      for (int d = 0; d < 4; ++d) acc[g][d] = fmaf(acc[g][d], corr, p * vx[d]);
      m[g] = mn;
    }
  }
  // merge the warps
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g >= group) break;
    if (lane == 0) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
#pragma unroll
    for (int d = 0; d < 4; ++d) s_acc[warp][g][4 * lane + d] = acc[g][d];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < group * kHd; idx += kAttnThreads) {
    const int g = idx / kHd, d = idx % kHd;
    float mx = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, s_m[w][g]);
    float ls = 0.0f, as = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = s_m[w][g] == -INFINITY ? 0.0f : exp2f(s_m[w][g] - mx);
      ls = fmaf(s_l[w][g], f, ls);
      as = fmaf(s_acc[w][g][d], f, as);
    }
    float* dst = part + ((int64_t)(h * group + g) * S + split) * (kHd + 2);
    dst[2 + d] = as;
    if (d == 0) {
      dst[0] = mx;
      dst[1] = ls;
    }
  }
}

// out[head] = merge of the S split partials, bf16.  One CTA per q head.
__global__ void attn_merge_kernel(const float* __restrict__ part, int S, uint16_t* __restrict__ out) {
  const int head = blockIdx.x, d = threadIdx.x;  // kHd threads
  const float* p = part + (int64_t)head * S * (kHd + 2);
  float mx = -INFINITY;
  for (int s = 0; s < S; ++s) mx = fmaxf(mx, p[s * (kHd + 2)]);
  float ls = 0.0f, as = 0.0f;
  for (int s = 0; s < S; ++s) {
    const float m = p[s * (kHd + 2)];
    const float f = m == -INFINITY ? 0.0f : exp2f(m - mx);
    ls = fmaf(p[s * (kHd + 2) + 1], f, ls);
    as = fmaf(p[s * (kHd + 2) + 2 + d], f, as);
  }
  out[(int64_t)head * kHd + d] = f32_to_bf16_bits(as / ls);
}

int attn_splits(int64_t L, int nkv, int sms) {
  const int want = std::max(1, sms / std::max(1, nkv));
  return (int)std::min<int64_t>(want, std::max<int64_t>(1, (L + 31) / 32));
}

struct StepWs {
  uint16_t *qkv, *q, *attn, *o, *h, *n, *xa, *xb;
  float* part;
  void* moe_ws;
  size_t moe_bytes, bytes;
};

StepWs carve_step(const b2_decoder_layer* layers, int n_layers, uint8_t* base, int sms) {
  const b2_attn_layer& a = layers[0].attn;
  const int64_t H = a.hidden, nq = a.n_heads, nkv = a.n_kv_heads;
  StepWs w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += a256(bytes);
    return p;
  };
  w.qkv = reinterpret_cast<uint16_t*>(take((size_t)(nq + 2 * nkv) * kHd * 2));
  w.q = reinterpret_cast<uint16_t*>(take((size_t)nq * kHd * 2));
  w.attn = reinterpret_cast<uint16_t*>(take((size_t)nq * kHd * 2));
  w.o = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.h = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.n = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.xa = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.xb = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  const int S = attn_splits(a.max_seq, (int)nkv, sms);
  w.part = reinterpret_cast<float*>(take((size_t)nq * S * (kHd + 2) * 4));
  size_t moe = 0;
  for (int i = 0; i < n_layers; ++i) moe = std::max(moe, decode_workspace_bytes(&layers[i].moe, 1));
  w.moe_bytes = moe;
  w.moe_ws = take(moe);
  w.bytes = off;
  return w;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

int validate_layers(const b2_decoder_layer* layers, int n_layers) {
  B2_REQUIRE(layers != nullptr && n_layers > 0, "[decode_step] no layers");
  const b2_attn_layer& a0 = layers[0].attn;
  for (int i = 0; i < n_layers; ++i) {
    const b2_attn_layer& a = layers[i].attn;
    B2_REQUIRE(a.head_dim == kHd, "[decode_step] head_dim must be %d (got %lld)", kHd, (long long)a.head_dim);
    B2_REQUIRE(a.n_heads > 0 && a.n_kv_heads > 0 && a.n_heads % a.n_kv_heads == 0 &&
                   a.n_heads / a.n_kv_heads <= kMaxGroup,
               "[decode_step] n_heads must be a multiple of n_kv_heads with at most %d q heads per kv head",
               kMaxGroup);
    B2_REQUIRE(a.hidden == a0.hidden && a.n_heads == a0.n_heads && a.n_kv_heads == a0.n_kv_heads &&
                   a.max_seq == a0.max_seq,
               "[decode_step] every layer must have the same attention shape");
    B2_REQUIRE(a.hidden % 16 == 0 && a.max_seq > 0, "[decode_step] invalid hidden / max_seq");
    B2_REQUIRE(a.attn_norm_w && a.mlp_norm_w && a.qkv_codes && a.qkv_scales && a.o_codes && a.o_scales &&
                   a.k_cache && a.v_cache,
               "[decode_step] layer %d: null attention pointer", i);
    B2_REQUIRE(reinterpret_cast<uintptr_t>(a.k_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(a.v_cache) % 16 == 0,
               "[decode_step] layer %d: KV caches must be 16-byte aligned", i);
    B2_REQUIRE(a.rope_theta > 0.0f && a.rms_eps >= 0.0f, "[decode_step] layer %d: invalid rope_theta / rms_eps", i);
    B2_REQUIRE(layers[i].moe.hidden == a.hidden, "[decode_step] layer %d: MoE hidden differs from attention", i);
    const int rc = validate_block(&layers[i].moe, "decode_step");
    if (rc) return rc;
  }
  return B2_OK;
}

}  // namespace
}  // namespace b2

extern "C" size_t b2_decode_step_workspace_size(const b2_decoder_layer* layers, int n_layers) {
  if (!layers || n_layers <= 0) return 0;
  return b2::carve_step(layers, n_layers, nullptr, b2::sm_count()).bytes;
}

extern "C" int b2_decode_step(const b2_decoder_layer* layers, int n_layers, const uint16_t* final_norm_w,
                              const uint16_t* x, int64_t pos, uint16_t* out, void* workspace, size_t workspace_bytes,
                              b2_stream_t stream) {
  using namespace b2;
  int rc = validate_layers(layers, n_layers);
  if (rc) return rc;
  const b2_attn_layer& a0 = layers[0].attn;
  B2_REQUIRE(x && out && final_norm_w && workspace, "[decode_step] null argument");
  B2_REQUIRE(pos >= 0 && pos < a0.max_seq, "[decode_step] position %lld outside the cache [0, %lld)", (long long)pos,
             (long long)a0.max_seq);
  B2_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "[decode_step] workspace must be 256-byte aligned");
  const int sms = sm_count();
  StepWs w = carve_step(layers, n_layers, static_cast<uint8_t*>(workspace), sms);
  B2_REQUIRE(workspace_bytes >= w.bytes, "[decode_step] workspace too small (%zu < %zu)", workspace_bytes, w.bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t H = a0.hidden, nq = a0.n_heads, nkv = a0.n_kv_heads, L = pos + 1;
  const int group = (int)(nq / nkv);
  const int S = attn_splits(a0.max_seq, (int)nkv, sms);
  const int chunk = (int)((L + S - 1) / S);
  const uint16_t* cur = x;
  for (int i = 0; i < n_layers; ++i) {
    const b2_attn_layer& a = layers[i].attn;
    uint16_t* nxt = (cur == w.xa) ? w.xb : w.xa;  // layer outputs alternate between two buffers
    rms_norm_kernel<<<1, kNormThreads, 0, st>>>(cur, nullptr, a.attn_norm_w, (int)H, a.rms_eps, nullptr, w.n);
    B2_CHECK_LAUNCH("decode_step: rms_norm");
    rc = qmm_bf16(w.n, a.qkv_codes, a.qkv_scales, 1, (nq + 2 * nkv) * kHd, H, w.qkv, st);
    if (rc) return rc;
    rope_cache_kernel<<<(unsigned)(nq + 2 * nkv), kHd / 2, 0, st>>>(w.qkv, (int)nq, (int)nkv, pos,
                                                                    log2f(a.rope_theta), a.max_seq, w.q, a.k_cache,
                                                                    a.v_cache);
    B2_CHECK_LAUNCH("decode_step: rope");
    const float qscale = (1.0f / sqrtf((float)kHd)) * 1.4426950408889634f;
    attn_partial_kernel<<<dim3((unsigned)nkv, (unsigned)S), kAttnThreads, 0, st>>>(w.q, group, a.k_cache, a.v_cache,
                                                                                   a.max_seq, (int)L, chunk, qscale,
                                                                                   w.part);
    B2_CHECK_LAUNCH("decode_step: attention");
    attn_merge_kernel<<<(unsigned)nq, kHd, 0, st>>>(w.part, S, w.attn);
    B2_CHECK_LAUNCH("decode_step: attention merge");
    rc = qmm_bf16(w.attn, a.o_codes, a.o_scales, 1, H, nq * kHd, w.o, st);
    if (rc) return rc;
    // h = x + attention; n = rms_norm(h)
    rms_norm_kernel<<<1, kNormThreads, 0, st>>>(cur, w.o, a.mlp_norm_w, (int)H, a.rms_eps, w.h, w.n);
    B2_CHECK_LAUNCH("decode_step: rms_norm");
    // x' = h + moe(n): the decode block with h as its residual
    rc = decode_forward(&layers[i].moe, w.n, 1, nullptr, w.h, nxt, nullptr, nullptr, w.moe_ws, w.moe_bytes, st);
    if (rc) return rc;
    cur = nxt;
  }
  rms_norm_kernel<<<1, kNormThreads, 0, st>>>(cur, nullptr, final_norm_w, (int)H, a0.rms_eps, nullptr, out);
  B2_CHECK_LAUNCH("decode_step: final norm");
  return B2_OK;
}
