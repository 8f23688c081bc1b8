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
// Kernels per layer: rms_norm (one CTA, vectorized; the second one fuses the
// attention residual), the fused q/k/v GEMV, one attention kernel (RoPE of
// q and of the new k, cache append, split-K attention over the cache with
// the splits merged by the last CTA of each kv head), the o GEMV, and the
// fused decode MoE kernel with the residual in its epilogue: 6 launches.
#include <algorithm>
#include <cmath>

#include "moe.cuh"
#include "moe_prefill.cuh"

namespace b2 {
namespace {

constexpr int kNormThreads = 256;
constexpr int kAttnThreads = 256;
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
// weight, as its kernels do.  One CTA per row; each thread holds 8
// consecutive values (one 16-byte load), H % 8 == 0, H <= 8 * kNormThreads * 4.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const uint16_t* __restrict__ x,
                                                                const uint16_t* __restrict__ add,
                                                                const uint16_t* __restrict__ w, int H, float eps,
                                                                uint16_t* __restrict__ h_out,
                                                                uint16_t* __restrict__ n_out) {
  constexpr int kPer = 4;  // 16-byte chunks per thread at most
  __shared__ float red[kNormThreads / 32];
  // the next kernel (a GEMV or the MoE block, launched as programmatic
  // dependents) may start its weight copies now; it waits for this grid
  // before it reads anything this kernel writes
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // inside a step this kernel is itself a programmatic dependent: x / add
  // are the previous kernel's output (a no-op after a plain launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x;
  x += (int64_t)row * H;
  if (add) add += (int64_t)row * H;
  if (h_out) h_out += (int64_t)row * H;
  n_out += (int64_t)row * H;
  const int chunks = H / 8;
  float v[kPer][8];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int c = threadIdx.x + u * kNormThreads;
    if (c < chunks) {
      const uint4 xv = *reinterpret_cast<const uint4*>(x + 8 * c);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
      uint4 av = make_uint4(0, 0, 0, 0);
      if (add) av = *reinterpret_cast<const uint4*>(add + 8 * c);
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
      uint32_t hw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float lo = __uint_as_float(xw[j] << 16), hi = __uint_as_float(xw[j] & 0xffff0000u);
        if (add) {
          lo = round_bf16(lo + __uint_as_float(aw[j] << 16));
          hi = round_bf16(hi + __uint_as_float(aw[j] & 0xffff0000u));
        }
        v[u][2 * j] = lo;
        v[u][2 * j + 1] = hi;
        hw[j] = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
      if (add) *reinterpret_cast<uint4*>(h_out + 8 * c) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int c = threadIdx.x + u * kNormThreads;
    if (c < chunks) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * c);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __uint_as_float(ww[j] << 16) * round_bf16(v[u][2 * j] * inv);
        const float hi = __uint_as_float(ww[j] & 0xffff0000u) * round_bf16(v[u][2 * j + 1] * inv);
        o[j] = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
      }
      *reinterpret_cast<uint4*>(n_out + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// rms_norm_kernel over one row.  `pdl`: as a programmatic dependent of the
// previous kernel -- only inside a step, where every kernel waits for its
// predecessor before it ends, so a kernel that has started implies that
// every kernel of the step before its predecessor has completed; the first
// norm of a step is a plain launch (the caller's kernels before it need not
// keep that rule).
int launch_norm(const uint16_t* x, const uint16_t* add, const uint16_t* w, int H, float eps, uint16_t* h_out,
                uint16_t* n_out, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[] = {(void*)&x, (void*)&add, (void*)&w, (void*)&H, (void*)&eps, (void*)&h_out, (void*)&n_out};
  cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)rms_norm_kernel, args);
  if (e != cudaSuccess && cfg.numAttrs == 1) {
    (void)cudaGetLastError();
    cfg.numAttrs = 0;
    e = cudaLaunchKernelExC(&cfg, (const void*)rms_norm_kernel, args);
  }
  return e == cudaSuccess ? B2_OK : check_cuda(e, "decode_step: rms_norm");
}

// Attention of one kv head's query group over a chunk of cache positions,
// one CTA per (kv head, split); the last CTA of a kv head to finish merges
// the splits (no separate merge launch).  Per CTA:
//   1. q heads of the group: RoPE (half-split pairs i, i + hd/2, angle =
//      pos * theta^(-2i/hd), f32, rounded to bf16 like MLX's RoPE output),
//      times hd^-0.5 * log2(e) into shared memory; the CTA whose chunk holds
//      `pos` also RoPEs the new k and appends k and v to the caches;
//   2. per piece of up to kPiece positions: the K and V rows are copied into
//      shared memory with every 16-byte copy in flight at once (K rows padded
//      to 272 bytes so that 8 consecutive rows cover all banks; the first
//      piece's copies are issued before the wait for the q/k/v GEMV, whose
//      output they do not need -- the kernel is a programmatic dependent of
//      that GEMV, so they overlap its tail), then
//      scores (thread = position x 4 heads, no cross-lane reduction), an
//      online softmax per head (warp = head) and P.V with lanes over the
//      head dims;
//   3. partial (max, sum, acc[hd]) per q head in f32; the last CTA (an
//      atomic count per kv head, reset by it) merges the S partials into the
//      bf16 attention output.
// Scores are in base 2 (exp2 of log2(e)-scaled logits).
constexpr int kPiece = 128;
constexpr int kKStride = kHd + 8;  // bf16 elements per staged K row (272 bytes)
// split partial of one q head: [max, sum, 2 unused, acc[kHd]] f32, so acc
// starts 16 bytes into a 16-byte-aligned row (float4 stores and loads)
constexpr int kPartStride = kHd + 4;
constexpr int kPartAcc = 4;
// At most this many splits per kv head: the merging CTA stages every
// partial of its kv head in shared memory (group x S rows of kPartStride).
constexpr int kMaxSplits = 40;
constexpr size_t kAttnMainSmem = (size_t)kPiece * kKStride * 2 + (size_t)kPiece * kHd * 2 +
                                 (size_t)kMaxGroup * kHd * 4 + (size_t)kMaxGroup * kPiece * 4 + 2 * kHd * 2;
constexpr size_t kAttnMergeSmem = (size_t)kMaxGroup * kMaxSplits * kPartStride * 4;
constexpr size_t kAttnSmem = kAttnMainSmem > kAttnMergeSmem ? kAttnMainSmem : kAttnMergeSmem;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void rope_pair(float x1, float x2, int i, int64_t pos, float log2_theta, uint16_t* o1,
                                          uint16_t* o2) {
  const float inv_freq = exp2f(-(float)(2 * i) / (float)kHd * log2_theta);
  float sn, cs;
  sincosf((float)pos * inv_freq, &sn, &cs);
  *o1 = f32_to_bf16_bits(x1 * cs - x2 * sn);
  *o2 = f32_to_bf16_bits(x1 * sn + x2 * cs);
}

__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const uint16_t* __restrict__ qkv, int nq, int nkv,
                                                            int group, int64_t pos, float log2_theta,
                                                            uint16_t* __restrict__ k_cache,
                                                            uint16_t* __restrict__ v_cache, int64_t max_seq, int L,
                                                            int chunk, float qscale, float* __restrict__ part,
                                                            unsigned* __restrict__ counters,
                                                            uint16_t* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  uint16_t* sK = reinterpret_cast<uint16_t*>(attn_smem);
  uint16_t* sV = sK + kPiece * kKStride;
  float* sQ = reinterpret_cast<float*>(sV + kPiece * kHd);  // [kMaxGroup][kHd]
  float* sP = sQ + kMaxGroup * kHd;                          // [kMaxGroup][kPiece]
  uint16_t* sNew = reinterpret_cast<uint16_t*>(sP + kMaxGroup * kPiece);  // new k row, new v row
  __shared__ float sF[kMaxGroup][kMaxSplits];
  __shared__ int s_last;
  const int h = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = split * chunk, j1 = min(L, j0 + chunk);
  const bool has_new = pos >= j0 && pos < j1;
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the o GEMV's weights
  const uint16_t* kb = k_cache + (int64_t)h * max_seq * kHd;
  const uint16_t* vb = v_cache + (int64_t)h * max_seq * kHd;
  // cached rows of a piece (every position but `pos`, whose row this launch
  // writes): written by earlier launches, which completed before the q/k/v
  // GEMV this kernel depends on was launched
  auto issue_piece = [&](int p0, int rows) {
    for (int idx = tid; idx < rows * 16; idx += kAttnThreads) {
      const int r = idx >> 4, c = idx & 15;
      if (p0 + r != pos) {
        cp_async16(sK + r * kKStride + 8 * c, kb + (int64_t)(p0 + r) * kHd + 8 * c);
        cp_async16(sV + r * kHd + 8 * c, vb + (int64_t)(p0 + r) * kHd + 8 * c);
      }
    }
  };
  if (j0 < j1) issue_piece(j0, min(kPiece, j1 - j0));
  // the q/k/v rows are the previous kernel's output
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // 1. q of the group (RoPE, bf16, scaled) and, in the CTA holding pos, the new k / v
  for (int t = tid; t < group * (kHd / 2); t += kAttnThreads) {
    const int g = t / (kHd / 2), i = t % (kHd / 2);
    const uint16_t* src = qkv + (int64_t)(h * group + g) * kHd;
    uint16_t o1, o2;
    rope_pair(bf16_bits_to_f32(src[i]), bf16_bits_to_f32(src[i + kHd / 2]), i, pos, log2_theta, &o1, &o2);
    sQ[g * kHd + i] = bf16_bits_to_f32(o1) * qscale;
    sQ[g * kHd + i + kHd / 2] = bf16_bits_to_f32(o2) * qscale;
  }
  if (has_new && tid < kHd) {
    const uint16_t* ksrc = qkv + (int64_t)(nq + h) * kHd;
    const uint16_t* vsrc = qkv + (int64_t)(nq + nkv + h) * kHd;
    if (tid < kHd / 2) {
      uint16_t o1, o2;
      rope_pair(bf16_bits_to_f32(ksrc[tid]), bf16_bits_to_f32(ksrc[tid + kHd / 2]), tid, pos, log2_theta, &o1, &o2);
      sNew[tid] = o1;
      sNew[tid + kHd / 2] = o2;
      uint16_t* kd = k_cache + ((int64_t)h * max_seq + pos) * kHd;
      kd[tid] = o1;
      kd[tid + kHd / 2] = o2;
    }
    const uint16_t v = vsrc[tid];
    sNew[kHd + tid] = v;
    v_cache[((int64_t)h * max_seq + pos) * kHd + tid] = v;
  }
  __syncthreads();

  float m_run = -INFINITY, l_run = 0.0f, acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // warp = head `warp`
  for (int p0 = j0; p0 < j1; p0 += kPiece) {
    const int rows = min(kPiece, j1 - p0);
    // 2a. stage the piece (the first was issued at entry; the new row comes
    // from shared memory)
    if (p0 != j0) issue_piece(p0, rows);
    if (pos >= p0 && pos < p0 + rows && tid < 16) {
      const int r = (int)(pos - p0);
      *reinterpret_cast<uint4*>(sK + r * kKStride + 8 * tid) = *reinterpret_cast<const uint4*>(sNew + 8 * tid);
      *reinterpret_cast<uint4*>(sV + r * kHd + 8 * tid) = *reinterpret_cast<const uint4*>(sNew + kHd + 8 * tid);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    // 2b. scores: thread = (position r, heads 4*half .. 4*half+3)
    {
      const int r = tid % kPiece, g0 = 4 * (tid / kPiece);
      if (r < rows && g0 < group) {
        float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint16_t* kr = sK + r * kKStride;
#pragma unroll 4
        for (int c = 0; c < kHd / 8; ++c) {
          const uint4 kv = *reinterpret_cast<const uint4*>(kr + 8 * c);
          const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
          float kx[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            kx[2 * j] = __uint_as_float(kw[j] << 16);
            kx[2 * j + 1] = __uint_as_float(kw[j] & 0xffff0000u);
          }
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const float4 qa = *reinterpret_cast<const float4*>(sQ + (g0 + g) * kHd + 8 * c);
            const float4 qb = *reinterpret_cast<const float4*>(sQ + (g0 + g) * kHd + 8 * c + 4);
            sc[g] = fmaf(qa.x, kx[0], sc[g]);
            sc[g] = fmaf(qa.y, kx[1], sc[g]);
            sc[g] = fmaf(qa.z, kx[2], sc[g]);
            sc[g] = fmaf(qa.w, kx[3], sc[g]);
            sc[g] = fmaf(qb.x, kx[4], sc[g]);
            sc[g] = fmaf(qb.y, kx[5], sc[g]);
            sc[g] = fmaf(qb.z, kx[6], sc[g]);
            sc[g] = fmaf(qb.w, kx[7], sc[g]);
          }
        }
#pragma unroll
        for (int g = 0; g < 4; ++g)
          if (g0 + g < group) sP[(g0 + g) * kPiece + r] = sc[g];
      }
    }
    __syncthreads();
    // 2c. online softmax and P.V: warp = head, lanes over 4 dims each
    if (warp < group) {
      float* pg = sP + warp * kPiece;
      float pm = -INFINITY;
      for (int r = lane; r < rows; r += 32) pm = fmaxf(pm, pg[r]);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o));
      const float mn = fmaxf(m_run, pm);
      const float corr = exp2f(m_run - mn);
      float ls = 0.0f;
      for (int r = lane; r < rows; r += 32) {
        const float pr = exp2f(pg[r] - mn);
        pg[r] = pr;
        ls += pr;
      }
      ls = warp_sum(ls);
      __syncwarp();
      l_run = fmaf(l_run, corr, ls);
#pragma unroll
      for (int d = 0; d < 4; ++d) acc[d] *= corr;
#pragma unroll 4
      for (int r = 0; r < rows; ++r) {
        const float pr = pg[r];
        const uint2 vr = *reinterpret_cast<const uint2*>(sV + r * kHd + 4 * lane);
        acc[0] = fmaf(pr, __uint_as_float(vr.x << 16), acc[0]);
        acc[1] = fmaf(pr, __uint_as_float(vr.x & 0xffff0000u), acc[1]);
        acc[2] = fmaf(pr, __uint_as_float(vr.y << 16), acc[2]);
        acc[3] = fmaf(pr, __uint_as_float(vr.y & 0xffff0000u), acc[3]);
      }
      m_run = mn;
    }
    __syncthreads();  // the piece may be refilled
  }

  // 3. partials, then the last CTA of this kv head merges
  if (warp < group) {
    float* dst = part + ((int64_t)(h * group + warp) * S + split) * kPartStride;
    *reinterpret_cast<float4*>(dst + kPartAcc + 4 * lane) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    if (lane == 0) {
      dst[0] = m_run;
      dst[1] = l_run;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&counters[h], 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // every partial of this kv head into shared memory (all copies in flight
  // at once; the staging area is free: the loop above ended on a barrier)
  float* sPart = reinterpret_cast<float*>(attn_smem);  // [group][S][kPartStride]
  {
    constexpr int kChunks = kPartStride / 4;  // 16-byte pieces per partial row
    const float* src = part + (int64_t)h * group * S * kPartStride;
    for (int idx = tid; idx < group * S * kChunks; idx += kAttnThreads) {
      const int row = idx / kChunks, c = idx % kChunks;
      cp_async16(sPart + row * kPartStride + 4 * c, src + (int64_t)row * kPartStride + 4 * c);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
  }
  if (warp < group) {
    const float* pb = sPart + warp * S * kPartStride;
    float* f = sF[warp];
    float mx = -INFINITY;
    for (int s2 = lane; s2 < S; s2 += 32) mx = fmaxf(mx, pb[s2 * kPartStride]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float ls = 0.0f;
    for (int s2 = lane; s2 < S; s2 += 32) {
      const float ms = pb[s2 * kPartStride];
      const float fs = ms == -INFINITY ? 0.0f : exp2f(ms - mx);
      f[s2] = fs;
      ls = fmaf(pb[s2 * kPartStride + 1], fs, ls);
    }
    ls = warp_sum(ls);
    __syncwarp();
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
    for (int s2 = 0; s2 < S; ++s2) {
      const float4 v = *reinterpret_cast<const float4*>(pb + s2 * kPartStride + kPartAcc + 4 * lane);
      const float fs = f[s2];
      a[0] = fmaf(v.x, fs, a[0]);
      a[1] = fmaf(v.y, fs, a[1]);
      a[2] = fmaf(v.z, fs, a[2]);
      a[3] = fmaf(v.w, fs, a[3]);
    }
    const float inv = 1.0f / ls;
    uint16_t* o = out + (int64_t)(h * group + warp) * kHd + 4 * lane;
    const uint32_t w0 = (uint32_t)f32_to_bf16_bits(a[0] * inv) | ((uint32_t)f32_to_bf16_bits(a[1] * inv) << 16);
    const uint32_t w1 = (uint32_t)f32_to_bf16_bits(a[2] * inv) | ((uint32_t)f32_to_bf16_bits(a[3] * inv) << 16);
    *reinterpret_cast<uint2*>(o) = make_uint2(w0, w1);
  }
  if (tid == 0) counters[h] = 0u;  // ready for the next launch
}

int attn_splits(int64_t L, int nkv, int sms) {
  const int want = std::max(1, std::min(kMaxSplits, sms / std::max(1, nkv)));
  return (int)std::min<int64_t>(want, std::max<int64_t>(1, (L + 31) / 32));
}

struct StepWs {
  uint16_t *qkv, *attn, *o, *h, *n, *xa, *xb;
  float* part;
  unsigned* counters;  // per kv head: attention CTAs done (zero between launches)
  void* moe_ws;
  size_t moe_bytes, bytes;
};

// The attention kernel as a programmatic dependent of the q/k/v GEMV before
// it (plain launch when the attribute is refused).
int launch_attn(const StepWs& w, int64_t nq, int64_t nkv, int group, int64_t pos, float log2_theta,
                uint16_t* k_cache, uint16_t* v_cache, int64_t max_seq, int64_t L, int chunk, float qscale, int S,
                cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nkv, (unsigned)S);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = kAttnSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const uint16_t* qkv = w.qkv;
  int inq = (int)nq, inkv = (int)nkv, iL = (int)L;
  float* part = w.part;
  unsigned* counters = w.counters;
  uint16_t* out = w.attn;
  void* args[] = {(void*)&qkv, (void*)&inq, (void*)&inkv, (void*)&group, (void*)&pos, (void*)&log2_theta,
                  (void*)&k_cache, (void*)&v_cache, (void*)&max_seq, (void*)&iL, (void*)&chunk, (void*)&qscale,
                  (void*)&part, (void*)&counters, (void*)&out};
  cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)attn_kernel, args);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    cfg.numAttrs = 0;
    e = cudaLaunchKernelExC(&cfg, (const void*)attn_kernel, args);
  }
  return e == cudaSuccess ? B2_OK : check_cuda(e, "decode_step: attention");
}

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
  w.attn = reinterpret_cast<uint16_t*>(take((size_t)nq * kHd * 2));
  w.o = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.h = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.n = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.xa = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  w.xb = reinterpret_cast<uint16_t*>(take((size_t)H * 2));
  const int S = attn_splits(a.max_seq, (int)nkv, sms);
  w.part = reinterpret_cast<float*>(take((size_t)nq * S * kPartStride * 4));
  w.counters = reinterpret_cast<unsigned*>(take((size_t)nkv * 4));
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
    B2_REQUIRE(a.hidden % 16 == 0 && a.hidden <= 8 * 256 * 4 && a.max_seq > 0,
               "[decode_step] hidden must be a multiple of 16 and at most 8192; max_seq positive");
    B2_REQUIRE(a.attn_norm_w && a.mlp_norm_w && a.qkv_codes && a.qkv_scales && a.o_codes && a.o_scales &&
                   a.k_cache && a.v_cache,
               "[decode_step] layer %d: null attention pointer", i);
    B2_REQUIRE(reinterpret_cast<uintptr_t>(a.k_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(a.v_cache) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.attn_norm_w) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.mlp_norm_w) % 16 == 0,
               "[decode_step] layer %d: KV caches and norm weights must be 16-byte aligned", i);
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
  B2_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(final_norm_w) % 16 == 0,
             "[decode_step] x, out and the norm weights must be 16-byte aligned");
  B2_REQUIRE(pos >= 0 && pos < a0.max_seq, "[decode_step] position %lld outside the cache [0, %lld)", (long long)pos,
             (long long)a0.max_seq);
  B2_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "[decode_step] workspace must be 256-byte aligned");
  const int sms = sm_count();
  rc = ensure_dynamic_smem((const void*)attn_kernel, kAttnSmem, "decode_step attention");
  if (rc) return rc;
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
    rc = launch_norm(cur, nullptr, a.attn_norm_w, (int)H, a.rms_eps, nullptr, w.n, i > 0, st);
    if (rc) return rc;
    rc = qmm_bf16(w.n, a.qkv_codes, a.qkv_scales, 1, (nq + 2 * nkv) * kHd, H, w.qkv, st);
    if (rc) return rc;
    const float qscale = (1.0f / sqrtf((float)kHd)) * 1.4426950408889634f;
    rc = launch_attn(w, nq, nkv, group, pos, log2f(a.rope_theta), a.k_cache, a.v_cache, a.max_seq, L, chunk,
                     qscale, S, st);
    if (rc) return rc;
    rc = qmm_bf16(w.attn, a.o_codes, a.o_scales, 1, H, nq * kHd, w.o, st);
    if (rc) return rc;
    // h = x + attention; n = rms_norm(h)
    rc = launch_norm(cur, w.o, a.mlp_norm_w, (int)H, a.rms_eps, w.h, w.n, true, st);
    if (rc) return rc;
    // x' = h + moe(n): the decode block with h as its residual
    rc = decode_forward(&layers[i].moe, w.n, 1, nullptr, w.h, nxt, nullptr, nullptr, w.moe_ws, w.moe_bytes, st);
    if (rc) return rc;
    cur = nxt;
  }
  return launch_norm(cur, nullptr, final_norm_w, (int)H, a0.rms_eps, nullptr, out, true, st);
}
