// Pieces shared by the fused decode MoE kernels (moe_decode.cu: MLX-layout
// banks streamed with cp.async; moe_decode_tma.cu: the prepared decode bank
// streamed with TMA bulk copies).
#pragma once

#include "moe.cuh"

namespace b2 {
namespace dec {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kRowPad = 16;
constexpr uint32_t kSpinLimit = 1u << 24;  // polls of a cross-CTA counter (~seconds)
constexpr int kMaxSlots = 32;

struct Params {
  const uint16_t* x;         // [T, H] bf16
  const void* router_w;      // [E, H]
  int router_w_dtype;
  const float* router_bias;  // [E] or null
  const float* logits_in;    // [T, E] or null
  const uint8_t* gcodes; const uint8_t* gscales;
  const uint8_t* ucodes; const uint8_t* uscales;
  const uint8_t* dcodes; const uint8_t* dscales;
  const uint16_t* residual;  // [T, H] or null
  uint16_t* out;             // [T, H]
  uint32_t* inds_out;        // [T, k]
  float* wts_out;            // [T, k]
  float* logits;             // scratch [T, E]
  uint16_t* act;             // scratch [T, k, F] bf16
  unsigned* counters;        // scratch: [0] logits, [1] exit, [8 + t] per-token activations
  unsigned* status;
  int T, E, H, F, k, mode, renorm;
  float routed_scale;
  int n_slots;               // ring slots in shared memory
  int slot_bytes;
  int n_gu;                  // gate/up tiles = T*k*(F/8)
  int n_items;               // n_gu + T*(H/2)
  int max_items;             // tiles per CTA, rounded up
  // prepared decode bank (b2_moe_prepare_decode_bank), or null
  const uint8_t* bank_gu;    // [E][F/8] tiles of 9*H bytes
  const uint8_t* bank_dn;    // [E][H/16] tiles of 9*F bytes
  int n_dn_slots;            // down-tile ring slots (prepared path)
  int router_smem;           // router rows of this CTA's logit tasks are bulk-copied to smem (prepared path)
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Two E2M1 codes (one byte) -> f16x2; byte 0 / byte 1 of `w`.
__device__ __forceinline__ uint32_t cvt_byte0(uint32_t w) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
      : "=r"(out)
      : "r"(w));
  return out;
}
__device__ __forceinline__ uint32_t cvt_byte1(uint32_t w) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b1;\n\t}"
      : "=r"(out)
      : "r"(w));
  return out;
}

// Scale bytes of rows r (low) and r+8 (high) -> f16x2 with MLX's E4M3 decode
// (bits 6..0 as the low bits of a half, times 256, bit 7 = sign).
__device__ __forceinline__ uint32_t scale_pair(uint32_t lo, uint32_t hi) {
  const uint32_t t = lo | (hi << 16);
  const uint32_t h = ((t & 0x007f007fu) << 7) | ((t & 0x00800080u) << 8);
  const __half2 k256 = __floats2half2_rn(256.0f, 256.0f);
  __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&h), k256);
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Arrive on `bar` once all of this thread's earlier cp.async copies landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Stage `nrows` rows of bf16 (global, read through L2) as f16 with a per-row
// power-of-two pre-scale so that max|x| * 2^-p < 2^15 (exact for every value
// >= 2^-17 * 2^p).  Executed by `nthreads` threads (local index ltid) that
// synchronise on named barrier `bar_id`; rows are contiguous in `src`.  The
// first kKeep chunks of each thread stay in registers between the row-max
// pass and the conversion pass, so the source is read once.
__device__ __forceinline__ void stage_chunk(uint4 v, int i, int chunks, const unsigned* red_max, __half* dst,
                                            int stride) {
  const int m = i / chunks, c = i - m * chunks;
  const unsigned e = (red_max[m] >> 7) & 0xffu;
  const float sc = (e >= 142u) ? __int_as_float((127 + 141 - (int)e) << 23) : 1.0f;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 hh = __floats2half2_rn(__uint_as_float(w[j] << 16) * sc, __uint_as_float(w[j] & 0xffff0000u) * sc);
    o[j] = *reinterpret_cast<uint32_t*>(&hh);
  }
  *reinterpret_cast<uint4*>(dst + (size_t)m * stride + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ unsigned chunk_absmax(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  unsigned mx = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) mx = max(mx, max(w[j] & 0x7fffu, (w[j] >> 16) & 0x7fffu));
  return mx;
}

__device__ inline void stage_rows(const uint16_t* src, int nrows, int K, __half* dst, int stride, int* xexp,
                                  unsigned* red_max, int ltid, int nthreads, int bar_id) {
  constexpr int kKeep = 4;
  const int chunks = K / 8;
  const int total = nrows * chunks;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  if (ltid < 32) red_max[ltid] = 0u;
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  uint4 kept[kKeep];
#pragma unroll
  for (int j = 0; j < kKeep; ++j) {
    const int i = ltid + j * nthreads;
    if (i < total) {
      kept[j] = __ldcg(s4 + i);
      const unsigned mx = chunk_absmax(kept[j]);
      if (mx) atomicMax(&red_max[i / chunks], mx);
    }
  }
  for (int i = ltid + kKeep * nthreads; i < total; i += nthreads) {
    const unsigned mx = chunk_absmax(__ldcg(s4 + i));
    if (mx) atomicMax(&red_max[i / chunks], mx);
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  if (ltid < nrows) {
    const unsigned e = (red_max[ltid] >> 7) & 0xffu;
    xexp[ltid] = (e >= 142u) ? (int)e - 141 : 0;
  }
#pragma unroll
  for (int j = 0; j < kKeep; ++j) {
    const int i = ltid + j * nthreads;
    if (i < total) stage_chunk(kept[j], i, chunks, red_max, dst, stride);
  }
  for (int i = ltid + kKeep * nthreads; i < total; i += nthreads) stage_chunk(__ldcg(s4 + i), i, chunks, red_max, dst, stride);
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
}

// Order-preserving 64-bit ranking key: larger key first, NaN last, -0 == +0,
// ties by the smaller index (the ranking order of the reference's top-k).
__device__ __forceinline__ unsigned long long rank_key(float f, int e) {
  uint32_t u = __float_as_uint(f);
  if (f == 0.0f) u = 0u;
  uint32_t k;
  if (isnan(f))
    k = 0u;
  else
    k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)k << 32) | (0xffffffffu - (uint32_t)e);
}

// Top-k of every token's logits by parallel rank counting (all threads):
// key e's rank is the number of keys that rank before it; keys of rank < k
// are the selection, in rank order.  keys / vals / rank: shared scratch.
__device__ inline void topk_ranked(const Params& p, const float* logits, uint32_t* inds, float* wts,
                            unsigned long long* keys, float* vals, unsigned* rank) {
  const int tid = threadIdx.x;
  const int E = p.E;
  const int parts = E >= (int)blockDim.x ? 1 : (int)blockDim.x / E;
  const int span = (E + parts - 1) / parts;
  for (int t = 0; t < p.T; ++t) {
    for (int e = tid; e < E; e += blockDim.x) {
      const float x = __ldcg(logits + (size_t)t * E + e);
      float kv, vv;
      if (p.mode == B2_ROUTER_SOFTMAX) {
        kv = x;
        vv = x;
      } else {
        vv = sigmoid_stable(x);
        kv = vv + (p.router_bias ? p.router_bias[e] : 0.0f);
      }
      keys[e] = rank_key(kv, e);
      vals[e] = vv;
      rank[e] = 0u;
    }
    __syncthreads();
    for (int idx = tid; idx < E * parts; idx += blockDim.x) {
      const int e = idx % E, part = idx / E;
      const unsigned long long ke = keys[e];
      const int j0 = part * span, j1 = min(E, j0 + span);
      unsigned cnt = 0;
      int j = j0;
      for (; j + 8 <= j1; j += 8) {
        unsigned long long kk[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) kk[u] = keys[j + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) cnt += kk[u] > ke ? 1u : 0u;
      }
      for (; j < j1; ++j) cnt += keys[j] > ke ? 1u : 0u;
      if (parts == 1)
        rank[e] = cnt;
      else if (cnt)
        atomicAdd(&rank[e], cnt);
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
      const unsigned r = rank[e];
      if (r < (unsigned)p.k) inds[t * p.k + r] = (uint32_t)e;
    }
    __syncthreads();
    if (tid < 32) {
      const int lane = tid;
      const float v = lane < p.k ? vals[inds[t * p.k + lane]] : 0.0f;
      float wv;
      if (p.mode == B2_ROUTER_SOFTMAX) {
        const float mx = __shfl_sync(0xffffffffu, v, 0);
        const float ev = lane < p.k ? b2_expf(__fsub_rn(v, mx)) : 0.0f;
        float tot = 0.0f;
        for (int s = 0; s < p.k; ++s) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, ev, s));
        wv = __fdiv_rn(ev, tot);
      } else {
        float tot = 0.0f;
        for (int s = 0; s < p.k; ++s) tot = __fadd_rn(__shfl_sync(0xffffffffu, v, s), tot);
        wv = p.renorm ? __fdiv_rn(v, tot) : v;
      }
      if (lane < p.k) wts[t * p.k + lane] = wv;
    }
    __syncthreads();
  }
}

__device__ __forceinline__ void release_tokens(const Params& p, unsigned* tokdone) {
  __threadfence();
  for (int t = 0; t < p.T; ++t)
    if (tokdone[t]) atomicAdd(&p.counters[8 + t], tokdone[t]);
}

// Phase 1 of both kernels: router logits (warps [0, R) of every CTA, one warp
// per (token, expert)), the f16 staging of the tokens (the other warps), the
// grid-wide wait for all logits and the redundant per-CTA top-k.  Leaves the
// selection in s_inds / s_wts (CTA 0 also writes the routing outputs) and
// clears *s_ok on a timed-out wait.  `scratch` must hold 16 bytes per expert.
int launch_tma(Params& p, const b2_moe_block* blk, cudaStream_t st);

__device__ __forceinline__ void phase1(const Params& p, __half* xs, int xstride, int* s_xexp, unsigned* s_red,
                                       uint32_t* s_inds, float* s_wts, int* s_ok, uint8_t* scratch,
                                       const uint8_t* rsm = nullptr, uint64_t* rbar = nullptr) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  // ---------------- phase 1: router logits (warps [0, R)) + token staging (the rest)
  const int tasks = p.logits_in ? 0 : p.T * p.E;
  const int per_cta = (tasks + G - 1) / G;
  const int R = min(kWarps, per_cta);
  if (warp < R) {
    // rsm: the router rows of this CTA's tasks (cta, cta + G, ...) in order,
    // landed in shared memory by bulk copies completing on rbar
    const int wsz = p.router_w_dtype == B2_DTYPE_F32 ? 4 : 2;
    if (rsm) mbar_wait_bounded(rbar, 0u, p.status);
    for (int task = cta + warp * G; task < tasks; task += G * R) {
      const int t = task / p.E, e = task % p.E;
      const uint16_t* xr = p.x + (int64_t)t * p.H;
      const uint8_t* wrow = rsm ? rsm + (size_t)((task - cta) / G) * p.H * wsz : nullptr;
      float a = 0.0f;
      const int chunks = p.H / 4;
      for (int base = lane; base < chunks; base += 32 * 8) {
        float4 w4[8];
        uint2 xv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c4 = base + 32 * u;
          if (c4 < chunks) {
            if (p.router_w_dtype == B2_DTYPE_F32) {
              w4[u] = wrow ? *reinterpret_cast<const float4*>(wrow + 16 * (size_t)c4)
                           : __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.router_w) +
                                                                   (int64_t)e * p.H + 4 * c4));
            } else {
              const uint2 wv = wrow ? *reinterpret_cast<const uint2*>(wrow + 8 * (size_t)c4)
                                    : __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p.router_w) +
                                                                           (int64_t)e * p.H + 4 * c4));
              w4[u] = make_float4(__uint_as_float(wv.x << 16), __uint_as_float(wv.x & 0xffff0000u),
                                  __uint_as_float(wv.y << 16), __uint_as_float(wv.y & 0xffff0000u));
            }
            xv[u] = __ldg(reinterpret_cast<const uint2*>(xr + 4 * c4));
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (base + 32 * u < chunks) {
            a = fmaf(__uint_as_float(xv[u].x << 16), w4[u].x, a);
            a = fmaf(__uint_as_float(xv[u].x & 0xffff0000u), w4[u].y, a);
            a = fmaf(__uint_as_float(xv[u].y << 16), w4[u].z, a);
            a = fmaf(__uint_as_float(xv[u].y & 0xffff0000u), w4[u].w, a);
          }
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) a = a + __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) {
        p.logits[(int64_t)t * p.E + e] = a;
        __threadfence();
        atomicAdd(&p.counters[0], 1u);
      }
    }
  }
  // warps beyond kWarps (a control warp) take no part in the staging
  if (R < kWarps) {
    if (warp >= R && warp < kWarps)
      stage_rows(p.x, p.T, p.H, xs, xstride, s_xexp, s_red, tid - R * 32, (kWarps - R) * 32, 1);
  } else if (warp < kWarps) {
    stage_rows(p.x, p.T, p.H, xs, xstride, s_xexp, s_red, tid, kThreads, 1);
  }

  // ---------------- top-k (every CTA, redundantly)
  if (tasks && tid == 0) {
    uint32_t i = 0;
    while (ld_acquire(&p.counters[0]) < (unsigned)tasks) {
      if (++i >= kSpinLimit) {
        report_status(p.status, B2_STATUS_WAIT_TIMEOUT);
        *s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  {
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(scratch);
    float* vals = reinterpret_cast<float*>(keys + p.E);
    unsigned* rank = reinterpret_cast<unsigned*>(vals + p.E);
    topk_ranked(p, p.logits_in ? p.logits_in : p.logits, s_inds, s_wts, keys, vals, rank);
  }
  if (cta == 0)
    for (int i = tid; i < p.T * p.k; i += blockDim.x) {
      p.inds_out[i] = s_inds[i];
      p.wts_out[i] = s_wts[i];
    }

}

}  // namespace dec
}  // namespace b2
