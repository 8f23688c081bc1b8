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

// Test hook state (b2_testing_set_decode_fault): the CTA that leaves its
// router logits unwritten (-1: none) and the cross-CTA wait bound.
void testing_decode_fault(int* skip_logit_cta, uint32_t* spin_limit);
constexpr int kMaxSlots = 32;

// Cross-launch state at the head of the workspace (kDecodeStateBytes; the
// prefill path never writes it).  u32 words:
//   [kActCnt, kActCnt + 16)  per-token activation counters, two sets of 8:
//                            a launch with epoch n counts in set n & 1 and
//                            clears set (n & 1) ^ 1 for the next launch;
//   [kEpochs, kEpochs + kMaxCtas)  launch epoch of each CTA index (every
//                            launch runs every CTA once, so all CTAs of a
//                            launch read the same value);
// then at byte kLogitWords the router logits of the launch, [8][1024] u64
// words (epoch + 1) << 32 | f32 bits, written with one 64-bit store each so
// a reader that sees its launch's tag also sees the value.  Nothing is reset
// at exit: no CTA waits for the others to finish, and a launch that gave up
// on a wait leaves nothing the next launch would trust.
constexpr int kActCnt = 16;
constexpr int kEpochs = 64;
constexpr int kMaxCtas = 960;
constexpr size_t kLogitWords = 4096;
static_assert(kLogitWords + 8 * 1024 * 8 == kDecodeStateBytes, "decode state layout");
static_assert(4 * (kEpochs + kMaxCtas) <= (int)kLogitWords, "decode state layout");

struct Params {
  const uint16_t* x;         // [T, H] bf16
  const void* router_w;      // [E, H]
  int router_w_dtype;
  const float* router_bias;  // [E] or null
  const float* logits_in;    // [T, E] or null
  const uint8_t* gcodes; const uint8_t* gscales;
  const uint8_t* ucodes; const uint8_t* uscales;
  const uint8_t* dcodes; const uint8_t* dscales;
  const uint16_t* shared;    // [T, H] shared-expert output or null
  const uint16_t* residual;  // [T, H] or null
  uint16_t* out;             // [T, H]
  uint32_t* inds_out;        // [T, k]
  float* wts_out;            // [T, k]
  unsigned long long* logit_words;  // scratch [T, E]: (epoch + 1) << 32 | f32 bits
  uint16_t* act;             // scratch [T, k, F] bf16
  unsigned* counters;        // cross-launch state: activation counter sets, launch epochs
  unsigned* status;
  uint32_t spin_limit;       // polls of a cross-CTA wait before it gives up
  int skip_logit_cta;        // test hook: this CTA leaves its logits unwritten (-1: none)
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
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The logit of this launch at *w (tag = epoch + 1), polled with a bound; on
// expiry the wait is reported, *ok cleared and 0 returned.
__device__ __forceinline__ float wait_logit(const unsigned long long* w, uint32_t tag, unsigned* status, int* ok,
                                            uint32_t limit) {
  if (!*reinterpret_cast<volatile int*>(ok)) return 0.0f;  // the CTA already gave up
  for (uint32_t i = 0; i < limit; ++i) {
    const unsigned long long v = ld_relaxed_u64(w);
    if ((uint32_t)(v >> 32) == tag) return __uint_as_float((uint32_t)v);
  }
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
  *ok = 0;
  return 0.0f;
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
// Row of flat chunk index i: i / chunks as a multiply-high by inv =
// floor((2^32 - 1) / chunks) + 1 (checked exhaustively: exact for every
// i < 8 * chunks with K = 8 * chunks a multiple of 256 up to 65536).
__device__ __forceinline__ int row_of(int i, uint32_t inv) { return (int)__umulhi((uint32_t)i, inv); }

__device__ __forceinline__ void stage_chunk(uint4 v, int i, int chunks, uint32_t inv, const unsigned* red_max,
                                            __half* dst, int stride) {
  const int m = row_of(i, inv), c = i - m * chunks;
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

// Not inlined: both decode kernels stage twice (tokens, then activations),
// and one shared copy keeps the kernels' code (and their instruction-cache
// misses) smaller.
static __device__ __noinline__ void stage_rows(const uint16_t* src, int nrows, int K, __half* dst, int stride, int* xexp,
                                  unsigned* red_max, int ltid, int nthreads, int bar_id) {
  constexpr int kKeep = 4;
  const int chunks = K / 8;
  const int total = nrows * chunks;
  const uint32_t inv = 0xffffffffu / (uint32_t)chunks + 1u;
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
      if (mx) atomicMax(&red_max[row_of(i, inv)], mx);
    }
  }
#pragma unroll 1
  for (int i = ltid + kKeep * nthreads; i < total; i += nthreads) {
    const unsigned mx = chunk_absmax(__ldcg(s4 + i));
    if (mx) atomicMax(&red_max[row_of(i, inv)], mx);
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  if (ltid < nrows) {
    const unsigned e = (red_max[ltid] >> 7) & 0xffu;
    xexp[ltid] = (e >= 142u) ? (int)e - 141 : 0;
  }
#pragma unroll
  for (int j = 0; j < kKeep; ++j) {
    const int i = ltid + j * nthreads;
    if (i < total) stage_chunk(kept[j], i, chunks, inv, red_max, dst, stride);
  }
#pragma unroll 1
  for (int i = ltid + kKeep * nthreads; i < total; i += nthreads)
    stage_chunk(__ldcg(s4 + i), i, chunks, inv, red_max, dst, stride);
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
// are the selection, in rank order.  The logits come from p.logits_in, or
// from this launch's tagged logit words (tag), each waited for by the thread
// that ranks it.  keys / vals / rank: shared scratch.
__device__ inline void topk_ranked(const Params& p, uint32_t tag, int* s_ok, uint32_t* inds, float* wts,
                                   unsigned long long* keys, float* vals, unsigned* rank) {
  const int tid = threadIdx.x;
  const int E = p.E;
  const int parts = E >= (int)blockDim.x ? 1 : (int)blockDim.x / E;
  const int span = (E + parts - 1) / parts;
#pragma unroll 1
  for (int t = 0; t < p.T; ++t) {
#pragma unroll 1
    for (int e = tid; e < E; e += blockDim.x) {
      const float x = p.logits_in ? __ldg(p.logits_in + (size_t)t * E + e)
                                  : wait_logit(p.logit_words + (size_t)t * E + e, tag, p.status, s_ok,
                                               p.spin_limit);
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
#pragma unroll 1
    for (int idx = tid; idx < E * parts; idx += blockDim.x) {
      const int e = idx % E, part = idx / E;
      const unsigned long long ke = keys[e];
      const int j0 = part * span, j1 = min(E, j0 + span);
      unsigned cnt = 0;
      int j = j0;
#pragma unroll 1
      for (; j + 8 <= j1; j += 8) {
        unsigned long long kk[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) kk[u] = keys[j + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) cnt += kk[u] > ke ? 1u : 0u;
      }
#pragma unroll 1
      for (; j < j1; ++j) cnt += keys[j] > ke ? 1u : 0u;
      if (parts == 1)
        rank[e] = cnt;
      else if (cnt)
        atomicAdd(&rank[e], cnt);
    }
    __syncthreads();
#pragma unroll 1
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
#pragma unroll 1
        for (int s = 0; s < p.k; ++s) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, ev, s));
        wv = __fdiv_rn(ev, tot);
      } else {
        float tot = 0.0f;
#pragma unroll 1
        for (int s = 0; s < p.k; ++s) tot = __fadd_rn(__shfl_sync(0xffffffffu, v, s), tot);
        wv = p.renorm ? __fdiv_rn(v, tot) : v;
      }
      if (lane < p.k) wts[t * p.k + lane] = wv;
    }
    __syncthreads();
  }
}

__device__ __forceinline__ void release_tokens(const Params& p, unsigned* act_cnt, unsigned* tokdone) {
  __threadfence();
  for (int t = 0; t < p.T; ++t)
    if (tokdone[t]) atomicAdd(&act_cnt[t], tokdone[t]);
}

// Phase 1 of both kernels: router logits (warps [0, R) of every CTA, one warp
// per (token, expert)), the f16 staging of the tokens (the other warps) and
// the redundant per-CTA top-k, whose threads wait for the logits they rank.
// Leaves the selection in s_inds / s_wts (CTA 0 also writes the routing
// outputs), clears *s_ok on a timed-out wait and returns the launch epoch.
// `scratch` must hold 16 bytes per expert; s_ep is one shared word.
int launch_tma(Params& p, const b2_moe_block* blk, cudaStream_t st);

__device__ __forceinline__ uint32_t phase1(const Params& p, __half* xs, int xstride, int* s_xexp, unsigned* s_red,
                                           uint32_t* s_inds, float* s_wts, int* s_ok, uint32_t* s_ep,
                                           uint8_t* scratch, const uint8_t* rsm = nullptr, uint64_t* rbar = nullptr) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  // ---------------- phase 1: router logits (warps [0, R)) + token staging (the rest)
  const int tasks = p.logits_in ? 0 : p.T * p.E;
  const int per_cta = (tasks + G - 1) / G;
  const int R = min(kWarps, per_cta);
  // The epoch is read here by the threads that store logits (and thread 0)
  // and advanced by thread 0 only after the CTA barrier below; the load's
  // latency hides behind the router-row copy.
  uint32_t ep = 0;
  if (tid == 0 || (warp < R && lane == 0)) ep = __ldcg(p.counters + kEpochs + cta);
  if (warp < R) {
    // rsm: the router rows of this CTA's tasks (cta, cta + G, ...) in order,
    // landed in shared memory by bulk copies completing on rbar
    const int wsz = p.router_w_dtype == B2_DTYPE_F32 ? 4 : 2;
    bool waited = rsm == nullptr;
    for (int task = cta + warp * G; task < tasks; task += G * R) {
      const int t = task / p.E, e = task % p.E;
      const uint16_t* xr = p.x + (int64_t)t * p.H;
      const bool wf32 = p.router_w_dtype == B2_DTYPE_F32;
      const uint8_t* wbase = rsm ? rsm + (size_t)((task - cta) / G) * p.H * wsz
                                 : static_cast<const uint8_t*>(p.router_w) + (size_t)e * p.H * wsz;
      float a = 0.0f;
      const int chunks = p.H / 4;
      // The x chunks of each 8-chunk group are loaded one group ahead (the
      // first group before the wait for the router rows), so the x loads
      // overlap the weight fetch; the FMA order is unchanged.
      uint2 xn[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (lane + 32 * u < chunks) xn[u] = __ldg(reinterpret_cast<const uint2*>(xr + 4 * (lane + 32 * u)));
      if (!waited) {
        mbar_wait_bounded(rbar, 0u, p.status);
        waited = true;
      }
      for (int base = lane; base < chunks; base += 32 * 8) {
        float4 w4[8];
        uint2 xv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) xv[u] = xn[u];
        if (base + 32 * 8 < chunks) {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c4 = base + 32 * 8 + 32 * u;
            if (c4 < chunks) xn[u] = __ldg(reinterpret_cast<const uint2*>(xr + 4 * c4));
          }
        }
        if (wf32) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (base + 32 * u < chunks) w4[u] = *reinterpret_cast<const float4*>(wbase + 16 * (size_t)(base + 32 * u));
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (base + 32 * u < chunks) {
              const uint2 wv = *reinterpret_cast<const uint2*>(wbase + 8 * (size_t)(base + 32 * u));
              w4[u] = make_float4(__uint_as_float(wv.x << 16), __uint_as_float(wv.x & 0xffff0000u),
                                  __uint_as_float(wv.y << 16), __uint_as_float(wv.y & 0xffff0000u));
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
      // a bf16 router weight gives bf16 logits (MLX's x.matmul(w.T) result
      // type, Laguna.swift:166 / RM:833-838); an f32 weight keeps the f32 sum
      if (!wf32) a = round_bf16(a);
      if (lane == 0 && cta != p.skip_logit_cta)
        st_relaxed_u64(p.logit_words + (int64_t)t * p.E + e,
                       ((unsigned long long)(ep + 1u) << 32) | __float_as_uint(a));
    }
  }
  if (tid == 0) *s_ep = ep;
  // warps beyond kWarps (a control warp) take no part in the staging
  if (R < kWarps) {
    if (warp >= R && warp < kWarps)
      stage_rows(p.x, p.T, p.H, xs, xstride, s_xexp, s_red, tid - R * 32, (kWarps - R) * 32, 1);
  } else if (warp < kWarps) {
    stage_rows(p.x, p.T, p.H, xs, xstride, s_xexp, s_red, tid, kThreads, 1);
  }

  // ---------------- top-k (every CTA, redundantly)
  __syncthreads();
  const uint32_t epoch = *s_ep;
  if (tid == 0) {
    p.counters[kEpochs + cta] = epoch + 1u;
    if (cta == 0)
      for (int t = 0; t < 8; ++t) p.counters[kActCnt + 8 * ((epoch & 1u) ^ 1u) + t] = 0u;
  }
  {
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(scratch);
    float* vals = reinterpret_cast<float*>(keys + p.E);
    unsigned* rank = reinterpret_cast<unsigned*>(vals + p.E);
    topk_ranked(p, epoch + 1u, s_ok, s_inds, s_wts, keys, vals, rank);
  }
  if (cta == 0)
    for (int i = tid; i < p.T * p.k; i += blockDim.x) {
      p.inds_out[i] = s_inds[i];
      p.wts_out[i] = s_wts[i];
    }
  return epoch;
}

}  // namespace dec
}  // namespace b2
