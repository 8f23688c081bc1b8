// Fused decode MoE block over the prepared decode bank.
//
// The prepared bank stores every expert tile the decode kernel reads as one
// contiguous block, so each tile arrives with a single TMA bulk copy (the TMA
// engine moves it; no load instructions on the SMs):
//   gate/up tile (expert e, 8-feature block f): 16 rows = gate rows 8f..8f+7
//     then up rows 8f..8f+7, codes [16][H/2] followed by scales [H/16][8][2]
//     (the scale bytes of rows p and p+8 adjacent), 9*H bytes;
//   down tile (expert e, 16-row block b): rows 16b..16b+15 of the down bank,
//     codes [16][F/2] then scales [F/16][8][2], 9*F bytes.
// Within each code row the 16-byte chunks are XOR-swizzled by (row & 7), so
// the eight rows a warp reads at one K offset fall in different banks.  The
// bank has exactly the bytes of the three MLX-layout banks (no padding).
//
// Kernel: phase 1 (router, top-k) as in moe_decode.cu; phase 2 prefetches
// every tile this CTA owns -- its gate/up tiles and its down items (token t,
// 16 hidden rows: the k slot experts' down tiles) -- into two smem rings with
// one bulk copy per tile, then computes them as they land.  All 16 warps
// split each gate/up tile's K range; for a down item warp w takes slot tile
// w % 8 and half of its K groups.  The last warp to finish a tile runs the
// epilogue (SwiGLU, or the slot-ordered weighted combine) and refills the
// slot.
#include <algorithm>

#include "moe_decode.cuh"
#include "moe_decode_common.cuh"
#include "moe_prefill.cuh"

namespace b2 {
namespace dec {
namespace {

constexpr int kMaxRing = 16;

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return (uint32_t)(chunk ^ (row & 7)); }

// ---------------------------------------------------------------- prepare
// One CTA per prepared tile.  tile < n_gu_tiles: gate/up tile (e, f);
// otherwise down tile (e, b).
__global__ void prepare_kernel(const uint8_t* __restrict__ gcodes, const uint8_t* __restrict__ gscales,
                               const uint8_t* __restrict__ ucodes, const uint8_t* __restrict__ uscales,
                               const uint8_t* __restrict__ dcodes, const uint8_t* __restrict__ dscales, int E, int H,
                               int F, uint8_t* __restrict__ bank) {
  const int64_t n_gu_tiles = (int64_t)E * (F / 8);
  const int64_t tile = blockIdx.x;
  const bool gu = tile < n_gu_tiles;
  const int K = gu ? H : F;
  const int64_t tile_bytes = 9 * (int64_t)K;
  uint8_t* dst = bank + (gu ? tile * tile_bytes : n_gu_tiles * 9 * (int64_t)H + (tile - n_gu_tiles) * tile_bytes);
  int64_t row_of[16];
  const uint8_t* cbase[16];
  const uint8_t* sbase[16];
  for (int r = 0; r < 16; ++r) {
    if (gu) {
      const int64_t e = tile / (F / 8), f = tile % (F / 8);
      row_of[r] = e * F + f * 8 + (r & 7);
      cbase[r] = (r < 8 ? gcodes : ucodes) + row_of[r] * (K / 2);
      sbase[r] = (r < 8 ? gscales : uscales) + row_of[r] * (K / 16);
    } else {
      const int64_t t2 = tile - n_gu_tiles;
      const int64_t e = t2 / (H / 16), b = t2 % (H / 16);
      row_of[r] = e * H + b * 16 + r;
      cbase[r] = dcodes + row_of[r] * (K / 2);
      sbase[r] = dscales + row_of[r] * (K / 16);
    }
  }
  const int chunks = K / 32;  // 16-byte chunks per code row
  for (int i = threadIdx.x; i < 16 * chunks; i += blockDim.x) {
    const int r = i / chunks, c = i % chunks;
    const uint4 v = *reinterpret_cast<const uint4*>(cbase[r] + 16 * c);
    *reinterpret_cast<uint4*>(dst + (size_t)r * (K / 2) + 16 * swz(r, c)) = v;
  }
  uint8_t* sd = dst + 16 * (K / 2);
  const int groups = K / 16;
  for (int i = threadIdx.x; i < groups * 16; i += blockDim.x) {
    const int g = i / 16, j = i % 16;  // j = 2*pair + half
    const int r = (j >> 1) + 8 * (j & 1);
    sd[i] = sbase[r][g];
  }
}

// ---------------------------------------------------------------- kernel
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Issue (one thread) the copies of gate/up item `it` into a gate/up slot.
// Expert ids were range-checked by phase 1; the guards below keep a corrupt
// id from ever becoming a copy source (it is recorded and expert 0 is read).
__device__ __forceinline__ uint32_t checked_expert(const Params& p, uint32_t e) {
  if (e >= (uint32_t)p.E) {
    report_status(p.status, B2_STATUS_BAD_INDEX);
    return 0u;
  }
  return e;
}

__device__ __forceinline__ void issue_gu(const Params& p, const uint32_t* inds, int it, uint8_t* slot, uint64_t* bar) {
  const int fb = p.F / 8;
  const int pair = it / fb, f = it % fb;
  const uint32_t bytes = 9u * (uint32_t)p.H;
  const uint8_t* src = p.bank_gu + ((uint64_t)checked_expert(p, inds[pair]) * fb + f) * bytes;
  mbar_expect_tx(bar, bytes);
  bulk_copy(slot, src, bytes, bar);
}

// Issue (one thread) the k tile copies of down item `it` (token t, block b).
__device__ __forceinline__ void issue_dn(const Params& p, const uint32_t* inds, int it, uint8_t* slot, uint64_t* bar) {
  const int hb = p.H / 16;
  const int t = it / hb, b = it % hb;
  const uint32_t bytes = 9u * (uint32_t)p.F;
  mbar_expect_tx(bar, bytes * (uint32_t)p.k);
  for (int s = 0; s < p.k; ++s) {
    const uint8_t* src = p.bank_dn + ((uint64_t)checked_expert(p, inds[t * p.k + s]) * hb + b) * bytes;
    bulk_copy(slot + (size_t)s * bytes, src, bytes, bar);
  }
}

// One 16-row prepared tile, groups grp0, grp0 + gstep, ...; B columns from
// staged rows xs (only rows < xcols are non-zero).  Accumulates D(16x8).
// Groups are processed 8 at a time: all their shared-memory loads are issued
// first and the MMAs alternate between two accumulators, so a warp has
// independent work in flight instead of one serial load->decode->mma chain.
__device__ __forceinline__ void tile_mma_prep(const uint8_t* tile, int K, int grp0, int gstep, const __half* xs,
                                              int xstride, int xcols, float acc[4]) {
  const int lane = threadIdx.x & 31;
  const int gi = lane >> 2, c = lane & 3;
  const int groups = K / 16;
  const int row_bytes = K / 2;
  const uint8_t* row0 = tile + (size_t)gi * row_bytes;
  const uint8_t* row8 = tile + (size_t)(gi + 8) * row_bytes;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(tile + 16 * (size_t)row_bytes) + gi;
  const uint32_t sel = (uint32_t)c | ((uint32_t)(4 + c) << 4);
  const bool bcol = gi < xcols;
  const __half* xr = xs + (size_t)gi * xstride + 2 * c;
  float acc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int base = grp0; base < groups; base += 8 * gstep) {
    uint2 w0[8], w8[8];
    uint32_t sb[8], b0[8], b1[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int grp = base + u * gstep;
      if (grp < groups) {
        const uint32_t off = (swz(gi, grp >> 1) << 4) + ((grp & 1) << 3);
        w0[u] = *reinterpret_cast<const uint2*>(row0 + off);
        w8[u] = *reinterpret_cast<const uint2*>(row8 + off);
        sb[u] = sc[grp * 8];
        b0[u] = bcol ? *reinterpret_cast<const uint32_t*>(xr + grp * 16) : 0u;
        b1[u] = bcol ? *reinterpret_cast<const uint32_t*>(xr + grp * 16 + 8) : 0u;
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int grp = base + u * gstep;
      if (grp < groups) {
        const uint32_t p0 = prmt(w0[u].x, w0[u].y, sel);
        const uint32_t p8 = prmt(w8[u].x, w8[u].y, sel);
        const uint32_t sp = scale_pair(sb[u] & 0xffu, sb[u] >> 8);
        const __half2 s2 = *reinterpret_cast<const __half2*>(&sp);
        const __half2 slo = __low2half2(s2), shi = __high2half2(s2);
        uint32_t a[4];
        a[0] = hmul2_u32(cvt_byte0(p0), *reinterpret_cast<const uint32_t*>(&slo));
        a[2] = hmul2_u32(cvt_byte1(p0), *reinterpret_cast<const uint32_t*>(&slo));
        a[1] = hmul2_u32(cvt_byte0(p8), *reinterpret_cast<const uint32_t*>(&shi));
        a[3] = hmul2_u32(cvt_byte1(p8), *reinterpret_cast<const uint32_t*>(&shi));
        float* d = (u & 1) ? acc1 : acc;
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0[u]), "r"(b1[u]));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] += acc1[j];
}

// Bounded spin until *cnt reaches `target` (one lane).
__device__ __forceinline__ void spin_smem(const unsigned* cnt, unsigned target, unsigned* status) {
  uint32_t i = 0;
  while (*reinterpret_cast<const volatile unsigned*>(cnt) < target)
    if (++i >= kSpinLimit) {
      report_status(status, B2_STATUS_WAIT_TIMEOUT);
      break;
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_block_tma_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t gbar[kMaxRing], dbar[kMaxRing];
  __shared__ unsigned gcnt[kMaxRing], dcnt[kMaxRing];
  __shared__ uint32_t s_inds[64];
  __shared__ float s_wts[64];
  __shared__ int s_xexp[8];
  __shared__ int s_aexp[8];
  __shared__ unsigned s_red[32];
  __shared__ unsigned s_tokdone[8];
  __shared__ int s_ok;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int ngs = p.n_slots, nds = p.n_dn_slots;
  const uint32_t gbytes = 9u * (uint32_t)p.H, dbytes = 9u * (uint32_t)p.F * (uint32_t)p.k;

  // carve: [x T x (H+8)] [a 8 x (F+8)] [partials: gate/up slots, down slots] [gate/up ring] [down ring]
  const int xstride = p.H + 8, astride = p.F + 8;
  __half* xs = reinterpret_cast<__half*>(smem);
  size_t off = ((size_t)p.T * xstride * 2 + 15) & ~size_t(15);
  __half* as = reinterpret_cast<__half*>(smem + off);
  off += ((size_t)8 * astride * 2 + 15) & ~size_t(15);
  float* gred = reinterpret_cast<float*>(smem + off);  // [ngs][kWarps][16]
  off += (size_t)ngs * kWarps * 16 * 4;
  float* dred = reinterpret_cast<float*>(smem + off);  // [nds][kWarps][16]
  off += (size_t)nds * kWarps * 16 * 4;
  off = (off + 127) & ~size_t(127);
  uint8_t* gring = smem + off;
  off += (size_t)ngs * gbytes;
  off = (off + 127) & ~size_t(127);
  uint8_t* dring = smem + off;

  if (tid == 0) {
    for (int i = 0; i < ngs; ++i) mbar_init(&gbar[i], 1);
    for (int i = 0; i < nds; ++i) mbar_init(&dbar[i], 1);
    fence_mbar_init();
    s_ok = 1;
  }
  if (tid < kMaxRing) {
    gcnt[tid] = 0u;
    dcnt[tid] = 0u;
  }
  if (tid < 8) s_tokdone[tid] = 0u;
  __syncthreads();

  phase1(p, xs, xstride, s_xexp, s_red, s_inds, s_wts, &s_ok, gring);  // the ring is unused until phase 2
  __syncthreads();

  // ---------------- phase 2
  const int n_dn = p.n_items - p.n_gu;
  const int gu_lo = (int)((int64_t)cta * p.n_gu / G), gu_hi = (int)((int64_t)(cta + 1) * p.n_gu / G);
  const int dn_lo = (int)((int64_t)cta * n_dn / G), dn_hi = (int)((int64_t)(cta + 1) * n_dn / G);
  const int my_gu = gu_hi - gu_lo, my_dn = dn_hi - dn_lo;
  if (tid == 0 && s_ok) {
    for (int q = 0; q < min(ngs, my_gu); ++q) issue_gu(p, s_inds, gu_lo + q, gring + (size_t)q * gbytes, &gbar[q]);
    for (int q = 0; q < min(nds, my_dn); ++q) issue_dn(p, s_inds, dn_lo + q, dring + (size_t)q * dbytes, &dbar[q]);
  }

  // gate/up tiles
  for (int q = 0; q < my_gu && s_ok; ++q) {
    const int it = gu_lo + q, sl = q % ngs;
    uint8_t* slot = gring + (size_t)sl * gbytes;
    mbar_wait_bounded(&gbar[sl], (uint32_t)((q / ngs) & 1), p.status);
    const int tok = (it / (p.F / 8)) / p.k;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    tile_mma_prep(slot, p.H, warp, kWarps, xs, xstride, p.T, acc);
    const int gi = lane >> 2, c = lane & 3;
    float* rp = gred + ((size_t)sl * kWarps + warp) * 16;
    if (c == (tok >> 1)) {
      rp[gi] = (tok & 1) ? acc[1] : acc[0];
      rp[gi + 8] = (tok & 1) ? acc[3] : acc[2];
    }
    __syncwarp();
    const unsigned use_done = (unsigned)kWarps * (unsigned)(q / ngs + 1);
    unsigned arrived = 0;
    if (lane == 0) {
      __threadfence_block();
      arrived = atomicAdd(&gcnt[sl], 1u);
    }
    arrived = __shfl_sync(0xffffffffu, arrived, 0);
    if (arrived == use_done - 1) {
      __threadfence_block();
      float v = 0.0f;
      if (lane < 16) {
        const float* rs = gred + (size_t)sl * kWarps * 16 + lane;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += rs[w * 16];
      }
      const float up = __shfl_down_sync(0xffffffffu, v, 8);
      if (lane < 8) {
        const int fb = p.F / 8;
        const int pair = it / fb, f0 = (it % fb) * 8;
        const float gv = round_bf16(ldexpf(v, s_xexp[tok]));
        const float uv = round_bf16(ldexpf(up, s_xexp[tok]));
        p.act[(int64_t)pair * p.F + f0 + lane] = f32_to_bf16_bits(swiglu_bf16(gv, uv));
      }
      if (lane == 0) {
        atomicAdd(&s_tokdone[tok], 1u);
        if (q + ngs < my_gu) issue_gu(p, s_inds, it + ngs, slot, &gbar[sl]);
      }
    }
  }

  // down items (token-major): transition per token
  int staged_tok = -1;
  bool released = false;
  for (int q = 0; q < my_dn; ++q) {
    const int it = dn_lo + q, sl = q % nds;
    uint8_t* slot = dring + (size_t)sl * dbytes;
    const int hb = p.H / 16;
    const int t = it / hb, b = it % hb;
    if (t != staged_tok) {
      __syncthreads();
      if (tid == 0) {
        if (!released) release_tokens(p, s_tokdone);
        uint32_t i = 0;
        while (s_ok && ld_acquire(&p.counters[8 + t]) < (unsigned)(p.k * (p.F / 8))) {
          if (++i >= kSpinLimit) {
            report_status(p.status, B2_STATUS_WAIT_TIMEOUT);
            s_ok = 0;
          }
        }
      }
      released = true;
      __syncthreads();
      if (!s_ok) break;
      stage_rows(p.act + (int64_t)t * p.k * p.F, p.k, p.F, as, astride, s_aexp, s_red, tid, kThreads, 1);
      staged_tok = t;
    }
    mbar_wait_bounded(&dbar[sl], (uint32_t)((q / nds) & 1), p.status);
    const int s = warp & 7, half = warp >> 3;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (s < p.k)
      tile_mma_prep(slot + (size_t)s * 9 * p.F, p.F, half, 2, as + (size_t)s * astride, astride, 1, acc);
    const int gi = lane >> 2, c = lane & 3;
    float* rp = dred + ((size_t)sl * kWarps + warp) * 16;
    if (c == 0) {
      rp[gi] = acc[0];
      rp[gi + 8] = acc[2];
    }
    __syncwarp();
    const unsigned use_done = (unsigned)kWarps * (unsigned)(q / nds + 1);
    unsigned arrived = 0;
    if (lane == 0) {
      __threadfence_block();
      arrived = atomicAdd(&dcnt[sl], 1u);
    }
    arrived = __shfl_sync(0xffffffffu, arrived, 0);
    if (arrived == use_done - 1) {
      __threadfence_block();
      if (lane < 16) {
        const float* rs = dred + (size_t)sl * kWarps * 16 + lane;
        float tot = 0.0f;
        for (int qq = 0; qq < p.k; ++qq) {
          const float dv = rs[qq * 16] + rs[(qq + 8) * 16];
          const float dr = round_bf16(ldexpf(dv, s_aexp[qq]));
          const float rw = round_bf16(s_wts[t * p.k + qq]);
          tot = round_bf16(__fadd_rn(round_bf16(__fmul_rn(dr, rw)), tot));
        }
        if (p.routed_scale != 1.0f) tot = round_bf16(__fmul_rn(tot, round_bf16(p.routed_scale)));
        const int64_t o = (int64_t)t * p.H + b * 16 + lane;
        if (p.residual) tot = round_bf16(__fadd_rn(tot, bf16_bits_to_f32(p.residual[o])));
        p.out[o] = f32_to_bf16_bits(tot);
      }
      if (lane == 0 && q + nds < my_dn) issue_dn(p, s_inds, it + nds, slot, &dbar[sl]);
    }
  }

  __syncthreads();
  if (tid == 0 && !released) release_tokens(p, s_tokdone);
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned done = atomicAdd(&p.counters[1], 1u);
    if (done == (unsigned)G - 1) {
      p.counters[0] = 0u;
      for (int t = 0; t < p.T; ++t) p.counters[8 + t] = 0u;
      __threadfence();
      p.counters[1] = 0u;
    }
  }
}

}  // namespace

size_t bank_bytes(const b2_moe_block* blk) {
  return (size_t)blk->n_experts * (size_t)(blk->ffn / 8) * 9 * (size_t)blk->hidden +
         (size_t)blk->n_experts * (size_t)(blk->hidden / 16) * 9 * (size_t)blk->ffn;
}

int prepare(const b2_moe_block* blk, void* dst, cudaStream_t st) {
  const int64_t tiles = blk->n_experts * (blk->ffn / 8) + blk->n_experts * (blk->hidden / 16);
  B2_REQUIRE(tiles <= INT32_MAX, "[prepare_decode_bank] too many tiles");
  prepare_kernel<<<(unsigned)tiles, 256, 0, st>>>(
      reinterpret_cast<const uint8_t*>(blk->gate_codes), blk->gate_scales,
      reinterpret_cast<const uint8_t*>(blk->up_codes), blk->up_scales,
      reinterpret_cast<const uint8_t*>(blk->down_codes), blk->down_scales, (int)blk->n_experts, (int)blk->hidden,
      (int)blk->ffn, static_cast<uint8_t*>(dst));
  B2_CHECK_LAUNCH("prepare_decode_bank");
  return B2_OK;
}

int launch_tma(Params& p, const b2_moe_block* blk, cudaStream_t st) {
  int dev = 0, sms = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa;
  int rc = check_cuda(cudaFuncGetAttributes(&fa, decode_block_tma_kernel), "moe_block");
  if (rc) return rc;
  const size_t avail = (size_t)optin - fa.sharedSizeBytes;
  // this kernel's down items are (token, 16 hidden rows)
  p.n_items = p.n_gu + p.T * (p.H / 16);
  const uint8_t* bank = static_cast<const uint8_t*>(blk->decode_bank);
  p.bank_gu = bank;
  p.bank_dn = bank + (size_t)p.E * (size_t)(p.F / 8) * 9 * (size_t)p.H;
  const int n_dn = p.n_items - p.n_gu;
  const int gu_max = (p.n_gu + sms - 1) / sms, dn_max = (n_dn + sms - 1) / sms;
  size_t fixed = ((size_t)p.T * (p.H + 8) * 2 + 15) & ~size_t(15);
  fixed += ((size_t)8 * (p.F + 8) * 2 + 15) & ~size_t(15);
  fixed += 256;  // alignment slack of the two rings
  const size_t gslot = 9 * (size_t)p.H + kWarps * 16 * 4;
  const size_t dslot = 9 * (size_t)p.F * p.k + kWarps * 16 * 4;
  B2_REQUIRE(avail > fixed + gslot + dslot, "[moe_block] hidden/ffn too large for the prepared decode kernel");
  p.n_dn_slots = (int)std::min<size_t>({(size_t)std::max(dn_max, 1), (size_t)2, (avail - fixed - gslot) / dslot});
  p.n_slots = (int)std::min<size_t>({(size_t)std::max(gu_max, 1), (size_t)kMaxRing,
                                     (avail - fixed - p.n_dn_slots * dslot) / gslot});
  // the gate/up ring doubles as the top-k ranking scratch (16 bytes per expert)
  B2_REQUIRE((size_t)p.n_slots * 9 * p.H >= (size_t)16 * p.E, "[moe_block] too many experts for the decode kernel");
  const size_t smem = fixed + p.n_slots * gslot + p.n_dn_slots * dslot;
  rc = ensure_dynamic_smem((const void*)decode_block_tma_kernel, smem, "moe_block");
  if (rc) return rc;
  void* args[] = {&p};
  return check_cuda(
      cudaLaunchCooperativeKernel((const void*)decode_block_tma_kernel, dim3(sms), dim3(kThreads), args, smem, st),
      "moe_block decode (prepared bank)");
}

}  // namespace dec
}  // namespace b2

extern "C" size_t b2_moe_decode_bank_size(const b2_moe_block* blk) {
  if (!blk || blk->n_experts <= 0 || blk->hidden <= 0 || blk->ffn <= 0) return 0;
  return b2::dec::bank_bytes(blk);
}

extern "C" int b2_moe_prepare_decode_bank(const b2_moe_block* blk, void* bank, size_t bank_bytes,
                                          b2_stream_t stream) {
  int rc = b2::validate_block(blk, "prepare_decode_bank");
  if (rc) return rc;
  B2_REQUIRE(bank != nullptr, "[prepare_decode_bank] destination is NULL");
  B2_REQUIRE(bank_bytes >= b2::dec::bank_bytes(blk), "[prepare_decode_bank] destination too small (%zu < %zu)",
             bank_bytes, b2::dec::bank_bytes(blk));
  B2_REQUIRE(reinterpret_cast<uintptr_t>(bank) % 16 == 0, "[prepare_decode_bank] destination must be 16-byte aligned");
  return b2::dec::prepare(blk, bank, reinterpret_cast<cudaStream_t>(stream));
}
