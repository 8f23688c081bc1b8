// Fused decode MoE block over the prepared decode bank.
//
// The prepared bank stores every expert tile the decode kernel reads as one
// contiguous block, so each tile arrives with a single TMA bulk copy:
//   gate/up tile (expert e, 8-feature block f): 16 rows = gate rows 8f..8f+7
//     then up rows 8f..8f+7 over K = H, 9*H bytes;
//   down tile (expert e, 16-row block b): rows 16b..16b+15 of the down bank
//     over K = F, 9*F bytes.
// A tile is consumed by `nsplit` warps (16 for gate/up, 2 for down); warp w
// takes the 32-element K blocks w, w + nsplit, w + 2*nsplit, ... (NB blocks).
// Layout of a tile, codes then scales:
//   codes  [w][NB/2][lane][16 bytes]: lane (gi, c) = (lane/4, lane%4) of an
//          m16n8k16 A fragment gets the code bytes of two blocks with one
//          16-byte load; per block and 16-element group one word whose bytes
//          hold the pairs (row gi, k 2c..2c+1), (row gi+8, k 2c..2c+1),
//          (row gi, k 2c+8..2c+9), (row gi+8, k 2c+8..2c+9) -- the four A
//          registers of that group;
//   scales [w][gi][NB][4 bytes]: per block the bytes of (row gi: group 0,
//          group 1; row gi+8: group 0, group 1), each the f16 bit pattern of
//          the decoded |scale| shifted right by 7 (exact: a decoded E4M3
//          scale has at most 4 significant bits), so two scales become an
//          f16x2 with one mask and one shift.  A negative scale byte is stored
//          as its magnitude and the sign bits of its 16 codes are flipped
//          instead ((-s) * q == s * (-q) exactly, signed zeros included).
// The bank has the same size as the three MLX-layout banks together.
//
// Kernel: phase 1 (router, top-k) as in moe_decode.cu; right after the top-k
// every warp issues pieces of the CTA's gate/up and down tiles into two rings
// of smem slots; the gate/up tiles are computed as they land; the CTA's down
// items (token t, 16 hidden rows: the k slot experts' down tiles) follow once
// every CTA's activations of token t are complete.  Two control warps run the
// epilogues (SwiGLU, or the slot-ordered weighted combine) and refill slots
// when a CTA has more tiles than slots.
#include <algorithm>
#include <cstdlib>

#include "moe_decode.cuh"
#include "moe_decode_common.cuh"
#include "moe_prefill.cuh"

namespace b2 {
namespace dec {
namespace {

constexpr int kMaxRing = 16;
// 16 compute warps + 2 control warps
constexpr int kCtlWarps = 2;
constexpr int kTmaThreads = kThreads + 32 * kCtlWarps;
// The first copies of a CTA's tiles are issued in pieces by the lanes of the
// control warps (a thread that issues bulk copies back to back stalls on each
// issue under load, so few issuing threads cap an SM far below its share of
// HBM): a gate/up tile in kGuPieces pieces, each expert's down tile in
// kDnPieces.
constexpr int kGuPieces = 8;
constexpr int kDnPieces = 2;

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
  const int nsplit = gu ? kWarps : 2;
  const int NB = K / 32 / nsplit;
  const int64_t tile_bytes = 9 * (int64_t)K;
  uint8_t* dst = bank + (gu ? tile * tile_bytes : n_gu_tiles * 9 * (int64_t)H + (tile - n_gu_tiles) * tile_bytes);
  __shared__ const uint8_t* cbase[16];
  __shared__ const uint8_t* sbase[16];
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    int64_t row;
    if (gu) {
      const int64_t e = tile / (F / 8), f = tile % (F / 8);
      row = e * F + f * 8 + (r & 7);
      cbase[r] = (r < 8 ? gcodes : ucodes) + row * (K / 2);
      sbase[r] = (r < 8 ? gscales : uscales) + row * (K / 16);
    } else {
      const int64_t e = (tile - n_gu_tiles) / (H / 16), b = (tile - n_gu_tiles) % (H / 16);
      row = e * H + b * 16 + r;
      cbase[r] = dcodes + row * (K / 2);
      sbase[r] = dscales + row * (K / 16);
    }
  }
  __syncthreads();
  // codes: one output word per (w, block u, group g, lane)
  const int words = 2 * K;  // 8K bytes / 4
  for (int i = threadIdx.x; i < words; i += blockDim.x) {
    const int w = i / (NB * 64), rem = i % (NB * 64);
    const int j = rem / 128, lane = (rem / 4) % 32, ub = (rem / 2) % 2, g = rem % 2;
    const int kb = w + nsplit * (2 * j + ub);
    const int gi = lane >> 2, c = lane & 3;
    const int k0 = kb * 32 + g * 16;
    uint32_t o = 0u;
#pragma unroll
    for (int bi = 0; bi < 4; ++bi) {
      const int r = gi + 8 * (bi & 1);
      const int kk = k0 + 2 * c + 8 * (bi >> 1);
      uint32_t byte = cbase[r][kk / 2];
      if (sbase[r][k0 / 16] & 0x80u) byte ^= 0x88u;
      o |= byte << (8 * bi);
    }
    reinterpret_cast<uint32_t*>(dst)[i] = o;
  }
  // scales: one output byte per (w, gi, block u, bi)
  uint8_t* sd = dst + 8 * (size_t)K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    const int w = i / (32 * NB), gi = (i / (4 * NB)) % 8, u = (i / 4) % NB, bi = i % 4;
    const int r = gi + 8 * (bi >> 1), g = bi & 1;
    const int kb = w + nsplit * u;
    sd[i] = prepared_scale_byte(sbase[r][kb * 2 + g]);
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

// Issue piece `j` (of `np`) of the copy of `bytes` bytes from src to dst.
__device__ __forceinline__ void issue_piece(uint8_t* dst, const uint8_t* src, uint32_t bytes, int j, int np,
                                            uint64_t* bar) {
  const uint32_t pb = bytes / (uint32_t)np;
  bulk_copy(dst + (size_t)j * pb, src + (size_t)j * pb, pb, bar);
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

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 16-element group: code word `cw` (four A-register byte pairs), scale
// pair `sp` (f16 row gi | row gi+8) -> the A fragment in f16 (exact products)
// and one mma into d.
__device__ __forceinline__ void group_mma(uint32_t cw, uint32_t sp, uint32_t b0, uint32_t b1, float (&d)[4]) {
  const __half2 s2 = *reinterpret_cast<const __half2*>(&sp);
  const __half2 slo = __low2half2(s2), shi = __high2half2(s2);
  const uint32_t lo = *reinterpret_cast<const uint32_t*>(&slo), hi = *reinterpret_cast<const uint32_t*>(&shi);
  mma16816(d, hmul2_u32(cvt_byte<0>(cw), lo), hmul2_u32(cvt_byte<1>(cw), hi), hmul2_u32(cvt_byte<2>(cw), lo),
           hmul2_u32(cvt_byte<3>(cw), hi), b0, b1);
}

// Scale word of one block -> f16x2 pairs (row gi, row gi+8) of groups 0, 1.
__device__ __forceinline__ uint32_t scale_g0(uint32_t sw) { return (sw & 0x00ff00ffu) << 7; }
__device__ __forceinline__ uint32_t scale_g1(uint32_t sw) { return (sw >> 1) & 0x7f807f80u; }

// B fragments (x columns = tokens gi < xcols, zero elsewhere) of the NB gate/up
// blocks of warp w; loaded once and reused for every gate/up tile.
template <int NB>
__device__ __forceinline__ void load_xfrag(const __half* xs, int xstride, int xcols, int w,
                                           uint32_t (&xb)[NB][2][2]) {
  const int lane = threadIdx.x & 31, gi = lane >> 2, c = lane & 3;
  const bool on = gi < xcols;
  const __half* xr = xs + (size_t)gi * xstride + 2 * c;
#pragma unroll
  for (int u = 0; u < NB; ++u)
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int k0 = (w + kWarps * u) * 32 + 16 * g;
      xb[u][g][0] = on ? *reinterpret_cast<const uint32_t*>(xr + k0) : 0u;
      xb[u][g][1] = on ? *reinterpret_cast<const uint32_t*>(xr + k0 + 8) : 0u;
    }
}

// Warp w's share (NB blocks) of a prepared gate/up tile: D(16x8) += A * X.
template <int NB>
__device__ __forceinline__ void gu_tile_mma(const uint8_t* tile, int K, int w, const uint32_t (&xb)[NB][2][2],
                                            float acc[4]) {
  const int lane = threadIdx.x & 31, gi = lane >> 2;
  const uint4* cp = reinterpret_cast<const uint4*>(tile + (size_t)w * NB * 256) + lane;
  const uint32_t* sp = reinterpret_cast<const uint32_t*>(tile + 8 * (size_t)K) + ((size_t)w * 8 + gi) * NB;
  uint4 cv[NB / 2];
  uint32_t sv[NB];
#pragma unroll
  for (int j = 0; j < NB / 2; ++j) cv[j] = cp[j * 32];
#pragma unroll
  for (int u = 0; u < NB; u += 2) {
    const uint2 t = *reinterpret_cast<const uint2*>(sp + u);
    sv[u] = t.x;
    sv[u + 1] = t.y;
  }
  float d[2][2][4] = {};
#pragma unroll
  for (int u = 0; u < NB; ++u) {
    const uint4 v = cv[u / 2];
    group_mma((u & 1) ? v.z : v.x, scale_g0(sv[u]), xb[u][0][0], xb[u][0][1], d[u & 1][0]);
    group_mma((u & 1) ? v.w : v.y, scale_g1(sv[u]), xb[u][1][0], xb[u][1][1], d[u & 1][1]);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] += (d[0][0][j] + d[0][1][j]) + (d[1][0][j] + d[1][1][j]);
}

// Warp w's share (of 2) of a prepared down tile against one staged
// activation row xrow (column 0; the other columns are zero).
__device__ __forceinline__ void dn_tile_mma(const uint8_t* tile, int K, int w, const __half* xrow, float acc[4]) {
  const int NB = K / 64;
  const int lane = threadIdx.x & 31, gi = lane >> 2, c = lane & 3;
  const bool on = gi == 0;
  const uint4* cp = reinterpret_cast<const uint4*>(tile + (size_t)w * NB * 256) + lane;
  const uint2* sp = reinterpret_cast<const uint2*>(tile + 8 * (size_t)K + ((size_t)w * 8 + gi) * NB * 4);
  const __half* xr = xrow + 2 * c;
  float d[2][2][4] = {};
#pragma unroll 1
  for (int j = 0; j < NB / 2; ++j) {
    const uint4 v = cp[j * 32];
    const uint2 sv = sp[j];
#pragma unroll
    for (int ub = 0; ub < 2; ++ub) {
      const int k0 = (w + 2 * (2 * j + ub)) * 32;
      const uint32_t sw = ub ? sv.y : sv.x;
      const uint32_t b00 = on ? *reinterpret_cast<const uint32_t*>(xr + k0) : 0u;
      const uint32_t b01 = on ? *reinterpret_cast<const uint32_t*>(xr + k0 + 8) : 0u;
      const uint32_t b10 = on ? *reinterpret_cast<const uint32_t*>(xr + k0 + 16) : 0u;
      const uint32_t b11 = on ? *reinterpret_cast<const uint32_t*>(xr + k0 + 24) : 0u;
      group_mma(ub ? v.z : v.x, scale_g0(sw), b00, b01, d[ub][0]);
      group_mma(ub ? v.w : v.y, scale_g1(sw), b10, b11, d[ub][1]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] += (d[0][0][j] + d[0][1][j]) + (d[1][0][j] + d[1][1][j]);
}

// NBG = H / 512: 32-element K blocks per compute warp of a gate/up tile.
template <int NBG>
__global__ void __launch_bounds__(kTmaThreads, 1) decode_block_tma_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  // gbar/dbar: tile data landed (TMA); gpar/dpar: all compute warps left
  // their partial sums of the slot's tile (kWarps arrivals)
  __shared__ uint64_t gbar[kMaxRing], dbar[kMaxRing], gpar[kMaxRing], dpar[kMaxRing];
  __shared__ uint64_t rbar;  // router rows landed
  __shared__ uint32_t s_inds[64];
  __shared__ float s_wts[64];
  __shared__ int s_xexp[8];
  __shared__ int s_aexp[8];
  __shared__ unsigned s_red[32];
  __shared__ unsigned s_tokdone[8];
  __shared__ int s_ok;
  __shared__ uint32_t s_ep;
  // last item whose copy each ring slot was armed for (-1: none), so a CTA
  // that gives up can wait for its copies in flight before it exits
  __shared__ int s_gu_last[kMaxRing], s_dn_last[kMaxRing];

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
    for (int i = 0; i < ngs; ++i) {
      mbar_init(&gbar[i], 1);
      mbar_init(&gpar[i], kWarps);
    }
    for (int i = 0; i < nds; ++i) {
      mbar_init(&dbar[i], 1);
      mbar_init(&dpar[i], kWarps);
    }
    mbar_init(&rbar, 1);
    fence_mbar_init();
    s_ok = 1;
  }
  if (tid < 8) s_tokdone[tid] = 0u;
  if (tid < kMaxRing) {
    s_gu_last[tid] = -1;
    s_dn_last[tid] = -1;
  }
  __syncthreads();

  // Prologue: only the router rows are read before the dependency wait (they
  // are weights; nothing earlier in the stream writes them).  With
  // programmatic dependent launch this overlaps the previous kernel's tail.
  const int n_tasks = p.logits_in ? 0 : p.T * p.E;
  const int rsm_off = (16 * p.E + 127) & ~127;  // after the top-k scratch
  const bool use_rsm = p.router_smem && n_tasks > 0;
  if (use_rsm && warp == kWarps && lane == 0) {
    const uint32_t rbytes = (uint32_t)p.H * (p.router_w_dtype == B2_DTYPE_F32 ? 4u : 2u);
    const int nt = cta < n_tasks ? (n_tasks - cta + G - 1) / G : 0;
    mbar_expect_tx(&rbar, rbytes * (uint32_t)nt);
    for (int j = 0; j < nt; ++j) {
      const int e = (cta + j * G) % p.E;
      bulk_copy(gring + rsm_off + (size_t)j * rbytes, static_cast<const uint8_t*>(p.router_w) + (size_t)e * rbytes,
                rbytes, &rbar);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // the ring is unused until phase 2 (top-k scratch, then the router rows)
  const uint32_t epoch = phase1(p, xs, xstride, s_xexp, s_red, s_inds, s_wts, &s_ok, &s_ep, gring,
                                use_rsm ? gring + rsm_off : nullptr, &rbar);
  unsigned* act_cnt = p.counters + kActCnt + 8 * (epoch & 1u);

  // this CTA's ranges of gate/up and down items (32-bit products: at most
  // 960 CTAs times T*k*F/8 or T*H/16 items stay far below 2^32)
  const unsigned n_dn = (unsigned)(p.n_items - p.n_gu), n_gu = (unsigned)p.n_gu, ug = (unsigned)G;
  const int gu_lo = (int)(cta * n_gu / ug), gu_hi = (int)((cta + 1) * n_gu / ug);
  const int dn_lo = (int)(cta * n_dn / ug), dn_hi = (int)((cta + 1) * n_dn / ug);
  const int my_gu = gu_hi - gu_lo, my_dn = dn_hi - dn_lo;
  // First fill of both rings, right after the top-k: the down tiles depend
  // only on the selection, so they stream in while the gate/up tiles are
  // computed.  Thread 0 arms the slots' barriers; the lanes of the control
  // warps then issue the pieces (tile-major, so the first tiles land first)
  // while the compute warps go straight to their first tile.  Pieces are
  // 16-byte multiples: 9*H/kGuPieces and 9*F/kDnPieces with H % 512 == 0 and
  // F % 128 == 0.
  const int n_gi = min(ngs, my_gu), n_di = min(nds, my_dn);
  if (tid == 0 && s_ok) {
    for (int q = 0; q < n_gi; ++q) {
      mbar_expect_tx(&gbar[q], gbytes);
      s_gu_last[q] = q;
    }
    for (int q = 0; q < n_di; ++q) {
      mbar_expect_tx(&dbar[q], dbytes);
      s_dn_last[q] = q;
    }
  }
  // the gate/up ring held the top-k scratch and router rows (generic proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  if (warp >= kWarps && s_ok) {
    const int fb = p.F / 8, hb = p.H / 16;
    const uint32_t tb = 9u * (uint32_t)p.F;
    const int gpieces = n_gi * kGuPieces, pieces = gpieces + n_di * p.k * kDnPieces;
#pragma unroll 1
    for (int j = (warp - kWarps) * 32 + lane; j < pieces; j += 32 * kCtlWarps) {
      if (j < gpieces) {
        const int q = j / kGuPieces, it = gu_lo + q, pair = it / fb, f = it % fb;
        const uint8_t* src = p.bank_gu + ((uint64_t)checked_expert(p, s_inds[pair]) * fb + f) * gbytes;
        issue_piece(gring + (size_t)q * gbytes, src, gbytes, j % kGuPieces, kGuPieces, &gbar[q]);
      } else {
        const int jj = j - gpieces, q = jj / (p.k * kDnPieces), s = (jj / kDnPieces) % p.k;
        const int it = dn_lo + q, t = it / hb, b = it % hb;
        const uint8_t* src = p.bank_dn + ((uint64_t)checked_expert(p, s_inds[t * p.k + s]) * hb + b) * tb;
        issue_piece(dring + (size_t)q * dbytes + (size_t)s * tb, src, tb, jj % kDnPieces, kDnPieces, &dbar[q]);
      }
    }
  }

  // ---------------- phase 2
  // Warps [0, kWarps) compute; the kCtlWarps control warps issue the bulk
  // copies and run the tile epilogues (tile q by control warp q % kCtlWarps)
  // once all compute warps have left their partial sums, refill the freed
  // slot and release this CTA's activation counts.  A bulk-copy issue can
  // stall for microseconds under memory back-pressure and an epilogue is a
  // long dependent chain, so neither sits in front of the tile math; two
  // control warps keep the epilogues level with the compute warps.
  const bool ctl = warp >= kWarps;
  const int cw = warp - kWarps;  // control warp index when ctl
  const int gi = lane >> 2, c = lane & 3;

  // gate/up tiles
  if (ctl) {
    const int fb = p.F / 8;
    for (int q = cw; q < my_gu && s_ok; q += kCtlWarps) {
      const int it = gu_lo + q, sl = q % ngs;
      const int pair = it / fb, tok = pair / p.k;
      if (!mbar_wait_bounded(&gpar[sl], (uint32_t)((q / ngs) & 1), p.status)) s_ok = 0;
      // row (lane & 15), warps 8*(lane >> 4) .. +7 as a fixed tree, then the
      // two halves
      float v;
      {
        const float* rs = gred + ((size_t)sl * kWarps + 8 * (lane >> 4)) * 16 + (lane & 15);
        float r[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) r[w] = rs[w * 16];
        v = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
      }
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      const float up = __shfl_down_sync(0xffffffffu, v, 8);
      if (lane < 8) {
        const int f0 = (it % fb) * 8;
        const float gv = round_bf16(mul_pow2(v, s_xexp[tok]));
        const float uv = round_bf16(mul_pow2(up, s_xexp[tok]));
        p.act[(int64_t)pair * p.F + f0 + lane] = f32_to_bf16_bits(swiglu_bf16(gv, uv));
      }
      __syncwarp();
      if (lane == 0) {
        atomicAdd(&s_tokdone[tok], 1u);
        if (q + ngs < my_gu && s_ok) {
          s_gu_last[sl] = q + ngs;
          issue_gu(p, s_inds, it + ngs, gring + (size_t)sl * gbytes, &gbar[sl]);
        }
      }
    }
    // both control warps' epilogues are done (and their smem counts visible)
    asm volatile("bar.sync 2, %0;" ::"r"(32 * kCtlWarps) : "memory");
    if (cw == 0 && lane == 0 && s_ok) release_tokens(p, act_cnt, s_tokdone);
  } else {
    uint32_t xb[NBG][2][2];
    load_xfrag<NBG>(xs, xstride, p.T, warp, xb);
    for (int q = 0; q < my_gu && s_ok; ++q) {
      const int it = gu_lo + q, sl = q % ngs;
      const uint8_t* slot = gring + (size_t)sl * gbytes;
      if (!mbar_wait_bounded(&gbar[sl], (uint32_t)((q / ngs) & 1), p.status)) s_ok = 0;
      const int tok = (it / (p.F / 8)) / p.k;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      gu_tile_mma<NBG>(slot, p.H, warp, xb, acc);
      float* rp = gred + ((size_t)sl * kWarps + warp) * 16;
      if (c == (tok >> 1)) {
        rp[gi] = (tok & 1) ? acc[1] : acc[0];
        rp[gi + 8] = (tok & 1) ? acc[3] : acc[2];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&gpar[sl]);
    }
  }

  // down items (token-major): at each token transition wait for every CTA's
  // activations of that token, then stage them
  int staged_tok = -1;
  for (int q = 0; q < my_dn; ++q) {
    const int it = dn_lo + q, sl = q % nds;
    const int hb = p.H / 16;
    const int t = it / hb, b = it % hb;
    if (t != staged_tok) {
      __syncthreads();
      if (tid == 0) {
        uint32_t i = 0;
        while (s_ok && ld_acquire(&act_cnt[t]) < (unsigned)(p.k * (p.F / 8))) {
          if (++i >= p.spin_limit) {
            report_status(p.status, B2_STATUS_WAIT_TIMEOUT);
            s_ok = 0;
          }
        }
      }
      __syncthreads();
      if (!s_ok) break;
      if (!ctl) stage_rows(p.act + (int64_t)t * p.k * p.F, p.k, p.F, as, astride, s_aexp, s_red, tid, kThreads, 1);
      staged_tok = t;
    }
    if (!ctl) {
      const uint8_t* slot = dring + (size_t)sl * dbytes;
      if (s_ok && !mbar_wait_bounded(&dbar[sl], (uint32_t)((q / nds) & 1), p.status)) s_ok = 0;
      const int s = warp & 7, half = warp >> 3;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (s < p.k) dn_tile_mma(slot + (size_t)s * 9 * p.F, p.F, half, as + (size_t)s * astride, acc);
      float* rp = dred + ((size_t)sl * kWarps + warp) * 16;
      if (c == 0) {
        rp[gi] = acc[0];
        rp[gi + 8] = acc[2];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&dpar[sl]);
    } else if (q % kCtlWarps == cw) {
      if (s_ok && !mbar_wait_bounded(&dpar[sl], (uint32_t)((q / nds) & 1), p.status)) s_ok = 0;
      if (lane < 16) {
        const float* rs = dred + (size_t)sl * kWarps * 16 + lane;
        float tot = 0.0f;
#pragma unroll 1
        for (int qq = 0; qq < p.k; ++qq) {
          const float dv = rs[qq * 16] + rs[(qq + 8) * 16];
          const float dr = round_bf16(mul_pow2(dv, s_aexp[qq]));
          const float rw = round_bf16(s_wts[t * p.k + qq]);
          tot = round_bf16(__fadd_rn(round_bf16(__fmul_rn(dr, rw)), tot));
        }
        if (p.routed_scale != 1.0f) tot = round_bf16(__fmul_rn(tot, round_bf16(p.routed_scale)));
        const int64_t o = (int64_t)t * p.H + b * 16 + lane;
        if (p.shared) tot = round_bf16(__fadd_rn(tot, bf16_bits_to_f32(p.shared[o])));
        if (p.residual) tot = round_bf16(__fadd_rn(tot, bf16_bits_to_f32(p.residual[o])));
        p.out[o] = f32_to_bf16_bits(tot);
      }
      __syncwarp();
      if (lane == 0 && s_ok && q + nds < my_dn) {
        s_dn_last[sl] = q + nds;
        issue_dn(p, s_inds, it + nds, dring + (size_t)sl * dbytes, &dbar[sl]);
      }
    }
  }

  // A CTA that gave up on a wait may still have bulk copies in flight into
  // its shared memory: before it exits, wait (bounded) for the last armed
  // phase of every ring slot and for the router rows.  Copies into a slot
  // complete in order, so the last phase completing means all have landed.
  __syncthreads();
  if (tid == 0 && !s_ok) {
    for (int sl = 0; sl < ngs; ++sl)
      if (s_gu_last[sl] >= 0) mbar_wait_bounded(&gbar[sl], (uint32_t)((s_gu_last[sl] / ngs) & 1), p.status);
    for (int sl = 0; sl < nds; ++sl)
      if (s_dn_last[sl] >= 0) mbar_wait_bounded(&dbar[sl], (uint32_t)((s_dn_last[sl] / nds) & 1), p.status);
    if (use_rsm) mbar_wait_bounded(&rbar, 0u, p.status);
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

// Programmatic dependent launch of the decode kernel (on unless the
// environment sets B2_DECODE_PDL=0).
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("B2_DECODE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int launch_tma(Params& p, const b2_moe_block* blk, cudaStream_t st) {
  int dev = 0, sms = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const void* fn = nullptr;
  switch (p.H / 512) {
    case 2: fn = (const void*)decode_block_tma_kernel<2>; break;
    case 4: fn = (const void*)decode_block_tma_kernel<4>; break;
    case 8: fn = (const void*)decode_block_tma_kernel<8>; break;
    default: break;
  }
  B2_REQUIRE(fn != nullptr && p.H % 512 == 0,
             "[moe_block] the prepared decode kernel supports hidden 1024, 2048 or 4096 (got %d)", p.H);
  B2_REQUIRE(p.F % 128 == 0, "[moe_block] the prepared decode kernel needs ffn %% 128 == 0 (got %d)", p.F);
  B2_REQUIRE(sms <= kMaxCtas, "[moe_block] the decode kernels support at most %d SMs (got %d)", kMaxCtas, sms);
  cudaFuncAttributes fa;
  int rc = check_cuda(cudaFuncGetAttributes(&fa, fn), "moe_block");
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
  {
    // router rows of a CTA's logit tasks in the gate/up ring, after the top-k
    // scratch (copies need 16-byte aligned rows)
    const int tasks = p.logits_in ? 0 : p.T * p.E;
    const size_t per_cta = (size_t)(tasks + sms - 1) / sms;
    const size_t rbytes = (size_t)p.H * (p.router_w_dtype == B2_DTYPE_F32 ? 4 : 2);
    const size_t roff = ((size_t)16 * p.E + 127) & ~size_t(127);
    static const bool rsm_env = [] {
      const char* v = std::getenv("B2_DECODE_ROUTER_SMEM");
      return !(v && v[0] == '0');
    }();
    p.router_smem = rsm_env && (reinterpret_cast<uintptr_t>(p.router_w) % 16 == 0) &&
                    roff + per_cta * rbytes <= (size_t)p.n_slots * 9 * p.H;
  }
  rc = ensure_dynamic_smem(fn, smem, "moe_block");
  if (rc) return rc;
  // Cooperative (every CTA resident: the kernel has grid-wide waits) and
  // programmatic dependent launch (the prologue overlaps the previous
  // kernel in the stream; the kernel waits on it before touching anything
  // but its router weights).  Falls back to a plain cooperative launch where
  // the combination is refused.
  void* args[] = {&p};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess && cfg.numAttrs == 2) {
    (void)cudaGetLastError();
    cfg.numAttrs = 1;
    e = cudaLaunchKernelExC(&cfg, fn, args);
  }
  return check_cuda(e, "moe_block decode (prepared bank)");
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
  B2_REQUIRE(blk->hidden == 1024 || blk->hidden == 2048 || blk->hidden == 4096,
             "[prepare_decode_bank] the prepared decode layout supports hidden 1024, 2048 or 4096 (got %lld)",
             (long long)blk->hidden);
  B2_REQUIRE(blk->ffn % 128 == 0, "[prepare_decode_bank] the prepared decode layout needs ffn %% 128 == 0 (got %lld)",
             (long long)blk->ffn);
  return b2::dec::prepare(blk, bank, reinterpret_cast<cudaStream_t>(stream));
}
