// Fused decode MoE block: ONE cooperative launch per block forward.
//
//   phase 1  router logits (one warp per (token, expert), spread over the
//            CTAs; the other warps stage the tokens as f16 meanwhile) ->
//            grid-wide counter -> every CTA ranks the top-k itself.
//   phase 2  every CTA owns a strided share of the block's 16-row expert
//            tiles:
//              gate/up tile = 8 gate rows + 8 up rows of one (token, slot)
//              expert -> SwiGLU -> act[t, s, 8 features] (global)
//              down tile    = 2 hidden rows of each of the k slot experts of
//              token t (B operand = the k slots' activations) -> weighted
//              combine in slot order -> out[t, 2 features]
//            Tiles stream into a ring of shared-memory slots with 16-byte
//            cp.async copies (one mbarrier per slot, 32 arrivals: the copying
//            warp's lanes); on B200 a CTA keeps ~150 KB in flight, so nearly
//            the whole ~21 MB block is requested at once across the chip.
//            All 16 warps split each tile's K range; each warp writes its
//            partial sums to the slot's reduction area and bumps the slot's
//            arrival counter; the warp that arrives last sums the partials
//            in warp order, runs the epilogue and refills the slot.  No
//            CTA-wide barrier per tile.
//
// Per 16-row tile the tensor cores do the multiply-adds (mma.sync m16n8k16,
// f16 in / f32 accumulate; weights are the 16-row A operand).  Thread (g, c)
// decodes code bytes c and c+4 of rows g and g+8 per 16-element group with one
// byte-permute and the hardware E2M1->f16 conversion and scales them by the
// group's E4M3 scale in f16 (exact: <= 6 significant bits, f16 normal range).
//
// Cross-CTA waits (logit counter, per-token activation counter) spin with an
// iteration bound; on expiry the CTA records B2_STATUS_WAIT_TIMEOUT and skips
// the dependent work.  The kernel is launched cooperatively so all CTAs are
// co-resident.  The counters live in two sets used by alternate launches (see
// moe_decode_common.cuh), so nothing is reset at exit.
#include <atomic>
#include <algorithm>

#include "moe.cuh"
#include "moe_decode.cuh"
#include "moe_decode_common.cuh"

namespace b2 {
namespace dec {
namespace {


struct TileGeo {
  int K;
  int code_stride;   // bytes per padded code row
  int scale_stride;  // bytes per padded scale row
  int scale_off;     // offset of the scale rows in a slot
};
__device__ __forceinline__ TileGeo geo(int K) {
  TileGeo g;
  g.K = K;
  g.code_stride = K / 2 + kRowPad;
  g.scale_stride = K / 16 + kRowPad;
  g.scale_off = 16 * g.code_stride;
  return g;
}

// Global row id of tile row r (0..15) of item `it` (gate/up: row in the gate
// bank for r < 8, in the up bank for r >= 8; down: row in the down bank).
__device__ __forceinline__ uint32_t item_row_id(const Params& p, const uint32_t* inds, int it, int r) {
  if (it < p.n_gu) {
    const int fb = p.F / 8;
    const int pair = it / fb, f0 = (it % fb) * 8;
    return inds[pair] * (uint32_t)p.F + (uint32_t)(f0 + (r & 7));
  }
  const int d = it - p.n_gu;
  const int hb = p.H / 2;
  const int t = d / hb, h0 = (d % hb) * 2;
  const int q = r >> 1, j = r & 1;
  return inds[t * p.k + min(q, p.k - 1)] * (uint32_t)p.H + (uint32_t)(h0 + j);
}

// Every thread of the CTA copies its share of item `it` (the q-th tile of
// this CTA; its 16 row ids are rows[q*16 ..]) into a ring slot with 16-byte
// cp.async chunks (code rows then scale rows, padded slot layout), then
// arrives on the slot's mbarrier (kThreads arrivals complete the phase once
// every chunk has landed).  Issue is spread over all warps because one
// warp's cp.async stream is limited to a few GB/s.
__device__ __forceinline__ void issue_item(const Params& p, const uint32_t* rows, uint8_t* slot_base, uint64_t* bar,
                                           int it, int q) {
  const bool gu = it < p.n_gu;
  const int K = gu ? p.H : p.F;
  const TileGeo g = geo(K);
  const int cch = K / 32, sch = K / 256;  // 16-byte chunks per code / scale row
  const int total = 16 * (cch + sch);
  const uint8_t* cb0 = gu ? p.gcodes : p.dcodes;
  const uint8_t* cb1 = gu ? p.ucodes : p.dcodes;
  const uint8_t* sb0 = gu ? p.gscales : p.dscales;
  const uint8_t* sb1 = gu ? p.uscales : p.dscales;
  for (int i = threadIdx.x; i < total; i += kThreads) {
    const bool code = i < 16 * cch;
    const int j = code ? i : i - 16 * cch;
    const int per = code ? cch : sch;
    const int r = j / per, c = j - r * per;
    const uint64_t row = rows[q * 16 + r];
    if (code) {
      const uint8_t* src = (r < 8 ? cb0 : cb1) + row * (uint64_t)(K / 2);
      cp_async16(slot_base + (size_t)r * g.code_stride + 16 * c, src + 16 * c);
    } else {
      const uint8_t* src = (r < 8 ? sb0 : sb1) + row * (uint64_t)(K / 16);
      cp_async16(slot_base + g.scale_off + (size_t)r * g.scale_stride + 16 * c, src + 16 * c);
    }
  }
  cp_async_arrive(bar);
}

// This warp's share of the K groups of one 16-row tile; accumulates D(16x8).
// xs: staged B rows (f16), xcols valid columns (others zero).
__device__ __forceinline__ void tile_mma(const uint8_t* slot, const TileGeo& g, const __half* xs, int xstride,
                                         int xcols, uint32_t* stab, float acc[4]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gi = lane >> 2, c = lane & 3;
  const int groups = g.K / 16;
  const int mine = (groups - warp + kWarps - 1) / kWarps;
  // per-warp scale table for this warp's groups: (row p, row p+8) f16 pairs
  for (int idx = lane; idx < mine * 8; idx += 32) {
    const int gl = idx >> 3, pr = idx & 7;
    const int grp = warp + gl * kWarps;
    const uint8_t* sb = slot + g.scale_off + grp;
    stab[gl * 8 + pr] = scale_pair(sb[(size_t)pr * g.scale_stride], sb[(size_t)(pr + 8) * g.scale_stride]);
  }
  __syncwarp();
  const uint32_t sel = (uint32_t)c | ((uint32_t)(4 + c) << 4);  // byte c of w.x, byte c of w.y
  const uint8_t* row0 = slot + (size_t)gi * g.code_stride;
  const uint8_t* row8 = slot + (size_t)(gi + 8) * g.code_stride;
  const bool bcol = gi < xcols;
  const __half* xr = xs + (size_t)gi * xstride + 2 * c;
#pragma unroll 2
  for (int gl = 0; gl < mine; ++gl) {
    const int grp = warp + gl * kWarps;
    const uint2 w0 = *reinterpret_cast<const uint2*>(row0 + grp * 8);
    const uint2 w8 = *reinterpret_cast<const uint2*>(row8 + grp * 8);
    const uint32_t p0 = prmt(w0.x, w0.y, sel);
    const uint32_t p8 = prmt(w8.x, w8.y, sel);
    const uint32_t sp = stab[gl * 8 + gi];
    const __half2 s2 = *reinterpret_cast<const __half2*>(&sp);
    const __half2 slo = __low2half2(s2), shi = __high2half2(s2);
    uint32_t a[4];
    a[0] = hmul2_u32(cvt_byte0(p0), *reinterpret_cast<const uint32_t*>(&slo));
    a[2] = hmul2_u32(cvt_byte1(p0), *reinterpret_cast<const uint32_t*>(&slo));
    a[1] = hmul2_u32(cvt_byte0(p8), *reinterpret_cast<const uint32_t*>(&shi));
    a[3] = hmul2_u32(cvt_byte1(p8), *reinterpret_cast<const uint32_t*>(&shi));
    uint32_t b[2] = {0u, 0u};
    if (bcol) {
      b[0] = *reinterpret_cast<const uint32_t*>(xr + grp * 16);
      b[1] = *reinterpret_cast<const uint32_t*>(xr + grp * 16 + 8);
    }
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_block_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bars[kMaxSlots];
  __shared__ unsigned s_cnt[kMaxSlots];
  __shared__ uint32_t s_inds[64];
  __shared__ float s_wts[64];
  __shared__ int s_xexp[8];
  __shared__ int s_aexp[8];
  __shared__ unsigned s_red[32];
  __shared__ unsigned s_tokdone[8];
  __shared__ int s_ok;
  __shared__ uint32_t s_ep;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;

  // shared-memory carve: [x T x (H+8)] [a 8 x (F+8)] [scale tables] [row ids] [red] [ring]
  const int xstride = p.H + 8, astride = p.F + 8;
  __half* xs = reinterpret_cast<__half*>(smem);
  size_t off = ((size_t)p.T * xstride * 2 + 15) & ~size_t(15);
  __half* as = reinterpret_cast<__half*>(smem + off);
  off += ((size_t)8 * astride * 2 + 15) & ~size_t(15);
  const int per_warp_g = (max(p.H, p.F) / 16 + kWarps - 1) / kWarps;
  uint32_t* stab = reinterpret_cast<uint32_t*>(smem + off) + (size_t)warp * per_warp_g * 8;
  off += (size_t)kWarps * per_warp_g * 8 * 4;
  uint32_t* rows = reinterpret_cast<uint32_t*>(smem + off);
  off += (size_t)p.max_items * 16 * 4;
  float* red = reinterpret_cast<float*>(smem + off);  // [slot][warp][16]
  off += (size_t)p.n_slots * kWarps * 16 * 4;
  off = (off + 127) & ~size_t(127);
  uint8_t* ring = smem + off;

  if (tid == 0) {
    for (int i = 0; i < p.n_slots; ++i) mbar_init(&bars[i], kThreads);
    fence_mbar_init();
    s_ok = 1;
  }
  if (tid < kMaxSlots) s_cnt[tid] = 0u;
  if (tid < 8) s_tokdone[tid] = 0u;
  __syncthreads();

  // the ring is unused until phase 2
  const uint32_t epoch = phase1(p, xs, xstride, s_xexp, s_red, s_inds, s_wts, &s_ok, &s_ep, ring);
  unsigned* act_cnt = p.counters + kActCnt + 8 * (epoch & 1u);

  // ---------------- phase 2: expert tiles through the ring
  // This CTA owns a contiguous range of gate/up tiles and a contiguous range
  // of down tiles (long runs of consecutive rows per expert for DRAM).
  const int n_dn = p.n_items - p.n_gu;
  const int gu_lo = (int)((int64_t)cta * p.n_gu / G), gu_hi = (int)((int64_t)(cta + 1) * p.n_gu / G);
  const int dn_lo = (int)((int64_t)cta * n_dn / G), dn_hi = (int)((int64_t)(cta + 1) * n_dn / G);
  const int my_gu = gu_hi - gu_lo;
  const int my_n = my_gu + (dn_hi - dn_lo);
  auto item_of = [&](int q) { return q < my_gu ? gu_lo + q : p.n_gu + dn_lo + (q - my_gu); };
  for (int i = tid; i < my_n * 16; i += blockDim.x) rows[i] = item_row_id(p, s_inds, item_of(i >> 4), i & 15);
  __syncthreads();
  const int first_fill = min(p.n_slots, my_n);
  if (s_ok)
    for (int q = 0; q < first_fill; ++q) issue_item(p, rows, ring + (size_t)q * p.slot_bytes, &bars[q], item_of(q), q);

  int staged_tok = -1;
  bool released = false;
  for (int q = 0; q < my_n; ++q) {
    const int it = item_of(q);
    const int sl = q % p.n_slots;
    uint8_t* slot = ring + (size_t)sl * p.slot_bytes;
    const bool is_gu = it < p.n_gu;
    if (!is_gu) {
      const int t = (it - p.n_gu) / (p.H / 2);
      if (t != staged_tok) {
        // CTA-wide transition to token t's down tiles: publish this CTA's
        // finished gate/up tiles once, wait for token t's activations, stage
        // them (all warps reach this point in the same tile order)
        __syncthreads();
        if (tid == 0) {
          if (!released) release_tokens(p, act_cnt, s_tokdone);
          uint32_t i = 0;
          while (s_ok && ld_acquire(&act_cnt[t]) < (unsigned)(p.k * (p.F / 8))) {
            if (++i >= p.spin_limit) {
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
    }
    if (!s_ok) break;
    // a wait that gives up only records the status: every warp keeps taking
    // the same path through the barriers of this loop
    mbar_wait_bounded(&bars[sl], (uint32_t)((q / p.n_slots) & 1), p.status);
    const TileGeo g = geo(is_gu ? p.H : p.F);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int tok = 0;
    if (is_gu) {
      tok = (it / (p.F / 8)) / p.k;
      tile_mma(slot, g, xs, xstride, p.T, stab, acc);
    } else {
      tile_mma(slot, g, as, astride, p.k, stab, acc);
    }
    // the 16 useful partial sums of this warp -> red[slot][warp][row]
    {
      const int gi = lane >> 2, c = lane & 3;
      float* rp = red + ((size_t)sl * kWarps + warp) * 16;
      if (is_gu) {
        // column = token
        if (c == (tok >> 1)) {
          rp[gi] = (tok & 1) ? acc[1] : acc[0];
          rp[gi + 8] = (tok & 1) ? acc[3] : acc[2];
        }
      } else {
        // row 2q+j, column q (slot)
        const int q0 = gi >> 1, q1 = 4 + (gi >> 1);
        if (c == (q0 >> 1)) rp[gi] = (q0 & 1) ? acc[1] : acc[0];
        if (c == (q1 >> 1)) rp[gi + 8] = (q1 & 1) ? acc[3] : acc[2];
      }
    }
    __syncwarp();
    // s_cnt[sl] counts warp arrivals over every use of the slot: use u of the
    // slot is complete when it reaches kWarps * (u + 1)
    const unsigned use_done = (unsigned)kWarps * (unsigned)(q / p.n_slots + 1);
    unsigned arrived = 0;
    if (lane == 0) {
      __threadfence_block();
      arrived = atomicAdd(&s_cnt[sl], 1u);
    }
    arrived = __shfl_sync(0xffffffffu, arrived, 0);
    if (arrived == use_done - 1) {
    // ---- this warp arrived last: epilogue
    __threadfence_block();
    float v = 0.0f;
    if (lane < 16) {
      const float* rs = red + (size_t)sl * kWarps * 16 + lane;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += rs[w * 16];
    }
    if (is_gu) {
      const float up = __shfl_down_sync(0xffffffffu, v, 8);
      if (lane < 8) {
        const int fb = p.F / 8;
        const int pair = it / fb, f0 = (it % fb) * 8;
        const float gv = round_bf16(ldexpf(v, s_xexp[tok]));
        const float uv = round_bf16(ldexpf(up, s_xexp[tok]));
        p.act[(int64_t)pair * p.F + f0 + lane] = f32_to_bf16_bits(swiglu_bf16(gv, uv));
      }
      if (lane == 0) atomicAdd(&s_tokdone[tok], 1u);
    } else {
      const int d = it - p.n_gu;
      const int hb = p.H / 2;
      const int t = d / hb, h0 = (d % hb) * 2;
      float tot = 0.0f;
      for (int qq = 0; qq < p.k; ++qq) {
        const float dv = __shfl_sync(0xffffffffu, v, 2 * qq + (lane & 1));
        const float dr = round_bf16(ldexpf(dv, s_aexp[qq]));
        const float rw = round_bf16(s_wts[t * p.k + qq]);
        tot = round_bf16(__fadd_rn(round_bf16(__fmul_rn(dr, rw)), tot));
      }
      if (lane < 2) {
        if (p.routed_scale != 1.0f) tot = round_bf16(__fmul_rn(tot, round_bf16(p.routed_scale)));
        if (p.shared) tot = round_bf16(__fadd_rn(tot, bf16_bits_to_f32(p.shared[(int64_t)t * p.H + h0 + lane])));
        if (p.residual) tot = round_bf16(__fadd_rn(tot, bf16_bits_to_f32(p.residual[(int64_t)t * p.H + h0 + lane])));
        p.out[(int64_t)t * p.H + h0 + lane] = f32_to_bf16_bits(tot);
      }
    }
    }
    // refill: every warp issues its share of tile q + n_slots once all warps
    // are done reading this slot (bounded spin on the slot's arrival count)
    if (q + p.n_slots < my_n) {
      if (lane == 0) {
        uint32_t i = 0;
        while (*reinterpret_cast<volatile unsigned*>(&s_cnt[sl]) < use_done) {
          if (++i >= p.spin_limit) {
            report_status(p.status, B2_STATUS_WAIT_TIMEOUT);
            break;
          }
        }
      }
      __syncwarp();
      issue_item(p, rows, slot, &bars[sl], item_of(q + p.n_slots), q + p.n_slots);
    }
  }

  // publish finished gate/up tiles if no down tile did it (or the loop stopped)
  __syncthreads();
  if (tid == 0 && !released) release_tokens(p, act_cnt, s_tokdone);
  // a CTA that stopped after issuing copies waits (bounded) for them to land
  if (!s_ok && tid == 0 && first_fill > 0)
    asm volatile("cp.async.wait_all;" ::: "memory");
}

size_t a256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

size_t scratch_bytes(const b2_moe_block* blk, int64_t T) {
  return kDecodeStateBytes + 2 * a256((size_t)T * blk->top_k * 4) + a256((size_t)T * blk->top_k * blk->ffn * 2) +
         shared_scratch_bytes(blk, T);
}

int forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, const float* logits, const uint16_t* residual,
            uint16_t* out, uint32_t* inds, float* weights, void* scratch, size_t scratch_len, cudaStream_t st) {
  B2_REQUIRE(T >= 1 && T <= 8, "[moe_block] decode path takes 1..8 tokens");
  B2_REQUIRE(scratch_len >= scratch_bytes(blk, T), "[moe_block] workspace too small (%zu < %zu)", scratch_len,
             scratch_bytes(blk, T));
  B2_REQUIRE(reinterpret_cast<uintptr_t>(scratch) % 256 == 0, "[moe_block] workspace must be 256-byte aligned");
  Params p{};
  p.x = x;
  p.router_w = blk->router_w;
  p.router_w_dtype = blk->router_w_dtype;
  p.router_bias = blk->router_bias;
  p.logits_in = logits;
  p.gcodes = reinterpret_cast<const uint8_t*>(blk->gate_codes);
  p.gscales = blk->gate_scales;
  p.ucodes = reinterpret_cast<const uint8_t*>(blk->up_codes);
  p.uscales = blk->up_scales;
  p.dcodes = reinterpret_cast<const uint8_t*>(blk->down_codes);
  p.dscales = blk->down_scales;
  p.residual = residual;
  p.out = out;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  size_t off = 0;
  p.counters = reinterpret_cast<unsigned*>(base + off);
  p.logit_words = reinterpret_cast<unsigned long long*>(base + kLogitWords);
  off += kDecodeStateBytes;
  p.inds_out = inds ? inds : reinterpret_cast<uint32_t*>(base + off);
  off += a256((size_t)T * blk->top_k * 4);
  p.wts_out = weights ? weights : reinterpret_cast<float*>(base + off);
  off += a256((size_t)T * blk->top_k * 4);
  p.act = reinterpret_cast<uint16_t*>(base + off);
  off += a256((size_t)T * blk->top_k * blk->ffn * 2);
  // the shared expert (if any) runs first, into the scratch after the
  // activations; the decode kernel adds its output in the epilogue
  {
    const int rc = shared_forward(blk, x, T, base + off, &p.shared, st);
    if (rc) return rc;
  }
  p.status = device_status_ptr();
  if (!p.status) return set_error(B2_ERR_CUDA, "[moe_block] device status word unavailable");
  testing_decode_fault(&p.skip_logit_cta, &p.spin_limit);  // (-1, the default bound) unless a test set it
  p.T = (int)T;
  p.E = (int)blk->n_experts;
  p.H = (int)blk->hidden;
  p.F = (int)blk->ffn;
  p.k = blk->top_k;
  p.mode = blk->router_mode;
  p.renorm = blk->renorm;
  p.routed_scale = blk->routed_scale;
  p.n_gu = p.T * p.k * (p.F / 8);
  p.n_items = p.n_gu + p.T * (p.H / 2);
  B2_REQUIRE((uint64_t)p.E * std::max(p.F, p.H) < (1ull << 32), "[moe_block] expert banks too large (32-bit row ids)");
  if (!logits) B2_REQUIRE(blk->router_w != nullptr, "[moe_block] router weight is NULL and no logits were given");

  if (blk->decode_bank) {
    B2_REQUIRE(reinterpret_cast<uintptr_t>(blk->decode_bank) % 16 == 0, "[moe_block] decode bank must be 16-byte aligned");
    return launch_tma(p, blk, st);
  }

  int dev = 0, sms = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  B2_REQUIRE(sms <= kMaxCtas, "[moe_block] the decode kernels support at most %d SMs (got %d)", kMaxCtas, sms);
  cudaFuncAttributes fa;
  int rc = check_cuda(cudaFuncGetAttributes(&fa, decode_block_kernel), "moe_block");
  if (rc) return rc;
  const size_t avail = (size_t)optin - fa.sharedSizeBytes;
  const int per_warp_g = (int)((std::max(blk->hidden, blk->ffn) / 16 + kWarps - 1) / kWarps);
  p.max_items = (p.n_gu + sms - 1) / sms + (p.n_items - p.n_gu + sms - 1) / sms;
  size_t fixed = ((size_t)p.T * (p.H + 8) * 2 + 15) & ~size_t(15);
  fixed += ((size_t)8 * (p.F + 8) * 2 + 15) & ~size_t(15);
  fixed += (size_t)kWarps * per_warp_g * 8 * 4 + (size_t)p.max_items * 16 * 4;
  const size_t slot_h = 16 * (size_t)(p.H / 2 + kRowPad) + 16 * (size_t)(p.H / 16 + kRowPad);
  const size_t slot_f = 16 * (size_t)(p.F / 2 + kRowPad) + 16 * (size_t)(p.F / 16 + kRowPad);
  p.slot_bytes = (int)((std::max(slot_h, slot_f) + 127) & ~size_t(127));
  const size_t per_slot = (size_t)p.slot_bytes + (size_t)kWarps * 16 * 4;
  B2_REQUIRE(avail > fixed + 128 + per_slot, "[moe_block] hidden/ffn too large for the decode kernel");
  p.n_slots = (int)std::min<size_t>({(avail - fixed - 128) / per_slot, (size_t)kMaxSlots, (size_t)p.max_items});
  // the ring doubles as the top-k ranking scratch (16 bytes per expert)
  while ((size_t)p.n_slots * p.slot_bytes < (size_t)16 * p.E && p.n_slots < kMaxSlots &&
         fixed + 128 + (size_t)(p.n_slots + 1) * per_slot <= avail)
    ++p.n_slots;
  B2_REQUIRE((size_t)p.n_slots * p.slot_bytes >= (size_t)16 * p.E, "[moe_block] too many experts for the decode kernel");
  const size_t smem = fixed + 128 + (size_t)p.n_slots * per_slot;
  rc = ensure_dynamic_smem((const void*)decode_block_kernel, smem, "moe_block");
  if (rc) return rc;
  void* args[] = {&p};
  return check_cuda(
      cudaLaunchCooperativeKernel((const void*)decode_block_kernel, dim3(sms), dim3(kThreads), args, smem, st),
      "moe_block decode");
}

// ---------------------------------------------------------------- test hook
namespace {
std::atomic<int> g_fault_skip_cta{-1};
std::atomic<uint32_t> g_fault_spin_limit{0};
}  // namespace

void testing_decode_fault(int* skip_logit_cta, uint32_t* spin_limit) {
  *skip_logit_cta = g_fault_skip_cta.load(std::memory_order_relaxed);
  const uint32_t s = g_fault_spin_limit.load(std::memory_order_relaxed);
  *spin_limit = s ? s : kSpinLimit;
}

}  // namespace dec
}  // namespace b2

extern "C" int b2_testing_set_decode_fault(int skip_logit_cta, unsigned spin_limit) {
  B2_REQUIRE(skip_logit_cta >= -1 && skip_logit_cta < b2::dec::kMaxCtas,
             "[testing_set_decode_fault] CTA index %d outside [-1, %d)", skip_logit_cta, b2::dec::kMaxCtas);
  b2::dec::g_fault_skip_cta.store(skip_logit_cta, std::memory_order_relaxed);
  b2::dec::g_fault_spin_limit.store(spin_limit, std::memory_order_relaxed);
  return B2_OK;
}
