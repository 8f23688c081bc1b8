// Prefill MoE expert block: expert-sorted grouped GEMMs on the 5th-generation
// tensor cores (tcgen05, accumulators in TMEM).
//
// Rows are the (token, slot) pairs in expert order (b2_moe_gather_sort); an
// expert's rows form M-tiles of 128.  A work unit is (M-tile, N-tile of 256
// output features); every CTA walks the units u = cta, cta + G, ... of the
// launch.  Per unit the K range is streamed in stages of 64:
//   A [128 x 64] f16: one tiled TMA copy per stage straight into the
//     128-byte-swizzled K-major layout the MMA reads (gate/up: the token rows
//     of x in expert order, pre-converted to f16 with a per-token
//     power-of-two pre-scale; down: the sorted SwiGLU rows, same treatment
//     per row);
//   B [256 x 64] f16: the stage's NVFP4 weights arrive as one 9 KB bulk copy
//     from the prefill bank (b2_moe_prepare_prefill_bank) and are dequantized
//     in shared memory (hardware E2M1 -> f16 conversion, times the f16 scale:
//     exact) into the same swizzled layout;
//   one thread issues 4 MMAs of 128x256x16 per stage into a TMEM accumulator
//   (two accumulators of 256 columns alternate between units, so the
//   epilogue of one unit overlaps the main loop of the next).
// Epilogues: gate/up -- the N-tile holds 128 gate and the matching 128 up
// features; g and u are scaled back, rounded to bf16 and combined by the
// reference's bf16 SwiGLU steps into act[row]; down -- the 256 hidden outputs
// are scaled back and rounded to bf16 into y[row] (the per-slot expert
// output; the ordered weighted combine follows in b2_moe_combine).
//
// Warp roles (20 warps): 0 MMA issue (+ TMEM allocation), 4 weight copies,
// 8 activation-row copies, 1-3/5-7/9-10 dequantizers, 12-19 epilogue (TMEM
// lane quarter = warp % 4, two warps per quarter split the columns).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "moe.cuh"
#include "moe_prefill_gemm.cuh"

namespace b2 {
namespace pf {
namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int MT = 1;                                 // 128-row MMA tiles per unit
constexpr int BMU = BM * MT;                          // rows per unit
constexpr int A_TILE = BM * BK * 2;                   // 16 KB per 128-row tile
constexpr int A_BYTES = A_TILE * MT;                  // per stage
constexpr int B_BYTES = BN * BK * 2;                  // 32 KB
constexpr int W_BYTES = BN * BK / 2 + BN * BK / 16;   // 9 KB packed stage
// Separate rings, deep where the source is far: packed weights come from
// HBM (SW stages ahead), activation rows from L2 (SA), dequantized weights
// are produced just in time from shared memory (SB).
constexpr int SW = 6, SA = 4, SB = 3;
// Warp roles.  Warps are spread over the SM's four sub-partitions by
// warp % 4, and an epilogue warp can only read the TMEM lane quarter
// warp % 4, so each sub-partition hosts two epilogue warps.  Sub-partition 0
// also hosts the MMA-issuing warp and the two copy-issuing warps (all mostly
// waiting), and the eight dequantizer warps fill sub-partitions 1-3, so the
// single MMA-issuing thread is not starved of issue slots.
constexpr int kWarps = 20;
constexpr int kThreads = kWarps * 32;
constexpr int W_MMA = 0, W_TMA = 4, W_A = 8, N_DQ = 8, N_EP = 8;
__device__ __forceinline__ int dq_index(int w) {  // warps 1,2,3,5,6,7,9,10 -> 0..7, else -1
  if (w < 12 && (w & 3) != 0 && w != 11) return (w >> 2) * 3 + (w & 3) - 1;
  return -1;
}
__device__ __forceinline__ bool is_epilogue(int w) { return w >= 12; }
constexpr int A_OFF = 0, B_OFF = SA * A_BYTES, W_OFF = B_OFF + SB * B_BYTES;
constexpr int kSmemBytes = W_OFF + SW * W_BYTES + 1024;
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr uint32_t kTmemCols = 512;

struct Params {
  const uint8_t* wbank;      // prepared [E][ntiles][nstages][W_BYTES]
  const __half* a16;         // gate/up: x rows [T][K]; down: activation rows [rows][K]
  const int* rexp;           // pre-scale exponent per a16 row
  const uint32_t* order;     // sorted row -> flat (token * k + slot)
  const uint32_t* offsets;   // [E + 1] first sorted row of each expert
  const uint32_t* tile_off;  // [E + 1] first unit row block (BMU rows) of each expert
  uint16_t* out;             // gate/up: act [rows][F]; down: y [rows][H]
  const uint16_t* silu_tab;  // exact bf16 SiLU table or null
  unsigned* status;
  int E, K, N, k, ntiles, nstages;
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  // K-major operand, 128-byte swizzle: start >> 4, LBO 16 B, SBO 1024 B (one
  // 8-row swizzle atom), descriptor version 1, layout type 2 (SWIZZLE_128B)
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16, f16 A and B (K-major), f32 accumulate, M = 128, N = 256
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

// byte offset of (row r, 16-byte chunk c) in a 128B-swizzled K-major tile
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Bounded mbarrier wait that gives up for good once any wait in the CTA has
// timed out (so a broken pipeline ends instead of stacking timeouts).
__device__ __forceinline__ void wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status) {
  if (*abort_flag) return;
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 255u) == 255u && *abort_flag) return;
  }
  *abort_flag = 1;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
}

// Spinning variant for the single MMA-issuing thread (mbarrier.test_wait
// never suspends the thread, so it resumes as soon as the phase completes).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void spin_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status) {
  if (*abort_flag) return;
  for (uint32_t i = 0; i < (kWaitLimit << 4); ++i) {
    if (mbar_test(bar, parity)) return;
    if ((i & 1023u) == 1023u && *abort_flag) return;
  }
  *abort_flag = 1;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
}

// unit u -> expert, first sorted row, valid rows, N-tile
struct Unit {
  int e, row0, nrows, n;
};
__device__ __forceinline__ Unit decode_unit(const Params& p, const uint32_t* s_toff, const uint32_t* s_off, int u) {
  Unit r;
  const int mt = u / p.ntiles;
  r.n = u - mt * p.ntiles;
  int lo = 0, hi = p.E;  // largest e with tile_off[e] <= mt
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if ((int)s_toff[mid] <= mt) lo = mid;
    else hi = mid;
  }
  r.e = lo;
  r.row0 = (int)s_off[lo] + (mt - (int)s_toff[lo]) * BMU;
  r.nrows = min(BMU, (int)s_off[lo + 1] - r.row0);
  return r;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(Params p, const __grid_constant__ CUtensorMap amap) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t afull[SA], aempty[SA], bfull[SB], bempty[SB], wfull[SW], wempty[SW], tfull_bar[2],
      tempty_bar[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ uint32_t s_toff[1025], s_off[1025];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  for (int i = tid; i <= p.E; i += kThreads) {
    s_toff[i] = p.tile_off[i];
    s_off[i] = p.offsets[i];
  }
  if (tid == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&afull[i], 1);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&bfull[i], N_DQ);
      mbar_init(&bempty[i], 1);
    }
    for (int i = 0; i < SW; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], N_DQ);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], N_EP);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == W_MMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  volatile int* abort_flag = &s_abort;
  const int U = (int)s_toff[p.E] * p.ntiles;
  const int NS = p.nstages;

  if (warp == W_MMA) {
    if (lane == 0) {
      // descriptors of slot 0; slot i adds its byte offset >> 4 (start field
      // stays below 2^14: shared memory is under 256 KB)
      const uint64_t adesc0 = sw128_desc(smem_u32(base + A_OFF)), bdesc0 = sw128_desc(smem_u32(base + B_OFF));
      uint32_t g = 0;
      int i = 0;
      for (int u = cta; u < U; u += G, ++i) {
        const Unit un = decode_unit(p, s_toff, s_off, u);
        // two accumulators of 256 columns alternate between units, so the
        // epilogue of one unit overlaps the main loop of the next
        const int acc = i & 1;
        wait_bar(&tempty_bar[acc], (uint32_t)(((i >> 1) & 1) ^ 1), abort_flag, p.status);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int s = 0; s < NS; ++s, ++g) {
          const uint32_t ia = g % SA, ib = g % SB;
          spin_bar(&afull[ia], (g / SA) & 1u, abort_flag, p.status);
          spin_bar(&bfull[ib], (g / SB) & 1u, abort_flag, p.status);
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t da0 = adesc0 + (uint64_t)(ia * (A_BYTES >> 4)), db0 = bdesc0 + (uint64_t)(ib * (B_BYTES >> 4));
          const uint32_t d = tmem + (uint32_t)(acc * BN);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // advancing K by 16 elements = 32 bytes = 2 in the descriptor's start field
            const uint32_t accum = (s > 0 || kk > 0) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred pd;\n\tsetp.ne.b32 pd, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pd;\n\t}\n" ::"r"(d),
                "l"(da0 + 2 * kk), "l"(db0 + 2 * kk), "r"(kIdesc), "r"(accum));
          }
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&aempty[ia]))
                       : "memory");
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&bempty[ib]))
                       : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&tfull_bar[acc]))
                     : "memory");
      }
    }
  } else if (warp == W_TMA) {
    if (lane == 0) {
      uint32_t g = 0;
      for (int u = cta; u < U; u += G) {
        const Unit un = decode_unit(p, s_toff, s_off, u);
        const uint8_t* src = p.wbank + (((size_t)un.e * p.ntiles + un.n) * NS) * (size_t)W_BYTES;
        for (int s = 0; s < NS; ++s, ++g) {
          const uint32_t iw = g % SW;
          wait_bar(&wempty[iw], ((g / SW) & 1u) ^ 1u, abort_flag, p.status);
          mbar_expect_tx(&wfull[iw], (uint32_t)W_BYTES);
          bulk_g2s(base + W_OFF + iw * W_BYTES, src + (size_t)s * W_BYTES, (uint32_t)W_BYTES, &wfull[iw]);
        }
      }
    }
  } else if (warp == W_A) {
    // activation rows: the unit's 128 sorted rows are contiguous (gate/up:
    // the f16 token rows already laid out in expert order; down: the sorted
    // SwiGLU rows), one tiled copy per stage; rows past the tensor read as
    // zeros, rows past the unit's end land in tile rows whose MMA output is
    // never stored
    if (lane == 0) {
      uint32_t g = 0;
      for (int u = cta; u < U; u += G) {
        const Unit un = decode_unit(p, s_toff, s_off, u);
        for (int s = 0; s < NS; ++s, ++g) {
          const uint32_t slot = g % SA;
          wait_bar(&aempty[slot], ((g / SA) & 1u) ^ 1u, abort_flag, p.status);
          mbar_expect_tx(&afull[slot], (uint32_t)A_BYTES);
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(base + A_OFF + slot * A_BYTES)),
              "l"(reinterpret_cast<uint64_t>(&amap)), "r"(s * BK), "r"(un.row0), "r"(smem_u32(&afull[slot]))
              : "memory");
        }
      }
    }
  } else if (dq_index(warp) >= 0) {
    // dequantizers: thread td takes the chunk pair (2(td%4), 2(td%4)+1) of rows
    // td/4 + 64j (j < 4): one 8-byte code load and one scale byte per pair;
    // every address is a per-thread base plus a constant
    static_assert(BN * 4 == N_DQ * 32 * 4, "four chunk pairs per dequantizer thread");
    const int td = dq_index(warp) * 32 + lane;
    const int cp = td & 3, rr = (td >> 2) & 7;
    const uint32_t w_code = (uint32_t)((td >> 2) * 32 + cp * 8);
    const uint32_t w_scale = (uint32_t)(BN * 32 + (td >> 2) * 4 + cp);
    const uint32_t b_base = (uint32_t)((td >> 5) * 1024 + rr * 128);
    const uint32_t b_c0 = (uint32_t)(((2 * cp) ^ rr) << 4), b_c1 = (uint32_t)(((2 * cp + 1) ^ rr) << 4);
    uint32_t g = 0;
    for (int u = cta; u < U; u += G) {
      for (int s = 0; s < NS; ++s, ++g) {
        const uint32_t iw = g % SW, ib = g % SB;
        wait_bar(&wfull[iw], (g / SW) & 1u, abort_flag, p.status);
        wait_bar(&bempty[ib], ((g / SB) & 1u) ^ 1u, abort_flag, p.status);
        const uint8_t* w = base + W_OFF + iw * W_BYTES;
        uint8_t* b = base + B_OFF + ib * B_BYTES + b_base;
        uint2 cw[4];
        uint32_t sb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          cw[j] = *reinterpret_cast<const uint2*>(w + w_code + j * 64 * 32);
          sb[j] = w[w_scale + j * 64 * 4];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t s2 = sb[j] * 0x00800080u;  // (sb << 7) | (sb << 23): the f16 scale in both halves
          uint4 o0, o1;
          o0.x = hmul2_u32(cvt_byte<0>(cw[j].x), s2);
          o0.y = hmul2_u32(cvt_byte<1>(cw[j].x), s2);
          o0.z = hmul2_u32(cvt_byte<2>(cw[j].x), s2);
          o0.w = hmul2_u32(cvt_byte<3>(cw[j].x), s2);
          o1.x = hmul2_u32(cvt_byte<0>(cw[j].y), s2);
          o1.y = hmul2_u32(cvt_byte<1>(cw[j].y), s2);
          o1.z = hmul2_u32(cvt_byte<2>(cw[j].y), s2);
          o1.w = hmul2_u32(cvt_byte<3>(cw[j].y), s2);
          *reinterpret_cast<uint4*>(b + j * 8192 + b_c0) = o0;
          *reinterpret_cast<uint4*>(b + j * 8192 + b_c1) = o1;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bfull[ib]);
          mbar_arrive(&wempty[iw]);
        }
      }
    }
  } else if (is_epilogue(warp)) {
    // epilogue: TMEM lane quarter q = warp % 4 (rows 32q.. of each 128-row
    // tile), the two warps of a quarter split the columns
    static_assert(N_EP == 8, "two epilogue warps per TMEM lane quarter");
    const int q = warp & 3, half = warp >= 16 ? 1 : 0;
    int i = 0;
    for (int u = cta; u < U; u += G, ++i) {
      const Unit un = decode_unit(p, s_toff, s_off, u);
      const int acc = i & 1;
      wait_bar(&tfull_bar[acc], (uint32_t)((i >> 1) & 1), abort_flag, p.status);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      {
        const int r = 32 * q + lane;
        const bool ok = r < un.nrows;
        const int row = un.row0 + r;
        const uint32_t t0 = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN);
        if (MODE == 0) {
          const int F = p.N / 2;
          const int ex = ok ? p.rexp[p.order[row] / (uint32_t)p.k] : 0;
          for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 16) {
            uint32_t gv[16], uv[16];
            tmem_ld16(t0 + c0, gv);
            tmem_ld16(t0 + 128 + c0, uv);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (ok) {
              uint32_t o[8];
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                const float a0 = swiglu_bf16_tab(round_bf16(mul_pow2(__uint_as_float(gv[j]), ex)),
                                                 round_bf16(mul_pow2(__uint_as_float(uv[j]), ex)), p.silu_tab);
                const float a1 = swiglu_bf16_tab(round_bf16(mul_pow2(__uint_as_float(gv[j + 1]), ex)),
                                                 round_bf16(mul_pow2(__uint_as_float(uv[j + 1]), ex)), p.silu_tab);
                o[j / 2] = (uint32_t)f32_to_bf16_bits(a0) | ((uint32_t)f32_to_bf16_bits(a1) << 16);
              }
              uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)row * F + un.n * 128 + c0);
              dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
              dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
          }
        } else {
          const int ex = ok ? p.rexp[row] : 0;
          for (int c0 = half * 128; c0 < half * 128 + 128; c0 += 16) {
            uint32_t dv[16];
            tmem_ld16(t0 + c0, dv);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (ok) {
              uint32_t o[8];
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                const float y0 = round_bf16(mul_pow2(__uint_as_float(dv[j]), ex));
                const float y1 = round_bf16(mul_pow2(__uint_as_float(dv[j + 1]), ex));
                o[j / 2] = (uint32_t)f32_to_bf16_bits(y0) | ((uint32_t)f32_to_bf16_bits(y1) << 16);
              }
              uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)row * p.N + un.n * BN + c0);
              dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
              dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == W_MMA)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ---------------------------------------------------------------- helpers
// Per-row power-of-two pre-scale and f16 copy: one warp per row of K bf16
// values; exp[row] = p with max|x| * 2^-p < 2^15 (the decode staging rule).
__global__ void to_f16_rows_kernel(const uint16_t* __restrict__ src, int64_t rows, int K, __half* __restrict__ dst,
                                   int* __restrict__ exps) {
  const int64_t row = blockIdx.x * (int64_t)(blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + row * K);
  unsigned mx = 0;
  for (int c = lane; c < K / 8; c += 32) {
    const uint4 v = __ldg(s4 + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) mx = max(mx, max(w[j] & 0x7fffu, (w[j] >> 16) & 0x7fffu));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const unsigned e = (mx >> 7) & 0xffu;
  const int pexp = (e >= 142u) ? (int)e - 141 : 0;
  const float sc = __int_as_float((127 - pexp) << 23);
  if (lane == 0) exps[row] = pexp;
  uint4* d4 = reinterpret_cast<uint4*>(dst + row * K);
  for (int c = lane; c < K / 8; c += 32) {
    const uint4 v = __ldg(s4 + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 hh = __floats2half2_rn(__uint_as_float(w[j] << 16) * sc, __uint_as_float(w[j] & 0xffff0000u) * sc);
      o[j] = *reinterpret_cast<uint32_t*>(&hh);
    }
    d4[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// dst[p] = src[order[p] / k]: f16 token rows copied into expert order (one
// 16-byte chunk per thread).
__global__ void gather_rows_kernel(const __half* __restrict__ src, const uint32_t* __restrict__ order, int k,
                                   int64_t rows, int K, __half* __restrict__ dst) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int chunks = K / 8;
  if (i >= rows * chunks) return;
  const int64_t p = i / chunks;
  const int c = (int)(i - p * chunks);
  const uint32_t t = order[p] / (uint32_t)k;
  reinterpret_cast<uint4*>(dst + p * K)[c] = __ldg(reinterpret_cast<const uint4*>(src + (int64_t)t * K) + c);
}

// tile_off[e] = sum over e' < e of ceil(n_e' / BMU) (unit row blocks)
__global__ void tile_offsets_kernel(const uint32_t* __restrict__ offsets, int E, uint32_t* __restrict__ tile_off) {
  if (threadIdx.x == 0) {
    uint32_t acc = 0;
    for (int e = 0; e < E; ++e) {
      tile_off[e] = acc;
      acc += (offsets[e + 1] - offsets[e] + BMU - 1) / BMU;
    }
    tile_off[E] = acc;
  }
}

// Prefill bank: tile (e, n, s) = [BN rows][32 code bytes] then [BN rows][4
// scale bytes] for K range 64s..64s+63.  Gate/up: rows 0..127 gate features
// 128n.., rows 128..255 the same up features; down: hidden rows 256n...
// Scale bytes as in the decode bank (f16 bits of |scale| >> 7; negative
// scales flip the sign bits of their group's codes).
__global__ void prepare_prefill_kernel(const uint8_t* __restrict__ gcodes, const uint8_t* __restrict__ gscales,
                                       const uint8_t* __restrict__ ucodes, const uint8_t* __restrict__ uscales,
                                       const uint8_t* __restrict__ dcodes, const uint8_t* __restrict__ dscales, int E,
                                       int H, int F, uint8_t* __restrict__ bank) {
  const int64_t gu_tiles = (int64_t)E * (F / 128) * (H / BK);
  const int64_t tile = blockIdx.x;
  const bool gu = tile < gu_tiles;
  const int r = threadIdx.x;  // BN threads: one row each
  int64_t crow;
  const uint8_t *cb, *sbp;
  int K, s;
  if (gu) {
    const int nst = H / BK, nt = F / 128;
    const int64_t e = tile / ((int64_t)nt * nst);
    const int n = (int)((tile / nst) % nt);
    s = (int)(tile % nst);
    K = H;
    crow = e * F + (int64_t)n * 128 + (r & 127);
    cb = r < 128 ? gcodes : ucodes;
    sbp = r < 128 ? gscales : uscales;
  } else {
    const int64_t t2 = tile - gu_tiles;
    const int nst = F / BK, nt = H / BN;
    const int64_t e = t2 / ((int64_t)nt * nst);
    const int n = (int)((t2 / nst) % nt);
    s = (int)(t2 % nst);
    K = F;
    crow = e * H + (int64_t)n * BN + r;
    cb = dcodes;
    sbp = dscales;
  }
  uint8_t* dst = bank + tile * (int64_t)W_BYTES;
  const uint8_t* code = cb + crow * (K / 2) + (int64_t)s * (BK / 2);
  const uint8_t* scl = sbp + crow * (K / 16) + (int64_t)s * (BK / 16);
  uint32_t sc4 = 0;
#pragma unroll
  for (int gq = 0; gq < 4; ++gq) sc4 |= (uint32_t)prepared_scale_byte(scl[gq]) << (8 * gq);
#pragma unroll
  for (int wq = 0; wq < 8; ++wq) {
    uint32_t w = *reinterpret_cast<const uint32_t*>(code + 4 * wq);
    if (scl[wq >> 1] & 0x80u) w ^= 0x88888888u;
    reinterpret_cast<uint32_t*>(dst + r * 32)[wq] = w;
  }
  reinterpret_cast<uint32_t*>(dst + BN * 32)[r] = sc4;
}

}  // namespace

size_t prefill_bank_bytes(const b2_moe_block* blk) {
  return (size_t)blk->n_experts * (size_t)(3 * blk->ffn) * (size_t)blk->hidden * 9 / 16;
}

bool prefill_gemm_supported(const b2_moe_block* blk) {
  return blk->hidden % BN == 0 && blk->ffn % 128 == 0 && blk->n_experts <= 1024;
}

int prepare_prefill(const b2_moe_block* blk, void* dst, cudaStream_t st) {
  (void)silu_table(st);  // setup call: build the SiLU table outside any capture
  const int64_t E = blk->n_experts, H = blk->hidden, F = blk->ffn;
  const int64_t tiles = E * (F / 128) * (H / BK) + E * (H / BN) * (F / BK);
  B2_REQUIRE(tiles <= INT32_MAX, "[prepare_prefill_bank] too many tiles");
  prepare_prefill_kernel<<<(unsigned)tiles, BN, 0, st>>>(
      reinterpret_cast<const uint8_t*>(blk->gate_codes), blk->gate_scales,
      reinterpret_cast<const uint8_t*>(blk->up_codes), blk->up_scales,
      reinterpret_cast<const uint8_t*>(blk->down_codes), blk->down_scales, (int)E, (int)H, (int)F,
      static_cast<uint8_t*>(dst));
  B2_CHECK_LAUNCH("prepare_prefill_bank");
  return B2_OK;
}

int to_f16_rows(const uint16_t* src, int64_t rows, int K, __half* dst, int* exps, cudaStream_t st) {
  if (rows == 0) return B2_OK;
  to_f16_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(src, rows, K, dst, exps);
  B2_CHECK_LAUNCH("to_f16_rows");
  return B2_OK;
}

int gather_rows(const __half* src, const uint32_t* order, int k, int64_t rows, int K, __half* dst, cudaStream_t st) {
  const int64_t total = rows * (K / 8);
  if (total == 0) return B2_OK;
  gather_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, order, k, rows, K, dst);
  B2_CHECK_LAUNCH("gather_rows");
  return B2_OK;
}

int tile_offsets(const uint32_t* offsets, int E, uint32_t* tile_off, cudaStream_t st) {
  tile_offsets_kernel<<<1, 32, 0, st>>>(offsets, E, tile_off);
  B2_CHECK_LAUNCH("tile_offsets");
  return B2_OK;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2-D f16 tensor [rows][cols] (row-major), 128-byte swizzle, box 64 x box_rows.
int make_tensor_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  B2_REQUIRE(enc != nullptr, "[prefill grouped gemm] cuTensorMapEncodeTiled is not available from the driver");
  B2_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0 && (cols * 2) % 16 == 0,
             "[prefill grouped gemm] activation rows must be 16-byte aligned");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2_REQUIRE(r == CUDA_SUCCESS, "[prefill grouped gemm] tensor map encoding failed (%d)", (int)r);
  return B2_OK;
}

}  // namespace

int grouped_gemm(int mode, const b2_moe_block* blk, const __half* a16, int64_t a_rows, const int* rexp,
                 const uint32_t* order, const uint32_t* offsets, const uint32_t* tile_off, uint16_t* out,
                 cudaStream_t st) {
  Params p;
  const int E = (int)blk->n_experts, H = (int)blk->hidden, F = (int)blk->ffn;
  p.wbank = static_cast<const uint8_t*>(blk->prefill_bank);
  if (mode == 1) p.wbank += (size_t)E * (F / 128) * (H / BK) * W_BYTES;
  p.a16 = a16;
  p.rexp = rexp;
  p.order = order;
  p.offsets = offsets;
  p.tile_off = tile_off;
  p.out = out;
  p.silu_tab = mode == 0 ? silu_table(st) : nullptr;
  p.status = device_status_ptr();
  p.E = E;
  p.k = blk->top_k;
  p.K = mode == 0 ? H : F;
  p.N = mode == 0 ? 2 * F : H;
  p.ntiles = p.N / BN;
  p.nstages = p.K / BK;
  const void* fn = mode == 0 ? (const void*)grouped_gemm_kernel<0> : (const void*)grouped_gemm_kernel<1>;
  int rc = ensure_dynamic_smem(fn, kSmemBytes, "prefill grouped gemm");
  if (rc) return rc;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  CUtensorMap amap;
  rc = make_tensor_map(&amap, a16, (uint64_t)a_rows, (uint64_t)p.K, (uint32_t)BM);
  if (rc) return rc;
  void* args[] = {&p, &amap};
  return check_cuda(cudaLaunchKernel(fn, dim3(sms), dim3(kThreads), args, kSmemBytes, st), "prefill grouped gemm");
}

}  // namespace pf
}  // namespace b2
