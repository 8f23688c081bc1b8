// Shared core of the NVFP4 GEMV kernels (decode-shaped quantized matmuls).
//
// Design (sm_100a):
//   * A CTA owns 8 groups of RT consecutive weight rows over the whole K range
//     (8 * RT rows).  Lane q of warp 0 issues one TMA bulk copy for the codes
//     of group q (RT rows, contiguous in the MLX layout: RT * K/2 bytes) and
//     one for its scales, all up front, so every CTA has its entire working
//     set in flight at once (HBM latency hidden by volume, not by warps) in a
//     few large copies (small bulk copies stream far below HBM bandwidth).
//     Groups are padded by 16 bytes in shared memory; MMA tile rt takes row
//     rt of every group, so the 8 rows a warp reads at one K offset fall in
//     distinct banks.
//   * The activations (<= 16*MT tokens) are staged as f16 with a per-token
//     power-of-two pre-scale chosen so the largest |x| stays below 2^15; the
//     conversion is exact for every bf16 value of magnitude >= 2^-17 times that
//     scale, and the scale is undone on the float result.
//   * The dot products run on the tensor cores with mma.sync m16n8k16 (f16 in,
//     f32 accumulate): tokens are the 16-row A side, eight weight rows the
//     8-column B side.  Thread (g, c) of a warp decodes, for weight row g and
//     each 16-element group, code bytes c and c+4 with the hardware
//     cvt.rn.f16x2.e2m1x2 (exact E2M1 -> f16) and multiplies them by the
//     group's E4M3 scale in f16 (exact: <= 6 significant bits, inside the f16
//     normal range), which is exactly the B fragment layout (k = 2c, 2c+1 and
//     2c+8, 2c+9).  The GEMV stays HBM-bound because the tensor core does the
//     multiply-adds and the ALU only decodes (two conversions and two f16
//     multiplies per 16 weights per thread).
//   * Warps split the groups of K round-robin; partial accumulators are
//     reduced through shared memory in a fixed order.
#pragma once

#include "common.cuh"

namespace b2 {

// Programmatic dependent launch of the GEMV kernels (on unless the
// environment sets B2_QMV_PDL=0).
bool qmv_pdl_enabled();

// Single-matrix streaming GEMV (qmv_stream.cu): 1 when the shape is outside
// its domain, else a b2 status.
int qmv_stream(const uint16_t* x, const uint8_t* codes, const uint8_t* scales, int M, int N, int K, uint16_t* y,
               cudaStream_t st);

namespace qmv {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowPad = 16;  // bytes of padding per shared-memory row

constexpr int kGroups = 8;  // row groups per CTA (the 8 columns of an MMA B fragment)

struct TileGeom {
  int K;            // reduction length (multiple of 256)
  int rg;           // consecutive rows per group (RT)
  int code_stride;  // padded bytes per group of code rows in smem
  int scale_stride; // padded bytes per group of scale rows in smem
  int x_stride;     // halves per staged activation row
};

__host__ __device__ inline TileGeom make_geom(int K, int rg) {
  TileGeom g;
  g.K = K;
  g.rg = rg;
  g.code_stride = rg * (K / 2) + kRowPad;
  g.scale_stride = rg * (K / 16) + kRowPad;
  g.x_stride = K + 8;  // 16 bytes of padding
  return g;
}

// Shared-memory bytes for the kGroups row groups, `xrows` staged activation
// rows and `red_floats` floats of reduction space.
__host__ __device__ inline size_t smem_bytes(const TileGeom& g, int xrows, int red_floats) {
  size_t b = 256;  // mbarrier + per-token exponents (<= 32 tokens)
  b += (size_t)kGroups * g.code_stride;
  b += (size_t)kGroups * g.scale_stride;
  b = (b + 15) & ~size_t(15);
  b += (size_t)xrows * g.x_stride * 2;
  b = (b + 15) & ~size_t(15);
  b += (size_t)red_floats * 4;
  return b;
}

struct Smem {
  uint64_t* bar;
  int* xexp;         // [32] per-token exponent p (x was multiplied by 2^-p)
  uint8_t* codes;    // [kGroups][code_stride]: rg rows of K/2 bytes each
  uint8_t* scales;   // [kGroups][scale_stride]: rg rows of K/16 bytes each
  __half* x;         // [xrows][x_stride]
  float* red;        // reduction space
};

__device__ inline Smem carve(uint8_t* base, const TileGeom& g, int xrows) {
  Smem s;
  s.bar = reinterpret_cast<uint64_t*>(base);
  s.xexp = reinterpret_cast<int*>(base + 64);
  size_t off = 256;
  s.codes = base + off;
  off += (size_t)kGroups * g.code_stride;
  s.scales = base + off;
  off += (size_t)kGroups * g.scale_stride;
  off = (off + 15) & ~size_t(15);
  s.x = reinterpret_cast<__half*>(base + off);
  off += (size_t)xrows * g.x_stride * 2;
  off = (off + 15) & ~size_t(15);
  s.red = reinterpret_cast<float*>(base + off);
  return s;
}

// Issue the bulk copies of the row groups: group q holds rows q*rg .. of
// this CTA, nvalid rows in all, starting at global code row `codes` and scale
// row `scales` (row-contiguous).  Called by warp 0.  The mbarrier must have
// been armed with expect_tx of nvalid * (K/2 + K/16) bytes.
__device__ inline void issue_groups(const Smem& s, const TileGeom& g, int nvalid, const uint8_t* codes,
                                    const uint8_t* scales) {
  const int q = threadIdx.x & 31;
  if (q >= kGroups) return;
  const int nr = min(g.rg, nvalid - q * g.rg);
  if (nr <= 0) return;
  bulk_g2s(s.codes + (size_t)q * g.code_stride, codes + (size_t)q * g.rg * (g.K / 2), (uint32_t)(nr * (g.K / 2)),
           s.bar);
  bulk_g2s(s.scales + (size_t)q * g.scale_stride, scales + (size_t)q * g.rg * (g.K / 16),
           (uint32_t)(nr * (g.K / 16)), s.bar);
}

// Stage activation rows into shared f16 with per-row power-of-two scaling.
// xrow(m) returns the bf16 row pointer (or nullptr for an all-zero row).
// Called by all threads; ends with __syncthreads().
template <typename XRow>
__device__ inline void stage_x(const Smem& s, const TileGeom& g, int nx, XRow xrow) {
  __shared__ unsigned red_max[32];
  const int tid = threadIdx.x;
  if (tid < 32) red_max[tid] = 0u;
  __syncthreads();
  const int chunks = g.K / 8;  // 16-byte chunks of 8 bf16
  // pass 1: max |x| per row (as bf16 magnitude bits; ordering of finite
  // magnitudes equals integer ordering, inf/NaN sort above).
  for (int m = 0; m < nx; ++m) {
    const uint16_t* xr = xrow(m);
    unsigned mx = 0;
    if (xr) {
      for (int c = tid; c < chunks; c += blockDim.x) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + 8 * c);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          mx = max(mx, w[j] & 0x7fffu);
          mx = max(mx, (w[j] >> 16) & 0x7fffu);
        }
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) atomicMax(&red_max[m], mx);
  }
  __syncthreads();
  if (tid < nx) {
    const unsigned e = (red_max[tid] >> 7) & 0xffu;  // biased exponent of max |x|
    // keep max|x| * 2^-p < 2^15: p = e - 127 - 14 when the exponent is >= 15
    s.xexp[tid] = (e >= 127u + 15u) ? (int)e - 127 - 14 : 0;
  }
  __syncthreads();
  // pass 2: convert
  for (int m = 0; m < nx; ++m) {
    const uint16_t* xr = xrow(m);
    const int p = s.xexp[m];
    const float sc = ldexpf(1.0f, -p);
    __half* dst = s.x + (size_t)m * g.x_stride;
    for (int c = tid; c < chunks; c += blockDim.x) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (xr) v = *reinterpret_cast<const uint4*>(xr + 8 * c);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __uint_as_float(w[j] << 16) * sc;
        const float hi = __uint_as_float(w[j] & 0xffff0000u) * sc;
        __half2 h = __floats2half2_rn(lo, hi);
        o[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();
}

// Decode the B fragment of one 16-element group for row j of group q of the
// smem tile: code bytes c and c+4 -> two f16x2 registers, times the scale.
__device__ __forceinline__ void load_b_frag(const Smem& s, const TileGeom& g, int q, int j, int grp, int c,
                                            uint32_t b[2]) {
  const uint8_t* cr = s.codes + (size_t)q * g.code_stride + (size_t)j * (g.K / 2) + (size_t)grp * 8;
  const uint2 w = *reinterpret_cast<const uint2*>(cr);
  const uint32_t sb = s.scales[(size_t)q * g.scale_stride + (size_t)j * (g.K / 16) + grp];
  const __half sh = e4m3_half(sb);
  const __half2 s2 = __halves2half2(sh, sh);
  const uint32_t su = *reinterpret_cast<const uint32_t*>(&s2);
  const uint32_t b0 = e2m1x2_to_f16x2((w.x >> (8 * c)) & 0xffu);
  const uint32_t b1 = e2m1x2_to_f16x2((w.y >> (8 * c)) & 0xffu);
  b[0] = hmul2_u32(b0, su);
  b[1] = hmul2_u32(b1, su);
}

// A fragment (tokens x 16 k) of group `grp` from staged rows
// [row0, row0 + nrows); fragment rows beyond nrows are zero.
__device__ __forceinline__ void load_a_frag(const Smem& s, const TileGeom& g, int grp, int lane,
                                            int row0, int nrows, uint32_t a[4]) {
  const int gi = lane >> 2, c = lane & 3;
  const int k = grp * 16 + 2 * c;
  const int r0 = gi, r1 = gi + 8;
  a[0] = a[1] = a[2] = a[3] = 0u;
  if (r0 < nrows) {
    const __half* xr = s.x + (size_t)(row0 + r0) * g.x_stride + k;
    a[0] = *reinterpret_cast<const uint32_t*>(xr);
    a[2] = *reinterpret_cast<const uint32_t*>(xr + 8);
  }
  if (r1 < nrows) {
    const __half* xr = s.x + (size_t)(row0 + r1) * g.x_stride + k;
    a[1] = *reinterpret_cast<const uint32_t*>(xr);
    a[3] = *reinterpret_cast<const uint32_t*>(xr + 8);
  }
}

}  // namespace qmv
}  // namespace b2
