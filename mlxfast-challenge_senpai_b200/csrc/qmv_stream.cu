// quantized_matmul (nvfp4, one weight matrix, bf16 x with M <= 32 rows,
// K <= 4096) as a streaming GEMV.
//
// Memory.  The N weight rows form sub-tiles of 8 rows (the 8 columns of an
// m16n8k16 B fragment); CTA g of G (one per SM) owns the contiguous sub-tiles
// [g*S/G, (g+1)*S/G), whose rows are one contiguous run of codes and one of
// scales in the MLX layout; all 512 threads copy it into shared memory with
// 16-byte cp.async (each warp instruction covers 512 contiguous bytes), one
// commit group per sub-tile, all issued at entry before the
// programmatic-launch dependency wait (the weights do not depend on the
// previous kernel in the stream).  Measured on this part: whole-row runs are
// needed (a row split over several SMs streamed at a fraction of the
// bandwidth), and issuing one bulk copy per row cost ~1.5 us per CTA at entry
// (the copy engine takes the issues one at a time), which many-thread
// cp.async avoids.  Rows are padded in shared memory (codes to 32 mod 128
// bytes, scales to an odd multiple of 16 bytes) so the fragment loads below
// are free of bank conflicts.
//
// Compute.  W warps split K: warp w owns the 64-element quads q = w, w + W,
// ... (W = 16 with 4 quads each, or 32 with 2 each for x of at most 8 rows).  It loads the x values of its quads for one 16-row tile of
// x straight into MMA fragment registers (f16, scaled by a power of two per
// row and warp that keeps the warp's largest |x| below 2^15: exact for every
// bf16 value above 2^-17 of it; undone on the f32 partial).  Inside a quad,
// thread (g, c) of the warp (g = lane / 4, c = lane % 4) loads the 8 code
// bytes of group 4q + c of weight row g (16 consecutive k) and their scale,
// and feeds four MMAs: MMA j takes code bytes 2j, 2j+1, which hold k =
// 16c + 4j + {0, 1} and {2, 3} of the quad.  That assignment of k to the
// MMA's k slots (2c, 2c+1) and (2c+8, 2c+9) is a permutation of the quad's
// 64 k; the x fragments use the same permutation, so each MMA still sums
// matching products, and each thread decodes one scale per 16 weights.
// Codes become f16 with cvt.rn.f16x2.e2m1x2 and are multiplied by the f16
// scale (exact).  Four accumulator sets (one per MMA of a quad) keep four
// independent MMA chains in flight.  x with more than 16 rows is processed
// in 16-row passes over the resident weights.
//
// Reduction, in a fixed order: a warp's four chains, then the W warps of a
// sub-tile through shared memory once the pass is done.  A row's result
// therefore does not depend on M or on the other rows of x.
#include <algorithm>
#include <mutex>
#include <vector>

#include "moe.cuh"
#include "qmv.cuh"

namespace b2 {
namespace qmvs {

// 16 warps split K, 4 quads each.  Measured alternatives that were slower
// at M = 1 (4096 x 4096): 32 warps of 2 quads (8.6 vs 7.0 us) and 64
// registers per thread so that two CTAs (this launch's and the next one's,
// programmatic dependent launch) share an SM (9.8 us; register spills).
template <bool HALF>
struct Cfg {
  static constexpr int kWarps = 16;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kQPW = 4;  // quads per warp
};
constexpr int kMaxK = 16 * 4 * 64;  // both configurations cover K <= 4096
constexpr int kMaxSub = 16;  // sub-tiles per CTA (commit groups in flight)

struct Args {
  const uint16_t* x;
  const uint8_t* codes;
  const uint8_t* scales;
  uint16_t* y;
  int M, N, K;
  int QC;          // quads of K
  int S, G;        // sub-tiles, CTAs
  int cstride;     // shared-memory row stride of codes
  int sstride;     // shared-memory row stride of scales
  int sub_bytes;   // shared-memory bytes of one sub-tile (codes then scales)
  int off_red;     // per-warp partials [sub-tile][warp][128 floats]
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Wait until at most n (0..kMaxSub-1) of this thread's commit groups are
// pending.
__device__ __forceinline__ void cp_async_wait_pending(int n) {
  switch (n) {
#define B2_WAIT_CASE(i) \
  case i:               \
    asm volatile("cp.async.wait_group " #i ";" ::: "memory"); \
    break;
    B2_WAIT_CASE(0) B2_WAIT_CASE(1) B2_WAIT_CASE(2) B2_WAIT_CASE(3) B2_WAIT_CASE(4) B2_WAIT_CASE(5)
    B2_WAIT_CASE(6) B2_WAIT_CASE(7) B2_WAIT_CASE(8) B2_WAIT_CASE(9) B2_WAIT_CASE(10) B2_WAIT_CASE(11)
    B2_WAIT_CASE(12) B2_WAIT_CASE(13) B2_WAIT_CASE(14)
#undef B2_WAIT_CASE
    default:
      asm volatile("cp.async.wait_group 15;" ::: "memory");
  }
}
__device__ __forceinline__ unsigned absmax8(const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  unsigned mx = 0;
#pragma unroll
  for (int h = 0; h < 4; ++h) mx = max(mx, max(w[h] & 0x7fffu, (w[h] >> 16) & 0x7fffu));
  return mx;
}
// 8 bf16 (one uint4) times 2^-p -> 4 f16x2 registers
__device__ __forceinline__ void to_f16x8(const uint4& v, float sc, uint32_t* o) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    __half2 hh = __floats2half2_rn(__uint_as_float(w[h] << 16) * sc, __uint_as_float(w[h] & 0xffff0000u) * sc);
    o[h] = *reinterpret_cast<uint32_t*>(&hh);
  }
}

// HALF: the 16-row tile has rows gi only (M <= 8), so the fragment rows
// gi + 8 are zero and are neither loaded nor held.
template <bool HALF>
__global__ void __launch_bounds__(Cfg<HALF>::kThreads, 1) qmv_stream_kernel(const Args a) {
  constexpr int kWarps = Cfg<HALF>::kWarps, kThreads = Cfg<HALF>::kThreads, kQPW = Cfg<HALF>::kQPW;
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s0 = (int)((int64_t)blockIdx.x * a.S / a.G);
  const int s1 = (int)((int64_t)(blockIdx.x + 1) * a.S / a.G);
  const int ns = s1 - s0;
  const int row0 = s0 * 8;
  const int R = min(ns * 8, a.N - row0);  // weight rows of this CTA
  const int K = a.K, M = a.M;
  float* red = reinterpret_cast<float*>(sm + a.off_red);

  // ---- weights: sub-tile j's rows in 16-byte chunks (K/32 of codes, then
  // K/256 of scales per row), one commit group per sub-tile
  {
    const int cpr = K / 32, spr = K / 256, per_row = cpr + spr;
    for (int j = 0; j < ns; ++j) {
      uint8_t* sub = sm + (size_t)j * a.sub_bytes;
      const int rows = min(8, R - 8 * j);
      for (int ch = tid; ch < rows * per_row; ch += kThreads) {
        const int r = ch / per_row, c = ch % per_row;
        const int64_t n = row0 + 8 * j + r;
        if (c < cpr)
          cp_async16(sub + r * a.cstride + 16 * c, a.codes + n * (K / 2) + 16 * c);
        else
          cp_async16(sub + 8 * a.cstride + r * a.sstride + 16 * (c - cpr), a.scales + n * (K / 16) + 16 * (c - cpr));
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }

  // ---- x depends on the previous kernel in the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int gi = lane >> 2, c = lane & 3;
  constexpr int NH = HALF ? 1 : 2;
  for (int m0 = 0; m0 < M; m0 += 16) {
    // x fragments of this warp's quads: rows m0 + gi (+ 8), 16 halves
    // k = 64q + 16c .. + 15 per row and quad
    uint32_t A[kQPW][NH][8];
    int pexp[NH];
#pragma unroll
    for (int hf = 0; hf < NH; ++hf) {
      const int m = m0 + gi + 8 * hf;
      uint4 v[kQPW][2];
      unsigned mx = 0;
#pragma unroll
      for (int qi = 0; qi < kQPW; ++qi) {
        const int q = warp + kWarps * qi;
        v[qi][0] = v[qi][1] = make_uint4(0, 0, 0, 0);
        if (q < a.QC && m < M) {
          const uint4* src = reinterpret_cast<const uint4*>(a.x + (int64_t)m * K + 64 * q + 16 * c);
          v[qi][0] = src[0];
          v[qi][1] = src[1];
        }
      }
#pragma unroll
      for (int qi = 0; qi < kQPW; ++qi) mx = max(mx, max(absmax8(v[qi][0]), absmax8(v[qi][1])));
      // the row's maximum over the warp's quads (the 4 lanes of row gi)
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const unsigned e = (mx >> 7) & 0xffu;
      const int p = (e >= 127u + 15u) ? (int)e - 127 - 14 : 0;
      pexp[hf] = p;
      const float scl = __int_as_float((127 - p) << 23);  // 2^-p, 0 <= p <= 114
#pragma unroll
      for (int qi = 0; qi < kQPW; ++qi) {
        to_f16x8(v[qi][0], scl, &A[qi][hf][0]);
        to_f16x8(v[qi][1], scl, &A[qi][hf][4]);
      }
    }

    for (int j = 0; j < ns; ++j) {
      if (m0 == 0) {
        // this thread's copies of sub-tile j have landed; after the barrier
        // every thread's have (later passes find them resident)
        cp_async_wait_pending(ns - 1 - j);
        __syncthreads();
      }
      float acc[4][4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[jj][e] = 0.0f;
      const uint8_t* sub = sm + (size_t)j * a.sub_bytes;
      const uint8_t* crow = sub + gi * a.cstride + 8 * c;
      const uint8_t* srow = sub + 8 * a.cstride + gi * a.sstride + c;
      {
#pragma unroll
        for (int qi = 0; qi < kQPW; ++qi) {
          const int q = warp + kWarps * qi;
          if (q < a.QC) {
            const uint2 w = *reinterpret_cast<const uint2*>(crow + 32 * q);
            const __half sh = e4m3_half(srow[4 * q]);
            const __half2 s2 = __halves2half2(sh, sh);
            const uint32_t su = *reinterpret_cast<const uint32_t*>(&s2);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const uint32_t wd = jj < 2 ? w.x : w.y;
              uint32_t bf[2];
              bf[0] = hmul2_u32((jj & 1) ? cvt_byte<2>(wd) : cvt_byte<0>(wd), su);
              bf[1] = hmul2_u32((jj & 1) ? cvt_byte<3>(wd) : cvt_byte<1>(wd), su);
              const uint32_t af[4] = {A[qi][0][2 * jj], HALF ? 0u : A[qi][NH - 1][2 * jj], A[qi][0][2 * jj + 1],
                                      HALF ? 0u : A[qi][NH - 1][2 * jj + 1]};
              mma_16816_f16(acc[jj], af, bf);
            }
          }
        }
      }
      float* rb = red + ((size_t)j * kWarps + warp) * 128;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (!HALF || e < 2)
          rb[e * 32 + lane] = mul_pow2(((acc[0][e] + acc[1][e]) + acc[2][e]) + acc[3][e], pexp[HALF ? 0 : (e >> 1)]);
    }
    __syncthreads();
    // 16 warps -> bf16 outputs of this pass, summed in warp order
    const int per_sub = HALF ? 64 : 128;
    for (int t = tid; t < ns * per_sub; t += kThreads) {
      const int j = t / per_sub, u = t % per_sub;
      const float* src = red + (size_t)j * kWarps * 128 + u;
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += src[(size_t)w * 128];
      const int ln = u & 31, e = u >> 5;
      const int m = m0 + (ln >> 2) + (e >= 2 ? 8 : 0);
      const int r = 8 * j + 2 * (ln & 3) + (e & 1);
      if (m < M && r < R) a.y[(int64_t)m * a.N + row0 + r] = f32_to_bf16_bits(v);
    }
    __syncthreads();  // the partials are rewritten by the next pass
  }
}

// CTAs of the kernel at `smem` bytes resident at once, one per SM.
int resident_ctas(const void* fn, int threads, size_t smem) {
  int dev = 0;
  cudaGetDevice(&dev);
  struct Entry {
    int dev;
    const void* fn;
    size_t smem;
    int n;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& en : cache)
    if (en.dev == dev && en.fn == fn && en.smem == smem) return en.n;
  int sms = 148, per_sm = 1;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem) != cudaSuccess) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  const int n = per_sm >= 1 ? sms : 1;
  cache.push_back({dev, fn, smem, n});
  return n;
}

}  // namespace qmvs

int qmv_stream(const uint16_t* x, const uint8_t* codes, const uint8_t* scales, int M, int N, int K, uint16_t* y,
               cudaStream_t st) {
  using namespace qmvs;
  if (M < 1 || M > 32 || K % 256 != 0 || K > kMaxK || N < 1) return 1;
  Args a = {};
  a.x = x;
  a.codes = codes;
  a.scales = scales;
  a.y = y;
  a.M = M;
  a.N = N;
  a.K = K;
  a.QC = K / 64;
  a.S = (N + 7) / 8;
  const int cb = K / 2;
  a.cstride = cb + ((32 - cb % 128) + 128) % 128;
  int sbytes = K / 16;  // a multiple of 16
  if ((sbytes / 16) % 2 == 0) sbytes += 16;
  a.sstride = sbytes;
  a.sub_bytes = (8 * (a.cstride + a.sstride) + 127) / 128 * 128;
  const bool half = M <= 8;
  const int warps = half ? Cfg<true>::kWarps : Cfg<false>::kWarps;
  const size_t per_sub = (size_t)a.sub_bytes + (size_t)warps * 128 * 4;
  const size_t budget = 200 * 1024;
  const int ns_cap = (int)std::min<size_t>(kMaxSub, budget / per_sub);
  const void* fn = half ? (const void*)qmv_stream_kernel<true> : (const void*)qmv_stream_kernel<false>;
  int rc = ensure_dynamic_smem(fn, budget, "quantized_matmul");
  if (rc) return rc;
  // one CTA per SM, never more than the sub-tiles; more (a second wave) only
  // when a CTA would otherwise hold more sub-tiles than fit
  const int G = std::max(std::min(a.S, resident_ctas(fn, warps * 32, budget)), (a.S + ns_cap - 1) / ns_cap);
  const int ns = (a.S + G - 1) / G;
  a.G = G;
  a.off_red = ns * a.sub_bytes;
  const size_t smem = (size_t)ns * per_sub;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3((unsigned)(warps * 32));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = qmv_pdl_enabled() ? 1 : 0;
  void* args[] = {(void*)&a};
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess && cfg.numAttrs == 1) {
    (void)cudaGetLastError();
    cfg.numAttrs = 0;
    e = cudaLaunchKernelExC(&cfg, fn, args);
  }
  return e == cudaSuccess ? 0 : check_cuda(e, "quantized_matmul");
}

}  // namespace b2
