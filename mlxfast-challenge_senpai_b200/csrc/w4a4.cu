// W4A4 path: NVFP4 activations x NVFP4 weights on the block-scaled tensor
// cores (tcgen05.mma kind::mxf4nvf4, one UE4M3 scale per 16 values).
//
// Semantics: the reference's qqmm in nvfp4 mode (MLX/ops.h:1524 qqmm,
// MLXC/ops.h:790 mlx_qqmm; CPU QQMatmul::eval_cpu,
// MLX/backend/cpu/quantized.cpp:1322-1360): the activations are quantized to
// NVFP4 by the reference's rule (fp_quantize_dequantize, :1094-1129: scale
// byte e4m3(max|x|/6), code by the threshold rounding of to_fp4_e2m1,
// :1064-1091), then y = xq . Wq^T accumulated in f32 -- on its CUDA backend
// the same product runs on cuBLASLt with CUDA_R_4F_E2M1 operands and
// VEC16_UE4M3 scales (MLX/backend/cuda/quantized/cublas_qqmm.cpp:19-32).
// The products E2M1 x E2M1 x scale x scale are exact in f32, so the result
// differs from an f32 restatement only by summation order.  Scale bytes are
// read with the hardware's UE4M3 meaning: MLX's quantizers produce bytes in
// [0, 0x7e], where both decodings agree (0x7f -- 480 for MLX, NaN for UE4M3
// -- and sign bits never come out of them).
//
// GEMM tile: A = 128 weight rows (M of the MMA), B = nt token rows (N of the
// MMA, nt = 128 or 256), D [128 x nt] f32 in TMEM; K in stages of 256 values
// (128 bytes per row, one 128-byte swizzle row) brought by tiled TMA copies
// of the packed codes and of the rows' 16 scale bytes of the stage; per
// stage 4 MMAs of K = 64.  The scale factors go shared memory -> registers
// -> TMEM (tcgen05.st) in the layout the MMA reads: for each MMA, 32-bit
// column c of TMEM lane l (replicated in all four lane quarters) holds the 4
// scale bytes (K groups 0..3 of that MMA) of row 32c + (l % 32).  (Loading
// the scale bytes from global memory in the scale warps instead serialised
// the pipeline on their ~2,400-cycle load latency, one stage at a time.)
// Epilogue: the accumulator is rounded to bf16 into shared memory (the
// drained stage buffers) and written out as 16-byte row chunks.
// Warp roles (9 warps): 0 and 6-8 TMA producers taking the stages in turn
// (producer i issues every stage g with g % 4 == i: one issuing thread keeps
// about one copy in flight, so a single producer left each 48 KB stage
// ~2 us in flight), 1 TMEM owner + MMA issuer, 2-5 scale loaders and the
// epilogue (TMEM lane quarter = warp % 4).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace b2 {
namespace w4 {
namespace {

constexpr int kStages = 4;
constexpr int kBK = 128;                  // bytes of K per stage per row (256 values)
constexpr int kABytes = 128 * kBK;        // 16 KB
constexpr int kBBytesMax = 256 * kBK;     // 32 KB
constexpr int kSfABytes = 128 * 16;        // 16 scale bytes per weight row
constexpr int kSfBBytesMax = 256 * 16;     // 16 scale bytes per token row
constexpr int kStageBytes = kABytes + kBBytesMax + kSfABytes + kSfBBytesMax;
static_assert(kStageBytes % 1024 == 0, "swizzled operands stay 1024-byte aligned");
constexpr int kSmem = kStages * kStageBytes + 1024;
constexpr int kSfSlots = 4;
constexpr int kSfaCols = 16;              // 4 MMAs x 4 columns
constexpr int kSfbColsMax = 32;           // 4 MMAs x 8 columns (nt = 256)
constexpr int kSfSlotCols = kSfaCols + kSfbColsMax;
constexpr uint32_t kSfBase = 256;         // after the accumulator (nt <= 256 columns)
constexpr uint32_t kTmemCols = 512;
static_assert(kSfBase + kSfSlots * kSfSlotCols <= kTmemCols, "TMEM budget");
constexpr int kProducers = 4;
static_assert(kProducers == kStages, "producer i owns stage slot i");
constexpr int kThreads = 288;
constexpr uint32_t kWaitLimit = 1u << 22;

struct Params {
  const uint8_t* sfa;  // weight scales [Nw, K/16]
  const uint8_t* sfb;  // activation scales [M, K/16]
  uint16_t* y;         // [M, Nw] bf16
  unsigned* status;
  int M, Nw, K, nt;
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  // K-major operand, 128-byte swizzle: start >> 4, LBO 16 B, SBO 1024 B,
  // descriptor version 1, layout type 2 (SWIZZLE_128B)
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status) {
  if (*abort_flag) return;
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 255u) == 255u && *abort_flag) return;
  }
  *abort_flag = 1;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mma_nvf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}


__device__ __forceinline__ uint32_t word_of(const uint4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

__global__ void __launch_bounds__(kThreads, 1) w4a4_gemm_kernel(Params p, const __grid_constant__ CUtensorMap map_a,
                                                                 const __grid_constant__ CUtensorMap map_b,
                                                                 const __grid_constant__ CUtensorMap map_sa,
                                                                 const __grid_constant__ CUtensorMap map_sb) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], sfull[kSfSlots], sempty[kSfSlots], accf;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * p.nt;
  const int KS = p.K / 256;
  const int nt = p.nt;
  const int sfb_per_mma = nt / 32;  // 4 or 8 columns

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kSfSlots; ++i) {
      mbar_init(&sfull[i], 4);  // the four scale-loading warps
      mbar_init(&sempty[i], 1);
    }
    mbar_init(&accf, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  volatile int* abort_flag = &s_abort;

  if (warp == 0 || warp >= 6) {
    if (lane == 0) {
      const int pi = warp == 0 ? 0 : warp - 5;  // this producer's stage slot
      const uint32_t tx = (uint32_t)kABytes + (uint32_t)nt * kBK + (uint32_t)kSfABytes + (uint32_t)nt * 16u;
      int last = -1;
      for (int g = pi; g < KS; g += kProducers) {
        wait_bar(&empty[pi], ((g / kStages) & 1) ^ 1, abort_flag, p.status);
        if (*abort_flag) break;
        uint8_t* st = base + pi * kStageBytes;
        mbar_expect_tx(&full[pi], tx);
        tma_load_2d(st, &map_a, g * kBK, m0, &full[pi]);
        tma_load_2d(st + kABytes, &map_b, g * kBK, n0, &full[pi]);
        tma_load_2d(st + kABytes + kBBytesMax, &map_sa, g * 16, m0, &full[pi]);
        tma_load_2d(st + kABytes + kBBytesMax + kSfABytes, &map_sb, g * 16, n0, &full[pi]);
        last = g;
      }
      // no copy may still be in flight into shared memory at exit (this
      // producer's slot holds at most its last stage)
      if (last >= 0) mbar_wait_bounded(&full[pi], (last / kStages) & 1, p.status, kWaitLimit);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = (1u << 7) | (1u << 10) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
      for (int g = 0; g < KS; ++g) {
        const int sl = g % kStages, ss = g % kSfSlots;
        wait_bar(&full[sl], (g / kStages) & 1, abort_flag, p.status);
        wait_bar(&sfull[ss], (g / kSfSlots) & 1, abort_flag, p.status);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (!*abort_flag) {
          const uint32_t sa = smem_u32(base + sl * kStageBytes);
          const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sa + kABytes);
          const uint32_t sfa = tmem + kSfBase + ss * kSfSlotCols;
          const uint32_t sfb = sfa + kSfaCols;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_nvf4(tmem, ad + 2 * j, bd + 2 * j, idesc, sfa + 4 * j, sfb + sfb_per_mma * j, (g | j) ? 1u : 0u);
        }
        mma_commit(&empty[sl]);
        mma_commit(&sempty[ss]);
      }
      mma_commit(&accf);
    }
  } else {
    // scale loaders: TMEM lane quarter q, lane l; every quarter writes the
    // same (replicated) columns
    const int q = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    for (int g = 0; g < KS; ++g) {
      const int ss = g % kSfSlots, sl = g % kStages;
      wait_bar(&sempty[ss], ((g / kSfSlots) & 1) ^ 1, abort_flag, p.status);
      wait_bar(&full[sl], (g / kStages) & 1, abort_flag, p.status);  // the stage's scale bytes landed
      const uint32_t col = kSfBase + ss * kSfSlotCols;
      const uint8_t* sfa_s = base + sl * kStageBytes + kABytes + kBBytesMax;
      const uint8_t* sfb_s = sfa_s + kSfABytes;
      {
        uint4 v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = *reinterpret_cast<const uint4*>(sfa_s + (lane + 32 * c) * 16);
        uint32_t r[16];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) r[4 * j + c] = word_of(v[c], j);
        tmem_st16(lane_base + col, r);
      }
      if (nt == 128) {
        uint4 v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = *reinterpret_cast<const uint4*>(sfb_s + (lane + 32 * c) * 16);
        uint32_t r[16];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) r[4 * j + c] = word_of(v[c], j);
        tmem_st16(lane_base + col + kSfaCols, r);
      } else {
        uint4 v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) v[c] = *reinterpret_cast<const uint4*>(sfb_s + (lane + 32 * c) * 16);
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // MMAs 2h, 2h+1: 16 columns
          uint32_t r[16];
#pragma unroll
          for (int jj = 0; jj < 2; ++jj)
#pragma unroll
            for (int c = 0; c < 8; ++c) r[8 * jj + c] = word_of(v[c], 2 * h + jj);
          tmem_st16(lane_base + col + kSfaCols + 16 * h, r);
        }
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfull[ss]);
    }
    // epilogue: weight row m0 + 32q + lane, tokens n0 .. n0 + nt
    wait_bar(&accf, 0, abort_flag, p.status);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // every stage has been consumed by the MMAs (accf), so the stage
    // buffers are free: bf16 tile [nt tokens][128 weight rows] there
    uint16_t* tile = reinterpret_cast<uint16_t*>(base);
    const int ml = 32 * q + lane;
    for (int c0 = 0; c0 < nt; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(lane_base + (uint32_t)c0, v);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int j = 0; j < 16; ++j) tile[(c0 + j) * 128 + ml] = f32_to_bf16_bits(__uint_as_float(v[j]));
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
    if (!*abort_flag) {
      const int et = tid - 64;  // 0..127 over warps 2-5
      const bool vec = (p.Nw % 8) == 0;
      for (int idx = et; idx < nt * 16; idx += 128) {
        const int n = idx >> 4, ch = idx & 15;
        const int row = n0 + n, col0 = m0 + 8 * ch;
        if (row >= p.M || col0 >= p.Nw) continue;
        const uint16_t* src = tile + n * 128 + 8 * ch;
        uint16_t* dst = p.y + (int64_t)row * p.Nw + col0;
        if (vec && col0 + 8 <= p.Nw) {
          *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        } else {
          for (int j = 0; j < 8 && col0 + j < p.Nw; ++j) dst[j] = src[j];
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1) {
    // every MMA has completed before TMEM is released (accf fired, or the
    // abort path: wait for the last commit)
    if (lane == 0) mbar_wait_bounded(&accf, 0, p.status, kWaitLimit);
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Activation quantizer (the reference qqmm's rule): one thread per
// 16-element group of bf16 x.  The rule codes rn(x / scale) by thresholds
// t in {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5} (">" at 0.25, 1.25, 2.5, 5 and
// ">=" at the others).  Here |x| is compared with t * scale instead, with no
// division and no branches, and the result is the same: t * scale is exact
// in f32 (t has at most 3 and an E4M3 scale at most 4 significant bits), and
// x is a bf16 value (at most 8 significant bits), so unless |x| == t * scale
// the two differ by at least 2^-9 of t * scale -- far more than the 2^-24
// relative rounding of x / scale, which therefore lies on the same side of t
// as |x| / scale does, and equality holds for both at once.  A zero scale
// codes every value 0 (the rule divides nothing then); NaN codes 7.
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

// Scale bytes [rows][K/16], box 16 bytes (one K stage) x box_rows, no swizzle.
int scales_map(const void* scales, uint64_t rows, uint64_t K, uint32_t box_rows, CUtensorMap* out) {
  auto enc = encoder();
  B2_REQUIRE(enc != nullptr, "[w4a4] cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {K / 16, rows};
  const cuuint64_t strides[1] = {K / 16};
  const cuuint32_t box[2] = {16u, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(scales), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2_REQUIRE(r == CUDA_SUCCESS, "[w4a4] tensor map encoding failed (%d)", (int)r);
  return B2_OK;
}

// Packed codes [rows][K/2] bytes, box 128 bytes x box_rows, 128-byte swizzle.
int codes_map(const void* codes, uint64_t rows, uint64_t K, uint32_t box_rows, CUtensorMap* out) {
  auto enc = encoder();
  B2_REQUIRE(enc != nullptr, "[w4a4] cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {K / 2, rows};
  const cuuint64_t strides[1] = {K / 2};
  const cuuint32_t box[2] = {128u, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(codes), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2_REQUIRE(r == CUDA_SUCCESS, "[w4a4] tensor map encoding failed (%d)", (int)r);
  return B2_OK;
}

}  // namespace

__global__ void quantize_activations_kernel(const uint16_t* __restrict__ x, int64_t groups,
                                            uint32_t* __restrict__ codes, uint8_t* __restrict__ scales) {
  const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const uint4 a = reinterpret_cast<const uint4*>(x)[2 * g];
  const uint4 b = reinterpret_cast<const uint4*>(x)[2 * g + 1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float v[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
  float amax = fabsf(v[0]);
#pragma unroll
  for (int i = 1; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const uint32_t sb = e4m3_encode_scale(__fdiv_rn(amax, 6.0f));
  const float sd = e4m3_value(sb);
  uint32_t c0 = 0, c1 = 0;
  if (sd != 0.0f) {
    const float t0 = 0.25f * sd, t1 = 0.75f * sd, t2 = 1.25f * sd, t3 = 1.75f * sd;
    const float t4 = 2.5f * sd, t5 = 3.5f * sd, t6 = 5.0f * sd;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = fabsf(v[i]);
      uint32_t c = (uint32_t)(a > t0) + (uint32_t)(a >= t1) + (uint32_t)(a > t2) + (uint32_t)(a >= t3) +
                   (uint32_t)(a > t4) + (uint32_t)(a >= t5) + (uint32_t)(a > t6);
      c |= (__float_as_uint(v[i]) >> 28) & 0x8u;  // sign
      if (a != a) c = 0x7u;                       // NaN
      if (i < 8) c0 |= c << (4 * i); else c1 |= c << (4 * (i - 8));
    }
  }
  codes[2 * g] = c0;
  codes[2 * g + 1] = c1;
  scales[g] = (uint8_t)sb;
}

int gemm(const uint32_t* xq, const uint8_t* xs, const uint32_t* wq, const uint8_t* ws, int64_t M, int64_t N, int64_t K,
         uint16_t* y, cudaStream_t st) {
  Params p;
  p.sfa = ws;
  p.sfb = xs;
  p.y = y;
  p.status = device_status_ptr();
  B2_REQUIRE(p.status != nullptr, "[w4a4] device status word unavailable");
  p.M = (int)M;
  p.Nw = (int)N;
  p.K = (int)K;
  p.nt = M <= 128 ? 128 : 256;
  CUtensorMap ma, mb;
  int rc = codes_map(wq, (uint64_t)N, (uint64_t)K, 128u, &ma);
  if (rc) return rc;
  rc = codes_map(xq, (uint64_t)M, (uint64_t)K, (uint32_t)p.nt, &mb);
  if (rc) return rc;
  CUtensorMap msa, msb;
  rc = scales_map(ws, (uint64_t)N, (uint64_t)K, 128u, &msa);
  if (rc) return rc;
  rc = scales_map(xs, (uint64_t)M, (uint64_t)K, (uint32_t)p.nt, &msb);
  if (rc) return rc;
  rc = ensure_dynamic_smem((const void*)w4a4_gemm_kernel, kSmem, "w4a4 gemm");
  if (rc) return rc;
  dim3 grid((unsigned)((N + 127) / 128), (unsigned)((M + p.nt - 1) / p.nt));
  w4a4_gemm_kernel<<<grid, kThreads, kSmem, st>>>(p, ma, mb, msa, msb);
  B2_CHECK_LAUNCH("w4a4 gemm");
  return B2_OK;
}

int quantize_activations(const uint16_t* x, int64_t rows, int64_t K, uint32_t* codes, uint8_t* scales,
                         cudaStream_t st) {
  const int64_t groups = rows * (K / 16);
  if (groups == 0) return B2_OK;
  quantize_activations_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, st>>>(x, groups, codes, scales);
  B2_CHECK_LAUNCH("quantize_activations");
  return B2_OK;
}

}  // namespace w4
}  // namespace b2

extern "C" int b2_fp_quantize_activations(const uint16_t* x, int64_t rows, int64_t K, uint32_t* codes,
                                          uint8_t* scales, b2_stream_t stream) {
  B2_REQUIRE(x && codes && scales, "[quantize_activations] null pointer argument");
  B2_REQUIRE(rows >= 0 && K > 0 && K % 16 == 0,
             "[quantize_activations] the last dimension (%lld) must be divisible by the nvfp4 group size 16",
             (long long)K);
  B2_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(codes) % 8 == 0,
             "[quantize_activations] x must be 16-byte aligned and codes 8-byte aligned");
  return b2::w4::quantize_activations(x, rows, K, codes, scales, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b2_nvfp4_gemm(const uint32_t* x_codes, const uint8_t* x_scales, const uint32_t* w_codes,
                             const uint8_t* w_scales, int64_t M, int64_t N, int64_t K, uint16_t* y,
                             b2_stream_t stream) {
  B2_REQUIRE(x_codes && x_scales && w_codes && w_scales && y, "[nvfp4_gemm] null pointer argument");
  B2_REQUIRE(M > 0 && N > 0 && K > 0 && K % 256 == 0, "[nvfp4_gemm] needs positive M, N and K %% 256 == 0");
  B2_REQUIRE(M <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX, "[nvfp4_gemm] shape too large");
  const auto al = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  B2_REQUIRE(al(x_codes) && al(x_scales) && al(w_codes) && al(w_scales),
             "[nvfp4_gemm] codes and scales must be 16-byte aligned");
  return b2::w4::gemm(x_codes, x_scales, w_codes, w_scales, M, N, K, y, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t b2_qqmm_workspace_size(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return (size_t)((M * K / 2 + 255) / 256 * 256) + (size_t)(M * K / 16);
}

extern "C" int b2_qqmm(const uint16_t* x, const uint32_t* w_codes, const uint8_t* w_scales, int64_t M, int64_t N,
                       int64_t K, uint16_t* y, void* workspace, size_t workspace_bytes, b2_stream_t stream) {
  B2_REQUIRE(x && workspace, "[qqmm] null pointer argument");
  B2_REQUIRE(workspace_bytes >= b2_qqmm_workspace_size(M, K), "[qqmm] workspace too small (%zu < %zu)",
             workspace_bytes, b2_qqmm_workspace_size(M, K));
  B2_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "[qqmm] workspace must be 256-byte aligned");
  uint32_t* xq = static_cast<uint32_t*>(workspace);
  uint8_t* xs = static_cast<uint8_t*>(workspace) + (M * K / 2 + 255) / 256 * 256;
  int rc = b2_fp_quantize_activations(x, M, K, xq, xs, stream);
  if (rc) return rc;
  return b2_nvfp4_gemm(xq, xs, w_codes, w_scales, M, N, K, y, stream);
}
