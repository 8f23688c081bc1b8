// MoE router: logits (fixed summation order) and top-k selection.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <vector>

#include "router.cuh"

#include <type_traits>

namespace b2 {
namespace {

template <typename W>
__device__ __forceinline__ float4 load_w4(const W* w, int64_t idx);
template <>
__device__ __forceinline__ float4 load_w4<float>(const float* w, int64_t idx) {
  return *reinterpret_cast<const float4*>(w + idx);
}
template <>
__device__ __forceinline__ float4 load_w4<__nv_bfloat16>(const __nv_bfloat16* w, int64_t idx) {
  const uint2 v = *reinterpret_cast<const uint2*>(w + idx);
  return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                     __uint_as_float(v.y & 0xffff0000u));
}

// The logit's value in MLX's result type of x.matmul(w.T): a bf16 router
// weight times bf16 tokens gives bf16 logits (rounded once, from the f32
// sum), which the gate then casts to f32 (Laguna.swift:166; the runtime's
// fused router stores bfloat(router_result), RM:833-838); an f32 weight
// promotes to f32 and leaves the sum as it is.
template <typename W>
__device__ __forceinline__ float logit_value(float a) {
  return std::is_same<W, __nv_bfloat16>::value ? round_bf16(a) : a;
}

// CTA = 8 warps; warp w owns EW experts, the CTA owns TT tokens whose rows are
// staged in shared memory.  Per (token, expert) the accumulation order is the
// contract of b2_moe_router_logits: lane l sums chunks c = l, l+32, ... (4
// elements each, fma in element order), then an xor butterfly.
template <typename W, int EW, int TT>
__global__ void __launch_bounds__(256)
router_logits_kernel(const uint16_t* __restrict__ x, const W* __restrict__ wr, int rows, int E, int H,
                     float* __restrict__ logits) {
  extern __shared__ __align__(16) uint16_t xs[];  // [TT][H]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * TT;
  const int tn = min(TT, rows - t0);
  // stage x rows (16-byte chunks)
  const int chunks8 = H / 8;
  for (int i = threadIdx.x; i < TT * chunks8; i += blockDim.x) {
    const int t = i / chunks8, c = i % chunks8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < tn) v = *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + t) * H + 8 * c);
    *reinterpret_cast<uint4*>(xs + (size_t)t * H + 8 * c) = v;
  }
  __syncthreads();
  const int e0 = (blockIdx.x * 8 + warp) * EW;
  float acc[TT][EW];
#pragma unroll
  for (int t = 0; t < TT; ++t)
#pragma unroll
    for (int e = 0; e < EW; ++e) acc[t][e] = 0.0f;
  const int chunks = H / 4;
  // the next chunk's router values are fetched while this one is used
  float4 wv[EW], wn[EW];
#pragma unroll
  for (int e = 0; e < EW; ++e) wv[e] = load_w4<W>(wr, (int64_t)min(e0 + e, E - 1) * H + 4 * lane);
  for (int c = lane; c < chunks; c += 32) {
    if (c + 32 < chunks) {
#pragma unroll
      for (int e = 0; e < EW; ++e) wn[e] = load_w4<W>(wr, (int64_t)min(e0 + e, E - 1) * H + 4 * (c + 32));
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const uint2 xv = *reinterpret_cast<const uint2*>(xs + (size_t)t * H + 4 * c);
      const float x0 = __uint_as_float(xv.x << 16), x1 = __uint_as_float(xv.x & 0xffff0000u);
      const float x2 = __uint_as_float(xv.y << 16), x3 = __uint_as_float(xv.y & 0xffff0000u);
#pragma unroll
      for (int e = 0; e < EW; ++e) {
        float a = acc[t][e];
        a = fmaf(x0, wv[e].x, a);
        a = fmaf(x1, wv[e].y, a);
        a = fmaf(x2, wv[e].z, a);
        a = fmaf(x3, wv[e].w, a);
        acc[t][e] = a;
      }
    }
#pragma unroll
    for (int e = 0; e < EW; ++e) wv[e] = wn[e];
  }
#pragma unroll
  for (int t = 0; t < TT; ++t)
#pragma unroll
    for (int e = 0; e < EW; ++e) {
      float a = acc[t][e];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) a = a + __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0 && t < tn && e0 + e < E) logits[(int64_t)(t0 + t) * E + e0 + e] = logit_value<W>(a);
    }
}

// Prefill: CTA = 32 tokens x 16 experts, K streamed in slabs of 256 that the
// TMA engine copies into a ring of three shared-memory buffers (x as bf16,
// router rows in their own type; rows past the tensors read as zeros), two
// slabs ahead of the warps (a slab's copy takes longer to land than its
// compute: one slab ahead left the warps waiting).  Warp w owns tokens 8(w%4).. and
// experts 8(w/4).., so every lane keeps 8 x 8 accumulators (as 4 token
// pairs x 8 experts of packed f32x2 FMAs: the kernel is issue bound) and each
// shared-memory load feeds 16 or 32 FMAs.  Lane l still sums exactly the
// chunks c = l, l+32, ... in increasing c (slab after slab), 4 elements per
// chunk with fma in element order, then the same xor butterfly: the same
// bits as router_logits_kernel.
constexpr int RT_T = 32, RT_E = 16, RT_SLAB = 256, RT_BUFS = 3;
constexpr uint32_t kRouterWaitLimit = 1u << 24;
template <typename W>
__host__ __device__ constexpr size_t router_buf_bytes() {
  return (size_t)RT_T * RT_SLAB * 2 + (size_t)RT_E * RT_SLAB * sizeof(W);
}
template <typename W>
__host__ __device__ constexpr size_t router_tile_smem() {
  return RT_BUFS * router_buf_bytes<W>() + 128;
}

__device__ __forceinline__ float4 smem_w4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Packed pair of f32 lanes (fma.rn.f32x2: each lane is one fmaf, the same
// single rounding; one issue slot for two FMAs).
__device__ __forceinline__ unsigned long long pack_f2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f2(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma_f2(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float4 smem_w4(const __nv_bfloat16* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                     __uint_as_float(v.y & 0xffff0000u));
}

template <typename W>
__global__ void __launch_bounds__(256, 2)
router_logits_tile_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                          int rows, int E, int H, float* __restrict__ logits, unsigned* status) {
  extern __shared__ __align__(128) uint8_t rsm[];
  __shared__ uint64_t full[RT_BUFS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * RT_T, e0 = blockIdx.x * RT_E;
  const int tg = (warp & 3) * 8, eg = (warp >> 2) * 8;
  constexpr uint32_t kBuf = (uint32_t)router_buf_bytes<W>();
  constexpr uint32_t kX = RT_T * RT_SLAB * 2;
  uint8_t* base = rsm + ((128u - (smem_u32(rsm) & 127u)) & 127u);
  const int nslab = H / RT_SLAB;
  if (threadIdx.x == 0) {
    for (int i = 0; i < RT_BUFS; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int sidx) {
    uint8_t* b = base + (sidx % RT_BUFS) * kBuf;
    uint64_t* bar = &full[sidx % RT_BUFS];
    mbar_expect_tx(bar, kBuf);
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(b)),
        "l"(reinterpret_cast<uint64_t>(&xmap)), "r"(sidx * RT_SLAB), "r"(t0), "r"(smem_u32(bar))
        : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(b + kX)),
        "l"(reinterpret_cast<uint64_t>(&wmap)), "r"(sidx * RT_SLAB), "r"(e0), "r"(smem_u32(bar))
        : "memory");
  };
  if (threadIdx.x == 0) {
    issue(0);
    if (nslab > 1) issue(1);
  }
  // acc2[tp][e]: tokens tg + 2tp (low lane) and tg + 2tp + 1 (high lane)
  unsigned long long acc2[4][8];
#pragma unroll
  for (int tp = 0; tp < 4; ++tp)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc2[tp][e] = 0ull;
  bool ok = true;
  for (int si = 0; si < nslab; ++si) {
    // the buffer slab si + 2 goes to held slab si - 1, released by the
    // barrier at the end of the previous iteration
    if (threadIdx.x == 0 && si + 2 < nslab) issue(si + 2);
    if (ok) ok = mbar_wait_bounded(&full[si % RT_BUFS], (uint32_t)((si / RT_BUFS) & 1), status, kRouterWaitLimit);
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(base + (si % RT_BUFS) * kBuf);  // [RT_T][RT_SLAB]
    const W* ws = reinterpret_cast<const W*>(base + (si % RT_BUFS) * kBuf + kX);           // [RT_E][RT_SLAB]
#pragma unroll 1
    for (int c = lane; c < RT_SLAB / 4; c += 32) {
      // xp[tp][j]: element j of the chunk for the token pair tp
      unsigned long long xp[4][4];
#pragma unroll
      for (int tp = 0; tp < 4; ++tp) {
        const uint2 q0 = *reinterpret_cast<const uint2*>(xs + (tg + 2 * tp) * RT_SLAB + 4 * c);
        const uint2 q1 = *reinterpret_cast<const uint2*>(xs + (tg + 2 * tp + 1) * RT_SLAB + 4 * c);
        xp[tp][0] = pack_f2(__uint_as_float(q0.x << 16), __uint_as_float(q1.x << 16));
        xp[tp][1] = pack_f2(__uint_as_float(q0.x & 0xffff0000u), __uint_as_float(q1.x & 0xffff0000u));
        xp[tp][2] = pack_f2(__uint_as_float(q0.y << 16), __uint_as_float(q1.y << 16));
        xp[tp][3] = pack_f2(__uint_as_float(q0.y & 0xffff0000u), __uint_as_float(q1.y & 0xffff0000u));
      }
#pragma unroll
      for (int eh = 0; eh < 8; eh += 4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 wv = smem_w4(ws + (eg + eh + e) * RT_SLAB + 4 * c);
          const unsigned long long w0 = pack_f2(wv.x, wv.x), w1 = pack_f2(wv.y, wv.y), w2 = pack_f2(wv.z, wv.z),
                                   w3 = pack_f2(wv.w, wv.w);
#pragma unroll
          for (int tp = 0; tp < 4; ++tp) {
            unsigned long long a = acc2[tp][eh + e];
            a = fma_f2(xp[tp][0], w0, a);
            a = fma_f2(xp[tp][1], w1, a);
            a = fma_f2(xp[tp][2], w2, a);
            a = fma_f2(xp[tp][3], w3, a);
            acc2[tp][eh + e] = a;
          }
        }
      }
    }
    __syncthreads();  // this buffer may be refilled
  }
#pragma unroll
  for (int t = 0; t < 8; ++t)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float lo, hi;
      unpack_f2(acc2[t >> 1][e], lo, hi);
      float a = (t & 1) ? hi : lo;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) a = a + __shfl_xor_sync(0xffffffffu, a, o);
      const int tt = t0 + tg + t, ee = e0 + eg + e;
      if (lane == 0 && tt < rows && ee < E) logits[(int64_t)tt * E + ee] = logit_value<W>(a);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 router_map_encoder() {
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

// 2-D row-major tensor [rows][cols] of 16- or 32-bit elements, no swizzle,
// box RT_SLAB x box_rows; cached per (base, rows, cols, type, box) since the
// map only describes the buffer.
int router_map(const void* base, uint64_t rows, uint64_t cols, CUtensorMapDataType dt, uint32_t esize,
               uint32_t box_rows, CUtensorMap* out) {
  struct Entry {
    const void* base;
    uint64_t rows, cols;
    int dt;
    uint32_t box_rows;
    CUtensorMap map;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& en : cache)
    if (en.base == base && en.rows == rows && en.cols == cols && en.dt == (int)dt && en.box_rows == box_rows) {
      *out = en.map;
      return B2_OK;
    }
  auto enc = router_map_encoder();
  B2_REQUIRE(enc != nullptr, "[router_logits] cuTensorMapEncodeTiled is not available from the driver");
  B2_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0 && (cols * esize) % 16 == 0,
             "[router_logits] rows must be 16-byte aligned");
  Entry en;
  en.base = base;
  en.rows = rows;
  en.cols = cols;
  en.dt = (int)dt;
  en.box_rows = box_rows;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * esize};
  const cuuint32_t box[2] = {(cuuint32_t)RT_SLAB, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&en.map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2_REQUIRE(r == CUDA_SUCCESS, "[router_logits] tensor map encoding failed (%d)", (int)r);
  if (cache.size() >= 16) cache.erase(cache.begin());
  cache.push_back(en);
  *out = en.map;
  return B2_OK;
}

template <typename W>
int launch_router_tile(const uint16_t* x, const W* wr, int64_t rows, int64_t E, int64_t H, float* logits,
                       cudaStream_t st) {
  CUtensorMap xmap, wmap;
  int rc = router_map(x, (uint64_t)rows, (uint64_t)H, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, RT_T, &xmap);
  if (rc) return rc;
  rc = router_map(wr, (uint64_t)E, (uint64_t)H,
                  sizeof(W) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                  (uint32_t)sizeof(W), RT_E, &wmap);
  if (rc) return rc;
  const void* fn = (const void*)router_logits_tile_kernel<W>;
  rc = ensure_dynamic_smem(fn, router_tile_smem<W>(), "router_logits");
  if (rc) return rc;
  dim3 grid((unsigned)((E + RT_E - 1) / RT_E), (unsigned)((rows + RT_T - 1) / RT_T));
  int ir = (int)rows, ie = (int)E, ih = (int)H;
  unsigned* status = device_status_ptr();
  void* args[] = {&xmap, &wmap, &ir, &ie, &ih, &logits, &status};
  return check_cuda(cudaLaunchKernel(fn, grid, dim3(256), args, router_tile_smem<W>(), st), "router_logits");
}

}  // namespace

int launch_router_logits(const uint16_t* x, const void* wr, int w_dtype, int64_t rows, int64_t E, int64_t H,
                         float* logits, cudaStream_t st) {
  if (rows == 0) return B2_OK;
  if (rows <= 4) {
    // decode: one expert per warp, one token per CTA row
    dim3 grid((unsigned)((E + 7) / 8), (unsigned)rows);
    const size_t smem = (size_t)H * 2;
    if (w_dtype == B2_DTYPE_F32)
      router_logits_kernel<float, 1, 1><<<grid, 256, smem, st>>>(x, (const float*)wr, (int)rows, (int)E, (int)H, logits);
    else
      router_logits_kernel<__nv_bfloat16, 1, 1><<<grid, 256, smem, st>>>(x, (const __nv_bfloat16*)wr, (int)rows,
                                                                        (int)E, (int)H, logits);
  } else if (rows <= 64 || (size_t)16 * H * 2 > 200 * 1024) {
    constexpr int EW = 2, TT = 8;
    dim3 grid((unsigned)((E + 8 * EW - 1) / (8 * EW)), (unsigned)((rows + TT - 1) / TT));
    const size_t smem = (size_t)TT * H * 2;
    const void* fn = (w_dtype == B2_DTYPE_F32) ? (const void*)router_logits_kernel<float, EW, TT>
                                               : (const void*)router_logits_kernel<__nv_bfloat16, EW, TT>;
    const int rc = ensure_dynamic_smem(fn, smem, "router_logits");
    if (rc) return rc;
    if (w_dtype == B2_DTYPE_F32)
      router_logits_kernel<float, EW, TT><<<grid, 256, smem, st>>>(x, (const float*)wr, (int)rows, (int)E, (int)H, logits);
    else
      router_logits_kernel<__nv_bfloat16, EW, TT><<<grid, 256, smem, st>>>(x, (const __nv_bfloat16*)wr, (int)rows,
                                                                          (int)E, (int)H, logits);
  } else if (H % RT_SLAB == 0) {
    // prefill: 32 x 16 (token, expert) tiles, both operands streamed by TMA
    const int rc = (w_dtype == B2_DTYPE_F32)
                       ? launch_router_tile<float>(x, (const float*)wr, rows, E, H, logits, st)
                       : launch_router_tile<__nv_bfloat16>(x, (const __nv_bfloat16*)wr, rows, E, H, logits, st);
    if (rc) return rc;
  } else {
    // 16 tokens per CTA (x rows staged once, router rows read by half as many
    // CTAs as with 8); same per-(token, expert) summation order
    constexpr int EW = 2, TT = 16;
    const size_t smem = (size_t)TT * H * 2;
    dim3 grid((unsigned)((E + 8 * EW - 1) / (8 * EW)), (unsigned)((rows + TT - 1) / TT));
    const void* fn = (w_dtype == B2_DTYPE_F32) ? (const void*)router_logits_kernel<float, EW, TT>
                                               : (const void*)router_logits_kernel<__nv_bfloat16, EW, TT>;
    const int rc = ensure_dynamic_smem(fn, smem, "router_logits");
    if (rc) return rc;
    if (w_dtype == B2_DTYPE_F32)
      router_logits_kernel<float, EW, TT><<<grid, 256, smem, st>>>(x, (const float*)wr, (int)rows, (int)E, (int)H, logits);
    else
      router_logits_kernel<__nv_bfloat16, EW, TT><<<grid, 256, smem, st>>>(x, (const __nv_bfloat16*)wr, (int)rows,
                                                                          (int)E, (int)H, logits);
  }
  B2_CHECK_LAUNCH("router_logits");
  return B2_OK;
}

namespace {

// One warp per row.  Keys live in registers (E/32 per lane, E <= 1024); k
// rounds of a warp-wide arg-best under the ranking order (larger key first,
// NaN last, ties by smaller index).  The order is carried by an unsigned
// code per entry: 0 for a padding lane or an entry already taken, 1 for NaN
// (all NaNs tie), else the order-preserving image of the key with -0 read as
// +0 (>= 0x007fffff, so above NaN); a round is then one redux max over the
// lanes' best codes and one redux min over the indices that reach it.
__device__ __forceinline__ uint32_t rank_code(float kv) {
  if (isnan(kv)) return 1u;
  if (kv == 0.0f) kv = 0.0f;  // -0 ties with +0
  const uint32_t u = __float_as_uint(kv);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int PER_LANE>
__global__ void __launch_bounds__(256)
topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int mode, int rows, int E, int k,
            int renorm, uint32_t* __restrict__ inds, float* __restrict__ weights) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;
  const float* l = logits + (int64_t)row * E;
  uint32_t code[PER_LANE];
  float val[PER_LANE];
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int e = j * 32 + lane;
    uint32_t c = 0u;
    float vv = 0.0f;
    if (e < E) {
      const float x = l[e];
      float kv;
      if (mode == B2_ROUTER_SOFTMAX) {
        kv = x;
        vv = x;
      } else {
        const float sg = sigmoid_stable(x);
        vv = sg;
        kv = sg + (bias ? bias[e] : 0.0f);
      }
      c = rank_code(kv);
    }
    code[j] = c;
    val[j] = vv;
  }
  uint32_t sel_idx = 0;
  float sel_val = 0.0f;
  for (int s = 0; s < k; ++s) {
    // this lane's best untaken entry (the smallest index among equal codes)
    uint32_t bc = 0u;
    int bj = 0;
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j)
      if (code[j] > bc) {
        bc = code[j];
        bj = j;
      }
    const uint32_t m = __reduce_max_sync(0xffffffffu, bc);
    const uint32_t cand = (bc == m) ? (uint32_t)(bj * 32 + lane) : 0xffffffffu;
    const uint32_t bi = __reduce_min_sync(0xffffffffu, cand);
    // the owner marks it taken and broadcasts its value
    const int owner = (int)(bi & 31u), slot = (int)(bi >> 5);
    float v = 0.0f;
    if (lane == owner) {
#pragma unroll
      for (int j = 0; j < PER_LANE; ++j)
        if (j == slot) {
          code[j] = 0u;
          v = val[j];
        }
    }
    v = __shfl_sync(0xffffffffu, v, owner);
    if (lane == s) {
      sel_idx = bi;
      sel_val = v;
    }
  }
  // weights (lanes 0..k-1 hold the selection in rank order)
  float wv;
  if (mode == B2_ROUTER_SOFTMAX) {
    const float mx = __shfl_sync(0xffffffffu, sel_val, 0);
    const float ev = (lane < k) ? b2_expf(__fsub_rn(sel_val, mx)) : 0.0f;
    float tot = 0.0f;
    for (int s = 0; s < k; ++s) tot += __shfl_sync(0xffffffffu, ev, s);
    wv = ev / tot;
  } else {
    float tot = 0.0f;
    for (int s = 0; s < k; ++s) tot = __shfl_sync(0xffffffffu, sel_val, s) + tot;
    wv = renorm ? sel_val / tot : sel_val;
  }
  if (lane < k) {
    inds[(int64_t)row * k + lane] = sel_idx;
    weights[(int64_t)row * k + lane] = wv;
  }
}

}  // namespace

int launch_router_topk(const float* logits, const float* bias, int mode, int64_t rows, int64_t E, int k, int renorm,
                       uint32_t* inds, float* weights, cudaStream_t st) {
  if (rows == 0) return B2_OK;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (E <= 128)
    topk_kernel<4><<<blocks, 256, 0, st>>>(logits, bias, mode, (int)rows, (int)E, k, renorm, inds, weights);
  else if (E <= 256)
    topk_kernel<8><<<blocks, 256, 0, st>>>(logits, bias, mode, (int)rows, (int)E, k, renorm, inds, weights);
  else
    topk_kernel<32><<<blocks, 256, 0, st>>>(logits, bias, mode, (int)rows, (int)E, k, renorm, inds, weights);
  B2_CHECK_LAUNCH("router_topk");
  return B2_OK;
}

}  // namespace b2

extern "C" int b2_moe_router_logits(const uint16_t* x, const void* router_w, int w_dtype, int64_t rows, int64_t E,
                                    int64_t H, float* logits, b2_stream_t stream) {
  B2_REQUIRE(x && router_w && logits, "[router_logits] null pointer argument");
  B2_REQUIRE(rows >= 0 && E > 0 && H > 0 && H % 8 == 0, "[router_logits] invalid shape (H must be a multiple of 8)");
  B2_REQUIRE(w_dtype == B2_DTYPE_F32 || w_dtype == B2_DTYPE_BF16, "[router_logits] router weight must be f32 or bf16");
  B2_REQUIRE(rows <= 65535 * 8, "[router_logits] too many rows");
  return b2::launch_router_logits(x, router_w, w_dtype, rows, E, H, logits, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b2_moe_router_topk(const float* logits, const float* bias, int mode, int64_t rows, int64_t E, int k,
                                  int renorm, uint32_t* inds, float* weights, b2_stream_t stream) {
  B2_REQUIRE(logits && inds && weights, "[router_topk] null pointer argument");
  B2_REQUIRE(mode == B2_ROUTER_SOFTMAX || mode == B2_ROUTER_SIGMOID_BIAS, "[router_topk] unknown router mode %d", mode);
  B2_REQUIRE(E > 0 && E <= 1024, "[router_topk] number of experts must be in [1, 1024] (got %lld)", (long long)E);
  B2_REQUIRE(k > 0 && k <= 32 && k <= E, "[router_topk] k must be in [1, min(32, E)] (got %d)", k);
  B2_REQUIRE(rows >= 0, "[router_topk] invalid row count");
  return b2::launch_router_topk(logits, bias, mode, rows, E, k, renorm, inds, weights,
                                reinterpret_cast<cudaStream_t>(stream));
}
