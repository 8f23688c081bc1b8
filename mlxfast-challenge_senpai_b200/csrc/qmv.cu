// quantized_matmul / gather_qmm for decode-shaped problems (few tokens per
// weight matrix).  See qmv.cuh for the design.
#include <cstdlib>

#include "qmv.cuh"

namespace b2 {

// Programmatic dependent launch of the GEMV (on unless the environment sets
// B2_QMV_PDL=0).
bool qmv_pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("B2_QMV_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

namespace {

using namespace qmv;

// Generic tensor-core GEMV: CTA = (RT tiles of 8 rows, one index pair).
//   x    bf16 [Bx, M, K]      (lhs[p] selects the batch; identity if null)
//   w    codes [E, N, K/8]    (rhs[p] selects the matrix; identity if null)
//   y    bf16 [P, M, N]
// M <= 16*MT.
template <int RT, int MT>
__global__ void __launch_bounds__(kThreads)
qmv_mma_kernel(const uint16_t* __restrict__ x, const uint8_t* __restrict__ codes,
               const uint8_t* __restrict__ scales, const uint32_t* __restrict__ lhs,
               const uint32_t* __restrict__ rhs, int64_t Bx, int64_t E, int M, int N, int K,
               uint16_t* __restrict__ y, unsigned* status) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const TileGeom g = make_geom(K, RT);
  constexpr int ROWS = RT * kGroups;
  const Smem s = carve(smem_raw, g, M);
  const int p = blockIdx.y;
  const int row0 = blockIdx.x * ROWS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int nvalid = min(ROWS, N - row0);
  if (threadIdx.x == 0) {
    mbar_init(s.bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Programmatic dependent launch: with a fixed weight matrix (no rhs
  // indices) the weights do not depend on the previous kernel in the stream,
  // so their copies start before the dependency wait and stream in while
  // that kernel finishes; the indices, x and y wait for it.
  const bool static_w = rhs == nullptr;
  auto issue = [&](uint32_t ri) {
    if (warp == 0) {
      const uint8_t* wbase = codes + (int64_t)ri * N * (K / 2);
      const uint8_t* sbase = scales + (int64_t)ri * N * (K / 16);
      if (lane == 0) mbar_expect_tx(s.bar, (uint32_t)nvalid * (uint32_t)(K / 2 + K / 16));
      __syncwarp();
      issue_groups(s, g, nvalid, wbase + (int64_t)row0 * (K / 2), sbase + (int64_t)row0 * (K / 16));
    }
  };
  if (static_w && p < E) issue((uint32_t)p);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const uint32_t li = lhs ? lhs[p] : (uint32_t)p;
  const uint32_t ri = rhs ? rhs[p] : (uint32_t)p;
  const bool bad = (int64_t)li >= Bx || (int64_t)ri >= E;
  if (bad) {
    if (threadIdx.x == 0) report_status(status, B2_STATUS_BAD_INDEX);
    for (int i = threadIdx.x; i < M * nvalid; i += blockDim.x) {
      const int m = i / nvalid, r = i % nvalid;
      y[((int64_t)p * M + m) * N + row0 + r] = 0;
    }
    // copies issued before the wait must land before the CTA exits
    if (static_w && p < E) mbar_wait_bounded(s.bar, 0, status);
    return;
  }
  if (!static_w) issue(ri);
  const uint16_t* xb = x + (int64_t)li * M * K;
  stage_x(s, g, M, [&](int m) { return xb + (int64_t)m * K; });
  if (!mbar_wait_bounded(s.bar, 0, status)) return;

  float acc[RT][MT][4];
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[rt][mt][j] = 0.0f;

  const int groups = K / 16;
  const int c = lane & 3, gi = lane >> 2;
  for (int grp = warp; grp < groups; grp += kWarps) {
    uint32_t a[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) load_a_frag(s, g, grp, lane, mt * 16, min(16, M - mt * 16), a[mt]);
#pragma unroll
    for (int rt = 0; rt < RT; ++rt) {
      uint32_t b[2];
      load_b_frag(s, g, gi, rt, grp, c, b);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) mma_16816_f16(acc[rt][mt], a[mt], b);
    }
  }

  // cross-warp reduction in fixed warp order
  float* red = s.red;
  constexpr int PER_WARP = RT * MT * 4 * 32;
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) red[warp * PER_WARP + ((rt * MT + mt) * 4 + j) * 32 + lane] = acc[rt][mt][j];
  __syncthreads();
  for (int i = threadIdx.x; i < PER_WARP; i += blockDim.x) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w * PER_WARP + i];
    const int ln = i & 31, j = (i >> 5) & 3, rm = i >> 7;
    const int mt = rm % MT, rt = rm / MT;
    const int m = mt * 16 + (ln >> 2) + ((j >= 2) ? 8 : 0);
    const int r = (2 * (ln & 3) + (j & 1)) * RT + rt;  // row rt of group (column) 2(ln&3)+(j&1)
    if (m < M && r < nvalid) {
      v = ldexpf(v, s.xexp[m]);
      y[((int64_t)p * M + m) * N + row0 + r] = f32_to_bf16_bits(v);
    }
  }
}

// Generic CUDA-core fallback for any activation dtype / K % 16 == 0: one warp
// per output row, lanes stride the groups, float FMA, shuffle reduction.
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(256)
qmv_fma_kernel(const T* __restrict__ x, const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
               const uint32_t* __restrict__ lhs, const uint32_t* __restrict__ rhs, int64_t Bx, int64_t E, int M,
               int N, int K, T* __restrict__ y, unsigned* status) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const int p = blockIdx.y;
  if (n >= N) return;
  const uint32_t li = lhs ? lhs[p] : (uint32_t)p;
  const uint32_t ri = rhs ? rhs[p] : (uint32_t)p;
  if ((int64_t)li >= Bx || (int64_t)ri >= E) {
    if (lane == 0) report_status(status, B2_STATUS_BAD_INDEX);
    for (int m = lane; m < M; m += 32) y[((int64_t)p * M + m) * N + n] = from_f32<T>(0.0f);
    return;
  }
  const uint8_t* wr = codes + ((int64_t)ri * N + n) * (K / 2);
  const uint8_t* sr = scales + ((int64_t)ri * N + n) * (K / 16);
  const T* xb = x + (int64_t)li * M * K;
  const int groups = K / 16;
  for (int m0 = 0; m0 < M; m0 += 8) {
    const int mc = min(8, M - m0);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int grp = lane; grp < groups; grp += 32) {
      const uint2 w = *reinterpret_cast<const uint2*>(wr + (int64_t)grp * 8);
      const float sc = e4m3_value(sr[grp]);
      float v[16];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = e2m1_value((w.x >> (4 * j)) & 15u);
        v[8 + j] = e2m1_value((w.y >> (4 * j)) & 15u);
      }
#pragma unroll
      for (int mm = 0; mm < 8; ++mm) {
        if (mm < mc) {
          const T* xr = xb + (int64_t)(m0 + mm) * K + grp * 16;
          float gs = 0.0f;
#pragma unroll
          for (int j = 0; j < 16; ++j) gs = fmaf(to_f32<T>(xr[j]), v[j], gs);
          acc[mm] = fmaf(sc, gs, acc[mm]);
        }
      }
    }
#pragma unroll
    for (int mm = 0; mm < 8; ++mm) {
      float a = acc[mm];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0 && mm < mc) y[((int64_t)p * M + m0 + mm) * N + n] = from_f32<T>(a);
    }
  }
}

template <int RT, int MT>
int launch_mma(const uint16_t* x, const uint8_t* codes, const uint8_t* scales, const uint32_t* lhs,
               const uint32_t* rhs, int64_t P, int64_t Bx, int64_t E, int M, int N, int K, uint16_t* y,
               cudaStream_t st) {
  const TileGeom g = make_geom(K, RT);
  const size_t smem = smem_bytes(g, M, kWarps * RT * MT * 128);
  if (smem > 200 * 1024) return -1;
  const int rc = ensure_dynamic_smem((const void*)qmv_mma_kernel<RT, MT>, smem, "quantized_matmul");
  if (rc) return rc;
  dim3 grid((unsigned)((N + RT * 8 - 1) / (RT * 8)), (unsigned)P);
  unsigned* status = device_status_ptr();
  void* args[] = {(void*)&x, (void*)&codes, (void*)&scales, (void*)&lhs, (void*)&rhs, (void*)&Bx, (void*)&E,
                  (void*)&M, (void*)&N, (void*)&K, (void*)&y, (void*)&status};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = qmv_pdl_enabled() ? 1 : 0;
  const void* fn = (const void*)qmv_mma_kernel<RT, MT>;
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess && cfg.numAttrs == 1) {
    (void)cudaGetLastError();
    cfg.numAttrs = 0;
    e = cudaLaunchKernelExC(&cfg, fn, args);
  }
  return e == cudaSuccess ? 0 : check_cuda(e, "quantized_matmul");
}

int run_qmv(const char* op, const void* x, int x_dtype, const uint32_t* codes, const uint8_t* scales,
            const uint32_t* lhs, const uint32_t* rhs, int64_t P, int64_t Bx, int64_t E, int64_t M, int64_t N,
            int64_t K, void* y, b2_stream_t stream) {
  B2_REQUIRE(x && codes && scales && y, "[%s] null pointer argument", op);
  B2_REQUIRE(M > 0 && N > 0 && K > 0 && P >= 0, "[%s] invalid shape M=%lld N=%lld K=%lld", op, (long long)M,
             (long long)N, (long long)K);
  B2_REQUIRE(K % 16 == 0,
             "[%s] the last dimension of x (%lld) must be divisible by the nvfp4 group size 16", op,
             (long long)K);
  B2_REQUIRE(N <= (int64_t)INT32_MAX && K <= (int64_t)INT32_MAX && M <= 65535, "[%s] shape too large", op);
  B2_REQUIRE(P <= 65535, "[%s] too many index pairs (%lld > 65535)", op, (long long)P);
  if (P == 0) return B2_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* status = device_status_ptr();
  const bool aligned = (reinterpret_cast<uintptr_t>(codes) % 16 == 0) && (reinterpret_cast<uintptr_t>(scales) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  if (x_dtype == B2_DTYPE_BF16 && K % 256 == 0 && aligned && M <= 32) {
    int rc;
    if (P == 1 && !lhs && !rhs) {
      // one weight matrix: the streaming kernel (qmv_stream.cu)
      rc = qmv_stream(static_cast<const uint16_t*>(x), reinterpret_cast<const uint8_t*>(codes), scales, (int)M,
                     (int)N, (int)K, static_cast<uint16_t*>(y), st);
      if (rc == 0) {
        B2_CHECK_LAUNCH(op);
        return B2_OK;
      }
      if (rc != 1) return rc;
    }
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    uint16_t* yb = static_cast<uint16_t*>(y);
    const uint8_t* cb = reinterpret_cast<const uint8_t*>(codes);
    if (M <= 16) {
      rc = launch_mma<2, 1>(xb, cb, scales, lhs, rhs, P, Bx, E, (int)M, (int)N, (int)K, yb, st);
    } else {
      rc = launch_mma<2, 2>(xb, cb, scales, lhs, rhs, P, Bx, E, (int)M, (int)N, (int)K, yb, st);
      if (rc < 0 && P == 1) {
        // 32 staged rows of this K do not fit in shared memory: two passes of
        // at most 16 rows (each output row is computed independently, so the
        // results are the same; the second pass finds the weights in L2)
        rc = launch_mma<2, 1>(xb, cb, scales, lhs, rhs, 1, 1, E, 16, (int)N, (int)K, yb, st);
        if (rc == 0) {
          B2_CHECK_LAUNCH(op);
          rc = launch_mma<2, 1>(xb + 16 * K, cb, scales, lhs, rhs, 1, 1, E, (int)M - 16, (int)N, (int)K,
                                yb + 16 * N, st);
        }
      }
    }
    if (rc == 0) {
      B2_CHECK_LAUNCH(op);
      return B2_OK;
    }
    if (rc > 0) return rc;
  }
  dim3 grid((unsigned)((N + 7) / 8), (unsigned)P);
  const uint8_t* cb = reinterpret_cast<const uint8_t*>(codes);
  switch (x_dtype) {
    case B2_DTYPE_BF16:
      qmv_fma_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, cb, scales, lhs, rhs, Bx, E,
                                                          (int)M, (int)N, (int)K, (__nv_bfloat16*)y, status);
      break;
    case B2_DTYPE_F16:
      qmv_fma_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, cb, scales, lhs, rhs, Bx, E, (int)M, (int)N,
                                                   (int)K, (__half*)y, status);
      break;
    case B2_DTYPE_F32:
      qmv_fma_kernel<float><<<grid, 256, 0, st>>>((const float*)x, cb, scales, lhs, rhs, Bx, E, (int)M, (int)N,
                                                  (int)K, (float*)y, status);
      break;
    default:
      return set_error(B2_ERR_INVALID_ARGUMENT, "[%s] unsupported activation dtype %d", op, x_dtype);
  }
  B2_CHECK_LAUNCH(op);
  return B2_OK;
}

}  // namespace

int qmm_bf16(const uint16_t* x, const uint32_t* codes, const uint8_t* scales, int64_t M, int64_t N, int64_t K,
             uint16_t* y, cudaStream_t st) {
  return run_qmv("shared_expert", x, B2_DTYPE_BF16, codes, scales, nullptr, nullptr, 1, 1, 1, M, N, K, y,
                 reinterpret_cast<b2_stream_t>(st));
}

}  // namespace b2

extern "C" int b2_quantized_matmul(const void* x, int x_dtype, const uint32_t* codes, const uint8_t* scales,
                                   void* y, int64_t M, int64_t N, int64_t K, b2_stream_t stream) {
  return b2::run_qmv("quantized_matmul", x, x_dtype, codes, scales, nullptr, nullptr, 1, 1, 1, M, N, K, y,
                     stream);
}

extern "C" int b2_gather_qmm(const void* x, int x_dtype, const uint32_t* codes, const uint8_t* scales,
                             const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t P, int64_t Bx,
                             int64_t E, int64_t M, int64_t N, int64_t K, int sorted_indices, void* y,
                             b2_stream_t stream) {
  (void)sorted_indices;
  B2_REQUIRE(lhs_indices || Bx == P, "[gather_qmm] lhs_indices is NULL but x batch (%lld) != pairs (%lld)",
             (long long)Bx, (long long)P);
  B2_REQUIRE(rhs_indices || E == P, "[gather_qmm] rhs_indices is NULL but w batch (%lld) != pairs (%lld)",
             (long long)E, (long long)P);
  return b2::run_qmv("gather_qmm", x, x_dtype, codes, scales, lhs_indices, rhs_indices, P, Bx, E, M, N, K, y,
                     stream);
}
