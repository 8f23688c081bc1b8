// NVFP4 quantize / dequantize kernels (MLX nvfp4 mode, group 16).
#include "common.cuh"

namespace b2 {
namespace {

// One thread per 16-element group.  q = w / decode(scale) and the code is the
// first LUT index minimising |q - LUT[j]| (MLX argmin: strict less-than, an
// initial NaN is never replaced), matching MLX/ops.cpp:4873-4978.
__global__ void quantize_kernel(const float* __restrict__ w, int64_t groups_total,
                                uint32_t* __restrict__ codes, uint8_t* __restrict__ scales) {
  const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (g >= groups_total) return;
  const float4* src = reinterpret_cast<const float4*>(w + g * 16);
  float v[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 t = src[i];
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
  float amax = fabsf(v[0]);
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    const float a = fabsf(v[i]);
    if (a > amax) amax = a;
  }
  const uint32_t sb = e4m3_encode_scale(__fdiv_rn(amax, 6.0f));
  const float sd = e4m3_value(sb);
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float q = __fdiv_rn(v[i], sd);
    uint32_t best = 0;
    float bv = fabsf(q - 0.0f);
#pragma unroll
    for (uint32_t j = 1; j < 16; ++j) {
      const float d = fabsf(__fsub_rn(q, e2m1_value(j)));
      if (d < bv) { bv = d; best = j; }
    }
    if (i < 8) w0 |= best << (4 * i); else w1 |= best << (4 * (i - 8));
  }
  codes[2 * g] = w0;
  codes[2 * g + 1] = w1;
  scales[g] = static_cast<uint8_t>(sb);
}

template <typename OutT>
__device__ __forceinline__ OutT from_float(float f);
template <> __device__ __forceinline__ float from_float<float>(float f) { return f; }
template <> __device__ __forceinline__ __half from_float<__half>(float f) { return __float2half_rn(f); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float f) {
  return __float2bfloat16_rn(f);
}

// One thread per code word (8 outputs).  value = LUT[code] * decode(scale) is
// exact in float and stays exact when narrowed to bf16/f16.
template <typename OutT>
__global__ void dequantize_kernel(const uint32_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                  int64_t words_total, OutT* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= words_total) return;
  const uint32_t w = codes[i];
  const float s = e4m3_value(scales[i >> 1]);
  OutT r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = from_float<OutT>(e2m1_value((w >> (4 * j)) & 15u) * s);
#pragma unroll
  for (int j = 0; j < 8; ++j) out[i * 8 + j] = r[j];
}

}  // namespace
}  // namespace b2

extern "C" int b2_fp_quantize(const float* w, int64_t rows, int64_t K, uint32_t* codes,
                              uint8_t* scales, b2_stream_t stream) {
  B2_REQUIRE(w && codes && scales, "[quantize] null pointer argument");
  B2_REQUIRE(rows >= 0 && K > 0, "[quantize] invalid shape rows=%lld K=%lld", (long long)rows, (long long)K);
  B2_REQUIRE(K % 16 == 0,
             "[quantize] nvfp4 quantization requires the last dimension (%lld) to be divisible by the group size 16",
             (long long)K);
  B2_REQUIRE(reinterpret_cast<uintptr_t>(w) % 16 == 0, "[quantize] w must be 16-byte aligned");
  const int64_t groups = rows * (K / 16);
  if (groups == 0) return B2_OK;
  const int threads = 256;
  const int64_t blocks = (groups + threads - 1) / threads;
  b2::quantize_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      w, groups, codes, scales);
  B2_CHECK_LAUNCH("quantize");
  return B2_OK;
}

extern "C" int b2_fp_dequantize(const uint32_t* codes, const uint8_t* scales, int64_t rows,
                                int64_t K, void* out, int out_dtype, b2_stream_t stream) {
  B2_REQUIRE(codes && scales && out, "[dequantize] null pointer argument");
  B2_REQUIRE(rows >= 0 && K > 0 && K % 16 == 0,
             "[dequantize] nvfp4 requires K (%lld) divisible by 16", (long long)K);
  const int64_t words = rows * (K / 8);
  if (words == 0) return B2_OK;
  const int threads = 256;
  const unsigned blocks = (unsigned)((words + threads - 1) / threads);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (out_dtype) {
    case B2_DTYPE_F32:
      b2::dequantize_kernel<float><<<blocks, threads, 0, s>>>(codes, scales, words, (float*)out);
      break;
    case B2_DTYPE_BF16:
      b2::dequantize_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(codes, scales, words,
                                                                     (__nv_bfloat16*)out);
      break;
    case B2_DTYPE_F16:
      b2::dequantize_kernel<__half><<<blocks, threads, 0, s>>>(codes, scales, words, (__half*)out);
      break;
    default:
      return b2::set_error(B2_ERR_INVALID_ARGUMENT, "[dequantize] unsupported output dtype %d", out_dtype);
  }
  B2_CHECK_LAUNCH("dequantize");
  return B2_OK;
}
