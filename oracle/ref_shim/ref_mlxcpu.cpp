// Shim that compiles the reference's own MLX CPU NVFP4 kernels in place and
// exports them with a C ABI, so tests can check the restatement in
// oracle/nvfp4_oracle.c against the reference itself.
//
// TEST INFRASTRUCTURE ONLY (built into oracle/_ref/, never shipped).
//
// The reference sources are compiled where they lie, by oracle/Makefile, with
// -I pointing at the reference's MLX tree; nothing is copied.  What is called:
//   fp_qmm_t<T,16,4>  backend/cpu/quantized.cpp:491-533 (T = float, bfloat16_t)
//   FromFP8 / ToFP8   backend/cpu/unary_ops.h:120-173
#include "mlx/backend/cpu/quantized.cpp"

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

REF_EXPORT void ref_fp_qmm_t_f32(float* y, const float* x, const uint32_t* w,
                                 const uint8_t* s, int M, int N, int K) {
  mlx::core::fp_qmm_t<float, 16, 4>(y, x, w, s, M, N, K);
}

REF_EXPORT void ref_fp_qmm_t_bf16(uint16_t* y, const uint16_t* x, const uint32_t* w,
                                  const uint8_t* s, int M, int N, int K) {
  using bf = mlx::core::bfloat16_t;
  mlx::core::fp_qmm_t<bf, 16, 4>(reinterpret_cast<bf*>(y), reinterpret_cast<const bf*>(x),
                                 w, s, M, N, K);
}

REF_EXPORT float ref_from_fp8(uint8_t b) { return mlx::core::detail::FromFP8{}(b); }
REF_EXPORT uint8_t ref_to_fp8(float f) { return mlx::core::detail::ToFP8{}(f); }

// The reference's activation fake-quantization for qqmm in nvfp4 mode
// (QQMatmul::eval_cpu -> fp_quantize_dequantize<bfloat16_t>,
// backend/cpu/quantized.cpp:1094-1129, 1322-1360), driven here over a plain
// buffer: per 16-group scale = dequantize_scale<float,16>(ToFP8(max|x|/6)),
// element code = to_fp4_e2m1(x / scale) (quantized.cpp:1064-1091),
// out = bf16(scale * FP4_LUT[code]).  Every step calls the reference's own
// function; codes and scale bytes are returned as well.
REF_EXPORT void ref_qdq_nvfp4_bf16(const uint16_t* x, size_t n, uint16_t* out, uint8_t* codes,
                                   uint8_t* scales) {
  using bf = mlx::core::bfloat16_t;
  const bf* w = reinterpret_cast<const bf*>(x);
  bf* o = reinterpret_cast<bf*>(out);
  for (size_t i = 0; i < n / 16; ++i) {
    const size_t idx = i * 16;
    float scale = -std::numeric_limits<float>::infinity();
    for (int j = 0; j < 16; ++j) scale = std::max(scale, static_cast<float>(std::abs(w[idx + j])));
    scale /= 6.0f;
    const uint8_t sb = mlx::core::detail::ToFP8()(scale);
    scales[i] = sb;
    scale = mlx::core::dequantize_scale<float, 16>(sb);
    for (int j = 0; j < 16; ++j) {
      const float w_el = scale == 0 ? 0.0f : w[idx + j] / scale;
      const uint8_t c = mlx::core::to_fp4_e2m1(w_el);
      codes[idx + j] = c;
      o[idx + j] = static_cast<bf>(scale * mlx::core::FP4_LUT[c]);
    }
  }
}

// The reference's CPU sigmoid (backend/cpu/unary_ops.h:77-84: stable form
// with MLX's own exp, simd/math.h) and softmax over one row
// (backend/cpu/softmax.cpp:18-110 for float with the scalar SIMD width of
// x86: max, exp(x - max) with MLX's exp, sum in order, times 1/sum).
REF_EXPORT float ref_sigmoid_f32(float x) { return mlx::core::detail::Sigmoid{}(x); }

REF_EXPORT void ref_softmax_f32(const float* x, int n, float* out) {
  namespace simd = mlx::core::simd;
  float maximum = -std::numeric_limits<float>::infinity();
  for (int i = 0; i < n; ++i) maximum = simd::maximum(simd::Simd<float, 1>(x[i]), simd::Simd<float, 1>(maximum)).value;
  float normalizer = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float e = simd::exp(simd::Simd<float, 1>(x[i] - maximum)).value;
    out[i] = e;
    normalizer = normalizer + e;
  }
  normalizer = 1 / normalizer;
  for (int i = 0; i < n; ++i) out[i] *= normalizer;
}

REF_EXPORT void ref_sigmoid_f32_array(const float* x, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = mlx::core::detail::Sigmoid{}(x[i]);
}
