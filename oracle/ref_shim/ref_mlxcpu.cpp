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
