// Shared device helpers for the NVFP4 MoE library (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2moe.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library is written for sm_100a only"
#endif

namespace b2 {

// Bytes at the head of every block workspace that hold the decode kernels'
// cross-launch state (activation counters, per-CTA launch epochs, tagged
// router logits for up to 8 tokens x 1024 experts).  Zero before the first
// call; the prefill path carves its buffers after it and never writes it.
constexpr size_t kDecodeStateBytes = 4096 + 8 * 1024 * 8;

// ---------------------------------------------------------------- host errors
// Records the message for b2_last_error() and forwards it to the user's
// handler (the shape of MLX's error channel, mlx-c error.h:15-33).
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

#define B2_CHECK_LAUNCH(what)                                  \
  do {                                                         \
    cudaError_t _e = cudaGetLastError();                       \
    if (_e != cudaSuccess) return ::b2::check_cuda(_e, what);  \
  } while (0)

#define B2_REQUIRE(cond, ...)                                           \
  do {                                                                  \
    if (!(cond)) return ::b2::set_error(B2_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

// Device-side status word: kernels that give up on a bounded wait record a
// code here instead of trapping; b2_device_status() reads and clears it.
__device__ __forceinline__ void report_status(unsigned* status, unsigned code) {
  if (status) atomicCAS(status, 0u, code);
}
unsigned* device_status_ptr();  // per-device status word (module-scope device variable)
// Opt `fn` into `bytes` of dynamic shared memory (per kernel and device).
int ensure_dynamic_smem(const void* fn, size_t bytes, const char* what);

// ---------------------------------------------------------------- bf16 / f16
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) {
  return __bfloat162float(__float2bfloat16_rn(f));
}

// ---------------------------------------------------------------- exp
// exp(x) by Cody-Waite argument reduction x = n*ln2 + r (ln2 split into the
// fdlibm hi/lo pair 0x3f317200 / 0x35bfbe8e so n*hi is exact), a degree-7
// Taylor polynomial of e^r on |r| <= ln2/2 in Horner form, and an exact
// scaling by 2^n.  Every step is an explicitly rounded IEEE operation, so the
// CPU checker (oracle/nvfp4_oracle.c, oracle_expf) computes the same bits.
// Max error about 2 ulp over the float range.
__device__ __forceinline__ float b2_expf(float x) {
  if (isnan(x)) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97208f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.42860676533018704e-06f, r);
  float p = 1.98412698412698413e-04f;            // 1/7!
  p = __fmaf_rn(p, r, 1.38888888888888889e-03f); // 1/6!
  p = __fmaf_rn(p, r, 8.33333333333333333e-03f); // 1/5!
  p = __fmaf_rn(p, r, 4.16666666666666667e-02f); // 1/4!
  p = __fmaf_rn(p, r, 1.66666666666666667e-01f); // 1/3!
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  return ldexpf(p, (int)n);
}

// ---------------------------------------------------------------- NVFP4 codec
// E2M1 code -> float (LUT of the MLX CPU backend, quantized.cpp:31-47).
__device__ __forceinline__ float e2m1_value(unsigned code) {
  const unsigned e = (code >> 1) & 3u, m = code & 1u;
  const float v = (e == 0u) ? 0.5f * static_cast<float>(m)
                            : 0.5f * static_cast<float>((2u + m) << (e - 1u));
  return (code & 8u) ? -v : v;
}

// E4M3 scale byte -> float with MLX's semantics (unary_ops.h:154-173): bits
// 6..0 are the low bits of an IEEE half whose exponent MSB is zero, times
// 256; bit 7 negates; 0x7f decodes to 480 (never NaN).  Exact in float.
__device__ __forceinline__ float e4m3_value(uint32_t b) {
  const __half h = __ushort_as_half(static_cast<unsigned short>((b & 0x7fu) << 7));
  const float v = __half2float(h) * 256.0f;
  return (b & 0x80u) ? -v : v;
}

// float -> E4M3 byte, round-to-nearest-even with saturation to 0x7e, the
// rounding MLX uses for scales (MLX/backend/cpu/unary_ops.h:120-152): below
// 2^-6 the value is added to 2^14 so the float adder rounds at the 2^-9
// subnormal step; above, a bias of (half an ulp - 1) plus the odd bit is added
// before truncating.  NaN and |f| >= 464 saturate to 448.
__device__ __forceinline__ uint32_t e4m3_encode_scale(float f) {
  uint32_t u = __float_as_uint(f);
  const uint32_t sign = u & 0x80000000u;
  uint32_t a = u ^ sign;
  uint32_t r;
  if (a >= (543u << 21)) {
    r = 0x7eu;
  } else if (a < (121u << 23)) {
    r = (__float_as_uint(__fadd_rn(__uint_as_float(a), __uint_as_float(141u << 23))) - (141u << 23)) & 0xffu;
  } else {
    const uint32_t odd = (a >> 20) & 1u;
    a += ((uint32_t)(7 - 127) << 23) + 0x7ffffu;
    a += odd;
    r = (a >> 20) & 0xffu;
  }
  return r | (sign >> 24);
}

// Same scale as an f16 (exact: every E4M3 value is an f16 normal or zero).
__device__ __forceinline__ __half e4m3_half(uint32_t b) {
  const __half h = __ushort_as_half(static_cast<unsigned short>(((b & 0x7fu) << 7) | ((b & 0x80u) << 8)));
  return __hmul(h, __float2half(256.0f));
}

// Two E2M1 codes packed in one byte (low nibble first) -> f16x2 in hardware
// (low half = low nibble).  Exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte_in_low_bits) {
  uint32_t out;
  asm("{\n\t.reg .b8 b;\n\tcvt.u8.u32 b, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b;\n\t}"
      : "=r"(out)
      : "r"(byte_in_low_bits));
  return out;
}

// Four f16x2 registers (8 consecutive E2M1 values, little-endian nibbles) from
// one 32-bit code word.
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t out[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
      : "r"(w));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// ---------------------------------------------------------------- mma.sync
// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
__device__ __forceinline__ void mma_16816_f16(float d[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// ---------------------------------------------------------------- mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (after recording B2_STATUS_WAIT_TIMEOUT) if the
// phase did not complete within `limit` polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* status,
                                                  uint32_t limit = (1u << 26)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared completing on an mbarrier (TMA engine).
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace b2
