// MoE epilogue helpers shared by the permute/combine kernels and the fused
// expert blocks.
#pragma once

#include "router.cuh"

namespace b2 {

// SwiGLU on bf16 values with the reference runtime's bf16 steps
// (RM:6843-6852): e = bf16(exp|g|), d = bf16(1+e), y = bf16(1/d),
// sig = g<0 ? y : bf16(1-y), a = bf16(bf16(g*sig) * u).  Every step is an
// explicitly rounded operation (no contraction) so it matches the CPU checker
// bit for bit for equal g and u.
// Two E2M1 codes (byte B of `w`) -> f16x2.
template <int B>
__device__ __forceinline__ uint32_t cvt_byte(uint32_t w) {
  static_assert(B >= 0 && B < 4, "byte index");
  uint32_t out;
  if (B == 0)
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
        : "=r"(out)
        : "r"(w));
  else if (B == 1)
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b1;\n\t}"
        : "=r"(out)
        : "r"(w));
  else if (B == 2)
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b2;\n\t}"
        : "=r"(out)
        : "r"(w));
  else
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b3;\n\t}"
        : "=r"(out)
        : "r"(w));
  return out;
}

// v * 2^e for 0 <= e <= 127: identical to ldexpf(v, e) there (a power of two
// in range scales exactly; overflow gives inf as ldexpf does).
__device__ __forceinline__ float mul_pow2(float v, int e) { return v * __int_as_float((127 + e) << 23); }

// Prepared scale byte (decode and prefill banks): bits 14..7 of the f16
// encoding of the MLX-decoded |scale| ((b & 127) << 7 as a half, times 256;
// exact, the decoded scale has at most 4 significant bits).  The sign of a
// negative scale byte is folded into its group's codes by the bank builders.
__device__ __forceinline__ uint8_t prepared_scale_byte(uint8_t sb) {
  const __half h = __hmul(__ushort_as_half((unsigned short)((sb & 0x7fu) << 7)), __float2half(256.0f));
  return (uint8_t)(__half_as_ushort(h) >> 7);
}

// 16 consecutive 32-bit TMEM columns of this thread's lane (warp-wide).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ float silu_bf16(float g) {
  const float e = round_bf16(b2_expf(fabsf(g)));
  const float d = round_bf16(__fadd_rn(1.0f, e));
  const float y = round_bf16(__frcp_rn(d));
  const float sig = g < 0.0f ? y : round_bf16(__fsub_rn(1.0f, y));
  return round_bf16(__fmul_rn(g, sig));
}
__device__ __forceinline__ float swiglu_bf16(float g, float u) { return round_bf16(__fmul_rn(silu_bf16(g), u)); }

// The same with the SiLU from the exact table (silu_table.cu) when present;
// g must already be a bf16 value.
__device__ __forceinline__ float swiglu_bf16_tab(float g, float u, const uint16_t* __restrict__ tab) {
  const float silu = tab ? bf16_bits_to_f32(__ldg(tab + (__float_as_uint(g) >> 16))) : silu_bf16(g);
  return round_bf16(__fmul_rn(silu, u));
}

// Tail of the weighted combine for 8 consecutive features of token t:
// optional * bf16(routed_scale), + shared, + residual (each rounded to bf16),
// then one 16-byte store.  (RM:7512-7526, RM:9426-9568)
__device__ __forceinline__ void finish_combine(float tot[8], int64_t t, int64_t h0, int64_t H, float routed_scale,
                                               const uint16_t* __restrict__ shared,
                                               const uint16_t* __restrict__ residual, uint16_t* __restrict__ out) {
  const float rs = round_bf16(routed_scale);
  uint4 sv = make_uint4(0, 0, 0, 0), rv = make_uint4(0, 0, 0, 0);
  if (shared) sv = *reinterpret_cast<const uint4*>(shared + t * H + h0);
  if (residual) rv = *reinterpret_cast<const uint4*>(residual + t * H + h0);
  const uint32_t s4[4] = {sv.x, sv.y, sv.z, sv.w}, r4[4] = {rv.x, rv.y, rv.z, rv.w};
  uint32_t o4[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v[2] = {tot[2 * j], tot[2 * j + 1]};
    const float sh[2] = {__uint_as_float(s4[j] << 16), __uint_as_float(s4[j] & 0xffff0000u)};
    const float re[2] = {__uint_as_float(r4[j] << 16), __uint_as_float(r4[j] & 0xffff0000u)};
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (routed_scale != 1.0f) v[q] = round_bf16(__fmul_rn(v[q], rs));
      if (shared) v[q] = round_bf16(__fadd_rn(v[q], sh[q]));
      if (residual) v[q] = round_bf16(__fadd_rn(v[q], re[q]));
    }
    o4[j] = (uint32_t)f32_to_bf16_bits(v[0]) | ((uint32_t)f32_to_bf16_bits(v[1]) << 16);
  }
  *reinterpret_cast<uint4*>(out + t * H + h0) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

// Device pointer of the exact bf16 SiLU table (built on first use outside a
// stream capture; nullptr while unavailable -- callers then use the chain).
const uint16_t* silu_table(cudaStream_t st);

// Multi-CTA stable sort for large n (same positions as launch_gather_sort);
// scratch: gather_sort_scratch_bytes(n, E) bytes (null -> single-CTA sort).
size_t gather_sort_scratch_bytes(int64_t n, int64_t E);
int launch_gather_sort_ws(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order, uint32_t* sorted_keys,
                          uint32_t* inverse, uint32_t* offsets, uint32_t* scratch, cudaStream_t st);
int launch_gather_sort(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order, uint32_t* sorted_keys,
                       uint32_t* inverse, uint32_t* offsets, cudaStream_t st);
int launch_combine(const uint16_t* d, const uint32_t* inverse, const float* w, int64_t T, int k, int64_t H,
                   float routed_scale, const uint16_t* shared, const uint16_t* residual, uint16_t* out,
                   cudaStream_t st);
int launch_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* a, cudaStream_t st);
// y[M, N] = x[M, K] . dequant(codes, scales)^T, bf16 in and out (the
// quantized_matmul kernels).
int qmm_bf16(const uint16_t* x, const uint32_t* codes, const uint8_t* scales, int64_t M, int64_t N, int64_t K,
             uint16_t* y, cudaStream_t st);

// Shared expert of the block (b2_moe_block.shared_gate_codes != NULL):
// scratch bytes for T tokens (0 without one), and the forward
// s = down(silu(gate(x)) * up(x)) into that scratch (*s = its output [T, H],
// nullptr without a shared expert).
size_t shared_scratch_bytes(const b2_moe_block* blk, int64_t T);
int shared_forward(const b2_moe_block* blk, const uint16_t* x, int64_t T, void* scratch, const uint16_t** s,
                   cudaStream_t st);

}  // namespace b2
