// Prefill grouped GEMMs (tcgen05, weights dequantized into TMEM) and their
// helpers; see moe_prefill_gemm.cu.
#pragma once

#include "common.cuh"

namespace b2 {
namespace pf {

// The gate/up grouped GEMM runs on f16 operands: each gathered token row is
// stored as f16 times 2^-p, with p >= 0 the smallest exponent that keeps
// max|x| * 2^-p below 2^15 (p = 0 for rows already below); every bf16 value
// of magnitude >= 2^-17 * 2^p converts exactly, and the GEMM epilogue
// multiplies each token's f32 sums by 2^p (exact).  With f16 operands the
// weights dequantize with one hardware E2M1 -> f16 conversion and one f16
// multiply per pair.  H <= 4096.
constexpr int kRowChunksPerLane = 16;

// One warp converts bf16 row `src` (H values) into dst and writes p to
// *p_out.  CPL = 16-byte chunks per lane (H / 256) when the row fits the
// warp's registers exactly; CPL = 0: any H (the row is read twice).
template <int CPL>
__device__ __forceinline__ void row_to_scaled_f16(const uint16_t* __restrict__ src, int H, uint16_t* __restrict__ dst,
                                                  int* __restrict__ p_out, int lane) {
  constexpr int N = CPL > 0 ? CPL : 1;
  const int chunks = H / 8;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  uint4 v[N];
  unsigned mx = 0;
  auto track = [&](const uint4& q) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) mx = max(mx, max(w[j] & 0x7fffu, (w[j] >> 16) & 0x7fffu));
  };
  if (CPL > 0) {
#pragma unroll
    for (int u = 0; u < N; ++u) {
      v[u] = __ldcg(s4 + lane + 32 * u);
      track(v[u]);
    }
  } else {
    for (int c = lane; c < chunks; c += 32) track(__ldcg(s4 + c));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const unsigned e = (mx >> 7) & 0xffu;
  const int p = (e >= 127u + 15u) ? (int)e - 127 - 14 : 0;
  const float sc = __int_as_float((127 - p) << 23);  // 2^-p
  auto convert = [&](const uint4& q) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 h = __floats2half2_rn(__uint_as_float(w[j] << 16) * sc, __uint_as_float(w[j] & 0xffff0000u) * sc);
      o[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  };
  if (CPL > 0) {
#pragma unroll
    for (int u = 0; u < N; ++u) d4[lane + 32 * u] = convert(v[u]);
  } else {
    for (int c = lane; c < chunks; c += 32) d4[c] = convert(__ldcg(s4 + c));
  }
  if (lane == 0) *p_out = p;
}

// Bytes of the prefill bank (the same as the three MLX-layout banks).
size_t prefill_bank_bytes(const b2_moe_block* blk);
// hidden % 128 == 0, ffn % 128 == 0, at most 1024 experts.
bool prefill_gemm_supported(const b2_moe_block* blk);
int prepare_prefill(const b2_moe_block* blk, void* dst, cudaStream_t st);
// Upper bound of the token tiles of `rows` expert-sorted rows over E experts.
int64_t max_tiles(int64_t E, int64_t rows);
// Whether the block's grouped GEMMs run as 2-CTA pairs (cta_group::2: two
// weight blocks per token tile, each CTA loading half the tile's rows): only
// when the environment sets B2_PREFILL_PAIR=1, for blocks whose gate/up and
// down weight-block counts are both even.
bool pair_mode(const b2_moe_block* blk);
// Token tiles from the expert offsets: tiles[j] = (first sorted row, rows,
// expert, rows rounded up to 16, or 32 for pair mode), *ntiles = count (both
// on the device).
int make_tiles(const uint32_t* offsets, int E, int4* tiles, int* ntiles, bool pair, cudaStream_t st);
// dst[p] = src[order[p] / k] for p < rows (16-bit rows of K values).
int gather_rows(const uint16_t* src, const uint32_t* order, int k, int64_t rows, int K, uint16_t* dst,
                cudaStream_t st);
// The same rows as scaled f16 (row_to_scaled_f16), exponents in xexp [rows].
int gather_rows_f16(const uint16_t* src, const uint32_t* order, int k, int64_t rows, int K, uint16_t* dst, int* xexp,
                    cudaStream_t st);
// mode 0: act[rows][F] = SwiGLU(tok * gate^T, tok * up^T); mode 1:
// y[rows][H] = tok * down^T (bf16 in, bf16 out; tok = the gathered token
// rows for mode 0, the SwiGLU rows for mode 1, both in expert-sorted order).
// Mode 1 writes sorted row r to y[out_order[r]] when out_order is given (the
// sort's order: y comes out in (token, slot) order), else to y[r].
// Expert parallel (mode 1 only): with peer_out, output row r = out_order[...]
// is written to peer_out[r / peer_rows] + (r % peer_rows) * H instead (a
// table of per-rank buffers in device memory, peer pointers included).
// Mode 0 takes the gathered rows as scaled f16 with their exponents
// (tok_exp, gather_rows_f16); mode 1 takes bf16 rows (tok_exp unused).
int expert_gemm(int mode, const b2_moe_block* blk, const uint16_t* tok, int64_t rows, const int4* tiles,
                const int* ntiles, uint16_t* out, const uint32_t* out_order, cudaStream_t st,
                uint16_t* const* peer_out = nullptr, uint32_t peer_rows = 0, const int* tok_exp = nullptr);

}  // namespace pf
}  // namespace b2
