// Prefill grouped GEMMs (tcgen05, weights dequantized into TMEM) and their
// helpers; see moe_prefill_gemm.cu.
#pragma once

#include "common.cuh"

namespace b2 {
namespace pf {

// Bytes of the prefill bank (the same as the three MLX-layout banks).
size_t prefill_bank_bytes(const b2_moe_block* blk);
// hidden % 128 == 0, ffn % 128 == 0, at most 1024 experts.
bool prefill_gemm_supported(const b2_moe_block* blk);
int prepare_prefill(const b2_moe_block* blk, void* dst, cudaStream_t st);
// Upper bound of the token tiles of `rows` expert-sorted rows over E experts.
int64_t max_tiles(int64_t E, int64_t rows);
// Token tiles from the expert offsets: tiles[j] = (first sorted row, rows,
// expert, rows rounded up to 16), *ntiles = count (both on the device).
int make_tiles(const uint32_t* offsets, int E, int4* tiles, int* ntiles, cudaStream_t st);
// dst[p] = src[order[p] / k] for p < rows (16-bit rows of K values).
int gather_rows(const uint16_t* src, const uint32_t* order, int k, int64_t rows, int K, uint16_t* dst,
                cudaStream_t st);
// mode 0: act[rows][F] = SwiGLU(tok * gate^T, tok * up^T); mode 1:
// y[rows][H] = tok * down^T (bf16 in, bf16 out; tok = the gathered token
// rows for mode 0, the SwiGLU rows for mode 1, both in expert-sorted order).
// Mode 1 writes sorted row r to y[out_order[r]] when out_order is given (the
// sort's order: y comes out in (token, slot) order), else to y[r].
// Expert parallel (mode 1 only): with peer_out, output row r = out_order[...]
// is written to peer_out[r / peer_rows] + (r % peer_rows) * H instead (a
// table of per-rank buffers in device memory, peer pointers included).
int expert_gemm(int mode, const b2_moe_block* blk, const uint16_t* tok, int64_t rows, const int4* tiles,
                const int* ntiles, uint16_t* out, const uint32_t* out_order, cudaStream_t st,
                uint16_t* const* peer_out = nullptr, uint32_t peer_rows = 0);

}  // namespace pf
}  // namespace b2
