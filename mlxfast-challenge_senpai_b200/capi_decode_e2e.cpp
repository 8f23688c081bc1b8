// End-to-end timing of decode-shaped MoE block forwards through the bare C
// ABI (include/b2moe.h), called the way a native host (the Swift worker over
// the SwiftPM C module) calls it: every step copies the token from pinned
// host memory, runs b2_moe_block_forward and copies the output back to
// pinned host memory, all on one stream; CUDA events bracket `steps` steps
// after `warmup` untimed ones.
//
// Shapes: BASELINE config 2 (hidden 2048, 128 experts, top-8, ffn 768,
// float32 router, softmax top-8 renormalised).  The weights are synthetic
// NVFP4 bytes (a code pattern and one positive scale byte, set on the
// device) and a seeded random router; `blocks` distinct blocks are rotated
// so the weights read per step come from HBM, not L2.
//
//   capi_decode_e2e [steps=200] [warmup=10] [blocks=16]
// prints one JSON object: {"us_per_step": ..., "steps": ..., "blocks": ...}
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include "b2moe.h"

#define CK(x)                                                                  \
  do {                                                                         \
    cudaError_t e_ = (x);                                                      \
    if (e_ != cudaSuccess) {                                                   \
      std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));            \
      std::exit(2);                                                            \
    }                                                                          \
  } while (0)
#define BK(x)                                                                  \
  do {                                                                         \
    int r_ = (x);                                                              \
    if (r_ != B2_OK) {                                                         \
      std::fprintf(stderr, "%s: %d %s\n", #x, r_, b2_last_error());            \
      std::exit(3);                                                            \
    }                                                                          \
  } while (0)

namespace {

constexpr int64_t H = 2048, F = 768, E = 128;
constexpr int K = 8;

void* dev_bytes(size_t n, int value) {
  void* p = nullptr;
  CK(cudaMalloc(&p, n));
  CK(cudaMemset(p, value, n));
  return p;
}

uint16_t bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

}  // namespace

int main(int argc, char** argv) {
  const int steps = argc > 1 ? std::atoi(argv[1]) : 200;
  const int warmup = argc > 2 ? std::atoi(argv[2]) : 10;
  const int nblk = argc > 3 ? std::atoi(argv[3]) : 16;
  if (steps <= 0 || warmup < 0 || nblk <= 0) return 1;
  cudaStream_t st;
  CK(cudaStreamCreate(&st));
  b2_stream_t bs = reinterpret_cast<b2_stream_t>(st);

  std::mt19937 rng(1234);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  std::vector<float> wr((size_t)E * H);
  std::vector<b2_moe_block> blocks(nblk);
  std::vector<void*> owned;
  size_t ws_bytes = 0;
  for (int b = 0; b < nblk; ++b) {
    b2_moe_block& blk = blocks[b];
    std::memset(&blk, 0, sizeof(blk));
    blk.hidden = H;
    blk.ffn = F;
    blk.n_experts = E;
    blk.top_k = K;
    blk.router_mode = B2_ROUTER_SOFTMAX;
    blk.renorm = 1;
    blk.router_w_dtype = B2_DTYPE_F32;
    blk.routed_scale = 1.0f;
    for (float& v : wr) v = 0.02f * nd(rng);
    void* rw = dev_bytes(wr.size() * 4, 0);
    CK(cudaMemcpy(rw, wr.data(), wr.size() * 4, cudaMemcpyHostToDevice));
    blk.router_w = rw;
    // code bytes such as 0x3a (the E2M1 pair 1.0, 1.5) and scale byte 0x20
    // (0.125 in E4M3): weights of magnitude ~0.1-0.2
    const size_t gu_codes = (size_t)E * F * H / 2, gu_scales = (size_t)E * F * H / 16;
    const size_t dn_codes = (size_t)E * H * F / 2, dn_scales = (size_t)E * H * F / 16;
    blk.gate_codes = static_cast<const uint32_t*>(dev_bytes(gu_codes, 0x3a));
    blk.gate_scales = static_cast<const uint8_t*>(dev_bytes(gu_scales, 0x20));
    blk.up_codes = static_cast<const uint32_t*>(dev_bytes(gu_codes, 0xa3));
    blk.up_scales = static_cast<const uint8_t*>(dev_bytes(gu_scales, 0x20));
    blk.down_codes = static_cast<const uint32_t*>(dev_bytes(dn_codes, 0x2b));
    blk.down_scales = static_cast<const uint8_t*>(dev_bytes(dn_scales, 0x20));
    owned.insert(owned.end(), {rw, (void*)blk.gate_codes, (void*)blk.gate_scales, (void*)blk.up_codes,
                               (void*)blk.up_scales, (void*)blk.down_codes, (void*)blk.down_scales});
    const size_t nb = b2_moe_decode_bank_size(&blk);
    void* bank = dev_bytes(nb, 0);
    owned.push_back(bank);
    BK(b2_moe_prepare_decode_bank(&blk, bank, nb, bs));
    blk.decode_bank = bank;
    const size_t w = b2_moe_block_workspace_size(&blk, 1);
    if (w > ws_bytes) ws_bytes = w;
  }
  void* ws = dev_bytes(ws_bytes, 0);  // zero before first use
  uint16_t *xh, *yh;
  CK(cudaMallocHost(&xh, H * 2));
  CK(cudaMallocHost(&yh, H * 2));
  for (int64_t i = 0; i < H; ++i) xh[i] = bf16_bits(nd(rng));
  void* xd = dev_bytes(H * 2, 0);
  void* yd = dev_bytes(H * 2, 0);
  void* inds = dev_bytes(K * 4, 0);
  void* wts = dev_bytes(K * 4, 0);
  CK(cudaStreamSynchronize(st));

  auto step = [&](int i) {
    CK(cudaMemcpyAsync(xd, xh, H * 2, cudaMemcpyHostToDevice, st));
    BK(b2_moe_block_forward(&blocks[i % nblk], static_cast<const uint16_t*>(xd), 1, nullptr, nullptr,
                            static_cast<uint16_t*>(yd), static_cast<uint32_t*>(inds), static_cast<float*>(wts), ws,
                            ws_bytes, bs));
    CK(cudaMemcpyAsync(yh, yd, H * 2, cudaMemcpyDeviceToHost, st));
  };
  for (int i = 0; i < warmup; ++i) step(i);
  CK(cudaStreamSynchronize(st));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(cudaEventRecord(e0, st));
  for (int i = 0; i < steps; ++i) step(i);
  CK(cudaEventRecord(e1, st));
  CK(cudaEventSynchronize(e1));
  float ms = 0.0f;
  CK(cudaEventElapsedTime(&ms, e0, e1));
  unsigned status = 0;
  BK(b2_device_status(&status, bs));
  std::printf("{\"us_per_step\": %.3f, \"steps\": %d, \"blocks\": %d, \"device_status\": %u}\n", 1e3 * ms / steps,
              steps, nblk, status);
  for (void* p : owned) cudaFree(p);
  cudaFree(ws);
  cudaFree(xd);
  cudaFree(yd);
  cudaFree(inds);
  cudaFree(wts);
  cudaFreeHost(xh);
  cudaFreeHost(yh);
  return status == 0 ? 0 : 4;
}
