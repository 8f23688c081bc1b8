// bf16 SiLU table: entry g (bf16 bits) = bf16 bits of silu(g) computed by
// the reference runtime's bf16 steps (RM:6843-6852: exp(|g|), 1/(1+e), sign
// select, g * sigma, each rounded to bf16).  silu depends only on the 16 input
// bits, so the table is an exact cache of that chain: SwiGLU becomes one
// lookup, one multiply by u and one rounding.  Kernels take the table pointer
// and fall back to the chain when it is null.
#include <mutex>

#include "moe.cuh"

namespace b2 {
namespace {

__device__ uint16_t g_silu_tab[65536];

__global__ void build_silu_table_kernel(uint16_t* tab) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536) tab[i] = f32_to_bf16_bits(silu_bf16(bf16_bits_to_f32((uint16_t)i)));
}

std::mutex g_tab_mu;
uint16_t* g_tab_ptr[64] = {};

}  // namespace

const uint16_t* silu_table(cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_tab_mu);
  if (g_tab_ptr[dev]) return g_tab_ptr[dev];
  // Built once per device on a private stream and waited for, never while the
  // caller's stream is being captured (a capturing caller gets the chain until
  // a later call builds the table).  Relaxed capture mode for this thread
  // keeps the wait from touching a capture running on another stream.
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_silu_tab) != cudaSuccess) return nullptr;
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  if (cudaThreadExchangeStreamCaptureMode(&mode) != cudaSuccess) return nullptr;
  cudaStream_t s = nullptr;
  bool ok = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess;
  if (ok) {
    build_silu_table_kernel<<<256, 256, 0, s>>>(static_cast<uint16_t*>(p));
    ok = cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(s) == cudaSuccess;
    cudaStreamDestroy(s);
  }
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (!ok) return nullptr;
  g_tab_ptr[dev] = static_cast<uint16_t*>(p);
  return g_tab_ptr[dev];
}

}  // namespace b2
