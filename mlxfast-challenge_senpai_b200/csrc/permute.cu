// Routed-row permutation (stable counting sort), SwiGLU product and the
// weighted combine.
#include "moe.cuh"

namespace b2 {
namespace {

constexpr int kSortThreads = 1024;

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Single-CTA stable counting sort (SWL:95-333 semantics: ties keep input
// order).  Pass 1 histograms all ids; an exclusive scan gives the expert
// offsets; pass 2 walks the ids in chunks of 1024, ranking equal ids inside a
// warp with match.any and across the warps of a chunk with per-warp
// histograms, so every id lands at offsets[e] + (number of earlier equal ids).
__global__ void __launch_bounds__(kSortThreads)
gather_sort_kernel(const uint32_t* __restrict__ inds, int n, int E, uint32_t* __restrict__ order,
                   uint32_t* __restrict__ sorted_keys, uint32_t* __restrict__ inverse, uint32_t* __restrict__ offsets,
                   unsigned* status) {
  extern __shared__ uint32_t sm[];
  uint32_t* run = sm;              // [E] running position per expert
  uint32_t* hist = sm + E;         // [32][E] per-warp counts of the current chunk
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E; e += blockDim.x) run[e] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const uint32_t e = inds[i];
    if (e < (uint32_t)E) atomicAdd(&run[e], 1u);
    else report_status(status, B2_STATUS_BAD_INDEX);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t acc = 0;
    for (int e = 0; e < E; ++e) {
      const uint32_t c = run[e];
      run[e] = acc;
      offsets[e] = acc;
      acc += c;
    }
    offsets[E] = acc;
  }
  __syncthreads();
  for (int base = 0; base < n; base += kSortThreads) {
    for (int j = tid; j < 32 * E; j += blockDim.x) hist[j] = 0;
    __syncthreads();
    const int i = base + tid;
    uint32_t key = 0xffffffffu;
    if (i < n) {
      key = inds[i];
      if (key >= (uint32_t)E) key = 0xffffffffu;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const uint32_t rank = __popc(peers & lanemask_lt());
    if (key != 0xffffffffu && rank == 0) hist[warp * E + key] = __popc(peers);
    __syncthreads();
    // per expert: prefix over the warps of this chunk
    for (int e = tid; e < E; e += blockDim.x) {
      uint32_t acc = run[e];
      for (int w = 0; w < 32; ++w) {
        const uint32_t c = hist[w * E + e];
        hist[w * E + e] = acc;
        acc += c;
      }
      run[e] = acc;
    }
    __syncthreads();
    if (key != 0xffffffffu) {
      const uint32_t pos = hist[warp * E + key] + rank;
      order[pos] = (uint32_t)i;
      sorted_keys[pos] = key;
      inverse[i] = pos;
    } else if (i < n) {
      inverse[i] = 0xffffffffu;
    }
    __syncthreads();
  }
}

// Multi-CTA version for large n (chunks of kSortThreads ids, one CTA each).
// Pass 1: per-chunk expert histograms.  Pass 2: every chunk derives its base
// position per expert (exclusive scan over experts of the totals plus the
// counts of the earlier chunks) and ranks its ids exactly as the single-CTA
// kernel does for one chunk, so positions are identical.
__global__ void __launch_bounds__(kSortThreads)
sort_hist_kernel(const uint32_t* __restrict__ inds, int n, int E, uint32_t* __restrict__ chunk_hist,
                 unsigned* status) {
  extern __shared__ uint32_t sh[];  // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int i = blockIdx.x * kSortThreads + threadIdx.x;
  if (i < n) {
    const uint32_t e = inds[i];
    if (e < (uint32_t)E) atomicAdd(&sh[e], 1u);
    else report_status(status, B2_STATUS_BAD_INDEX);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_hist[(size_t)blockIdx.x * E + e] = sh[e];
}

__global__ void __launch_bounds__(kSortThreads)
sort_scatter_kernel(const uint32_t* __restrict__ inds, int n, int E, const uint32_t* __restrict__ chunk_hist,
                    uint32_t* __restrict__ order, uint32_t* __restrict__ sorted_keys, uint32_t* __restrict__ inverse,
                    uint32_t* __restrict__ offsets) {
  extern __shared__ uint32_t sm[];
  uint32_t* run = sm;        // [E] this chunk's next position per expert
  uint32_t* hist = sm + E;   // [32][E] per-warp counts of the chunk
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, C = gridDim.x;
  // totals and this chunk's prefix per expert (eight chunk counts in flight
  // per thread: the loads are independent, the integer sums exact)
  for (int e = tid; e < E; e += blockDim.x) {
    uint32_t tot = 0, pre = 0;
    int cc = 0;
    for (; cc + 8 <= C; cc += 8) {
      uint32_t h[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) h[u] = chunk_hist[(size_t)(cc + u) * E + e];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (cc + u < c) pre += h[u];
        tot += h[u];
      }
    }
    for (; cc < C; ++cc) {
      const uint32_t h = chunk_hist[(size_t)cc * E + e];
      if (cc < c) pre += h;
      tot += h;
    }
    run[e] = tot;
    hist[e] = pre;  // scratch until the scan below
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the totals: lane = a run of E/32 experts
    const int per = (E + 31) / 32, b0 = min(E, lane * per), b1 = min(E, b0 + per);
    uint32_t seg = 0;
    for (int e = b0; e < b1; ++e) seg += run[e];
    uint32_t inc = seg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    uint32_t acc = inc - seg;
    for (int e = b0; e < b1; ++e) {
      const uint32_t t = run[e];
      run[e] = acc;
      acc += t;
    }
    if (lane == 31 && c == 0) offsets[E] = inc;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    if (c == 0) offsets[e] = run[e];
    run[e] += hist[e];
  }
  __syncthreads();
  for (int j = tid; j < 32 * E; j += blockDim.x) hist[j] = 0;
  __syncthreads();
  const int i = c * kSortThreads + tid;
  uint32_t key = 0xffffffffu;
  if (i < n) {
    key = inds[i];
    if (key >= (uint32_t)E) key = 0xffffffffu;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  const uint32_t rank = __popc(peers & lanemask_lt());
  if (key != 0xffffffffu && rank == 0) hist[warp * E + key] = __popc(peers);
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    uint32_t acc = run[e];
    for (int w = 0; w < 32; ++w) {
      const uint32_t cnt = hist[w * E + e];
      hist[w * E + e] = acc;
      acc += cnt;
    }
  }
  __syncthreads();
  if (key != 0xffffffffu) {
    const uint32_t pos = hist[warp * E + key] + rank;
    order[pos] = (uint32_t)i;
    sorted_keys[pos] = key;
    inverse[i] = pos;
  } else if (i < n) {
    inverse[i] = 0xffffffffu;
  }
}

__global__ void silu_mul_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u, int64_t n,
                                uint16_t* __restrict__ a) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) a[i] = f32_to_bf16_bits(swiglu_bf16(bf16_bits_to_f32(g[i]), bf16_bits_to_f32(u[i])));
}

// bf16x2 arithmetic for the combine: for bf16 inputs, bf16(a * b) and
// bf16(a + b) computed once in f32 and rounded to bf16 equal the single
// bf16 roundings of these instructions (a product of two bf16 values is exact
// in f32; a sum is exact in f32 unless the exponents differ by more than 16,
// and then the smaller operand is far below half a bf16 ulp of the larger
// for both paths), so these are the reference's steps, two features at a time.
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One thread per (token, 8 consecutive hidden features): the ordered
// weighted fold tot = bf16(bf16(d_s * w_s) + tot) over s = 0..k-1, then the
// finish (RM:7512-7526, RM:9426-9568): * bf16(routed_scale), + shared,
// + residual, each rounded to bf16.
__global__ void combine_kernel(const uint16_t* __restrict__ d, const uint32_t* __restrict__ inverse,
                               const float* __restrict__ w, int64_t T, int k, int64_t H, float routed_scale,
                               const uint16_t* __restrict__ shared, const uint16_t* __restrict__ residual,
                               uint16_t* __restrict__ out) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t hc = H / 8;
  if (idx >= T * hc) return;
  const int64_t t = idx / hc, h0 = (idx % hc) * 8;
  uint32_t tot[4] = {0u, 0u, 0u, 0u};  // +0 in both halves
  // all k (<= 8) rows are loaded before the ordered fold, so their latencies overlap
  uint4 v[8];
  uint32_t rw[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    if (s < k) {
      const int64_t flat = t * k + s;
      const int64_t row = inverse ? (int64_t)inverse[flat] : flat;
      rw[s] = (uint32_t)f32_to_bf16_bits(w[flat]) * 0x00010001u;
      v[s] = *reinterpret_cast<const uint4*>(d + row * H + h0);
    }
  }
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    if (s < k) {
      tot[0] = badd2(bmul2(v[s].x, rw[s]), tot[0]);
      tot[1] = badd2(bmul2(v[s].y, rw[s]), tot[1]);
      tot[2] = badd2(bmul2(v[s].z, rw[s]), tot[2]);
      tot[3] = badd2(bmul2(v[s].w, rw[s]), tot[3]);
    }
  }
  for (int s = 8; s < k; ++s) {  // more than 8 slots: the rest in order, one at a time
    const int64_t flat = t * k + s;
    const int64_t row = inverse ? (int64_t)inverse[flat] : flat;
    const uint32_t r = (uint32_t)f32_to_bf16_bits(w[flat]) * 0x00010001u;
    const uint4 q = *reinterpret_cast<const uint4*>(d + row * H + h0);
    tot[0] = badd2(bmul2(q.x, r), tot[0]);
    tot[1] = badd2(bmul2(q.y, r), tot[1]);
    tot[2] = badd2(bmul2(q.z, r), tot[2]);
    tot[3] = badd2(bmul2(q.w, r), tot[3]);
  }
  if (routed_scale != 1.0f) {
    const uint32_t rs = (uint32_t)f32_to_bf16_bits(routed_scale) * 0x00010001u;
#pragma unroll
    for (int j = 0; j < 4; ++j) tot[j] = bmul2(tot[j], rs);
  }
  if (shared) {
    const uint4 sv = *reinterpret_cast<const uint4*>(shared + t * H + h0);
    tot[0] = badd2(tot[0], sv.x);
    tot[1] = badd2(tot[1], sv.y);
    tot[2] = badd2(tot[2], sv.z);
    tot[3] = badd2(tot[3], sv.w);
  }
  if (residual) {
    const uint4 rv = *reinterpret_cast<const uint4*>(residual + t * H + h0);
    tot[0] = badd2(tot[0], rv.x);
    tot[1] = badd2(tot[1], rv.y);
    tot[2] = badd2(tot[2], rv.z);
    tot[3] = badd2(tot[3], rv.w);
  }
  *reinterpret_cast<uint4*>(out + t * H + h0) = make_uint4(tot[0], tot[1], tot[2], tot[3]);
}

}  // namespace

int launch_gather_sort(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order, uint32_t* sorted_keys,
                       uint32_t* inverse, uint32_t* offsets, cudaStream_t st) {
  const size_t smem = (size_t)(E + 32 * E) * 4;
  const int rc = ensure_dynamic_smem((const void*)gather_sort_kernel, smem, "gather_sort");
  if (rc) return rc;
  gather_sort_kernel<<<1, kSortThreads, smem, st>>>(inds, (int)n, (int)E, order, sorted_keys, inverse, offsets,
                                                    device_status_ptr());
  B2_CHECK_LAUNCH("gather_sort");
  return B2_OK;
}

size_t gather_sort_scratch_bytes(int64_t n, int64_t E) {
  return (size_t)((n + kSortThreads - 1) / kSortThreads) * (size_t)E * 4;
}

int launch_gather_sort_ws(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order, uint32_t* sorted_keys,
                          uint32_t* inverse, uint32_t* offsets, uint32_t* scratch, cudaStream_t st) {
  if (n <= 2 * kSortThreads || scratch == nullptr)
    return launch_gather_sort(inds, n, E, order, sorted_keys, inverse, offsets, st);
  const unsigned C = (unsigned)((n + kSortThreads - 1) / kSortThreads);
  int rc = ensure_dynamic_smem((const void*)sort_hist_kernel, (size_t)E * 4, "gather_sort");
  if (rc) return rc;
  const size_t smem = (size_t)(E + 32 * E) * 4;
  rc = ensure_dynamic_smem((const void*)sort_scatter_kernel, smem, "gather_sort");
  if (rc) return rc;
  sort_hist_kernel<<<C, kSortThreads, (size_t)E * 4, st>>>(inds, (int)n, (int)E, scratch, device_status_ptr());
  B2_CHECK_LAUNCH("gather_sort");
  sort_scatter_kernel<<<C, kSortThreads, smem, st>>>(inds, (int)n, (int)E, scratch, order, sorted_keys, inverse,
                                                     offsets);
  B2_CHECK_LAUNCH("gather_sort");
  return B2_OK;
}

int launch_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* a, cudaStream_t st) {
  if (n == 0) return B2_OK;
  silu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, n, a);
  B2_CHECK_LAUNCH("silu_mul");
  return B2_OK;
}

int launch_combine(const uint16_t* d, const uint32_t* inverse, const float* w, int64_t T, int k, int64_t H,
                   float routed_scale, const uint16_t* shared, const uint16_t* residual, uint16_t* out,
                   cudaStream_t st) {
  const int64_t total = T * (H / 8);
  if (total == 0) return B2_OK;
  combine_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(d, inverse, w, T, k, H, routed_scale, shared,
                                                                  residual, out);
  B2_CHECK_LAUNCH("combine");
  return B2_OK;
}

}  // namespace b2

extern "C" int b2_moe_gather_sort(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order, uint32_t* sorted_keys,
                                  uint32_t* inverse, uint32_t* offsets, b2_stream_t stream) {
  B2_REQUIRE(inds && order && sorted_keys && inverse && offsets, "[gather_sort] null pointer argument");
  B2_REQUIRE(n >= 0 && n <= (int64_t)INT32_MAX, "[gather_sort] invalid count");
  B2_REQUIRE(E > 0 && E <= 1536, "[gather_sort] number of experts must be in [1, 1536]");
  return b2::launch_gather_sort(inds, n, E, order, sorted_keys, inverse, offsets,
                                reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t b2_moe_gather_sort_scratch_size(int64_t n, int64_t E) {
  if (n < 0 || E <= 0) return 0;
  return b2::gather_sort_scratch_bytes(n, E);
}

extern "C" int b2_moe_gather_sort_ws(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order,
                                     uint32_t* sorted_keys, uint32_t* inverse, uint32_t* offsets, void* scratch,
                                     size_t scratch_bytes, b2_stream_t stream) {
  B2_REQUIRE(inds && order && sorted_keys && inverse && offsets, "[gather_sort] null pointer argument");
  B2_REQUIRE(n >= 0 && n <= (int64_t)INT32_MAX, "[gather_sort] invalid count");
  B2_REQUIRE(E > 0 && E <= 1536, "[gather_sort] number of experts must be in [1, 1536]");
  B2_REQUIRE(scratch != nullptr && scratch_bytes >= b2::gather_sort_scratch_bytes(n, E),
             "[gather_sort] scratch too small (%zu < %zu bytes)", scratch_bytes, b2::gather_sort_scratch_bytes(n, E));
  B2_REQUIRE(reinterpret_cast<uintptr_t>(scratch) % 4 == 0, "[gather_sort] scratch must be 4-byte aligned");
  return b2::launch_gather_sort_ws(inds, n, E, order, sorted_keys, inverse, offsets, static_cast<uint32_t*>(scratch),
                                   reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b2_moe_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* a, b2_stream_t stream) {
  B2_REQUIRE(g && u && a, "[silu_mul] null pointer argument");
  B2_REQUIRE(n >= 0, "[silu_mul] invalid count");
  if (n == 0) return B2_OK;
  b2::silu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(g, u, n, a);
  B2_CHECK_LAUNCH("silu_mul");
  return B2_OK;
}

extern "C" int b2_moe_combine(const uint16_t* d, const uint32_t* inverse, const float* weights, int64_t T, int k,
                              int64_t H, float routed_scale, const uint16_t* shared, const uint16_t* residual,
                              uint16_t* out, b2_stream_t stream) {
  B2_REQUIRE(d && weights && out, "[combine] null pointer argument");
  B2_REQUIRE(T >= 0 && k > 0 && H > 0 && H % 8 == 0, "[combine] invalid shape (H must be a multiple of 8)");
  return b2::launch_combine(d, inverse, weights, T, k, H, routed_scale, shared, residual, out,
                            reinterpret_cast<cudaStream_t>(stream));
}
