// Router helpers shared by the router kernels and the fused MoE blocks.
#pragma once

#include "common.cuh"

namespace b2 {

// Ranking order of the top-k selection: larger key first, NaN after every
// number, equal keys (including -0 == +0) by the smaller expert index.  This
// is the comparator of the reference's top-8 kernels (RM:8392-8411,
// RM:8542-8567).  True if (ka, ia) ranks before (kb, ib).
__device__ __forceinline__ bool ranks_before(float ka, int ia, float kb, int ib) {
  const bool na = isnan(ka), nb = isnan(kb);
  if (na != nb) return nb;
  if (!na && ka != kb) return ka > kb;
  return ia < ib;
}

// Stable logistic function in the reference's form (RM:8316-8318, MLX
// unary_ops.h:77-84): y = 1/(1+exp(|x|)); x < 0 ? y : 1 - y, with the
// library's own exp so that the value is reproducible bit for bit.
__device__ __forceinline__ float sigmoid_stable(float x) {
  const float y = __frcp_rn(__fadd_rn(1.0f, b2_expf(fabsf(x))));
  return x < 0.0f ? y : __fsub_rn(1.0f, y);
}

int launch_router_logits(const uint16_t* x, const void* wr, int w_dtype, int64_t rows, int64_t E, int64_t H,
                         float* logits, cudaStream_t st);
int launch_router_topk(const float* logits, const float* bias, int mode, int64_t rows, int64_t E, int k, int renorm,
                       uint32_t* inds, float* weights, cudaStream_t st);

}  // namespace b2
