/*
 * CPU restatement of the reference's NVFP4 / MoE arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in mlxfast-challenge_senpai_b200/csrc.  Only tests/, the smoke entry
 * point and bench.py's CPU-baseline leg load it.  The product path never calls
 * into it and has no CPU fallback.
 *
 * Paths below are relative to the reference project root.  Shorthand:
 *   MLX  = Vendor/mlx-swift/Source/Cmlx/mlx/mlx
 *   CPUQ = MLX/backend/cpu/quantized.cpp
 *   RM   = Sources/MLXFastModel/LagunaRuntimeModel.swift
 *   SWL  = Vendor/mlx-swift-lm/Libraries/MLXLMCommon/SwitchLayers.swift
 *   LAG  = Vendor/mlx-swift-lm/Libraries/MLXLLM/Models/Laguna.swift
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no FMA contraction, so
 * that separate multiply/add steps round exactly like the reference's scalar
 * x86 loops; fmaf() is called explicitly where the CUDA kernels fuse).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* bit helpers                                                          */
/* ------------------------------------------------------------------ */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* float -> bf16, round to nearest even; NaN becomes the canonical quiet NaN. */
EXPORT uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
EXPORT float oracle_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }
static inline float rbf(float f) { return oracle_bf16_to_f32(oracle_f32_to_bf16(f)); }

/* exp(x) as the CUDA library computes it (csrc/common.cuh b2_expf):
 * Cody-Waite reduction with the fdlibm ln2 hi/lo split, degree-7 Taylor
 * polynomial in Horner form with fmaf, exact 2^n scaling.  Same operations in
 * the same order, so CPU and GPU agree bit for bit. */
EXPORT float oracle_expf(float x) {
  if (isnan(x)) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.97208f) return 0.0f;
  const float n = rintf(x * 1.44269504088896341f);
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.42860676533018704e-06f, r);
  float p = 1.98412698412698413e-04f;
  p = fmaf(p, r, 1.38888888888888889e-03f);
  p = fmaf(p, r, 8.33333333333333333e-03f);
  p = fmaf(p, r, 4.16666666666666667e-02f);
  p = fmaf(p, r, 1.66666666666666667e-01f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  return ldexpf(p, (int)n);
}

/* ------------------------------------------------------------------ */
/* a1: NVFP4 codec                                                      */
/* ------------------------------------------------------------------ */
/* E2M1 value of a 4-bit code: bit 3 sign, bits 2..1 exponent, bit 0
 * mantissa; codes 0..7 = 0, .5, 1, 1.5, 2, 3, 4, 6 (CPUQ:31-47). */
EXPORT float oracle_e2m1_value(unsigned code) {
  unsigned mag = code & 7u, e = mag >> 1, m = mag & 1u;
  float v = (e == 0) ? 0.5f * (float)m : ldexpf(1.0f + 0.5f * (float)m, (int)e - 1);
  return (code & 8u) ? -v : v;
}

/* E4M3 scale byte -> float, following MLX's FromFP8
 * (MLX/backend/cpu/unary_ops.h:154-173): bits 6..0 are read as the low bits
 * of an IEEE half with a 5-bit exponent field whose top bit is zero, the
 * half is multiplied by 256, bit 7 negates.  Never NaN: 0x7f -> 480. */
EXPORT float oracle_e4m3_value(uint8_t b) {
  unsigned e = (b >> 3) & 15u, m = b & 7u;
  float v = (e == 0) ? ldexpf((float)m, -9) : ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
  return (b & 0x80u) ? -v : v;
}

/* float -> E4M3 byte with round-to-nearest-even and saturation to 0x7e
 * (448), as MLX's ToFP8 (MLX/backend/cpu/unary_ops.h:120-152).
 * Magnitudes below 2^-6 are rounded by adding 2^14 in float arithmetic so the
 * hardware add performs RNE at the 2^-9 subnormal step; larger magnitudes are
 * rounded with the integer bias trick (add half-ulp-minus-one plus the odd
 * bit, then truncate).  NaN and |f| >= 464 saturate. */
EXPORT uint8_t oracle_e4m3_encode(float f) {
  uint32_t u = f2u(f);
  uint32_t sign = u & 0x80000000u;
  uint32_t a = u ^ sign;
  uint8_t r;
  if (a >= (543u << 21)) {
    r = 0x7e;
  } else if (a < (121u << 23)) {
    const float magic = u2f(141u << 23); /* 2^14 */
    r = (uint8_t)(f2u(u2f(a) + magic) - (141u << 23));
  } else {
    uint32_t odd = (a >> 20) & 1u;
    a += ((uint32_t)(7 - 127) << 23) + 0x7ffffu;
    a += odd;
    r = (uint8_t)(a >> 20);
  }
  return (uint8_t)(r | (sign >> 24));
}

/* a2: NVFP4 quantization of float rows (ops.cpp:4873-4978, nvfp4, no global
 * scale).  Per 16-group: scale = e4m3(max|w| / 6); q = w / decode(scale);
 * code = first index j minimising |q - LUT[j]| (MLX argmin keeps the first
 * minimum and never replaces an initial NaN: backend/cpu/arg_reduce.cpp:41-48).
 * Codes are packed eight per u32, low nibble first. */
EXPORT void oracle_fp_quantize(const float* w, int64_t rows, int64_t K, uint32_t* codes,
                               uint8_t* scales) {
  float lut[16];
  for (int j = 0; j < 16; ++j) lut[j] = oracle_e2m1_value((unsigned)j);
  int64_t groups = K / 16;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t g = 0; g < groups; ++g) {
      const float* src = w + r * K + g * 16;
      float amax = fabsf(src[0]);
      for (int i = 1; i < 16; ++i) {
        float v = fabsf(src[i]);
        if (v > amax) amax = v;
      }
      uint8_t sb = oracle_e4m3_encode(amax / 6.0f);
      scales[r * groups + g] = sb;
      float sd = oracle_e4m3_value(sb);
      uint32_t w0 = 0, w1 = 0;
      for (int i = 0; i < 16; ++i) {
        float q = src[i] / sd;
        unsigned best = 0;
        float bv = fabsf(q - lut[0]);
        for (unsigned j = 1; j < 16; ++j) {
          float d = fabsf(q - lut[j]);
          if (d < bv) { bv = d; best = j; }
        }
        if (i < 8) w0 |= best << (4 * i); else w1 |= best << (4 * (i - 8));
      }
      codes[r * (K / 8) + g * 2] = w0;
      codes[r * (K / 8) + g * 2 + 1] = w1;
    }
  }
}

/* Dequantization (ops.cpp:5120-5241): LUT[code] * decode(scale), exact in
 * f32/bf16/f16 because both factors have few significant bits. */
EXPORT void oracle_fp_dequantize_f32(const uint32_t* codes, const uint8_t* scales, int64_t rows,
                                     int64_t K, float* out) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t k = 0; k < K; ++k) {
      uint32_t word = codes[r * (K / 8) + k / 8];
      unsigned nib = (word >> (4 * (k % 8))) & 15u;
      out[r * K + k] = oracle_e2m1_value(nib) * oracle_e4m3_value(scales[r * (K / 16) + k / 16]);
    }
}

/* ------------------------------------------------------------------ */
/* a3/a4: quantized_matmul and gather_qmm                               */
/* ------------------------------------------------------------------ */
/* y[M,N] = x[M,K] . W^T with float accumulation in the exact order of
 * fp_qmm_t<float,16,4> (CPUQ:491-533): per group a running gsum of x*lut,
 * then sum += scale * gsum. */
EXPORT void oracle_qmm_f32(const float* x, const uint32_t* w, const uint8_t* s, float* y,
                           int64_t M, int64_t N, int64_t K) {
  float lut[16];
  for (int j = 0; j < 16; ++j) lut[j] = oracle_e2m1_value((unsigned)j);
  const int64_t kw = K / 8, kg = K / 16;
  for (int64_t m = 0; m < M; ++m) {
    const float* xr = x + m * K;
    for (int64_t n = 0; n < N; ++n) {
      const uint8_t* wb = (const uint8_t*)(w + n * kw);
      const uint8_t* sr = s + n * kg;
      float sum = 0.0f;
      for (int64_t g = 0; g < kg; ++g) {
        float scale = oracle_e4m3_value(sr[g]);
        float gsum = 0.0f;
        for (int b = 0; b < 8; ++b) {
          uint8_t byte = wb[g * 8 + b];
          gsum += xr[g * 16 + 2 * b] * lut[byte & 15];
          gsum += xr[g * 16 + 2 * b + 1] * lut[(byte >> 4) & 15];
        }
        sum += scale * gsum;
      }
      y[m * N + n] = sum;
    }
  }
}

/* The parity oracle for bf16 activations: MLX CPU quantized_matmul run on
 * astype(x, float32) with the float result rounded to bf16. */
EXPORT void oracle_qmm_bf16(const uint16_t* x, const uint32_t* w, const uint8_t* s, uint16_t* y,
                            int64_t M, int64_t N, int64_t K) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K));
  float* yf = (float*)malloc(sizeof(float) * (size_t)(M * N));
  for (int64_t i = 0; i < M * K; ++i) xf[i] = oracle_bf16_to_f32(x[i]);
  oracle_qmm_f32(xf, w, s, yf, M, N, K);
  for (int64_t i = 0; i < M * N; ++i) y[i] = oracle_f32_to_bf16(yf[i]);
  free(xf);
  free(yf);
}

/* gather_qmm (ops.cpp:5338-5437, CPUQ:805-844): for pair i,
 * y[i] = x[lhs[i]] . W[rhs[i]]^T.  x is [Bx, M, K], W is [E, N, K/8],
 * y is [P, M, N]. */
EXPORT void oracle_gather_qmm_bf16(const uint16_t* x, const uint32_t* w, const uint8_t* s,
                                   const uint32_t* lhs, const uint32_t* rhs, int64_t P, int64_t M,
                                   int64_t N, int64_t K, uint16_t* y) {
  for (int64_t i = 0; i < P; ++i) {
    const uint16_t* xi = x + (int64_t)lhs[i] * M * K;
    const uint32_t* wi = w + (int64_t)rhs[i] * N * (K / 8);
    const uint8_t* si = s + (int64_t)rhs[i] * N * (K / 16);
    oracle_qmm_bf16(xi, wi, si, y + i * M * N, M, N, K);
  }
}

/* ------------------------------------------------------------------ */
/* a5: router                                                           */
/* ------------------------------------------------------------------ */
/* Router logits logits[r,e] = x[r,:] . Wr[e,:] (x bf16, Wr float32), in the
 * summation order the CUDA router kernels use: 32 lane partials, lane l
 * owns 4-element chunks c = l, l+32, ... and accumulates them with fused
 * multiply-add in element order; then an xor-butterfly over offsets
 * 16,8,4,2,1.  H must be a multiple of 4. */
EXPORT void oracle_router_logits(const uint16_t* x, const float* wr, int64_t rows, int64_t E,
                                 int64_t H, float* logits) {
  int64_t chunks = H / 4;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t e = 0; e < E; ++e) {
      float acc[32];
      for (int l = 0; l < 32; ++l) {
        float a = 0.0f;
        for (int64_t c = l; c < chunks; c += 32)
          for (int j = 0; j < 4; ++j)
            a = fmaf(oracle_bf16_to_f32(x[r * H + 4 * c + j]), wr[e * H + 4 * c + j], a);
        acc[l] = a;
      }
      for (int off = 16; off >= 1; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = acc[l] + acc[l ^ off];
        memcpy(acc, nxt, sizeof(acc));
      }
      logits[r * E + e] = acc[0];
    }
  }
}

/* Total order used for selection: larger key first, NaN after every number,
 * equal keys (including -0 == +0) by smaller expert index.  This is the
 * comparator of the reference's decode/prefill top-k kernels
 * (RM:8392-8411, RM:8542-8567). Returns nonzero if (ka,ia) ranks before
 * (kb,ib). */
static int ranks_before(float ka, uint32_t ia, float kb, uint32_t ib) {
  int na = isnan(ka), nb = isnan(kb);
  if (na != nb) return nb;
  if (!na && ka != kb) return ka > kb;
  return ia < ib;
}

static void select_topk(const float* key, int64_t E, int k, uint32_t* out) {
  /* k rounds of selection of the best remaining element; O(kE). */
  unsigned char* used = (unsigned char*)calloc((size_t)E, 1);
  for (int s = 0; s < k; ++s) {
    int64_t best = -1;
    for (int64_t e = 0; e < E; ++e) {
      if (used[e]) continue;
      if (best < 0 || ranks_before(key[e], (uint32_t)e, key[best], (uint32_t)best)) best = e;
    }
    used[best] = 1;
    out[s] = (uint32_t)best;
  }
  free(used);
}

/* Softmax router (BASELINE mode): top-k of softmax(logits) renormalised over
 * the selected experts.  Selection uses the logits themselves (softmax is
 * monotone, so this is the softmax order with its rounding ties broken by
 * the logit and then the index).  Weights: exp(l_i - max) / sum over the
 * selected in rank order. */
EXPORT void oracle_topk_softmax(const float* logits, int64_t rows, int64_t E, int k,
                                uint32_t* inds, float* weights) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* l = logits + r * E;
    uint32_t* ir = inds + r * k;
    select_topk(l, E, k, ir);
    float mx = l[ir[0]];
    float tot = 0.0f, ev[64];
    for (int s = 0; s < k; ++s) { ev[s] = oracle_expf(l[ir[s]] - mx); tot += ev[s]; }
    for (int s = 0; s < k; ++s) weights[r * k + s] = ev[s] / tot;
  }
}

/* Sigmoid + correction-bias router (Laguna mode, LAG:165-180, RM:8290-8411):
 * s = sigmoid(l) in the stable form x<0 ? y : 1-y with y = 1/(1+exp(|x|));
 * choice key = s + bias; weights = s[idx], renormalised (when renorm) by a
 * left fold total = s_i + total in rank order. */
EXPORT void oracle_topk_sigmoid_bias(const float* logits, const float* bias, int64_t rows,
                                     int64_t E, int k, int renorm, uint32_t* inds,
                                     float* weights) {
  float* sc = (float*)malloc(sizeof(float) * (size_t)E);
  float* key = (float*)malloc(sizeof(float) * (size_t)E);
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t e = 0; e < E; ++e) {
      float x = logits[r * E + e];
      float y = 1.0f / (1.0f + oracle_expf(fabsf(x)));
      sc[e] = x < 0.0f ? y : 1.0f - y;
      key[e] = sc[e] + (bias ? bias[e] : 0.0f);
    }
    uint32_t* ir = inds + r * k;
    select_topk(key, E, k, ir);
    float tot = 0.0f;
    for (int s = 0; s < k; ++s) tot = sc[ir[s]] + tot;
    for (int s = 0; s < k; ++s) weights[r * k + s] = renorm ? sc[ir[s]] / tot : sc[ir[s]];
  }
  free(sc);
  free(key);
}

/* ------------------------------------------------------------------ */
/* a6: stable counting sort of routed rows (SWL:95-372)                 */
/* ------------------------------------------------------------------ */
/* inds: n flat expert ids (token-major, k per token).  Outputs:
 *   order[p]          flat index of the p-th row in expert order (stable)
 *   sorted_keys[p]    expert id of that row
 *   inverse[i]        position p of flat index i
 *   offsets[E+1]      first position of each expert */
EXPORT void oracle_gather_sort(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order,
                               uint32_t* sorted_keys, uint32_t* inverse, uint32_t* offsets) {
  memset(offsets, 0, sizeof(uint32_t) * (size_t)(E + 1));
  for (int64_t i = 0; i < n; ++i) offsets[inds[i] + 1]++;
  for (int64_t e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
  uint32_t* cur = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)E);
  memcpy(cur, offsets, sizeof(uint32_t) * (size_t)E);
  for (int64_t i = 0; i < n; ++i) {
    uint32_t p = cur[inds[i]]++;
    order[p] = (uint32_t)i;
    sorted_keys[p] = inds[i];
    inverse[i] = p;
  }
  free(cur);
}

/* ------------------------------------------------------------------ */
/* a7: SwiGLU in bf16 steps, as the reference runtime's fused kernels    */
/* (RM:6843-6852): e = bf16(exp|g|), d = bf16(1+e), y = bf16(1/d),      */
/* sig = g<0 ? y : bf16(1-y), a = bf16(bf16(g*sig) * u).                */
/* ------------------------------------------------------------------ */
EXPORT float oracle_swiglu_one(float g, float u) {
  float e = rbf(oracle_expf(fabsf(g)));
  float d = rbf(1.0f + e);
  float y = rbf(1.0f / d);
  float sig = g < 0.0f ? y : rbf(1.0f - y);
  float silu = rbf(g * sig);
  return rbf(silu * u);
}

EXPORT void oracle_swiglu_bf16(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* a) {
  for (int64_t i = 0; i < n; ++i)
    a[i] = oracle_f32_to_bf16(oracle_swiglu_one(oracle_bf16_to_f32(g[i]), oracle_bf16_to_f32(u[i])));
}

/* ------------------------------------------------------------------ */
/* a8: weighted combine (SWL:31-36 stock, fused form RM:7512-7526)       */
/* ------------------------------------------------------------------ */
/* out[t,h] = fold over slots s=0..k-1 of total = bf16(bf16(d*bf16(w)) + total)
 * starting at bf16 zero; then optional * bf16(routed_scale), + shared,
 * + residual, each rounded to bf16.  d is [T, k, H] (token-slot order). */
EXPORT void oracle_combine_bf16(const uint16_t* d, const float* w, int64_t T, int k, int64_t H,
                                float routed_scale, const uint16_t* shared,
                                const uint16_t* residual, uint16_t* out) {
  float rs = rbf(routed_scale);
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < H; ++h) {
      float total = 0.0f;
      for (int s = 0; s < k; ++s) {
        float rw = rbf(w[t * k + s]);
        float prod = rbf(oracle_bf16_to_f32(d[(t * k + s) * H + h]) * rw);
        total = rbf(prod + total);
      }
      if (routed_scale != 1.0f) total = rbf(total * rs);
      if (shared) total = rbf(total + oracle_bf16_to_f32(shared[t * H + h]));
      if (residual) total = rbf(total + oracle_bf16_to_f32(residual[t * H + h]));
      out[t * H + h] = oracle_f32_to_bf16(total);
    }
}

/* ------------------------------------------------------------------ */
/* a10: MoE block for a subset of tokens                                */
/* ------------------------------------------------------------------ */
/* Routed SwitchGLU block for the tokens listed in `tok` (all tokens when
 * tok == NULL), given precomputed routing (inds/weights [T,k]).  Banks:
 * gate/up [E, F, H/8] codes + [E, F, H/16] scales, down [E, H, F/8] +
 * [E, H, F/16].  Writes out rows for the listed tokens only. */
EXPORT void oracle_moe_experts(const uint16_t* x, int64_t T, int64_t H, int64_t F, int k,
                               const uint32_t* inds, const float* weights,
                               const uint32_t* gw, const uint8_t* gs, const uint32_t* uw,
                               const uint8_t* us, const uint32_t* dw, const uint8_t* ds,
                               float routed_scale, const uint16_t* shared,
                               const uint16_t* residual, const int64_t* tok, int64_t ntok,
                               uint16_t* out) {
  uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)F);
  uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)F);
  uint16_t* a = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)F);
  uint16_t* d = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(k * H));
  int64_t count = tok ? ntok : T;
  for (int64_t i = 0; i < count; ++i) {
    int64_t t = tok ? tok[i] : i;
    for (int s = 0; s < k; ++s) {
      uint32_t e = inds[t * k + s];
      oracle_qmm_bf16(x + t * H, gw + (int64_t)e * F * (H / 8), gs + (int64_t)e * F * (H / 16), g, 1, F, H);
      oracle_qmm_bf16(x + t * H, uw + (int64_t)e * F * (H / 8), us + (int64_t)e * F * (H / 16), u, 1, F, H);
      oracle_swiglu_bf16(g, u, F, a);
      oracle_qmm_bf16(a, dw + (int64_t)e * H * (F / 8), ds + (int64_t)e * H * (F / 16), d + s * H, 1, H, F);
    }
    oracle_combine_bf16(d, weights + t * k, 1, k, H, routed_scale,
                        shared ? shared + t * H : NULL, residual ? residual + t * H : NULL,
                        out + t * H);
  }
  free(g);
  free(u);
  free(a);
  free(d);
}

/* E2M1 code of x by the threshold rule of the reference's activation
 * quantizer (to_fp4_e2m1, MLX/backend/cpu/quantized.cpp:1064-1091): ties
 * round up in magnitude at 0.75, 1.75, 3.5 and down at 0.25, 1.25, 2.5, 5;
 * NaN -> 7; sign from the sign bit. */
static uint8_t fp4_threshold(float x) {
  if (isnan(x)) return 0x7;
  const uint8_t sign = signbit(x) ? 0x8 : 0x0;
  x = fabsf(x);
  uint8_t b;
  if (x > 5.0f) b = 7;
  else if (x >= 3.5f) b = 6;
  else if (x > 2.5f) b = 5;
  else if (x >= 1.75f) b = 4;
  else if (x > 1.25f) b = 3;
  else if (x >= 0.75f) b = 2;
  else if (x > 0.25f) b = 1;
  else b = 0;
  return b | sign;
}

/* Activation NVFP4 quantization of the reference's qqmm (QQMatmul::eval_cpu
 * -> fp_quantize_dequantize, MLX/backend/cpu/quantized.cpp:1094-1129,
 * 1322-1360) on bf16 rows [rows, K]: per 16-group scale byte
 * e4m3(max|x| / 6), element code by the threshold rule of x / decode(scale)
 * (code 0 when the scale decodes to 0); codes packed in MLX's layout (u32
 * [rows, K/8], low nibble first), plus the fake-quantized values
 * bf16(decode(scale) * LUT[code]) in xhat (nullable). */
EXPORT void oracle_quantize_activations(const uint16_t* x, int64_t rows, int64_t K, uint32_t* codes,
                                        uint8_t* scales, uint16_t* xhat) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t g = 0; g < K / 16; ++g) {
      const uint16_t* v = x + r * K + g * 16;
      float amax = -INFINITY;
      for (int j = 0; j < 16; ++j) {
        const float a = fabsf(oracle_bf16_to_f32(v[j]));
        if (a > amax) amax = a;
      }
      const uint8_t sb = oracle_e4m3_encode(amax / 6.0f);
      const float sd = oracle_e4m3_value(sb);
      scales[r * (K / 16) + g] = sb;
      uint32_t w0 = 0, w1 = 0;
      for (int j = 0; j < 16; ++j) {
        const float q = sd == 0.0f ? 0.0f : oracle_bf16_to_f32(v[j]) / sd;
        const uint8_t c = fp4_threshold(q);
        if (j < 8) w0 |= (uint32_t)c << (4 * j); else w1 |= (uint32_t)c << (4 * (j - 8));
        if (xhat) xhat[r * K + g * 16 + j] = oracle_f32_to_bf16(sd * oracle_e2m1_value(c));
      }
      codes[(r * K + g * 16) / 8] = w0;
      codes[(r * K + g * 16) / 8 + 1] = w1;
    }
}
