/*
 * b2moe.h -- C ABI of the B200 (sm_100a) NVFP4 quantized-matmul and MoE
 * expert-block library.
 *
 * This is the drop-in boundary for the reference runtime's MoE hot path
 * (morganmcg1/mlxfast-challenge_senpai, Swift over MLX).  Each entry point
 * names the reference interface it replaces (paths relative to the reference
 * root; MLXC = Vendor/mlx-swift/Source/Cmlx/mlx-c/mlx/c, MLX =
 * Vendor/mlx-swift/Source/Cmlx/mlx/mlx, RM =
 * Sources/MLXFastModel/LagunaRuntimeModel.swift, SWL =
 * Vendor/mlx-swift-lm/Libraries/MLXLMCommon/SwitchLayers.swift).
 *
 * Conventions (mirroring the MLX C ABI, MLXC/error.h:15-33 and ops.h):
 *   - every function returns 0 on success and a positive B2_ERR_* code on
 *     failure; the message is available from b2_last_error() (thread-local)
 *     and is passed to the handler installed with b2_set_error_handler();
 *   - all tensor pointers are device pointers owned by the caller, row-major
 *     and contiguous; inputs are read-only;
 *   - work is enqueued on the given CUDA stream (0 = legacy default stream)
 *     and is asynchronous; no function synchronizes unless documented;
 *   - NVFP4 tensors use MLX's layout: codes uint32 [..., rows, K/8] with eight
 *     E2M1 values per word, least-significant nibble first; scales uint8
 *     [..., rows, K/16], one E4M3 byte per 16 consecutive K elements
 *     (MLX/ops.cpp:4873-4978, group_size 16, bits 4, mode "nvfp4").
 *   - bf16/f16 values are passed as raw 16-bit storage.
 *
 * Device addresses of the library's module-scope variables are looked up
 * once per device and kept, so do not keep using the library across a
 * cudaDeviceReset.
 *
 * No entry point allocates device memory except b2_ep_create (the
 * expert-parallel context, allocated once like a communicator): scratch
 * comes from the caller (b2_moe_block_workspace_size) and the status word is
 * a module-scope device variable of the library.
 */
#ifndef B2MOE_H
#define B2MOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2_API __attribute__((visibility("default")))
#else
#define B2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* b2_stream_t; /* same type as cudaStream_t */

/* status codes */
#define B2_OK 0
#define B2_ERR_INVALID_ARGUMENT 1
#define B2_ERR_CUDA 2
#define B2_ERR_UNSUPPORTED 3
#define B2_ERR_DEVICE_STATUS 4

/* device status word values (b2_device_status) */
#define B2_STATUS_OK 0u
#define B2_STATUS_WAIT_TIMEOUT 1u
#define B2_STATUS_BAD_INDEX 2u

/* element types */
#define B2_DTYPE_BF16 0
#define B2_DTYPE_F16 1
#define B2_DTYPE_F32 2

/* router modes */
#define B2_ROUTER_SOFTMAX 0      /* softmax top-k renormalised */
#define B2_ROUTER_SIGMOID_BIAS 1 /* sigmoid + e_score_correction_bias (Laguna, RM:9292-9404) */

/* ------------------------------------------------------------------ */
/* library                                                             */
/* ------------------------------------------------------------------ */
B2_API const char* b2_version(void);

/* Message of the last failing call on this thread ("" if none).
 * Replaces the message channel of mlx_error (MLXC/error.h:15-33). */
B2_API const char* b2_last_error(void);

/* Install a process-wide error callback (NULL restores the default, which
 * only records the message).  Mirrors mlx_set_error_handler
 * (MLXC/error.h:22-26). */
typedef void (*b2_error_handler_func)(const char* msg, void* data);
B2_API void b2_set_error_handler(b2_error_handler_func handler, void* data);

/* Read and clear the current device's status word, which kernels set instead
 * of trapping when a bounded wait gives up or an index is out of range.
 * Synchronizes `stream`. *status receives one of B2_STATUS_*. */
B2_API int b2_device_status(unsigned* status, b2_stream_t stream);

/* ------------------------------------------------------------------ */
/* NVFP4 codec                                                          */
/* ------------------------------------------------------------------ */
/* Quantize float32 rows [rows, K] (K % 16 == 0) to NVFP4 codes/scales,
 * bit-exact to the MLX CPU composition (MLX/ops.cpp:4873-4978; the MLX C
 * entry point is mlx_quantize, MLXC/ops.h:790). */
B2_API int b2_fp_quantize(const float* w, int64_t rows, int64_t K, uint32_t* codes, uint8_t* scales,
                   b2_stream_t stream);

/* Dequantize to `out_dtype` [rows, K] (exact in every dtype).
 * Replaces mlx_dequantize in nvfp4 mode (MLXC/ops.h:359, MLX/ops.cpp:5120-5241). */
B2_API int b2_fp_dequantize(const uint32_t* codes, const uint8_t* scales, int64_t rows, int64_t K,
                     void* out, int out_dtype, b2_stream_t stream);

/* ------------------------------------------------------------------ */
/* quantized matmuls                                                    */
/* ------------------------------------------------------------------ */
/* y[M,N] = x[M,K] . W^T with W = dequant(codes[N,K/8], scales[N,K/16]);
 * y has x's dtype; float32 accumulation.
 * Replaces mlx_quantized_matmul(res, x, w, scales, biases=NULL,
 * transpose=true, group_size=16, bits=4, mode="nvfp4", s)
 * (MLXC/ops.h:809-818, MLX/ops.cpp:4549). */
B2_API int b2_quantized_matmul(const void* x, int x_dtype, const uint32_t* codes, const uint8_t* scales,
                        void* y, int64_t M, int64_t N, int64_t K, b2_stream_t stream);

/* Gathered quantized matmul over P index pairs:
 *   y[i] = x[lhs[i]] . W[rhs[i]]^T,   x [Bx, M, K], W [E, N, K/8] (+ scales),
 *   y [P, M, N] in x's dtype.
 * lhs == NULL means lhs[i] = i (requires Bx == P); rhs == NULL means
 * rhs[i] = i (requires E == P).  Indices outside [0,Bx) / [0,E) are rejected
 * on the device: the pair's output is zeroed and B2_STATUS_BAD_INDEX is
 * recorded.  `sorted_indices` is a hint that rhs is non-decreasing.
 * Replaces mlx_gather_qmm(..., transpose=true, group 16, bits 4, "nvfp4",
 * sorted_indices) (MLXC/ops.h:475-488, MLX/ops.cpp:5338-5437). */
B2_API int b2_gather_qmm(const void* x, int x_dtype, const uint32_t* codes, const uint8_t* scales,
                  const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t P, int64_t Bx,
                  int64_t E, int64_t M, int64_t N, int64_t K, int sorted_indices, void* y,
                  b2_stream_t stream);

/* ------------------------------------------------------------------ */
/* W4A4: NVFP4 activations on the block-scaled tensor cores             */
/* ------------------------------------------------------------------ */
/* Quantize bf16 activations [rows, K] (K % 16 == 0) to NVFP4 in MLX's
 * layout (codes u32 [rows, K/8], scale bytes [rows, K/16]) with the rule of
 * the reference's qqmm (MLX/backend/cpu/quantized.cpp:1094-1129 and
 * :1064-1091: scale byte e4m3(max|x| / 6), code by threshold rounding of
 * x / decode(scale)); bit-exact to it.  x 16-byte aligned. */
B2_API int b2_fp_quantize_activations(const uint16_t* x, int64_t rows, int64_t K, uint32_t* codes,
                                      uint8_t* scales, b2_stream_t stream);

/* y[M, N] (bf16) = Xq . Wq^T for NVFP4 X [M, K] and W [N, K] (codes + scale
 * bytes, MLX layout), f32 accumulation on tcgen05 kind::mxf4nvf4 with one
 * UE4M3 scale per 16 values.  K % 256 == 0; all buffers 16-byte aligned;
 * scale bytes in [0, 0x7e] (what MLX's quantizers produce).  The product of
 * the reference's qqmm after its activation quantization. */
B2_API int b2_nvfp4_gemm(const uint32_t* x_codes, const uint8_t* x_scales, const uint32_t* w_codes,
                         const uint8_t* w_scales, int64_t M, int64_t N, int64_t K, uint16_t* y,
                         b2_stream_t stream);

/* y = qqmm(x, W) in nvfp4 mode: b2_fp_quantize_activations into the
 * workspace (b2_qqmm_workspace_size bytes, 256-byte aligned) then
 * b2_nvfp4_gemm.  Replaces mlx_qqmm(res, x, w, w_scales, group 16, bits 4,
 * "nvfp4", global_scale_x = NULL, global_scale_w = NULL, s)
 * (MLXC/ops.h:790, MLX/ops.h:1524; Ops.swift quantizedQuantizedMM). */
B2_API size_t b2_qqmm_workspace_size(int64_t M, int64_t K);
B2_API int b2_qqmm(const uint16_t* x, const uint32_t* w_codes, const uint8_t* w_scales, int64_t M, int64_t N,
                   int64_t K, uint16_t* y, void* workspace, size_t workspace_bytes, b2_stream_t stream);

/* ------------------------------------------------------------------ */
/* MoE routing, permutation and combine                                 */
/* ------------------------------------------------------------------ */
/* Router logits[rows, E] (float32) = x[rows, H] (bf16) . Wr^T, Wr [E, H] in
 * float32 or bf16 (`w_dtype`).  Summation order (part of the contract, so
 * that top-k indices are reproducible bit for bit): 32 lane partials where
 * lane l accumulates the 4-element chunks c = l, l+32, ... with fused
 * multiply-add in element order, then an xor butterfly over 16,8,4,2,1.
 * H % 4 == 0.  Replaces x.matmul(weight.T).asType(.float32) of the MoE gate
 * (Laguna.swift:166, RM:823-1067 router logits). */
B2_API int b2_moe_router_logits(const uint16_t* x, const void* router_w, int w_dtype, int64_t rows,
                         int64_t E, int64_t H, float* logits, b2_stream_t stream);

/* Top-k routing from float32 logits [rows, E] (E <= 1024, k <= 32).
 *   B2_ROUTER_SOFTMAX: select by logit (the softmax order), weights =
 *     exp(l - lmax) renormalised over the selected experts (renorm ignored);
 *   B2_ROUTER_SIGMOID_BIAS: s = sigmoid(l), select by s + bias[e] (bias may be
 *     NULL), weights = s (divided by their rank-order sum when renorm).
 * Ranking order: larger key first, NaN last, ties (incl. -0 == +0) by the
 * smaller expert index.  inds uint32 [rows, k] in rank order, weights float32
 * [rows, k].  Replaces LagunaRuntimeMoEGate.callAsFunction(x, logits:)
 * (RM:9312, kernels RM:8290-8715, RM:8859-9290; stock LAG:165-180). */
B2_API int b2_moe_router_topk(const float* logits, const float* bias, int mode, int64_t rows, int64_t E,
                       int k, int renorm, uint32_t* inds, float* weights, b2_stream_t stream);

/* Stable counting sort of n = rows*k flat expert ids [n] (< E):
 *   order[p] = flat index of the p-th row in expert order,
 *   sorted_keys[p] = its expert, inverse[i] = position of flat index i,
 *   offsets[E+1] = first position of each expert.
 * Replaces gatherSort / the fused counting-sort scatter (SWL:249-364). */
B2_API int b2_moe_gather_sort(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order,
                       uint32_t* sorted_keys, uint32_t* inverse, uint32_t* offsets,
                       b2_stream_t stream);

/* The same permutation computed by several CTAs (for large n): pass
 * scratch of b2_moe_gather_sort_scratch_size(n, E) bytes (device, 4-byte
 * aligned; contents need no initialisation).  Positions are identical to
 * b2_moe_gather_sort.  No reference counterpart beyond gatherSort itself. */
B2_API size_t b2_moe_gather_sort_scratch_size(int64_t n, int64_t E);
B2_API int b2_moe_gather_sort_ws(const uint32_t* inds, int64_t n, int64_t E, uint32_t* order,
                                 uint32_t* sorted_keys, uint32_t* inverse, uint32_t* offsets, void* scratch,
                                 size_t scratch_bytes, b2_stream_t stream);

/* a[i] = silu(g[i]) * u[i] on bf16 with the reference runtime's bf16 steps
 * (RM:6843-6852).  Replaces compiledSiluProduct (SWL:19-29). */
B2_API int b2_moe_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* a,
                    b2_stream_t stream);

/* Weighted combine of per-(token, slot) expert rows d (bf16, H wide):
 *   out[t] = fold_s total = bf16(bf16(d[t,s] * bf16(w[t,s])) + total)
 * then * bf16(routed_scale) (skipped when 1), + shared[t], + residual[t]
 * (both nullable), all bf16.  d row of (t,s) is d[inverse[t*k+s]] when
 * inverse != NULL (rows in expert-sorted order), else d[t*k+s].
 * Replaces weightedExpertSum (SWL:31-36) with the fused tail of RM:7512-7526
 * and RM:9426-9568. */
B2_API int b2_moe_combine(const uint16_t* d, const uint32_t* inverse, const float* weights, int64_t T,
                   int k, int64_t H, float routed_scale, const uint16_t* shared,
                   const uint16_t* residual, uint16_t* out, b2_stream_t stream);

/* ------------------------------------------------------------------ */
/* MoE expert block                                                     */
/* ------------------------------------------------------------------ */
typedef struct b2_moe_block {
  int64_t hidden;          /* H */
  int64_t ffn;             /* F, per-expert intermediate size */
  int64_t n_experts;       /* E */
  int32_t top_k;           /* k */
  int32_t router_mode;     /* B2_ROUTER_* */
  int32_t renorm;          /* renormalise top-k weights (sigmoid mode) */
  int32_t router_w_dtype;  /* B2_DTYPE_F32 or B2_DTYPE_BF16 */
  float routed_scale;      /* 1.0 for the BASELINE configs, 2.5 for Laguna */
  const void* router_w;    /* [E, H] */
  const float* router_bias;/* [E] or NULL */
  const uint32_t* gate_codes; const uint8_t* gate_scales; /* [E, F, H/8], [E, F, H/16] */
  const uint32_t* up_codes;   const uint8_t* up_scales;   /* [E, F, H/8], [E, F, H/16] */
  const uint32_t* down_codes; const uint8_t* down_scales; /* [E, H, F/8], [E, H, F/16] */
  const void* decode_bank; /* prepared decode bank (b2_moe_prepare_decode_bank) or NULL */
  const void* prefill_bank; /* prepared prefill bank (b2_moe_prepare_prefill_bank) or NULL */
  /* Optional shared expert (Laguna's LagunaRuntimeMLP, RM:7971-8275): a dense
   * NVFP4 SwiGLU MLP hidden -> shared_ffn -> hidden on every token, whose
   * bf16 output is added after the routed scale and before the residual:
   * out = bf16(bf16(routed * scale) + shared) (+ residual) (RM:10170-10186).
   * shared_gate_codes == NULL means none.  For a fused [gate; up] bank pass
   * gate = the bank and up = the bank + shared_ffn rows. */
  int64_t shared_ffn;
  const uint32_t* shared_gate_codes; const uint8_t* shared_gate_scales; /* [Fs, H/8], [Fs, H/16] */
  const uint32_t* shared_up_codes;   const uint8_t* shared_up_scales;   /* [Fs, H/8], [Fs, H/16] */
  const uint32_t* shared_down_codes; const uint8_t* shared_down_scales; /* [H, Fs/8], [H, Fs/16] */
} b2_moe_block;

/* Bytes of the prepared decode bank of `blk` (same as its three NVFP4 banks).
 * No counterpart in the reference API: it is this library's load-time weight
 * re-layout, the analogue of the runtime's prepareFusedRoutedGateUp /
 * packed-scale side bank (RM:9707-9840). */
B2_API size_t b2_moe_decode_bank_size(const b2_moe_block* blk);

/* Re-lay the block's gate/up/down banks into the prepared decode bank: every
 * tile the fused decode kernel streams (8 gate + 8 up rows of one expert; 16
 * down rows of one expert) becomes one contiguous, bank-conflict-swizzled
 * block so it arrives with a single TMA bulk copy.  Run once after loading
 * the weights; set blk->decode_bank to `bank` to use it.  bank: 16-byte
 * aligned device buffer of b2_moe_decode_bank_size(blk) bytes. */
B2_API int b2_moe_prepare_decode_bank(const b2_moe_block* blk, void* bank, size_t bank_bytes,
                                      b2_stream_t stream);

/* SwitchGLU over given routing (SwitchLayers.swift:476-524 with sorted
 * indices): y[t, s] = down_e(silu(gate_e(x[t])) * up_e(x[t])) for
 * e = inds[t, s], bf16 x [tokens, H] -> bf16 y [tokens, k, H], the same
 * arithmetic as the prefill path of b2_moe_block_forward without router and
 * combine.  Needs the block's prepared prefill bank.  inds uint32 [tokens, k]
 * (< n_experts; k in [1, 8], independent of blk->top_k).  Workspace: 256-byte
 * aligned, b2_moe_switch_glu_workspace_size(blk, tokens, k) bytes. */
B2_API size_t b2_moe_switch_glu_workspace_size(const b2_moe_block* blk, int64_t tokens, int k);
B2_API int b2_moe_switch_glu(const b2_moe_block* blk, const uint16_t* x, int64_t tokens, const uint32_t* inds,
                             int k, uint16_t* y, void* workspace, size_t workspace_bytes, b2_stream_t stream);

/* dst[i] = src[idx[i]] for rows of K 16-bit values (K % 8 == 0, 16-byte
 * aligned rows): the row gather of the token permute (gatherSort's
 * x[row_order], SwitchLayers.swift:335-364). */
B2_API int b2_gather_rows16(const void* src, const uint32_t* idx, int64_t n, int64_t K, void* dst,
                            b2_stream_t stream);

/* Bytes of the prepared prefill bank (the same as the three MLX-layout
 * banks together).  No reference counterpart: the reference's prefill GEMMs
 * (gather_qmm, CUQ/quantized.cpp:159-262; Metal MTLQ:2193-2299) read the MLX
 * layout directly. */
B2_API size_t b2_moe_prefill_bank_size(const b2_moe_block* blk);

/* Re-lay the block's banks into the prepared prefill bank: per (expert,
 * 256-row output tile, 64-wide K stage) one contiguous 9 KB tile (codes,
 * then scales pre-decoded to f16 bit patterns) that the grouped GEMM reads
 * with one bulk copy.  Gate/up output tiles hold 128 gate rows followed by
 * the same 128 up rows.  Requires hidden % 256 == 0 and ffn % 128 == 0.
 * Set blk->prefill_bank to `bank` to route calls with more than 8 tokens
 * through the tensor-core grouped GEMMs. */
B2_API int b2_moe_prepare_prefill_bank(const b2_moe_block* blk, void* bank, size_t bank_bytes,
                                       b2_stream_t stream);

/* Device scratch bytes b2_moe_block_forward needs for `tokens` tokens.
 * The workspace must be 256-byte aligned and zero-filled before its first
 * use; its head (69,632 bytes) holds the decode kernels' cross-launch state
 * (per-launch epochs, two alternating sets of counters, tagged router
 * logits), which every call leaves valid for the next, so one workspace can
 * be reused by consecutive calls on a stream, for blocks of any shape and for
 * decode and prefill calls alike (calls that overlap on the GPU need separate
 * workspaces). */
B2_API size_t b2_moe_block_workspace_size(const b2_moe_block* blk, int64_t tokens);

/* Routed expert block for x [tokens, H] (bf16): router logits (or the given
 * `logits` [tokens, E] when non-NULL), top-k, SwiGLU experts, weighted
 * combine, optional `residual` [tokens, H] added last.  out [tokens, H]
 * bf16.  inds/weights (nullable) receive the routing.  Decode-shaped calls
 * (tokens <= 8) take the fused gathered-GEMV path; larger calls take the
 * sorted grouped-GEMM path.  Replaces
 * LagunaRuntimeSparseMoEBlock.callAsFunction(x, residual:, routerLogits:,
 * routerKeys:) (RM:9860-10187) and, for router_mode SOFTMAX with scale 1, the
 * stock SwitchGLU + weightedExpertSum composition (SWL:476-524). */
B2_API int b2_moe_block_forward(const b2_moe_block* blk, const uint16_t* x, int64_t tokens,
                         const float* logits, const uint16_t* residual, uint16_t* out,
                         uint32_t* inds, float* weights, void* workspace, size_t workspace_bytes,
                         b2_stream_t stream);

/* Decode-shaped block forward (tokens <= 8) that allocates nothing and takes
 * no workspace.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory -- a custom-op callback inside another
 * framework's runtime, whose allocator owns all device buffers and hands the
 * callback only the op's inputs and outputs, or a process held to a fixed
 * device-memory budget -- and so cannot supply b2_moe_block_forward's
 * workspace.  Scratch is a 512 KiB static device array inside the library
 * (every GPU that loads the library holds it until exit); calls whose scratch
 * need (b2_moe_block_workspace_size) exceeds it are rejected with
 * B2_ERR_INVALID_ARGUMENT.  The first call on each device looks up the
 * array's device address, so make it before any stream capture.  All calls
 * share the one array and it keeps what the last call left: its head is the
 * decode kernels' cross-launch state (launch epochs, alternating counter sets,
 * tagged logits), which every call leaves valid for the next whatever block
 * that is, and every other byte is written before it is read, so nothing is
 * cleared between calls.  Calls that overlap on the GPU (several streams or
 * host threads at once) race; serialize them.  Arguments as
 * b2_moe_block_forward. */
B2_API int b2_moe_block_decode_static(const b2_moe_block* blk, const uint16_t* x, int64_t tokens,
                                      const float* logits, const uint16_t* residual, uint16_t* out,
                                      uint32_t* inds, float* weights, b2_stream_t stream);

/* ------------------------------------------------------------------ */
/* decode step of a decoder stack (attention + MoE per layer)           */
/* ------------------------------------------------------------------ */
/* Attention half of one decoder layer: RMSNorm, fused NVFP4 q/k/v
 * projection, RoPE (half-split pairs, angle pos * theta^(-2i/head_dim)),
 * KV-cache append, grouped-query attention over positions 0..pos, NVFP4
 * output projection, residual.  Shapes and semantics of the decoder layer
 * of Laguna.swift:22-128 / LagunaRuntimeModel.swift:446-6130 as BASELINE's
 * 4-layer decode configuration states them: no per-head q/k norm, no output
 * gate, no sliding window, full-head RoPE. */
typedef struct b2_attn_layer {
  int64_t hidden;      /* H */
  int64_t n_heads;     /* q heads */
  int64_t n_kv_heads;  /* k/v heads (n_heads % n_kv_heads == 0, <= 8 q heads per kv head) */
  int64_t head_dim;    /* 128 */
  int64_t max_seq;     /* cache length */
  float rope_theta;    /* e.g. 1e6 */
  float rms_eps;       /* e.g. 1e-6 */
  const uint16_t* attn_norm_w;  /* [H] bf16 */
  const uint32_t* qkv_codes; const uint8_t* qkv_scales; /* [(nq + 2 nkv) hd, H/8], [.., H/16]: q rows, k rows, v rows */
  const uint32_t* o_codes;   const uint8_t* o_scales;   /* [H, nq hd / 8], [H, nq hd / 16] */
  const uint16_t* mlp_norm_w;   /* [H] bf16 */
  uint16_t* k_cache;            /* [nkv, max_seq, hd] bf16, 16-byte aligned */
  uint16_t* v_cache;            /* [nkv, max_seq, hd] bf16, 16-byte aligned */
} b2_attn_layer;

/* One decoder layer: x' = h + moe(rms_norm(h)), h = x + attn(x). */
typedef struct b2_decoder_layer {
  b2_attn_layer attn;
  b2_moe_block moe;
} b2_decoder_layer;

/* Workspace bytes of b2_decode_step (256-byte aligned, zero before the first
 * call; reusable by every later call on the stream, like the block
 * workspace whose decode state it holds). */
B2_API size_t b2_decode_step_workspace_size(const b2_decoder_layer* layers, int n_layers);

/* One token (B = 1) through `n_layers` layers at position `pos` (the caches
 * hold positions 0..pos-1; this call writes pos), then the final RMSNorm:
 * out [H] bf16.  Replaces the per-token forward of the reference's decoder
 * stack (LagunaModelInner.callAsFunction over its layers, Laguna.swift;
 * the runtime's decode step, LagunaRuntimeModel.swift). */
B2_API int b2_decode_step(const b2_decoder_layer* layers, int n_layers, const uint16_t* final_norm_w,
                          const uint16_t* x, int64_t pos, uint16_t* out, void* workspace, size_t workspace_bytes,
                          b2_stream_t stream);

/* Test hook, no counterpart in the reference: lets a test drive the decode
 * kernels' timeout path without any GPU fault.  While set, CTA
 * `skip_logit_cta` (>= 0) of every decode-kernel launch leaves its router
 * logits unwritten, so the waits for them run out after `spin_limit` polls
 * (0 = the library's default bound), the launch records
 * B2_STATUS_WAIT_TIMEOUT and returns without touching expert weights.
 * b2_testing_set_decode_fault(-1, 0) restores normal operation.  Process-wide;
 * read when a call is launched. */
B2_API int b2_testing_set_decode_fault(int skip_logit_cta, unsigned spin_limit);

/* ------------------------------------------------------------------ */
/* expert-parallel prefill over NVLink peer memory                      */
/* ------------------------------------------------------------------ */
/* One process per GPU; rank r of `world` owns experts [r*E/world,
 * (r+1)*E/world) and routes its own shard of tokens_per_rank tokens.  The
 * reference runtime has no expert parallelism (its MLX collectives have no
 * all-to-all, MLX/distributed/nccl/nccl.cpp); this is the sharded form of
 * b2_moe_block_forward's sorted prefill branch (RM:9867-10187,
 * SWL:476-524): every rank's output equals b2_moe_block_forward on its own
 * tokens bit for bit.  Dispatch and return are NVLink peer loads and stores
 * into CUDA-IPC-mapped buffers with flag barriers in peer memory; nothing
 * goes through the host between calls. */
#define B2_EP_MAX_RANKS 8
#define B2_EP_HANDLE_BYTES 128
#define B2_EP_PHASE_EVENTS 8

typedef struct b2_ep_ctx b2_ep_ctx;

typedef struct b2_ep_config {
  int32_t rank;             /* this process's rank, [0, world) */
  int32_t world;            /* ranks (GPUs), 1..B2_EP_MAX_RANKS */
  int64_t tokens_per_rank;  /* tokens every rank passes to each call */
  int32_t wait_timeout_ms;  /* bound of each cross-GPU wait (<= 0: 10000) */
  /* Expert placement (nullable; the same on every rank): slot[e] in [0, E),
   * a permutation; expert e lives on rank slot[e] / (E/world) as its local
   * expert slot[e] % (E/world).  NULL: slot[e] = e (contiguous ranges).  A
   * load-balanced placement (hot experts spread over the ranks) evens the
   * ranks' expert work under skewed routing. */
  const int32_t* expert_slot;
} b2_ep_config;

/* Create this rank's context on the current device.  `blk` describes the
 * whole block's router (n_experts = E, router_w [E, H], mode, bias, renorm,
 * routed_scale) but its six bank pointers (and prefill_bank, if set) hold
 * only this rank's E/world experts in MLX layout, in local-slot order (see
 * expert_slot); without a prefill_bank the context prepares one.  Allocates the context's device memory (exported
 * region + scratch, about (world*T*k)*(2H+2F+20) bytes) once, here, as a
 * communicator init does; b2_moe_ep_prefill allocates nothing.  Writes this
 * rank's B2_EP_HANDLE_BYTES-byte handle to `handle`; the host exchanges the
 * handles (any channel: torch.distributed, MPI, a TCP store) and passes all
 * of them, in rank order, to b2_ep_connect.  The context is the
 * communicator handle of this path, in the place of the NCCL communicator
 * of the reference's distributed group (MLX/distributed/distributed.h). */
B2_API int b2_ep_create(const b2_moe_block* blk, const b2_ep_config* cfg, b2_ep_ctx** ctx, void* handle);

/* Map every peer's exported region (CUDA IPC) from `handles`
 * [world][B2_EP_HANDLE_BYTES].  Call once on every rank after all ranks
 * created their contexts. */
B2_API int b2_ep_connect(b2_ep_ctx* ctx, const void* handles);

/* Expert-parallel block forward on this rank's tokens: x [T, H] bf16 with
 * T = tokens_per_rank (on every rank), optional router `logits` [T, E] f32
 * (else computed from x), optional `residual` [T, H]; out [T, H] bf16;
 * inds uint32 / weights f32 [T, k] (nullable) receive the routing.  Every
 * rank must make the same sequence of calls (each call holds two cross-GPU
 * barriers).  A barrier that gives up records B2_STATUS_WAIT_TIMEOUT
 * (b2_device_status) and leaves the context unusable: destroy it. */
B2_API int b2_moe_ep_prefill(b2_ep_ctx* ctx, const uint16_t* x, int64_t tokens, const float* logits,
                             const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights,
                             b2_stream_t stream);

/* Phase timing (no reference counterpart): when enabled, each call records
 * B2_EP_PHASE_EVENTS CUDA events; b2_ep_phase_times then writes the
 * B2_EP_PHASE_EVENTS - 1 intervals of the last call in ms: route, barrier A,
 * keys+sort+gather, gate/up GEMM, down GEMM (with the peer stores),
 * barrier B, combine. */
B2_API int b2_ep_set_phase_timing(b2_ep_ctx* ctx, int enable);
B2_API int b2_ep_phase_times(b2_ep_ctx* ctx, float* ms);

/* Release the context (synchronizes the device).  Peers map this rank's
 * region: destroy only after every rank's last call has completed (a host
 * barrier after a device synchronize). */
B2_API int b2_ep_destroy(b2_ep_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* B2MOE_H */
