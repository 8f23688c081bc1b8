"""ctypes/numpy front end of the CPU checker libraries.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py.  The CUDA product path never imports this module.

Two libraries are wrapped:
  * oracle/_build/liboracle.so   -- the C restatement (nvfp4_oracle.c)
  * oracle/_ref/libref_mlxcpu.so -- the reference's own MLX CPU NVFP4 kernels
    (backend/cpu/quantized.cpp fp_qmm_t, backend/cpu/unary_ops.h FromFP8/ToFP8),
    compiled in place from the reference tree by oracle/Makefile.  Optional:
    `ref_available()` reports whether it was built.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(HERE, "_build", "liboracle.so")
_REF = os.path.join(HERE, "_ref", "libref_mlxcpu.so")

_lib = None
_ref = None

P = ctypes.c_void_p
I64 = ctypes.c_int64


def reference_root():
    """The reference checkout the shim compiles from: $B2_REFERENCE_ROOT, else a
    `reference` directory beside this repository; None when neither exists."""
    cand = os.environ.get("B2_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(cand) else None


def build() -> None:
    """Compile the checker (and the reference shim when the tree exists)."""
    cmd = ["make", "-s", "-C", HERE]
    root = reference_root()
    if root:
        cmd.append(f"REF_ROOT={root}")
    subprocess.run(cmd, check=True)


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB) or os.path.getmtime(_LIB) < os.path.getmtime(
            os.path.join(HERE, "nvfp4_oracle.c")
        ):
            build()
        lib = ctypes.CDLL(_LIB)
        lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
        lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.oracle_e2m1_value.restype = ctypes.c_float
        lib.oracle_e2m1_value.argtypes = [ctypes.c_uint]
        lib.oracle_e4m3_value.restype = ctypes.c_float
        lib.oracle_e4m3_value.argtypes = [ctypes.c_uint8]
        lib.oracle_e4m3_encode.restype = ctypes.c_uint8
        lib.oracle_e4m3_encode.argtypes = [ctypes.c_float]
        lib.oracle_swiglu_one.restype = ctypes.c_float
        lib.oracle_swiglu_one.argtypes = [ctypes.c_float, ctypes.c_float]
        for name in (
            "oracle_quantize_activations",
            "oracle_fp_quantize",
            "oracle_fp_dequantize_f32",
            "oracle_qmm_f32",
            "oracle_qmm_bf16",
            "oracle_gather_qmm_bf16",
            "oracle_router_logits",
            "oracle_topk_softmax",
            "oracle_topk_sigmoid_bias",
            "oracle_gather_sort",
            "oracle_swiglu_bf16",
            "oracle_combine_bf16",
            "oracle_moe_experts",
        ):
            getattr(lib, name).restype = None
        _lib = lib
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF)


def _load_ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError("oracle/_ref/libref_mlxcpu.so not built (reference tree absent)")
        r = ctypes.CDLL(_REF)
        r.ref_from_fp8.restype = ctypes.c_float
        r.ref_from_fp8.argtypes = [ctypes.c_uint8]
        r.ref_to_fp8.restype = ctypes.c_uint8
        r.ref_to_fp8.argtypes = [ctypes.c_float]
        r.ref_fp_qmm_t_f32.restype = None
        r.ref_fp_qmm_t_bf16.restype = None
        r.ref_qdq_nvfp4_bf16.restype = None
        _ref = r
    return _ref


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(P)


# ---------------------------------------------------------------- bf16 utils
def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- codec
def e2m1_value(code: int) -> float:
    return _load().oracle_e2m1_value(code)


def e4m3_value(b: int) -> float:
    return _load().oracle_e4m3_value(b)


def e4m3_encode(f: float) -> int:
    return _load().oracle_e4m3_encode(f)


def fp_quantize(w: np.ndarray):
    """w float32 [..., K] -> (codes uint32 [..., K/8], scales uint8 [..., K/16])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    K = w.shape[-1]
    if K % 16:
        raise ValueError("[quantize] last dimension must be divisible by 16")
    rows = w.size // K
    codes = np.zeros(w.shape[:-1] + (K // 8,), np.uint32)
    scales = np.zeros(w.shape[:-1] + (K // 16,), np.uint8)
    _load().oracle_fp_quantize(_p(w), I64(rows), I64(K), _p(codes), _p(scales))
    return codes, scales


def fp_dequantize(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    K = codes.shape[-1] * 8
    rows = codes.size // codes.shape[-1]
    out = np.zeros(codes.shape[:-1] + (K,), np.float32)
    _load().oracle_fp_dequantize_f32(_p(codes), _p(scales), I64(rows), I64(K), _p(out))
    return out


# ---------------------------------------------------------------- matmuls
def qmm_f32(x: np.ndarray, w: np.ndarray, s: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.zeros((M, N), np.float32)
    _load().oracle_qmm_f32(_p(x), _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(s)),
                           _p(y), I64(M), I64(N), I64(K))
    return y


def qmm_bf16(x_bf16: np.ndarray, w: np.ndarray, s: np.ndarray) -> np.ndarray:
    """bf16 bits in, bf16 bits out (float32 accumulation)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[0]
    y = np.zeros((M, N), np.uint16)
    _load().oracle_qmm_bf16(_p(x), _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(s)),
                            _p(y), I64(M), I64(N), I64(K))
    return y


def gather_qmm_bf16(x_bf16, w, s, lhs, rhs) -> np.ndarray:
    """x [Bx, M, K] bf16 bits; w [E, N, K/8]; pairs (lhs[i], rhs[i]) -> [P, M, N]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    Bx, M, K = x.shape
    E, N, _ = w.shape
    lhs = np.ascontiguousarray(lhs, dtype=np.uint32).reshape(-1)
    rhs = np.ascontiguousarray(rhs, dtype=np.uint32).reshape(-1)
    Pn = lhs.size
    y = np.zeros((Pn, M, N), np.uint16)
    _load().oracle_gather_qmm_bf16(_p(x), _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(s)),
                                   _p(lhs), _p(rhs), I64(Pn), I64(M), I64(N), I64(K), _p(y))
    return y


# ---------------------------------------------------------------- router
def router_logits(x_bf16: np.ndarray, wr: np.ndarray, bf16_weight: bool = False) -> np.ndarray:
    """f32 logits x . wr^T in the library's fixed summation order.  With
    bf16_weight (wr holds bf16 values) each logit is rounded to bf16 once:
    MLX's result type of a bf16 x bf16 matmul, which the reference gate casts
    to f32 (Laguna.swift:166; RM:833-838 stores bfloat(router_result))."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    wr = np.ascontiguousarray(wr, dtype=np.float32)
    T, H = x.shape
    E = wr.shape[0]
    out = np.zeros((T, E), np.float32)
    _load().oracle_router_logits(_p(x), _p(wr), I64(T), I64(E), I64(H), _p(out))
    if bf16_weight:
        out = bf16_to_f32(f32_to_bf16(out))
    return out


def topk_softmax(logits: np.ndarray, k: int):
    l = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = l.shape
    inds = np.zeros((T, k), np.uint32)
    w = np.zeros((T, k), np.float32)
    _load().oracle_topk_softmax(_p(l), I64(T), I64(E), ctypes.c_int(k), _p(inds), _p(w))
    return inds, w


def topk_sigmoid_bias(logits: np.ndarray, bias, k: int, renorm: bool = True):
    l = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = l.shape
    inds = np.zeros((T, k), np.uint32)
    w = np.zeros((T, k), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    _load().oracle_topk_sigmoid_bias(_p(l), None if b is None else _p(b), I64(T), I64(E),
                                     ctypes.c_int(k), ctypes.c_int(int(renorm)), _p(inds), _p(w))
    return inds, w


def gather_sort(inds: np.ndarray, E: int):
    i = np.ascontiguousarray(inds, dtype=np.uint32).reshape(-1)
    n = i.size
    order = np.zeros(n, np.uint32)
    keys = np.zeros(n, np.uint32)
    inv = np.zeros(n, np.uint32)
    offs = np.zeros(E + 1, np.uint32)
    _load().oracle_gather_sort(_p(i), I64(n), I64(E), _p(order), _p(keys), _p(inv), _p(offs))
    return order, keys, inv, offs


def swiglu_bf16(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.uint16)
    u = np.ascontiguousarray(u, dtype=np.uint16)
    a = np.zeros_like(g)
    _load().oracle_swiglu_bf16(_p(g), _p(u), I64(g.size), _p(a))
    return a


def combine_bf16(d, w, routed_scale=1.0, shared=None, residual=None) -> np.ndarray:
    d = np.ascontiguousarray(d, dtype=np.uint16)
    T, k, H = d.shape
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros((T, H), np.uint16)
    sh = None if shared is None else np.ascontiguousarray(shared, dtype=np.uint16)
    rs = None if residual is None else np.ascontiguousarray(residual, dtype=np.uint16)
    _load().oracle_combine_bf16(_p(d), _p(w), I64(T), ctypes.c_int(k), I64(H),
                                ctypes.c_float(routed_scale), None if sh is None else _p(sh),
                                None if rs is None else _p(rs), _p(out))
    return out


def moe_experts(x_bf16, inds, weights, bank, routed_scale=1.0, shared=None, residual=None,
                tokens=None) -> np.ndarray:
    """Routed experts + combine for the listed tokens (all when None).

    bank = dict(gate_w, gate_s, up_w, up_s, down_w, down_s) as numpy arrays.
    Returns out bf16 [T, H]; rows not listed are left zero."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T, H = x.shape
    k = inds.shape[1]
    F = bank["gate_w"].shape[1]
    out = np.zeros((T, H), np.uint16)
    tok = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int64)
    c = lambda a: _p(np.ascontiguousarray(a))
    sh = None if shared is None else np.ascontiguousarray(shared, dtype=np.uint16)
    rs = None if residual is None else np.ascontiguousarray(residual, dtype=np.uint16)
    _load().oracle_moe_experts(
        _p(x), I64(T), I64(H), I64(F), ctypes.c_int(k),
        c(np.ascontiguousarray(inds, dtype=np.uint32)), c(np.ascontiguousarray(weights, dtype=np.float32)),
        c(bank["gate_w"]), c(bank["gate_s"]), c(bank["up_w"]), c(bank["up_s"]),
        c(bank["down_w"]), c(bank["down_s"]), ctypes.c_float(routed_scale),
        None if sh is None else _p(sh), None if rs is None else _p(rs),
        None if tok is None else _p(tok), I64(0 if tok is None else tok.size), _p(out))
    return out


# ---------------------------------------------------------------- reference shim
def ref_from_fp8(b: int) -> float:
    return _load_ref().ref_from_fp8(b)


def ref_to_fp8(f: float) -> int:
    return _load_ref().ref_to_fp8(f)


def ref_qmm_f32(x, w, s) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.zeros((M, N), np.float32)
    _load_ref().ref_fp_qmm_t_f32(_p(y), _p(x), _p(np.ascontiguousarray(w)),
                                 _p(np.ascontiguousarray(s)), ctypes.c_int(M), ctypes.c_int(N),
                                 ctypes.c_int(K))
    return y


def ref_qmm_bf16(x_bf16, w, s) -> np.ndarray:
    """The reference's stock bf16 CPU path (bf16 accumulators)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[0]
    y = np.zeros((M, N), np.uint16)
    _load_ref().ref_fp_qmm_t_bf16(_p(y), _p(x), _p(np.ascontiguousarray(w)),
                                  _p(np.ascontiguousarray(s)), ctypes.c_int(M), ctypes.c_int(N),
                                  ctypes.c_int(K))
    return y


def ref_qdq_nvfp4_bf16(x_bf16):
    """The reference's own activation fake-quantization for qqmm (shim over
    fp_quantize_dequantize's steps): (xhat bf16, per-element codes, scales)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    out = np.zeros_like(x)
    codes = np.zeros(x.shape, np.uint8)
    scales = np.zeros(x.shape[:-1] + (x.shape[-1] // 16,), np.uint8)
    _load_ref().ref_qdq_nvfp4_bf16(_p(x), ctypes.c_size_t(x.size), _p(out), _p(codes), _p(scales))
    return out, codes, scales


def ref_sigmoid(x):
    """The reference's CPU sigmoid (MLX unary_ops.h Sigmoid, MLX's exp)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    _load_ref().ref_sigmoid_f32_array(_p(x), ctypes.c_size_t(x.size), _p(out))
    return out


def ref_softmax_rows(x):
    """The reference's CPU softmax over the last axis (float32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    n = x.shape[-1]
    for r in range(x.size // n):
        _load_ref().ref_softmax_f32(_p(x.reshape(-1, n)[r]), ctypes.c_int(n), _p(out.reshape(-1, n)[r]))
    return out


def select_by_keys(keys, k):
    """Top-k expert ids by the reference runtime's total order (larger key
    first, NaN last, ties by smaller index; RM:8392-8411)."""
    keys = np.asarray(keys, np.float64)
    order = np.lexsort((np.arange(keys.shape[-1])[None, :].repeat(keys.shape[0], 0), -np.nan_to_num(keys, nan=-np.inf)),
                       axis=-1)
    return order[:, :k].astype(np.uint32)


# ---------------------------------------------------------------- W4A4 (qqmm, nvfp4)
def quantize_activations(x_bf16):
    """NVFP4 codes (u32 [rows, K/8]), scale bytes and fake-quantized values of
    bf16 activations, by the reference qqmm's activation quantizer."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, K = x.shape
    codes = np.zeros((rows, K // 8), np.uint32)
    scales = np.zeros((rows, K // 16), np.uint8)
    xhat = np.zeros_like(x)
    _load().oracle_quantize_activations(_p(x), I64(rows), I64(K), _p(codes), _p(scales), _p(xhat))
    return codes, scales, xhat


def qqmm_bf16(x_bf16, w, s):
    """y = qdq(x) . W^T with f32 accumulation, rounded to bf16: the W4A4
    product the block-scaled tensor cores compute (the reference's qqmm on
    its CUDA backend, cuBLASLt with VEC16_UE4M3 scales)."""
    _, _, xhat = quantize_activations(x_bf16)
    return qmm_bf16(xhat, w, s)


# ---------------------------------------------------------------- decode step (config 4)
# numpy restatement of the decoder-layer semantics (Laguna.swift:22-128; MLX
# fast rms_norm / RoPE / scaled_dot_product_attention), rounding to bf16 at
# the same points as the library's kernels.
def rms_norm_bf16(x_bits, w_bits, eps, add_bits=None):
    """(h, n): h = bf16(x + add) (x when add is None), n = bf16(w *
    bf16(h * rsqrt(mean(h^2) + eps))) -- MLX's rms_norm in f32."""
    h = bf16_to_f32(x_bits)
    if add_bits is not None:
        h = bf16_to_f32(f32_to_bf16(h + bf16_to_f32(add_bits)))
    inv = np.float32(1.0) / np.sqrt(np.float32(np.mean(h.astype(np.float64) ** 2)) + np.float32(eps))
    n = bf16_to_f32(f32_to_bf16((h * inv).astype(np.float32)))
    return f32_to_bf16(h), f32_to_bf16((bf16_to_f32(w_bits) * n).astype(np.float32))


def rope_bf16(heads_bits, pos, theta):
    """MLX RoPE, traditional=False: pairs (i, i + hd/2), angle = pos *
    theta^(-2i/hd), in f32, result rounded to bf16.  heads [n, hd]."""
    x = bf16_to_f32(heads_bits).astype(np.float32)
    hd = x.shape[-1]
    i = np.arange(hd // 2, dtype=np.float32)
    inv = np.exp2(-(2 * i / np.float32(hd)) * np.float32(np.log2(theta))).astype(np.float32)
    ang = (np.float32(pos) * inv).astype(np.float32)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
    return f32_to_bf16(np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1).astype(np.float32))


def attention_bf16(q_bits, k_bits, v_bits):
    """softmax(q k^T / sqrt(hd)) v per q head (kv head = q head // group), in
    float64, rounded to bf16.  q [nq, hd], k/v [nkv, L, hd]."""
    q = bf16_to_f32(q_bits).astype(np.float64)
    k = bf16_to_f32(k_bits).astype(np.float64)
    v = bf16_to_f32(v_bits).astype(np.float64)
    nq, hd = q.shape
    group = nq // k.shape[0]
    out = np.empty((nq, hd))
    for hq in range(nq):
        s = k[hq // group] @ q[hq] / np.sqrt(hd)
        p = np.exp(s - s.max())
        out[hq] = (p / p.sum()) @ v[hq // group]
    return f32_to_bf16(out.astype(np.float32))


def decode_step(x_bits, layers, final_norm_w, pos, caches, n_heads, n_kv_heads, theta=1e6, eps=1e-6, top_k=8):
    """One token through the stack.  layers: dicts with attn_norm_w, qkv
    (codes, scales), o (codes, scales), mlp_norm_w, router (f32 [E, H]) and
    bank (moe_experts layout); caches: per layer [k, v] bf16 arrays
    [nkv, max_seq, hd], updated at pos.  Returns the final-normed hidden."""
    hd = 128
    cur = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(1, -1)
    for L, (kc, vc) in zip(layers, caches):
        _, n = rms_norm_bf16(cur, L["attn_norm_w"], eps)
        qkv = qmm_bf16(n, *L["qkv"]).reshape(-1, hd)
        q = rope_bf16(qkv[:n_heads], pos, theta)
        kc[:, pos] = rope_bf16(qkv[n_heads:n_heads + n_kv_heads], pos, theta)
        vc[:, pos] = qkv[n_heads + n_kv_heads:]
        a = attention_bf16(q, kc[:, : pos + 1], vc[:, : pos + 1]).reshape(1, -1)
        o = qmm_bf16(a, *L["o"])
        h, n2 = rms_norm_bf16(cur, L["mlp_norm_w"], eps, add_bits=o)
        ri, rw = topk_softmax(router_logits(n2, L["router"]), top_k)
        cur = moe_experts(n2, ri, rw, L["bank"], residual=h)
    return rms_norm_bf16(cur, final_norm_w, eps)[1]
