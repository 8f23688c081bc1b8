"""Python front end of libb2moe (the B200 NVFP4 / MoE C ABI in include/b2moe.h).

The functions mirror the reference's operator API for this path -- MLX's
``quantize`` / ``dequantize`` / ``quantized_matmul`` / ``gather_qmm`` in
``mode="nvfp4"`` and the MoE gate / SwitchGLU / sparse-block modules -- with the
same argument meaning and MLX-style ``[op] ...`` error messages (ValueError for
invalid arguments).  Tensors are torch CUDA tensors; device memory, streams
and ``torch.distributed`` are plumbing only: every op runs a kernel from
libb2moe.so.  There is no CPU fallback: without the library or a GPU the
calls raise.
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libb2moe.so")

B2_OK = 0
B2_ERR_INVALID_ARGUMENT = 1
B2_ERR_CUDA = 2
B2_ERR_UNSUPPORTED = 3
B2_ERR_DEVICE_STATUS = 4

STATUS_OK = 0
STATUS_WAIT_TIMEOUT = 1
STATUS_BAD_INDEX = 2

DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2
ROUTER_SOFTMAX, ROUTER_SIGMOID_BIAS = 0, 1

_DT = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16, torch.float32: DTYPE_F32}

_VP = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

_lib = None


class B2Error(RuntimeError):
    pass


class _Block(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int64),
        ("ffn", ctypes.c_int64),
        ("n_experts", ctypes.c_int64),
        ("top_k", ctypes.c_int32),
        ("router_mode", ctypes.c_int32),
        ("renorm", ctypes.c_int32),
        ("router_w_dtype", ctypes.c_int32),
        ("routed_scale", ctypes.c_float),
        ("router_w", _VP),
        ("router_bias", _VP),
        ("gate_codes", _VP), ("gate_scales", _VP),
        ("up_codes", _VP), ("up_scales", _VP),
        ("down_codes", _VP), ("down_scales", _VP),
        ("decode_bank", _VP),
        ("prefill_bank", _VP),
        ("shared_ffn", ctypes.c_int64),
        ("shared_gate_codes", _VP), ("shared_gate_scales", _VP),
        ("shared_up_codes", _VP), ("shared_up_scales", _VP),
        ("shared_down_codes", _VP), ("shared_down_scales", _VP),
    ]


def lib() -> ctypes.CDLL:
    """Load libb2moe.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libb2moe.so not built: run python {os.path.join(HERE, 'build.py')}")
        L = ctypes.CDLL(LIB_PATH)
        L.b2_version.restype = ctypes.c_char_p
        L.b2_last_error.restype = ctypes.c_char_p
        L.b2_moe_block_workspace_size.restype = ctypes.c_size_t
        L.b2_moe_block_workspace_size.argtypes = [ctypes.POINTER(_Block), _I64]
        L.b2_moe_decode_bank_size.restype = ctypes.c_size_t
        L.b2_moe_decode_bank_size.argtypes = [ctypes.POINTER(_Block)]
        L.b2_moe_gather_sort_scratch_size.restype = ctypes.c_size_t
        L.b2_moe_gather_sort_scratch_size.argtypes = [_I64, _I64]
        L.b2_moe_switch_glu_workspace_size.restype = ctypes.c_size_t
        L.b2_moe_switch_glu_workspace_size.argtypes = [ctypes.POINTER(_Block), _I64, _I]
        L.b2_moe_prefill_bank_size.restype = ctypes.c_size_t
        L.b2_moe_prefill_bank_size.argtypes = [ctypes.POINTER(_Block)]
        for name in ("b2_fp_quantize", "b2_fp_dequantize", "b2_quantized_matmul", "b2_gather_qmm",
                     "b2_moe_router_logits", "b2_moe_router_topk", "b2_moe_gather_sort", "b2_moe_silu_mul",
                     "b2_moe_combine", "b2_moe_block_forward", "b2_device_status", "b2_moe_prepare_decode_bank",
                     "b2_moe_prepare_prefill_bank", "b2_moe_gather_sort_ws",
                     "b2_moe_switch_glu", "b2_gather_rows16", "b2_fp_quantize_activations", "b2_nvfp4_gemm",
                     "b2_qqmm"):
            getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def version() -> str:
    return lib().b2_version().decode()


def _check(rc: int) -> None:
    if rc != B2_OK:
        msg = lib().b2_last_error().decode()
        if rc == B2_ERR_INVALID_ARGUMENT:
            raise ValueError(msg)
        raise B2Error(f"b2moe error {rc}: {msg}")


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("b2moe operates on CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("b2moe requires contiguous tensors")
    return _VP(t.data_ptr())


def _stream(t: Optional[torch.Tensor] = None):
    dev = t.device if t is not None else torch.device("cuda", torch.cuda.current_device())
    return _VP(torch.cuda.current_stream(dev).cuda_stream)


def device_status() -> int:
    """Read and clear the device status word (B2_STATUS_*)."""
    v = ctypes.c_uint(0)
    _check(lib().b2_device_status(ctypes.byref(v), _stream()))
    return v.value


def _nvfp4_params(op: str, group_size, bits, mode: str, biases, transpose=True):
    if mode != "nvfp4":
        raise ValueError(f"[{op}] only mode='nvfp4' is implemented by this library (got '{mode}').")
    if group_size not in (None, 16):
        raise ValueError(f"[{op}] nvfp4 quantization requires group size 16 but got {group_size}.")
    if bits not in (None, 4):
        raise ValueError(f"[{op}] nvfp4 quantization requires bits to be 4 but got {bits}.")
    if biases is not None:
        raise ValueError(f"[{op}] biases must be null for quantization mode 'nvfp4'.")
    if not transpose:
        raise ValueError(f"[{op}] only transpose=True is supported for nvfp4.")


# ---------------------------------------------------------------------- codec
def quantize(w: torch.Tensor, group_size: Optional[int] = None, bits: Optional[int] = None,
             mode: str = "nvfp4"):
    """mx.quantize(w, mode="nvfp4") -> (codes uint32 [..., K/8], scales uint8 [..., K/16])."""
    _nvfp4_params("quantize", group_size, bits, mode, None)
    if w.dtype != torch.float32:
        raise ValueError("[quantize] this library quantizes float32 weights")
    w = w.contiguous()
    K = w.shape[-1]
    if K % 16:
        raise ValueError(f"[quantize] The last dimension of the matrix needs to be divisible by the "
                         f"quantization group size 16. However the provided matrix has shape {tuple(w.shape)}")
    rows = w.numel() // K
    codes = torch.empty(*w.shape[:-1], K // 8, dtype=torch.int32, device=w.device)
    scales = torch.empty(*w.shape[:-1], K // 16, dtype=torch.uint8, device=w.device)
    _check(lib().b2_fp_quantize(_ptr(w), _I64(rows), _I64(K), _ptr(codes), _ptr(scales), _stream(w)))
    return codes, scales


def dequantize(codes: torch.Tensor, scales: torch.Tensor, biases=None, group_size: Optional[int] = None,
               bits: Optional[int] = None, mode: str = "nvfp4", dtype: torch.dtype = torch.bfloat16):
    _nvfp4_params("dequantize", group_size, bits, mode, biases)
    K = codes.shape[-1] * 8
    if tuple(scales.shape[:-1]) != tuple(codes.shape[:-1]) or scales.shape[-1] * 16 != K:
        raise ValueError("[dequantize] Shape of scales does not match the matrix given the quantization "
                         f"parameters. Provided matrix of shape {tuple(codes.shape)} and scales of shape "
                         f"{tuple(scales.shape)}.")
    rows = codes.numel() // codes.shape[-1]
    out = torch.empty(*codes.shape[:-1], K, dtype=dtype, device=codes.device)
    _check(lib().b2_fp_dequantize(_ptr(codes), _ptr(scales), _I64(rows), _I64(K), _ptr(out), _I(_DT[dtype]),
                                  _stream(codes)))
    return out


# ---------------------------------------------------------------------- matmuls
def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases=None, transpose: bool = True,
                     group_size: Optional[int] = None, bits: Optional[int] = None, mode: str = "nvfp4"):
    """mx.quantized_matmul(x, w, scales, transpose=True, mode="nvfp4"): x [..., M, K] -> [..., M, N]."""
    _nvfp4_params("quantized_matmul", group_size, bits, mode, biases, transpose)
    if w.dim() != 2:
        raise ValueError("[quantized_matmul] batched weights are handled by gather_qmm")
    N, K = w.shape[0], w.shape[1] * 8
    if x.shape[-1] != K:
        raise ValueError(f"[quantized_matmul] Last dimension of first input with shape (..., {x.shape[-1]}) "
                         f"does not match the expanded quantized matrix ({N}, {K}) computed from shape "
                         f"{tuple(w.shape)} with group_size=16, bits=4 and transpose=true")
    x = x.contiguous()
    M = x.numel() // K
    y = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    if M == 0:
        return y
    _check(lib().b2_quantized_matmul(_ptr(x), _I(_DT[x.dtype]), _ptr(w), _ptr(scales), _ptr(y), _I64(M), _I64(N),
                                     _I64(K), _stream(x)))
    return y


def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases=None,
               lhs_indices: Optional[torch.Tensor] = None, rhs_indices: Optional[torch.Tensor] = None,
               transpose: bool = True, group_size: Optional[int] = None, bits: Optional[int] = None,
               mode: str = "nvfp4", sorted_indices: bool = False):
    """mx.gather_qmm in nvfp4 mode.

    x [*Bx, M, K], w [*E, N, K/8]; the indices (broadcast together) select the
    batch entries; output shape = indices.shape + [M, N]."""
    _nvfp4_params("gather_qmm", group_size, bits, mode, biases, transpose)
    if lhs_indices is None and rhs_indices is None:
        return quantized_matmul(x, w, scales, transpose=True, mode=mode) if w.dim() == 2 else \
            _batched_qmm(x, w, scales)
    N, K = w.shape[-2], w.shape[-1] * 8
    if x.shape[-1] != K:
        raise ValueError(f"[gather_qmm] Last dimension of first input with shape (..., {x.shape[-1]}) does not "
                         f"match the expanded quantized matrix ({N}, {K})")
    M = x.shape[-2]
    Bx = x.numel() // (M * K)
    E = w.numel() // (N * w.shape[-1])
    if lhs_indices is None:
        lhs_indices = torch.arange(Bx, device=x.device, dtype=torch.int32).reshape(x.shape[:-2])
    if rhs_indices is None:
        rhs_indices = torch.arange(E, device=x.device, dtype=torch.int32).reshape(w.shape[:-2])
    for t, nm in ((lhs_indices, "lhs_indices"), (rhs_indices, "rhs_indices")):
        if t.dtype.is_floating_point:
            raise ValueError(f"[gather_qmm] Got {nm} with invalid dtype. Indices must be integral.")
    lhs_b, rhs_b = torch.broadcast_tensors(lhs_indices, rhs_indices)
    out_shape = tuple(lhs_b.shape) + (M, N)
    lhs_c = lhs_b.reshape(-1).to(torch.int32).contiguous()
    rhs_c = rhs_b.reshape(-1).to(torch.int32).contiguous()
    P = lhs_c.numel()
    x = x.contiguous()
    y = torch.empty(P, M, N, dtype=x.dtype, device=x.device)
    if P:
        _check(lib().b2_gather_qmm(_ptr(x), _I(_DT[x.dtype]), _ptr(w.contiguous()), _ptr(scales.contiguous()),
                                   _ptr(lhs_c), _ptr(rhs_c), _I64(P), _I64(Bx), _I64(E), _I64(M), _I64(N), _I64(K),
                                   _I(int(sorted_indices)), _ptr(y), _stream(x)))
    return y.reshape(out_shape)


def _batched_qmm(x, w, scales):
    E = w.numel() // (w.shape[-2] * w.shape[-1])
    idx = torch.arange(E, device=x.device, dtype=torch.int32).reshape(w.shape[:-2])
    return gather_qmm(x, w, scales, rhs_indices=idx)


# ---------------------------------------------------------------------- W4A4
def quantize_activations(x: torch.Tensor):
    """NVFP4 codes (int32 view of u32 [..., K/8]) and scale bytes of bf16
    activations by the reference qqmm's activation rule."""
    if x.dtype != torch.bfloat16:
        raise ValueError("[quantize_activations] x must be bf16")
    x = x.contiguous()
    K = x.shape[-1]
    rows = x.numel() // K
    codes = torch.empty(*x.shape[:-1], K // 8, dtype=torch.int32, device=x.device)
    scales = torch.empty(*x.shape[:-1], K // 16, dtype=torch.uint8, device=x.device)
    _check(lib().b2_fp_quantize_activations(_ptr(x), _I64(rows), _I64(K), _ptr(codes), _ptr(scales), _stream(x)))
    return codes, scales


def nvfp4_gemm(x_codes, x_scales, w_codes, w_scales) -> torch.Tensor:
    """y [M, N] bf16 = Xq . Wq^T on the block-scaled tensor cores."""
    M, K = x_codes.shape[0], x_codes.shape[1] * 8
    N = w_codes.shape[0]
    y = torch.empty(M, N, dtype=torch.bfloat16, device=x_codes.device)
    _check(lib().b2_nvfp4_gemm(_ptr(x_codes.contiguous()), _ptr(x_scales.contiguous()), _ptr(w_codes.contiguous()),
                               _ptr(w_scales.contiguous()), _I64(M), _I64(N), _I64(K), _ptr(y), _stream(x_codes)))
    return y


def qqmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, group_size: Optional[int] = None,
         bits: Optional[int] = None, mode: str = "nvfp4", workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mx.qqmm(x, w, scales, mode="nvfp4"): x bf16 [..., M, K] quantized to
    NVFP4 on the fly, times the NVFP4 weight W [N, K/8] (transpose)."""
    _nvfp4_params("qqmm", group_size, bits, mode, None)
    N, K = w.shape[0], w.shape[1] * 8
    if x.shape[-1] != K:
        raise ValueError(f"[qqmm] Last dimension of x ({x.shape[-1]}) does not match K = {K} of w")
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    L = lib()
    L.b2_qqmm_workspace_size.restype = ctypes.c_size_t
    need = int(L.b2_qqmm_workspace_size(_I64(M), _I64(K)))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    _check(L.b2_qqmm(_ptr(x2), _ptr(w.contiguous()), _ptr(scales.contiguous()), _I64(M), _I64(N), _I64(K), _ptr(y),
                     _ptr(workspace), ctypes.c_size_t(workspace.numel()), _stream(x)))
    return y.reshape(*x.shape[:-1], N)


# ---------------------------------------------------------------------- routing
def router_logits(x: torch.Tensor, router_w: torch.Tensor) -> torch.Tensor:
    """float32 logits [T, E] = x [T, H] (bf16) . router_w^T (router_w f32 or bf16 [E, H])."""
    T, H = x.shape
    E = router_w.shape[0]
    out = torch.empty(T, E, dtype=torch.float32, device=x.device)
    _check(lib().b2_moe_router_logits(_ptr(x.contiguous()), _ptr(router_w.contiguous()), _I(_DT[router_w.dtype]),
                                      _I64(T), _I64(E), _I64(H), _ptr(out), _stream(x)))
    return out


def router_topk(logits: torch.Tensor, k: int, mode: int = ROUTER_SOFTMAX, bias: Optional[torch.Tensor] = None,
                renorm: bool = True):
    T, E = logits.shape
    inds = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    _check(lib().b2_moe_router_topk(_ptr(logits.contiguous()), _ptr(bias), _I(mode), _I64(T), _I64(E), _I(k),
                                    _I(int(renorm)), _ptr(inds), _ptr(w), _stream(logits)))
    return inds, w


def gather_sort(inds: torch.Tensor, n_experts: int, multi_cta: bool = False):
    """Stable expert-order permutation of flattened routed rows (SwitchLayers gatherSort).
    multi_cta: the several-CTA variant (identical positions, faster for large n)."""
    flat = inds.reshape(-1).to(torch.int32).contiguous()
    n = flat.numel()
    dev = inds.device
    order = torch.empty(n, dtype=torch.int32, device=dev)
    keys = torch.empty(n, dtype=torch.int32, device=dev)
    inv = torch.empty(n, dtype=torch.int32, device=dev)
    offs = torch.empty(n_experts + 1, dtype=torch.int32, device=dev)
    if multi_cta:
        nb = int(lib().b2_moe_gather_sort_scratch_size(_I64(n), _I64(n_experts)))
        scratch = torch.empty(max(nb, 4), dtype=torch.uint8, device=dev)
        _check(lib().b2_moe_gather_sort_ws(_ptr(flat), _I64(n), _I64(n_experts), _ptr(order), _ptr(keys), _ptr(inv),
                                           _ptr(offs), _ptr(scratch), ctypes.c_size_t(scratch.numel()),
                                           _stream(inds)))
    else:
        _check(lib().b2_moe_gather_sort(_ptr(flat), _I64(n), _I64(n_experts), _ptr(order), _ptr(keys), _ptr(inv),
                                        _ptr(offs), _stream(inds)))
    return order, keys, inv, offs


def gather_rows(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """dst[i] = src[idx[i]] for a [rows, K] tensor of 16-bit values."""
    n = idx.numel()
    K = src.shape[-1]
    dst = torch.empty(n, K, dtype=src.dtype, device=src.device)
    if n:
        _check(lib().b2_gather_rows16(_ptr(src.contiguous()), _ptr(idx.reshape(-1).to(torch.int32).contiguous()),
                                      _I64(n), _I64(K), _ptr(dst), _stream(src)))
    return dst


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    a = torch.empty_like(g)
    _check(lib().b2_moe_silu_mul(_ptr(g.contiguous()), _ptr(u.contiguous()), _I64(g.numel()), _ptr(a), _stream(g)))
    return a


def combine(d: torch.Tensor, weights: torch.Tensor, inverse: Optional[torch.Tensor] = None,
            routed_scale: float = 1.0, shared: Optional[torch.Tensor] = None,
            residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Weighted expert sum: d [T*k, H] (token-slot order, or expert-sorted with `inverse`)."""
    T, k = weights.shape
    H = d.shape[-1]
    out = torch.empty(T, H, dtype=torch.bfloat16, device=d.device)
    _check(lib().b2_moe_combine(_ptr(d.contiguous()), _ptr(inverse), _ptr(weights.contiguous()), _I64(T), _I(k),
                                _I64(H), ctypes.c_float(routed_scale), _ptr(shared), _ptr(residual), _ptr(out),
                                _stream(d)))
    return out


# ---------------------------------------------------------------------- block
@dataclass
class ExpertBank:
    """Routed SwitchGLU bank in MLX nvfp4 layout."""
    gate_codes: torch.Tensor   # [E, F, H/8] int32 (u32 bits)
    gate_scales: torch.Tensor  # [E, F, H/16] uint8
    up_codes: torch.Tensor
    up_scales: torch.Tensor
    down_codes: torch.Tensor   # [E, H, F/8]
    down_scales: torch.Tensor  # [E, H, F/16]


@dataclass
class SharedExpert:
    """Dense NVFP4 SwiGLU MLP run on every token (Laguna's shared expert,
    LagunaRuntimeMLP): gate/up [Fs, H/8] + [Fs, H/16], down [H, Fs/8] +
    [H, Fs/16]."""
    gate_codes: torch.Tensor
    gate_scales: torch.Tensor
    up_codes: torch.Tensor
    up_scales: torch.Tensor
    down_codes: torch.Tensor
    down_scales: torch.Tensor


class MoEBlock:
    """Routed MoE expert block (router -> top-k -> SwiGLU experts -> combine).

    Mirrors LagunaRuntimeSparseMoEBlock.callAsFunction(x, residual:,
    routerLogits:) for the routed part and, in softmax mode with scale 1, the
    stock SwitchGLU + weightedExpertSum composition."""

    def __init__(self, bank: ExpertBank, router_w: torch.Tensor, top_k: int, router_mode: int = ROUTER_SOFTMAX,
                 router_bias: Optional[torch.Tensor] = None, renorm: bool = True, routed_scale: float = 1.0,
                 prepare_decode: bool = False, prepare_prefill: bool = False,
                 shared: Optional[SharedExpert] = None):
        E, F, H8 = bank.gate_codes.shape
        self.bank = bank
        self.router_w = router_w.contiguous()
        self.router_bias = None if router_bias is None else router_bias.contiguous().float()
        b = _Block()
        b.hidden, b.ffn, b.n_experts = H8 * 8, F, E
        b.top_k, b.router_mode, b.renorm = top_k, router_mode, int(renorm)
        b.router_w_dtype = _DT[self.router_w.dtype]
        b.routed_scale = routed_scale
        b.router_w = self.router_w.data_ptr()
        b.router_bias = None if self.router_bias is None else self.router_bias.data_ptr()
        for nm in ("gate_codes", "gate_scales", "up_codes", "up_scales", "down_codes", "down_scales"):
            setattr(b, nm, getattr(bank, nm).data_ptr())
        self.shared = None
        if shared is not None:
            names = ("gate_codes", "gate_scales", "up_codes", "up_scales", "down_codes", "down_scales")
            self.shared = SharedExpert(**{nm: getattr(shared, nm).contiguous() for nm in names})
            b.shared_ffn = self.shared.gate_codes.shape[0]
            for nm in names:
                setattr(b, "shared_" + nm, getattr(self.shared, nm).data_ptr())
        self._blk = b
        self._ws = None
        # block workspaces, one per (device, stream): calls on one stream run
        # in order and can share one; calls on two streams may overlap on the
        # GPU and must not (the workspace head carries state between calls)
        self._ws_by_stream = {}
        # per (device, stream, tokens): the routing outputs of calls that do
        # not return them, reused call after call
        self._routing_by_stream = {}
        self._ws_need = {}
        self._fwd = None
        self.decode_bank = None
        self.prefill_bank = None
        if prepare_decode:
            self.prepare_decode_bank()
        if prepare_prefill:
            self.prepare_prefill_bank()

    def prepare_decode_bank(self) -> None:
        """Build the prepared decode bank (one contiguous tile per TMA copy)."""
        n = int(lib().b2_moe_decode_bank_size(ctypes.byref(self._blk)))
        dev = self.bank.gate_codes.device
        self.decode_bank = torch.empty(n, dtype=torch.uint8, device=dev)
        self._blk.decode_bank = None
        _check(lib().b2_moe_prepare_decode_bank(ctypes.byref(self._blk), _ptr(self.decode_bank),
                                                 ctypes.c_size_t(n), _stream(self.decode_bank)))
        self._blk.decode_bank = self.decode_bank.data_ptr()
        self._ws_need.clear()  # the workspace size may depend on the prepared banks

    def prepare_prefill_bank(self) -> None:
        """Build the prepared prefill bank: calls with more than 8 tokens then
        run the tensor-core grouped GEMMs."""
        n = int(lib().b2_moe_prefill_bank_size(ctypes.byref(self._blk)))
        dev = self.bank.gate_codes.device
        self.prefill_bank = torch.empty(n, dtype=torch.uint8, device=dev)
        self._blk.prefill_bank = None
        _check(lib().b2_moe_prepare_prefill_bank(ctypes.byref(self._blk), _ptr(self.prefill_bank),
                                                  ctypes.c_size_t(n), _stream(self.prefill_bank)))
        self._blk.prefill_bank = self.prefill_bank.data_ptr()
        self._ws_need.clear()  # the workspace size may depend on the prepared banks

    def switch_glu(self, x: torch.Tensor, inds: torch.Tensor) -> torch.Tensor:
        """SwitchGLU over given routing: x [T, H] bf16, inds [T, k] -> y [T, k, H]
        (SwitchLayers SwitchGLU.callAsFunction with sorted indices; needs the
        prepared prefill bank)."""
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        T = x2.shape[0]
        k = inds.shape[-1] if inds.dim() > 1 else 1
        y = torch.empty(T, k, x2.shape[-1], dtype=torch.bfloat16, device=x.device)
        if T == 0:
            return y
        need = int(lib().b2_moe_switch_glu_workspace_size(ctypes.byref(self._blk), _I64(T), _I(k)))
        # SwitchGLU carries no state between calls: one scratch per block
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
        ii = inds.reshape(T, k).to(torch.int32).contiguous()
        _check(lib().b2_moe_switch_glu(ctypes.byref(self._blk), _ptr(x2), _I64(T), _ptr(ii), _I(k), _ptr(y),
                                       _ptr(self._ws), ctypes.c_size_t(self._ws.numel()), _stream(x)))
        return y

    @property
    def hidden(self) -> int:
        return self._blk.hidden

    def workspace_bytes(self, tokens: int) -> int:
        return int(lib().b2_moe_block_workspace_size(ctypes.byref(self._blk), _I64(tokens)))

    def _workspace(self, tokens: int, device, stream: Optional[int] = None) -> torch.Tensor:
        if stream is None:
            stream = torch.cuda.current_stream(device).cuda_stream
        key = (str(device), stream)
        ws = self._ws_by_stream.get(key)
        need = self._ws_need.get(tokens)
        if need is None:
            need = self._ws_need[tokens] = self.workspace_bytes(tokens)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)
            self._ws_by_stream[key] = ws
        return ws

    def _forward_fn(self):
        # a typed handle of its own: ctypes then converts plain ints without
        # building argument objects on every call
        if self._fwd is None:
            f = lib()["b2_moe_block_forward"]
            f.argtypes = [_VP, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_size_t, _VP]
            f.restype = ctypes.c_int
            self._fwd = f
        return self._fwd

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 logits: Optional[torch.Tensor] = None, return_routing: bool = False,
                 out: Optional[torch.Tensor] = None):
        shape = x.shape
        x2 = x if (x.dim() == 2 and x.is_contiguous()) else x.reshape(-1, shape[-1]).contiguous()
        if not x2.is_cuda:
            raise ValueError("b2moe operates on CUDA tensors")
        T = x2.shape[0]
        dev = x2.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        if out is None:
            out = torch.empty_like(x2)
        elif not (out.is_cuda and out.is_contiguous() and out.dtype == torch.bfloat16 and out.numel() == x2.numel()):
            raise ValueError("[moe_block] out must be a contiguous bf16 tensor shaped like x")
        k = self._blk.top_k
        if return_routing:
            inds = torch.empty(T, k, dtype=torch.int32, device=dev)
            wts = torch.empty(T, k, dtype=torch.float32, device=dev)
        else:
            key = (str(dev), stream, T)
            rw = self._routing_by_stream.get(key)
            if rw is None:
                rw = (torch.empty(T, k, dtype=torch.int32, device=dev), torch.empty(T, k, dtype=torch.float32, device=dev))
                self._routing_by_stream[key] = rw
            inds, wts = rw
        ws = self._workspace(T, dev, stream)
        res = None if residual is None else residual.reshape(-1, shape[-1]).contiguous()
        lg = None if logits is None else _ptr(logits)
        rc = self._forward_fn()(ctypes.addressof(self._blk), x2.data_ptr(), T, lg,
                                None if res is None else _ptr(res), out.data_ptr(), inds.data_ptr(), wts.data_ptr(),
                                ws.data_ptr(), ws.numel(), stream)
        _check(rc)
        out = out.reshape(shape)
        return (out, inds, wts) if return_routing else out


# ---------------------------------------------------------------------- decode step
class _AttnLayer(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int64), ("n_heads", ctypes.c_int64), ("n_kv_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64), ("max_seq", ctypes.c_int64),
        ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("attn_norm_w", _VP), ("qkv_codes", _VP), ("qkv_scales", _VP), ("o_codes", _VP), ("o_scales", _VP),
        ("mlp_norm_w", _VP), ("k_cache", _VP), ("v_cache", _VP),
    ]


class _DecoderLayer(ctypes.Structure):
    _fields_ = [("attn", _AttnLayer), ("moe", _Block)]


@dataclass
class AttentionWeights:
    """One layer's attention half: RMSNorm weights (bf16 [H]) and the NVFP4
    projections -- fused q;k;v rows [(nq + 2 nkv) hd, H/8] (+ scales) and
    o [H, nq hd / 8] (+ scales)."""
    attn_norm_w: torch.Tensor
    qkv_codes: torch.Tensor
    qkv_scales: torch.Tensor
    o_codes: torch.Tensor
    o_scales: torch.Tensor
    mlp_norm_w: torch.Tensor


class DecoderStack:
    """B=1 decode step of a decoder stack: per layer attention (RMSNorm,
    NVFP4 q/k/v, RoPE, KV cache, GQA) + the MoE block, then a final RMSNorm
    (b2_decode_step).  Owns the bf16 KV caches [layers][nkv, max_seq, hd]."""

    def __init__(self, attn: Sequence[AttentionWeights], moe: Sequence[MoEBlock], final_norm_w: torch.Tensor,
                 n_heads: int, n_kv_heads: int, max_seq: int, head_dim: int = 128, rope_theta: float = 1e6,
                 rms_eps: float = 1e-6):
        if len(attn) != len(moe) or not attn:
            raise ValueError("[decode_step] one attention half and one MoE block per layer")
        dev = final_norm_w.device
        H = final_norm_w.shape[0]
        self.attn, self.moe, self.final_norm_w = list(attn), list(moe), final_norm_w.contiguous()
        self.H, self.max_seq = H, max_seq
        self.k_cache = [torch.zeros(n_kv_heads, max_seq, head_dim, dtype=torch.bfloat16, device=dev) for _ in attn]
        self.v_cache = [torch.zeros(n_kv_heads, max_seq, head_dim, dtype=torch.bfloat16, device=dev) for _ in attn]
        arr = (_DecoderLayer * len(attn))()
        for i, (a, m) in enumerate(zip(self.attn, self.moe)):
            L = arr[i]
            L.attn.hidden, L.attn.n_heads, L.attn.n_kv_heads = H, n_heads, n_kv_heads
            L.attn.head_dim, L.attn.max_seq = head_dim, max_seq
            L.attn.rope_theta, L.attn.rms_eps = rope_theta, rms_eps
            for nm in ("attn_norm_w", "qkv_codes", "qkv_scales", "o_codes", "o_scales", "mlp_norm_w"):
                t = getattr(a, nm)
                if not t.is_contiguous():
                    raise ValueError(f"[decode_step] {nm} must be contiguous")
                setattr(L.attn, nm, t.data_ptr())
            L.attn.k_cache, L.attn.v_cache = self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr()
            L.moe = m._blk
        self._layers = arr
        L_ = lib()
        L_.b2_decode_step_workspace_size.restype = ctypes.c_size_t
        L_.b2_decode_step_workspace_size.argtypes = [ctypes.POINTER(_DecoderLayer), _I]
        L_.b2_decode_step.restype = ctypes.c_int
        n = int(L_.b2_decode_step_workspace_size(arr, len(attn)))
        self._ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=dev)

    def step(self, x: torch.Tensor, pos: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x bf16 [H] (or [1, H]) at position pos -> final-normed hidden [1, H]."""
        x = x.reshape(1, self.H).contiguous()
        if out is None:
            out = torch.empty_like(x)
        _check(lib().b2_decode_step(self._layers, _I(len(self.attn)), _ptr(self.final_norm_w), _ptr(x), _I64(pos),
                                    _ptr(out), _ptr(self._ws), ctypes.c_size_t(self._ws.numel()), _stream(x)))
        return out
