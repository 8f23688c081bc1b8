"""GPU parity tests of the NVFP4 operators through the C ABI (libb2moe.so)
against the CPU checker (oracle/) and the golden fixtures made from the
reference's own kernels.  Bit-exact for codes, scales, dequantized values,
router indices and permutations; bf16 outputs within max-abs 2e-2 and mean
relative 1e-3 (the tolerance the path's contract states)."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import oracle as O
from _util import (assert_bf16_close, bf16_normal, det_source, from_torch_bf16, normal_weights, to_torch,
                   to_torch_bf16, to_torch_u32)

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _u32(t):
    return t.cpu().numpy().view(np.uint32)


# ---------------------------------------------------------------- codec
@pytest.mark.parametrize("shape,src", [((64, 2048), "normal"), ((33, 256), "det"), ((8, 4096), "edge")])
def test_quantize_bit_exact(cuda, shape, src):
    import b2moe

    rng = np.random.default_rng(5)
    if src == "normal":
        w = normal_weights(rng, shape)
    elif src == "det":
        w = det_source(shape, 59)
    else:
        w = normal_weights(rng, shape, std=1.0)
        w[0, :16] = 0.0  # all-zero group
        w[1, :16] = 1e-9  # tiny -> subnormal e4m3 scale
        w[2, :16] = 1e6  # saturating scale
        w[3, 5] = -0.0
        w[4, :16] = np.linspace(-3, 3, 16)
    c_ref, s_ref = O.fp_quantize(w)
    c, s = b2moe.quantize(to_torch(w, cuda))
    assert np.array_equal(_u32(c), c_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_dequantize_exact(cuda, dtype):
    import torch
    import b2moe

    rng = np.random.default_rng(6)
    c = rng.integers(0, 2**32, size=(40, 64), dtype=np.uint64).astype(np.uint32)
    s = rng.integers(0, 256, size=(40, 32), dtype=np.uint8)
    ref = O.fp_dequantize(c, s)
    td = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    out = b2moe.dequantize(to_torch_u32(c, cuda), to_torch(s, cuda), dtype=td).float().cpu().numpy()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_dequantize_nibble_order_kat(cuda):
    import torch
    import b2moe

    k = json.load(open(os.path.join(GOLD, "kat.json")))["nibble_order"]
    out = b2moe.dequantize(to_torch_u32(np.array(k["codes"], np.uint32), cuda),
                           to_torch(np.array(k["scales"], np.uint8), cuda), dtype=torch.float32)
    assert out.cpu().numpy().tolist() == k["expected"]


# ---------------------------------------------------------------- quantized_matmul
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (1, 64, 256), (3, 40, 768), (8, 128, 2048), (16, 24, 512),
                                   (17, 64, 256), (32, 4096, 4096), (2, 96, 48)])
def test_qmm_bf16_matches_oracle(cuda, M, N, K):
    import b2moe

    rng = np.random.default_rng(M * 1000 + N + K)
    c, s = O.fp_quantize(normal_weights(rng, (N, K)))
    xb = bf16_normal(rng, (M, K))
    y = b2moe.quantized_matmul(to_torch_bf16(xb, cuda), to_torch_u32(c, cuda), to_torch(s, cuda))
    assert_bf16_close(from_torch_bf16(y), O.qmm_bf16(xb, c, s), what=f"qmm M={M} N={N} K={K}")


def test_qmm_rows_independent_of_batch(cuda):
    """M = 32 with K = 4096 runs as two 16-row passes: every output row must be
    bit-identical to the same row computed in a call of its own."""
    import torch
    import b2moe

    rng = np.random.default_rng(5)
    c, s = O.fp_quantize(normal_weights(rng, (256, 4096)))
    x = to_torch_bf16(bf16_normal(rng, (32, 4096)), cuda)
    ct, st = to_torch_u32(c, cuda), to_torch(s, cuda)
    y = b2moe.quantized_matmul(x, ct, st)
    parts = torch.cat([b2moe.quantized_matmul(x[:16].contiguous(), ct, st),
                       b2moe.quantized_matmul(x[16:].contiguous(), ct, st)])
    assert torch.equal(y.view(torch.int16), parts.view(torch.int16))
    one = torch.cat([b2moe.quantized_matmul(x[m:m + 1].contiguous(), ct, st) for m in (0, 17, 31)])
    assert torch.equal(y[[0, 17, 31]].view(torch.int16), one.view(torch.int16))


@pytest.mark.parametrize("case", ["det", "normal_m1", "normal_m32"])
def test_qmm_against_reference_golden(cuda, case):
    import torch
    import b2moe

    g = np.load(os.path.join(GOLD, "ref_qmm.npz"))
    c, s, x = g[f"{case}/codes"], g[f"{case}/scales"], g[f"{case}/x"]
    ref = O.f32_to_bf16(g[f"{case}/y_f32"])
    y = b2moe.quantized_matmul(to_torch_bf16(O.f32_to_bf16(x), cuda), to_torch_u32(c, cuda), to_torch(s, cuda))
    assert_bf16_close(from_torch_bf16(y), ref, what=case)
    # float32 activations (CUDA-core path) against the reference's float kernel
    yf = b2moe.quantized_matmul(to_torch(x, cuda), to_torch_u32(c, cuda), to_torch(s, cuda))
    assert yf.dtype == torch.float32
    assert np.abs(yf.cpu().numpy() - g[f"{case}/y_f32"]).max() <= 1e-4 * max(1.0, np.abs(g[f"{case}/y_f32"]).max())


def test_qmm_large_activations_are_prescaled(cuda):
    import b2moe

    rng = np.random.default_rng(9)
    c, s = O.fp_quantize(normal_weights(rng, (64, 512)))
    x = rng.standard_normal((2, 512), dtype=np.float32)
    x[0] *= 3e5  # beyond the f16 range: the staged copy must be pre-scaled
    xb = O.f32_to_bf16(x)
    y = b2moe.quantized_matmul(to_torch_bf16(xb, cuda), to_torch_u32(c, cuda), to_torch(s, cuda))
    ref = O.qmm_bf16(xb, c, s)
    a, b = O.bf16_to_f32(from_torch_bf16(y)), O.bf16_to_f32(ref)
    assert np.all(np.isfinite(a))
    assert np.abs(a - b).max() <= 2e-3 * np.abs(b).max()


def test_qmm_all_ones_split_k_shape(cuda):
    import torch
    import b2moe

    c, s = b2moe.quantize(torch.ones(128, 64, device=cuda))
    y = b2moe.quantized_matmul(torch.ones(32, 64, device=cuda), c, s)
    ref = torch.ones(32, 64, device=cuda) @ b2moe.dequantize(c, s, dtype=torch.float32).T
    assert (y - ref).abs().max().item() <= 1e-4


# The streaming GEMV (K <= 4096, K % 256 == 0) with K warps partly idle (K <
# 4096), ragged N (last 8-row sub-tile partly filled), M on both sides of 8
# and 16 (one or two 16-row passes), and the generic kernel beyond K = 4096.
@pytest.mark.parametrize("M,N,K", [(1, 1000, 768), (3, 100, 1536), (16, 520, 2048), (17, 64, 2560),
                                   (32, 1000, 3072), (5, 300, 8192), (32, 136, 5120), (9, 77, 6144),
                                   (1, 5120, 2048), (8, 2049, 4096), (24, 12, 256)])
def test_qmm_streaming_shapes(cuda, M, N, K):
    import b2moe

    rng = np.random.default_rng(M * 7 + N * 3 + K)
    c, s = O.fp_quantize(normal_weights(rng, (N, K)))
    xb = bf16_normal(rng, (M, K))
    y = b2moe.quantized_matmul(to_torch_bf16(xb, cuda), to_torch_u32(c, cuda), to_torch(s, cuda))
    assert_bf16_close(from_torch_bf16(y), O.qmm_bf16(xb, c, s), what=f"qmm M={M} N={N} K={K}")


@pytest.mark.parametrize("K", [768, 2048, 4096, 8192])
def test_qmm_row_results_independent_of_m(cuda, K):
    """Each 16-row pass of x computes its rows with the same K split, so a row
    of x gives the same bits whatever the other rows and M are."""
    import torch
    import b2moe

    rng = np.random.default_rng(K)
    c, s = O.fp_quantize(normal_weights(rng, (203, K)))
    x = to_torch_bf16(bf16_normal(rng, (32, K)), cuda)
    ct, st = to_torch_u32(c, cuda), to_torch(s, cuda)
    y = b2moe.quantized_matmul(x, ct, st)
    y16 = b2moe.quantized_matmul(x[8:24].contiguous(), ct, st)
    assert torch.equal(y[8:24].view(torch.int16), y16.view(torch.int16))
    for m in (0, 15, 16, 31):
        y1 = b2moe.quantized_matmul(x[m:m + 1].contiguous(), ct, st)
        assert torch.equal(y[m:m + 1].view(torch.int16), y1.view(torch.int16))


# ---------------------------------------------------------------- gather_qmm
@pytest.mark.parametrize("N,K", [(512, 2048), (2048, 512)])
@pytest.mark.parametrize("tokens", [1, 8])
def test_routed_gather_all_256_experts(cuda, N, K, tokens):
    """LagunaNVFP4KernelTests.swift:152-330: 256 experts with distinct constant
    codes, selected ids include 255, against the dequantized gather."""
    import torch
    import b2moe

    E = 256
    codes = torch.tensor([((e % 7) + 1) * 0x11111111 for e in range(E)], dtype=torch.int64, device=cuda)
    codes = codes.to(torch.int32).view(E, 1, 1).expand(E, N, K // 8).contiguous()
    scales = torch.full((E, N, K // 16), 0x38, dtype=torch.uint8, device=cuda)
    sel = [0, 7, 42, 255, 3, 128, 17, 99]
    x = torch.full((1, tokens, 1, 1, K), 0.25, dtype=torch.bfloat16, device=cuda)
    rhs = torch.tensor(sel * tokens, dtype=torch.int32, device=cuda).view(1, tokens, 8)
    lhs = torch.arange(tokens, dtype=torch.int32, device=cuda).view(1, tokens, 1).expand(1, tokens, 8)
    y = b2moe.gather_qmm(x.view(tokens, 1, K), codes, scales, lhs_indices=lhs, rhs_indices=rhs)
    assert tuple(y.shape) == (1, tokens, 8, 1, N)
    deq = b2moe.dequantize(codes[sel], scales[sel], dtype=torch.float32)  # [8, N, K]
    ref = torch.einsum("k,enk->en", torch.full((K,), 0.25, device=cuda), deq)
    err = (y.float().view(tokens, 8, N) - ref.unsqueeze(0)).abs().max().item()
    assert err <= 1e-4


@pytest.mark.parametrize("E,N,K,rows,idx,sorted_", [
    (4, 512, 2048, 1, [3, 0, 2, 1, 3, 1, 0, 2], False),
    (4, 512, 2048, 32, [0, 3, 1, 2], False),
    (4, 2048, 512, 1, [0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3], True),
])
def test_gather_matches_non_gather(cuda, E, N, K, rows, idx, sorted_):
    """NVFP4QuantizedMMTests.swift:309-459 shapes (deterministic source)."""
    import b2moe

    c, s = O.fp_quantize(det_source((E, N, K), 59))
    x = O.f32_to_bf16(det_source((len(idx), rows, K), 72))
    y = b2moe.gather_qmm(to_torch_bf16(x, cuda), to_torch_u32(c, cuda), to_torch(s, cuda),
                         rhs_indices=to_torch(np.array(idx, np.int32), cuda), sorted_indices=sorted_)
    ref = O.gather_qmm_bf16(x, c, s, np.arange(len(idx), dtype=np.uint32), np.array(idx, np.uint32))
    assert_bf16_close(from_torch_bf16(y).reshape(ref.shape), ref, what="gather")


def test_gather_bad_index_reports_status(cuda):
    import torch
    import b2moe

    b2moe.device_status()  # clear
    c = torch.zeros(2, 16, 32, dtype=torch.int32, device=cuda)
    s = torch.full((2, 16, 16), 0x38, dtype=torch.uint8, device=cuda)
    x = torch.ones(1, 1, 256, dtype=torch.bfloat16, device=cuda)
    y = b2moe.gather_qmm(x, c, s, lhs_indices=torch.zeros(1, dtype=torch.int32, device=cuda),
                         rhs_indices=torch.tensor([5], dtype=torch.int32, device=cuda))
    torch.cuda.synchronize()
    assert b2moe.device_status() == b2moe.STATUS_BAD_INDEX
    assert torch.all(y == 0)
    assert b2moe.device_status() == b2moe.STATUS_OK


# ---------------------------------------------------------------- router
@pytest.mark.parametrize("T,E,H,wdt", [(1, 128, 2048, "f32"), (37, 128, 2048, "f32"), (5, 256, 2048, "bf16"),
                                       (300, 128, 2048, "f32"), (97, 40, 640, "bf16"), (2048, 128, 2048, "f32")])
def test_router_logits_bit_exact(cuda, T, E, H, wdt):
    import torch
    import b2moe

    rng = np.random.default_rng(T + E)
    x = bf16_normal(rng, (T, H))
    w = rng.standard_normal((E, H), dtype=np.float32)
    if wdt == "bf16":
        wb = O.f32_to_bf16(w)
        ref = O.router_logits(x, O.bf16_to_f32(wb), bf16_weight=True)
        wt = to_torch_bf16(wb, cuda)
    else:
        ref = O.router_logits(x, w)
        wt = to_torch(w, cuda)
    got = b2moe.router_logits(to_torch_bf16(x, cuda), wt).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("E", [128, 40, 256, 1000])
@pytest.mark.parametrize("mode", ["softmax", "sigmoid"])
def test_router_topk_bit_exact(cuda, mode, E):
    import b2moe

    rng = np.random.default_rng(17 + E)
    T, k = 300, 8
    l = rng.standard_normal((T, E), dtype=np.float32)
    l[0, :] = 0.5  # all ties
    l[1, 3] = np.nan
    l[2, :10] = -0.0
    l[2, 10:20] = 0.0
    l[3] = np.round(l[3], 1)  # many exact ties
    l[4, :] = np.nan  # NaN ranks last: the first k indices
    l[5, 5:] = -np.inf
    if mode == "softmax":
        ri, rw = O.topk_softmax(l, k)
        gi, gw = b2moe.router_topk(to_torch(l, cuda), k, b2moe.ROUTER_SOFTMAX)
    else:
        bias = (rng.standard_normal(E, dtype=np.float32) * 0.1).astype(np.float32)
        ri, rw = O.topk_sigmoid_bias(l, bias, k, renorm=True)
        gi, gw = b2moe.router_topk(to_torch(l, cuda), k, b2moe.ROUTER_SIGMOID_BIAS, bias=to_torch(bias, cuda))
    assert np.array_equal(gi.cpu().numpy().view(np.uint32), ri)
    assert np.allclose(gw.cpu().numpy(), rw, rtol=2e-6, atol=1e-7, equal_nan=True)


@pytest.mark.parametrize("multi", [False, True])
@pytest.mark.parametrize("n,E", [(8, 128), (16384, 128), (5000, 1000), (65536, 256), (3000, 1)])
def test_gather_sort_bit_exact(cuda, n, E, multi):
    import b2moe

    rng = np.random.default_rng(n)
    inds = rng.integers(0, E, size=n, dtype=np.uint32)
    if n == 65536:  # skewed: a few hot experts, many empty ones
        inds = (rng.zipf(1.3, size=n) % E).astype(np.uint32)
    ro, rk, rinv, roff = O.gather_sort(inds, E)
    go, gk, ginv, goff = b2moe.gather_sort(to_torch_u32(inds, cuda), E, multi_cta=multi)
    for a, b in ((go, ro), (gk, rk), (ginv, rinv), (goff, roff)):
        assert np.array_equal(_u32(a), b)


def test_silu_mul_bit_exact(cuda):
    import b2moe

    rng = np.random.default_rng(2)
    g = O.f32_to_bf16(rng.standard_normal(4096, dtype=np.float32) * 4)
    u = bf16_normal(rng, (4096,))
    a = b2moe.silu_mul(to_torch_bf16(g, cuda), to_torch_bf16(u, cuda))
    assert np.array_equal(from_torch_bf16(a), O.swiglu_bf16(g, u))


def test_combine_wide_exponents_bit_exact(cuda):
    """Slot outputs, weights and residuals spread over 2^-40 .. 2^40 (sums
    whose operands differ by far more than 16 exponents, signed zeros,
    cancellations) through the bf16 fold, with 8 and with 10 slots."""
    import b2moe

    rng = np.random.default_rng(11)
    for T, k, H in ((17, 8, 128), (9, 10, 64)):
        mag = np.ldexp(rng.random((T, k, H)).astype(np.float32) + 0.5, rng.integers(-40, 41, (T, k, H)))
        d = O.f32_to_bf16(np.where(rng.random((T, k, H)) < 0.5, -mag, mag).astype(np.float32))
        d[0, :, :4] = 0x8000  # -0 rows
        d[1, 1] = d[1, 0] ^ 0x8000  # exact cancellation against slot 0 when weights match
        w = np.ldexp(rng.random((T, k)).astype(np.float32) + 0.5, rng.integers(-20, 21, (T, k))).astype(np.float32)
        w[1, 1] = w[1, 0]
        res = O.f32_to_bf16(np.ldexp(rng.standard_normal((T, H)).astype(np.float32), rng.integers(-30, 31, (T, H))))
        ref = O.combine_bf16(d, w, routed_scale=2.5, residual=res)
        out = b2moe.combine(to_torch_bf16(d.reshape(T * k, H), cuda), to_torch(w, cuda), routed_scale=2.5,
                            residual=to_torch_bf16(res, cuda))
        assert np.array_equal(from_torch_bf16(out), ref), f"T={T} k={k}"


@pytest.mark.parametrize("sorted_rows", [False, True])
def test_combine_bit_exact(cuda, sorted_rows):
    import b2moe

    rng = np.random.default_rng(4)
    T, k, H = 33, 8, 256
    d = bf16_normal(rng, (T, k, H))
    w = rng.random((T, k), dtype=np.float32)
    res = bf16_normal(rng, (T, H))
    ref = O.combine_bf16(d, w, routed_scale=2.5, residual=res)
    dd = d.reshape(T * k, H)
    inv = None
    if sorted_rows:
        perm = rng.permutation(T * k).astype(np.uint32)  # row i of d lives at position inv[i]
        dd = np.empty_like(dd)
        dd[perm] = d.reshape(T * k, H)
        inv = to_torch_u32(perm, cuda)
    out = b2moe.combine(to_torch_bf16(dd, cuda), to_torch(w, cuda), inverse=inv, routed_scale=2.5,
                        residual=to_torch_bf16(res, cuda))
    assert np.array_equal(from_torch_bf16(out), ref)
