"""W4A4 path (the reference's qqmm in nvfp4 mode): the activation quantizer
bit-exact against the checker (itself pinned to the reference's own
fp_quantize_dequantize steps, tests/test_oracle.py), and the block-scaled
tcgen05 GEMM against the checker's f32 product of the same NVFP4 operands.
The E2M1 x E2M1 x scale x scale products are exact in f32, so only the
summation order differs: the W4A4 tolerance is the contract's bf16
tolerance, max-abs 2e-2 and mean relative 1e-3 on outputs of unit scale
(the qqmm outputs here are scaled to unit magnitude by the weight scale)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from _util import assert_bf16_close, bf16_normal, from_torch_bf16, to_torch, to_torch_bf16

pytestmark = pytest.mark.gpu


def _act(rng, shape):
    x = (rng.standard_normal(shape, dtype=np.float32) * np.exp(rng.uniform(-6, 6, (shape[0], 1)))).astype(np.float32)
    xb = O.f32_to_bf16(x)
    xb[0, :16] = 0  # an all-zero group (scale 0)
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5, 6, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5, -6], np.float32)
    xb[min(1, shape[0] - 1), 16:32] = O.f32_to_bf16(ties)  # threshold ties at scale 1
    return xb


@pytest.mark.parametrize("rows,K", [(1, 256), (37, 512), (300, 2048)])
def test_quantize_activations_bit_exact(cuda, rows, K):
    import b2moe

    x = _act(np.random.default_rng(rows + K), (rows, K))
    c, s = b2moe.quantize_activations(to_torch_bf16(x, cuda))
    rc, rs, _ = O.quantize_activations(x)
    assert np.array_equal(c.cpu().numpy().view(np.uint32), rc)
    assert np.array_equal(s.cpu().numpy(), rs)


def _bf16_step(bits, d):
    """The bf16 value d steps of the last place away from `bits` (same sign)."""
    return np.uint16(int(bits) + d)


def test_quantize_activations_threshold_neighbours(cuda):
    """Groups whose scale takes every E4M3 mantissa (normal and subnormal)
    over a range of exponents, holding t * scale and the bf16 values one step
    either side of it for every threshold t: the quantizer's division-free
    threshold test must code them exactly as the rule's rn(x / scale)."""
    import b2moe

    ts = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    scales = [m / 8 * 2.0 ** e for e in range(-8, 9, 2) for m in range(8, 16)]
    scales += [m / 8 * 2.0 ** -6 for m in range(1, 8)]  # subnormal E4M3
    groups = []
    for sd in scales:
        for sign in (1.0, -1.0):
            # element 0 sets the group maximum to 6 * scale, so the group's
            # scale is `sd`; the other 15 are the threshold neighbourhoods
            vals = []
            for t in ts:
                c = O.f32_to_bf16(np.array([sign * t * sd], np.float32))[0]
                vals += [_bf16_step(c, -1), c, _bf16_step(c, 1)]
            head = O.f32_to_bf16(np.array([6.0 * sd], np.float32))[0]
            for i in range(0, len(vals), 15):
                part = vals[i:i + 15]
                part += [np.uint16(0)] * (15 - len(part))
                groups.append([head] + part)
    g = np.array(groups, np.uint16)
    pad = (-len(g)) % 16
    g = np.concatenate([g, np.zeros((pad, 16), np.uint16)])
    x = g.reshape(-1, 256)
    c, s = b2moe.quantize_activations(to_torch_bf16(x, cuda))
    rc, rs, _ = O.quantize_activations(x)
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(c.cpu().numpy().view(np.uint32), rc)


@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (37, 384, 512), (128, 256, 2048), (300, 640, 1024),
                                   (1024, 4096, 4096)])
def test_nvfp4_gemm_matches_oracle(cuda, M, N, K):
    import b2moe

    rng = np.random.default_rng(M * 7 + N)
    x = bf16_normal(rng, (M, K))
    w, ws = O.fp_quantize((rng.standard_normal((N, K), dtype=np.float32) * np.float32(1.0 / np.sqrt(K))).astype(
        np.float32))
    xc, xs, _ = O.quantize_activations(x)
    y = b2moe.nvfp4_gemm(to_torch(xc.view(np.int32), cuda), to_torch(xs, cuda), to_torch(w.view(np.int32), cuda),
                         to_torch(ws, cuda))
    # the checker: f32 product of the dequantized operands, rounded to bf16
    xf = O.fp_dequantize(xc, xs)
    if M * N * K > 1 << 30:  # large case: a sample of rows keeps the check fast on the CPU
        rows = np.unique(np.r_[0, M - 1, rng.choice(M, 31, replace=False)])
        ref = O.f32_to_bf16(xf[rows] @ O.fp_dequantize(w, ws).T)
        assert_bf16_close(from_torch_bf16(y)[rows], ref, what=f"nvfp4 gemm {M}x{N}x{K} (sampled rows)")
    else:
        ref = O.f32_to_bf16(xf @ O.fp_dequantize(w, ws).T)
        assert_bf16_close(from_torch_bf16(y), ref, what=f"nvfp4 gemm {M}x{N}x{K}")


def test_qqmm_is_quantize_then_gemm(cuda):
    import torch
    import b2moe

    rng = np.random.default_rng(5)
    M, N, K = 64, 256, 1024
    x = bf16_normal(rng, (M, K))
    w, ws = O.fp_quantize((rng.standard_normal((N, K), dtype=np.float32) * 0.03).astype(np.float32))
    wt, wst = to_torch(w.view(np.int32), cuda), to_torch(ws, cuda)
    y = b2moe.qqmm(to_torch_bf16(x, cuda), wt, wst)
    xc, xs = b2moe.quantize_activations(to_torch_bf16(x, cuda))
    assert torch.equal(y, b2moe.nvfp4_gemm(xc, xs, wt, wst))
    assert_bf16_close(from_torch_bf16(y), O.qqmm_bf16(x, w, ws), what="qqmm vs checker")
    with pytest.raises(ValueError):
        b2moe.qqmm(to_torch_bf16(x[:, :1000], cuda), wt, wst)
