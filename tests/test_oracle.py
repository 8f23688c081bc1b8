"""CPU tests of the checker: the restatement in oracle/nvfp4_oracle.c against
the reference's known-answer tests and against the reference's own MLX CPU
kernels (golden fixtures, and the in-place build when the tree is present)."""
from __future__ import annotations

import json
import math
import os

import numpy as np
import pytest

import oracle as O
from _util import det_source

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def kat():
    with open(os.path.join(GOLD, "kat.json")) as f:
        return json.load(f)


def f32_bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


# ------------------------------------------------------------------ codec KATs
def test_nibble_order_and_e4m3_scale_bytes():
    k = kat()["nibble_order"]
    out = O.fp_dequantize(np.array(k["codes"], np.uint32), np.array(k["scales"], np.uint8))
    assert f32_bits_equal(out, np.array(k["expected"], np.float32))


def test_packed_nibbles_decode_low_nibble_first():
    k = kat()["low_nibble_first"]
    nib = k["nibbles"]
    words = [sum((nib[8 * w + j] & 15) << (4 * j) for j in range(8)) for w in range(2)]
    out = O.fp_dequantize(np.array([words], np.uint32), np.array(k["scales"], np.uint8))
    assert np.array_equal(out, np.array(k["expected"], np.float32))


def test_e4m3_scales_decode_per_group():
    k = kat()["group_scales"]
    out = O.fp_dequantize(np.array(k["codes"], np.uint32), np.array(k["scales"], np.uint8))
    assert np.array_equal(out, np.array(k["expected"], np.float32))


def test_e4m3_decode_all_bytes_matches_reference():
    g = np.load(os.path.join(GOLD, "ref_fp8.npz"))
    ours = np.array([O.e4m3_value(b) for b in range(256)], np.float32)
    assert f32_bits_equal(ours, g["decode"])
    assert O.e4m3_value(0x7F) == 480.0 and O.e4m3_value(0xFF) == -480.0  # never NaN


def test_e4m3_encode_matches_reference_sweep():
    g = np.load(os.path.join(GOLD, "ref_fp8.npz"))
    ours = np.array([O.e4m3_encode(float(v)) for v in g["encode_in"]], np.uint8)
    assert np.array_equal(ours, g["encode_out"])


@pytest.mark.skipif(not O.ref_available(), reason="reference shim not built here")
def test_e4m3_encode_matches_reference_dense():
    # every 997th float bit pattern in the finite range below 2^10 plus negatives
    bits = np.arange(0, 0x44800000, 997, dtype=np.uint32)
    vals = np.concatenate([bits, bits | 0x80000000]).view(np.float32)
    vals = vals[::7]
    mism = sum(1 for v in vals if O.e4m3_encode(float(v)) != O.ref_to_fp8(float(v)))
    assert mism == 0


def test_quantize_round_trip_on_lut_values():
    # MLX test_quantized.py:113-162: LUT values (+3e-6) with one 6 per group
    # survive a quantize/dequantize round trip within 1e-5.
    rng = np.random.default_rng(0)
    lut = np.array([O.e2m1_value(j) for j in range(16)], np.float32)
    w = lut[rng.integers(0, 16, size=(128, 512))].reshape(-1, 16)
    w[:, 0] = 6
    w = (w + np.float32(3e-6)).astype(np.float32).reshape(128, 512)
    c, s = O.fp_quantize(w)
    back = O.fp_dequantize(c, s)
    assert np.allclose(back, w, rtol=1e-5, atol=1e-5)


def test_quantize_zeros():
    c, s = O.fp_quantize(np.zeros((256, 512), np.float32))
    assert np.all(O.fp_dequantize(c, s) == 0)


def test_quantize_ties_follow_argmin_first_index():
    # q = 0.25 is equidistant from +0 and 0.5 -> +0 (index 0); q = 5 between 4
    # and 6 -> 4 (first index); -0.25 -> +0.  Group max 6 gives scale 1.0.
    w = np.zeros((1, 16), np.float32)
    w[0, :4] = [6.0, 0.25, 5.0, -0.25]
    c, s = O.fp_quantize(w)
    assert s[0, 0] == 0x38
    nib = [(int(c[0, 0]) >> (4 * j)) & 15 for j in range(4)]
    assert nib == [7, 0, 6, 0]


# ------------------------------------------------------------------ qmm vs reference kernels
@pytest.mark.parametrize("case", ["det", "normal_m1", "normal_m32"])
def test_qmm_f32_bit_exact_with_reference(case):
    g = np.load(os.path.join(GOLD, "ref_qmm.npz"))
    c, s, x = g[f"{case}/codes"], g[f"{case}/scales"], g[f"{case}/x"]
    assert f32_bits_equal(O.qmm_f32(x, c, s), g[f"{case}/y_f32"])


def test_reference_bf16_path_error_is_reported_not_a_target():
    # The stock MLX CPU path with bf16 x accumulates in bf16; it is the timed
    # CPU baseline but cannot meet the float tolerance, so its error is
    # reported here rather than used as a parity target.
    g = np.load(os.path.join(GOLD, "ref_qmm.npz"))
    ref = g["normal_m1/y_f32"]
    bfp = O.bf16_to_f32(g["normal_m1/y_bf16path"])
    err = np.abs(bfp - ref).max()
    assert 0 < err < 0.5


@pytest.mark.skipif(not O.ref_available(), reason="reference shim not built here")
def test_qmm_f32_bit_exact_with_reference_random_shapes():
    rng = np.random.default_rng(7)
    for (M, N, K) in [(1, 48, 64), (5, 33, 256), (2, 17, 768)]:
        w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
        c, s = O.fp_quantize(w)
        x = rng.standard_normal((M, K), dtype=np.float32)
        assert f32_bits_equal(O.qmm_f32(x, c, s), O.ref_qmm_f32(x, c, s))


def test_split_k_all_ones_shape():
    # LagunaNVFP4KernelTests.swift:8-56: all-ones M=32 N=128 K=64 equals the
    # dequantized matmul within 1e-4.
    c, s = O.fp_quantize(np.ones((128, 64), np.float32))
    y = O.qmm_f32(np.ones((32, 64), np.float32), c, s)
    ref = np.ones((32, 64), np.float32) @ O.fp_dequantize(c, s).T
    assert np.abs(y - ref).max() <= 1e-4


def test_routed_gather_256_experts_kat():
    k = kat()["routed_gather"]
    N, K = 64, 256  # reduced rows; addressing is what the case pins
    E = k["n_experts"]
    codes = np.zeros((E, N, K // 8), np.uint32)
    for e in range(E):
        codes[e] = np.uint32(((e % 7) + 1) * 0x11111111)
    scales = np.full((E, N, K // 16), k["scale"], np.uint8)
    sel = np.array(k["selected"], np.uint32)
    x = O.f32_to_bf16(np.full((1, 1, K), k["x_value"], np.float32))
    y = O.gather_qmm_bf16(x, codes, scales, np.zeros(8, np.uint32), sel)
    for i, e in enumerate(sel):
        v = O.e2m1_value((e % 7) + 1)
        assert np.all(O.bf16_to_f32(y[i]) == np.float32(k["x_value"] * v * K))


# ------------------------------------------------------------------ router
def test_topk_total_order_ties_nan_signed_zero():
    l = np.array([[1.0, 3.0, 3.0, np.nan, -0.0, 0.0, 2.0, 3.0]], np.float32)
    inds, w = O.topk_softmax(l, 6)
    assert inds[0].tolist() == [1, 2, 7, 6, 0, 4]
    assert abs(w.sum() - 1) < 1e-6
    inds, _ = O.topk_softmax(l, 8)
    assert inds[0, -1] == 3  # NaN ranks last
    assert inds[0].tolist()[4:7] == [0, 4, 5]  # -0 == +0, by index


def test_topk_sigmoid_bias_choice_differs_from_weight():
    l = np.array([[0.0, 0.1, -0.2, 0.3]], np.float32)
    bias = np.array([0.0, 0.0, 1.0, 0.0], np.float32)
    inds, w = O.topk_sigmoid_bias(l, bias, 2, renorm=True)
    assert inds[0].tolist() == [2, 3]
    s2 = 1 / (1 + math.exp(0.2))
    s3 = 1 - 1 / (1 + math.exp(0.3))
    assert abs(w[0, 0] - s2 / (s2 + s3)) < 1e-6


def test_oracle_expf_accuracy():
    xs = np.linspace(-80, 80, 20001, dtype=np.float32)
    lib = O._load()
    lib.oracle_expf.restype = __import__("ctypes").c_float
    lib.oracle_expf.argtypes = [__import__("ctypes").c_float]
    ours = np.array([lib.oracle_expf(float(x)) for x in xs], np.float64)
    ref = np.exp(xs.astype(np.float64))
    ulp = np.abs(ours - ref) / np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    assert ulp.max() <= 2.0


def test_router_logits_fixed_order_matches_float64_closely():
    rng = np.random.default_rng(3)
    x = O.f32_to_bf16(rng.standard_normal((3, 256), dtype=np.float32))
    w = rng.standard_normal((16, 256), dtype=np.float32)
    l = O.router_logits(x, w)
    ref = O.bf16_to_f32(x).astype(np.float64) @ w.T.astype(np.float64)
    assert np.abs(l - ref).max() < 1e-4


# ------------------------------------------------------------------ permute / combine
def test_gather_sort_is_stable():
    inds = np.array([3, 1, 3, 0, 1, 3, 2, 0], np.uint32)
    order, keys, inv, offs = O.gather_sort(inds, 4)
    assert keys.tolist() == sorted(inds.tolist())
    assert order.tolist() == [3, 7, 1, 4, 6, 0, 2, 5]
    assert offs.tolist() == [0, 2, 4, 5, 8]
    assert np.array_equal(order[inv], np.arange(8))


def test_combine_bf16_fold_order():
    d = O.f32_to_bf16(np.array([[[1.0, 2.0], [3.0, 4.0]]], np.float32))
    w = np.array([[0.5, 0.25]], np.float32)
    out = O.bf16_to_f32(O.combine_bf16(d, w))
    assert out.tolist() == [[1.25, 2.0]]
    out = O.bf16_to_f32(O.combine_bf16(d, w, routed_scale=2.5))
    assert out.tolist() == [[3.125, 5.0]]


def test_swiglu_matches_float_formula_within_bf16():
    g = O.f32_to_bf16(np.linspace(-6, 6, 101, dtype=np.float32))
    u = O.f32_to_bf16(np.full(101, 1.5, np.float32))
    a = O.bf16_to_f32(O.swiglu_bf16(g, u))
    gf = O.bf16_to_f32(g).astype(np.float64)
    ref = gf / (1 + np.exp(-gf)) * 1.5
    assert np.abs(a - ref).max() < 0.06


def test_moe_experts_matches_composed_ops():
    rng = np.random.default_rng(11)
    E, H, F, k, T = 6, 256, 256, 2, 3
    bank = {}
    for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
        c, s = O.fp_quantize((rng.standard_normal(shp, dtype=np.float32) * 0.02).astype(np.float32))
        bank[nm + "_w"], bank[nm + "_s"] = c, s
    x = O.f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32))
    inds = np.array([[0, 5], [2, 2], [4, 1]], np.uint32)
    wts = np.array([[0.7, 0.3], [0.5, 0.5], [0.9, 0.1]], np.float32)
    out = O.moe_experts(x, inds, wts, bank)
    # compose by hand
    d = np.zeros((T, k, H), np.uint16)
    for t in range(T):
        for s_ in range(k):
            e = inds[t, s_]
            g = O.qmm_bf16(x[t:t + 1], bank["gate_w"][e], bank["gate_s"][e])
            u = O.qmm_bf16(x[t:t + 1], bank["up_w"][e], bank["up_s"][e])
            a = O.swiglu_bf16(g, u)
            d[t, s_] = O.qmm_bf16(a, bank["down_w"][e], bank["down_s"][e])[0]
    assert np.array_equal(out, O.combine_bf16(d, wts))


@pytest.mark.skipif(not O.ref_available(), reason="reference shim not built")
def test_activation_quantizer_pinned_to_reference():
    """The checker's qqmm activation quantizer equals the reference's own
    fp_quantize_dequantize steps (to_fp4_e2m1 threshold rounding, ToFP8,
    dequantize_scale) on wide-range data, ties and zero groups."""
    rng = np.random.default_rng(11)
    x = O.f32_to_bf16((rng.standard_normal((64, 512)) * np.exp(rng.uniform(-10, 10, (64, 1)))).astype(np.float32))
    x[0, :16] = 0
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5, 6, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5, -6], np.float32)
    x[1, :16] = O.f32_to_bf16(ties)
    c, s, xh = O.quantize_activations(x)
    rh, rc, rs = O.ref_qdq_nvfp4_bf16(x)
    assert np.array_equal(s, rs) and np.array_equal(xh, rh)
    assert np.array_equal(((c[:, :, None] >> (4 * np.arange(8))) & 15).reshape(x.shape).astype(np.uint8), rc)


@pytest.mark.skipif(not O.ref_available(), reason="reference shim not built")
def test_router_selection_against_reference_primitives(capsys):
    """Router parity against the reference's own CPU primitives on seeded
    inputs of the two router modes, 4096 tokens each:
      * Laguna mode (bf16 logits, E = 256, sigmoid + bias, top-8): the
        selection keys built with the reference's sigmoid (MLX unary_ops.h,
        MLX's exp) against the library's (its own exp): the sigmoid values
        differ by at most a few ulp, and every token whose top-8 set differs
        is a near-tie (keys within 4 ulp at the selection boundary);
      * softmax mode (f32 logits, E = 128, top-8): the reference selects on
        its softmax probabilities (softmax.cpp), the library on the logits
        (the same order, exactly, wherever the probabilities do not tie);
        the renormalised weights agree to 2e-6 relative.
    The disagreement rates are printed (tie rate of the seeded configs)."""
    rng = np.random.default_rng(21)
    T, k = 4096, 8
    # Laguna mode
    E = 256
    logits = O.bf16_to_f32(O.f32_to_bf16((rng.standard_normal((T, E)) * 2).astype(np.float32)))
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    ours_i, ours_s = O.topk_sigmoid_bias(logits, bias, k, renorm=False)
    ref_s = O.ref_sigmoid(logits)
    ref_keys = (ref_s + bias).astype(np.float32)
    ref_i = O.select_by_keys(ref_keys, k)
    sel = np.take_along_axis(ref_s, ours_i.astype(np.int64), axis=1)
    ulps = np.abs(sel.view(np.int32).astype(np.int64) - ours_s.view(np.int32).astype(np.int64))
    diff_rows = [t for t in range(T) if set(ours_i[t]) != set(ref_i[t])]
    for t in diff_rows:
        srt = np.sort(ref_keys[t])[::-1]
        gap = (srt[k - 1] - srt[k]) / max(abs(srt[k - 1]), 1e-30)
        assert gap <= 4 * np.finfo(np.float32).eps, f"token {t}: selection differs away from a tie"
    laguna_rate = len(diff_rows) / T
    # softmax mode
    E = 128
    logits = rng.standard_normal((T, E)).astype(np.float32) * 2
    ours_i2, ours_w2 = O.topk_softmax(logits, k)
    p = O.ref_softmax_rows(logits)
    ref_i2 = O.select_by_keys(p, k)
    diff2 = [t for t in range(T) if set(ours_i2[t]) != set(ref_i2[t])]
    for t in diff2:
        srt = np.sort(p[t])[::-1]
        assert srt[k - 1] == srt[k], f"token {t}: softmax selection differs away from a probability tie"
    same = [t for t in range(T) if t not in set(diff2)]
    pw = np.take_along_axis(p, ours_i2.astype(np.int64), axis=1)[same]
    ref_w = pw / pw.sum(axis=1, keepdims=True)
    np.testing.assert_allclose(ours_w2[same], ref_w, rtol=2e-6, atol=0)
    with capsys.disabled():
        print(f"\n[router parity] laguna: sigmoid max diff {int(ulps.max())} ulp, top-8 set disagreements "
              f"{len(diff_rows)}/{T} (all near-ties); softmax: disagreements {len(diff2)}/{T} (probability ties)")
    assert laguna_rate <= 1e-2 and len(diff2) / T <= 1e-2


def _rank_code(keys: np.ndarray) -> np.ndarray:
    """The top-k kernel's unsigned ranking code (csrc/router.cu rank_code):
    1 for NaN, else the order-preserving image of the key with -0 read as
    +0; a larger code ranks first, equal codes by the smaller index."""
    k = np.where(keys == 0.0, np.float32(0.0), keys).astype(np.float32)
    bits = k.view(np.uint32)
    code = np.where(bits & np.uint32(0x80000000), ~bits, bits | np.uint32(0x80000000)).astype(np.uint32)
    return np.where(np.isnan(keys), np.uint32(1), code).astype(np.uint32)


@pytest.mark.parametrize("E", [40, 128, 256])
def test_topk_rank_code_order_matches_checker(E):
    """Selecting by (code descending, index ascending) -- what each warp
    reduction round of the GPU top-k computes -- gives the checker's top-k
    (larger key first, NaN last, -0 == +0, ties by index) on rows with ties,
    NaNs, signed zeros and infinities."""
    rng = np.random.default_rng(E)
    T, k = 64, 8
    l = rng.standard_normal((T, E), dtype=np.float32)
    l[0, :] = 0.5
    l[1, 3] = np.nan
    l[2, :10] = -0.0
    l[2, 10:20] = 0.0
    l[3] = np.round(l[3], 1)
    l[4, :] = np.nan
    l[5, 5:] = -np.inf
    l[6, ::3] = np.inf
    l[7, :] = -0.0
    ref, _ = O.topk_softmax(l, k)
    code = _rank_code(l)
    idx = np.arange(E)
    for t in range(T):
        order = np.lexsort((idx, -code[t].astype(np.int64)))[:k]
        assert np.array_equal(order.astype(np.uint32), ref[t]), f"row {t}"
