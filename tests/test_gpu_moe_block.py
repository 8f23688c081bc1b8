"""GPU parity tests of the MoE expert block (b2_moe_block_forward) against the
CPU checker: router indices bit-exact, bf16 outputs within max-abs 2e-2 and
mean relative 1e-3."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from _util import assert_bf16_close, bf16_normal, from_torch_bf16, to_torch, to_torch_bf16

pytestmark = pytest.mark.gpu


def make_bank(cuda, E, H, F, seed):
    """N(0, 0.02) expert weights generated and quantized on the GPU; returns the
    torch bank and numpy copies for the checker."""
    import torch
    import b2moe

    gen = torch.Generator(device=cuda).manual_seed(seed)
    t, n = {}, {}
    for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
        w = torch.randn(shp, generator=gen, device=cuda, dtype=torch.float32) * 0.02
        c, s = b2moe.quantize(w)
        del w
        t[nm + "_codes"], t[nm + "_scales"] = c, s
        n[nm + "_w"], n[nm + "_s"] = c.cpu().numpy().view(np.uint32), s.cpu().numpy()
    return b2moe.ExpertBank(**t), n


@pytest.fixture(scope="module")
def config2(cuda):
    """H=2048, E=128, top-8, F=768, fp32 router, softmax."""
    E, H, F = 128, 2048, 768
    bank, nbank = make_bank(cuda, E, H, F, seed=2)
    rng = np.random.default_rng(22)
    wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    return dict(E=E, H=H, F=F, bank=bank, nbank=nbank, wr=wr, wr_t=to_torch(wr, cuda))


@pytest.mark.parametrize("prepared", [False, True])
@pytest.mark.parametrize("T", [1, 2, 5, 8])
def test_decode_block_matches_oracle(cuda, config2, T, prepared):
    import b2moe

    c = config2
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, prepare_decode=prepared)
    rng = np.random.default_rng(100 + T)
    x = bf16_normal(rng, (T, c["H"]))
    out, inds, wts = blk(to_torch_bf16(x, cuda), return_routing=True)
    logits = O.router_logits(x, c["wr"])
    ri, rw = O.topk_softmax(logits, 8)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri), "router indices must be bit-exact"
    assert np.allclose(wts.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    ref = O.moe_experts(x, ri, rw, c["nbank"])
    assert_bf16_close(from_torch_bf16(out), ref, what=f"decode block T={T}")


@pytest.mark.parametrize("prepared", [False, True])
def test_decode_block_with_given_logits_residual_and_scale(cuda, config2, prepared):
    import b2moe

    c = config2
    rng = np.random.default_rng(7)
    bias = (rng.standard_normal(c["E"], dtype=np.float32) * 0.05).astype(np.float32)
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, router_mode=b2moe.ROUTER_SIGMOID_BIAS,
                         router_bias=to_torch(bias, cuda), routed_scale=2.5, prepare_decode=prepared)
    T = 3
    x = bf16_normal(rng, (T, c["H"]))
    res = bf16_normal(rng, (T, c["H"]))
    logits = rng.standard_normal((T, c["E"]), dtype=np.float32)
    out, inds, wts = blk(to_torch_bf16(x, cuda), residual=to_torch_bf16(res, cuda), logits=to_torch(logits, cuda),
                         return_routing=True)
    ri, rw = O.topk_sigmoid_bias(logits, bias, 8, renorm=True)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri)
    ref = O.moe_experts(x, ri, rw, c["nbank"], routed_scale=2.5, residual=res)
    assert_bf16_close(from_torch_bf16(out), ref, what="laguna-style decode")


@pytest.mark.parametrize("prepared", [False, True])
def test_block_repeatable(cuda, config2, prepared):
    import torch
    import b2moe

    c = config2
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, prepare_decode=prepared)
    x = to_torch_bf16(bf16_normal(np.random.default_rng(1), (1, c["H"])), cuda)
    a = blk(x)
    b = blk(x)
    assert torch.equal(a, b)


def prepared_scale_bytes(sb):
    """Prepared scale byte: bits 14..7 of the f16 encoding of the MLX-decoded
    |scale| ((b & 127) << 7 as a half, times 256)."""
    m = (sb.astype(np.uint16) & 0x7F) << 7
    h = (m.view(np.float16).astype(np.float32) * 256.0).astype(np.float16)
    return (h.view(np.uint16) >> 7).astype(np.uint8)


def prepared_tile(codes, scales, nsplit):
    """Numpy statement of one prepared tile: codes [16, K/2] u8, scales
    [16, K/16] u8 (MLX layout) -> 9K bytes (codes then scales)."""
    K = codes.shape[1] * 2
    NB = K // 32 // nsplit
    i = np.arange(2 * K)
    w, rem = i // (NB * 64), i % (NB * 64)
    j, lane, ub, g = rem // 128, (rem // 4) % 32, (rem // 2) % 2, rem % 2
    kb = w + nsplit * (2 * j + ub)
    gi, c = lane // 4, lane % 4
    k0 = kb * 32 + 16 * g
    words = np.zeros(2 * K, np.uint32)
    for bi in range(4):
        r = gi + 8 * (bi & 1)
        kk = k0 + 2 * c + 8 * (bi >> 1)
        byte = codes[r, kk // 2].astype(np.uint32)
        byte ^= np.where(scales[r, k0 // 16] & 0x80, 0x88, 0).astype(np.uint32)
        words |= byte << (8 * bi)
    i = np.arange(K)
    w, gi, u, bi = i // (32 * NB), (i // (4 * NB)) % 8, (i // 4) % NB, i % 4
    r, g = gi + 8 * (bi >> 1), bi & 1
    sbytes = prepared_scale_bytes(scales[r, (w + nsplit * u) * 2 + g])
    return np.concatenate([words.view(np.uint8), sbytes])


def check_prepared_tiles(bank_u8, nb, E, H, F, picks):
    """Compare the listed gate/up tiles (e, f) and down tiles (e, b) of a
    prepared bank with the numpy statement of the layout."""
    n_gu = E * (F // 8)
    for kind, e, t in picks:
        if kind == "gu":
            rows = np.arange(8) + 8 * t
            codes = np.concatenate([nb["gate_w"][e, rows].view(np.uint8), nb["up_w"][e, rows].view(np.uint8)])
            scales = np.concatenate([nb["gate_s"][e, rows], nb["up_s"][e, rows]])
            off, K, ns = (e * (F // 8) + t) * 9 * H, H, 16
        else:
            rows = np.arange(16) + 16 * t
            codes = nb["down_w"][e, rows].view(np.uint8)
            scales = nb["down_s"][e, rows]
            off, K, ns = n_gu * 9 * H + (e * (H // 16) + t) * 9 * F, F, 2
        want = prepared_tile(codes.reshape(16, K // 2), scales.reshape(16, K // 16), ns)
        got = bank_u8[off:off + 9 * K]
        assert np.array_equal(got, want), f"prepared {kind} tile ({e}, {t}) differs"


def test_prepared_decode_bank_layout(cuda, config2):
    import b2moe

    c = config2
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, prepare_decode=True)
    E, H, F = c["E"], c["H"], c["F"]
    assert blk.decode_bank.numel() == E * (F // 8) * 9 * H + E * (H // 16) * 9 * F
    bank = blk.decode_bank.cpu().numpy()
    check_prepared_tiles(bank, c["nbank"], E, H, F,
                         [("gu", 0, 0), ("gu", 5, 17), ("gu", E - 1, F // 8 - 1), ("dn", 0, 0), ("dn", 77, 3),
                          ("dn", E - 1, H // 16 - 1)])


def test_prepared_bank_negative_scales(cuda):
    """Scale bytes with the sign bit set (MLX decodes them as negative) go
    through the prepared bank as |scale| with the group's code signs flipped;
    the decode output must still match the checker."""
    import torch
    import b2moe

    E, H, F = 8, 1024, 256
    bank, nb = make_bank(cuda, E, H, F, seed=31)
    rng = np.random.default_rng(5)
    t = {}
    for nm in ("gate", "up", "down"):
        s = nb[nm + "_s"].copy()
        flip = rng.random(s.shape) < 0.3
        s[flip] |= 0x80
        nb[nm + "_s"] = s
        t[nm + "_scales"] = torch.from_numpy(s).to(cuda)
        t[nm + "_codes"] = getattr(bank, nm + "_codes")
    bank2 = b2moe.ExpertBank(**t)
    wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.05).astype(np.float32)
    blk = b2moe.MoEBlock(bank2, to_torch(wr, cuda), top_k=2, prepare_decode=True)
    check_prepared_tiles(blk.decode_bank.cpu().numpy(), nb, E, H, F,
                         [("gu", e, f) for e in range(E) for f in (0, 7, F // 8 - 1)] +
                         [("dn", e, b) for e in range(E) for b in (0, H // 16 - 1)])
    for T in (1, 3):
        x = bf16_normal(rng, (T, H))
        out, inds, wts = blk(to_torch_bf16(x, cuda), return_routing=True)
        ri, rw = O.topk_softmax(O.router_logits(x, wr), 2)
        assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri)
        ref = O.moe_experts(x, ri, rw, nb)
        assert_bf16_close(from_torch_bf16(out), ref, what=f"negative scales T={T}")
