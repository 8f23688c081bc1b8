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


def test_block_repeatable(cuda, config2):
    import torch
    import b2moe

    c = config2
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8)
    x = to_torch_bf16(bf16_normal(np.random.default_rng(1), (1, c["H"])), cuda)
    a = blk(x)
    b = blk(x)
    assert torch.equal(a, b)


def test_prepared_decode_bank_is_a_byte_permutation(cuda, config2):
    import torch
    import b2moe

    c = config2
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, prepare_decode=True)
    raw = torch.cat([t.reshape(-1).view(torch.uint8) for t in (c["bank"].gate_codes, c["bank"].gate_scales,
                                                              c["bank"].up_codes, c["bank"].up_scales,
                                                              c["bank"].down_codes, c["bank"].down_scales)])
    assert blk.decode_bank.numel() == raw.numel()
    assert torch.equal(torch.bincount(blk.decode_bank.long(), minlength=256), torch.bincount(raw.long(), minlength=256))
