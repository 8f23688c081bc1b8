"""GPU parity tests of the prefill path (more than 8 tokens): router, expert
sort and the tensor-core grouped GEMMs (b2_moe_prepare_prefill_bank) against
the CPU checker at small sizes, and against the decode path (itself checked
against the checker) at BASELINE sizes.  Router indices must be bit-exact;
bf16 outputs within max-abs 2e-2 and mean relative 1e-3."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as O
from _util import assert_bf16_close, bf16_normal, from_torch_bf16, to_torch, to_torch_bf16
from test_gpu_moe_block import make_bank

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small(cuda):
    E, H, F = 8, 1024, 256
    bank, nbank = make_bank(cuda, E, H, F, seed=41)
    rng = np.random.default_rng(41)
    wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.05).astype(np.float32)
    return dict(E=E, H=H, F=F, bank=bank, nbank=nbank, wr=wr, wr_t=to_torch(wr, cuda))


@pytest.fixture(scope="module")
def config2(cuda):
    E, H, F = 128, 2048, 768
    bank, nbank = make_bank(cuda, E, H, F, seed=2)
    rng = np.random.default_rng(22)
    wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    return dict(E=E, H=H, F=F, bank=bank, nbank=nbank, wr=wr, wr_t=to_torch(wr, cuda))


@pytest.mark.parametrize("T,k", [(9, 2), (64, 4), (300, 2)])
def test_prefill_small_matches_oracle(cuda, small, T, k):
    import b2moe

    c = small
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=k, prepare_prefill=True)
    rng = np.random.default_rng(500 + T)
    x = bf16_normal(rng, (T, c["H"]))
    out, inds, wts = blk(to_torch_bf16(x, cuda), return_routing=True)
    ri, rw = O.topk_softmax(O.router_logits(x, c["wr"]), k)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri), "router indices must be bit-exact"
    assert np.allclose(wts.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    ref = O.moe_experts(x, ri, rw, c["nbank"])
    assert_bf16_close(from_torch_bf16(out), ref, what=f"prefill T={T} k={k}")


def test_prefill_one_hot_expert_many_tiles(cuda, small):
    """Every token routed to the same experts (given logits): two experts own
    300 rows each (two balanced token tiles of 150), the others none."""
    import b2moe

    c = small
    T, k = 300, 2
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=k, prepare_prefill=True)
    rng = np.random.default_rng(9)
    x = bf16_normal(rng, (T, c["H"]))
    logits = np.full((T, c["E"]), -5.0, np.float32)
    logits[:, 3] = 4.0
    logits[:, 6] = 3.0 + rng.random(T, dtype=np.float32)
    out, inds, wts = blk(to_torch_bf16(x, cuda), logits=to_torch(logits, cuda), return_routing=True)
    ri, rw = O.topk_softmax(logits, k)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri)
    ref = O.moe_experts(x, ri, rw, c["nbank"])
    assert_bf16_close(from_torch_bf16(out), ref, what="one hot expert")


def test_prefill_sigmoid_bias_residual_scale(cuda, small):
    import b2moe

    c = small
    T, k = 40, 4
    rng = np.random.default_rng(13)
    bias = (rng.standard_normal(c["E"], dtype=np.float32) * 0.1).astype(np.float32)
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=k, router_mode=b2moe.ROUTER_SIGMOID_BIAS,
                         router_bias=to_torch(bias, cuda), routed_scale=2.5, prepare_prefill=True)
    x = bf16_normal(rng, (T, c["H"]))
    res = bf16_normal(rng, (T, c["H"]))
    out, inds, wts = blk(to_torch_bf16(x, cuda), residual=to_torch_bf16(res, cuda), return_routing=True)
    ri, rw = O.topk_sigmoid_bias(O.router_logits(x, c["wr"]), bias, k, renorm=True)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri)
    ref = O.moe_experts(x, ri, rw, c["nbank"], routed_scale=2.5, residual=res)
    assert_bf16_close(from_torch_bf16(out), ref, what="prefill sigmoid/bias + residual + scale")


def test_prefill_config2_matches_oracle(cuda, config2):
    import b2moe

    c = config2
    T = 24
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, prepare_prefill=True)
    rng = np.random.default_rng(77)
    x = bf16_normal(rng, (T, c["H"]))
    out, inds, wts = blk(to_torch_bf16(x, cuda), return_routing=True)
    ri, rw = O.topk_softmax(O.router_logits(x, c["wr"]), 8)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri)
    ref = O.moe_experts(x, ri, rw, c["nbank"])
    assert_bf16_close(from_torch_bf16(out), ref, what="prefill config2 T=24")


@pytest.mark.parametrize("T", [512, 2048])
def test_prefill_config3_matches_decode_path(cuda, config2, T):
    """BASELINE config 3 shapes: the grouped-GEMM path against the decode
    path (checked against the checker above) on the same tokens."""
    import torch
    import b2moe

    c = config2
    gemm = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, prepare_prefill=True)
    dec = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8)
    gen = torch.Generator(device=cuda).manual_seed(T)
    x = torch.randn(T, c["H"], generator=gen, device=cuda).to(torch.bfloat16)
    a, ia, wa = gemm(x, return_routing=True)
    b, ib, wb = dec(x, return_routing=True)
    assert torch.equal(ia, ib) and torch.equal(wa, wb), "routing must not depend on the path"
    assert_bf16_close(from_torch_bf16(a), from_torch_bf16(b), what=f"gemm vs decode path T={T}")


def test_prefill_config3_sampled_tokens_match_oracle(cuda, config2):
    """BASELINE config 3 at full size (2048 tokens, near-uniform routing: every
    expert gets 94-174 rows, so tiles of every height and tile boundaries
    inside experts occur): routing of all tokens bit-exact, and 96 sampled
    tokens -- the first and last token of the batch plus a seeded sample --
    checked directly against the checker."""
    import b2moe

    c = config2
    T = 2048
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=8, prepare_prefill=True)
    rng = np.random.default_rng(2048)
    x = bf16_normal(rng, (T, c["H"]))
    out, inds, wts = blk(to_torch_bf16(x, cuda), return_routing=True)
    ri, rw = O.topk_softmax(O.router_logits(x, c["wr"]), 8)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri)
    counts = np.bincount(ri.reshape(-1), minlength=c["E"])
    assert counts.min() > 0, "every expert must get rows at this size"
    sample = np.unique(np.concatenate([[0, T - 1], rng.choice(T, 94, replace=False)]))
    ref = O.moe_experts(x, ri, rw, c["nbank"], tokens=sample)
    got = from_torch_bf16(out)
    assert_bf16_close(got[sample], ref[sample], what=f"config3 T={T}, {sample.size} sampled tokens")


def test_prefill_repeatable(cuda, small):
    import torch
    import b2moe

    c = small
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=4, prepare_prefill=True)
    x = to_torch_bf16(bf16_normal(np.random.default_rng(3), (200, c["H"])), cuda)
    assert torch.equal(blk(x), blk(x))


def test_prefill_other_hidden_sizes(cuda):
    """hidden 768 / 512 and ffn 256 / 512 through the GEMM path (six and four
    128-row down blocks; 4 and 8 gate/up blocks of 64 features); the last
    case gives every expert about 150 rows (one token tile of N = 160)."""
    import b2moe

    for E, H, F, T in ((3, 768, 256, 20), (2, 512, 512, 33), (4, 512, 256, 300)):
        bank, nb = make_bank(cuda, E, H, F, seed=H)
        rng = np.random.default_rng(H)
        wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.05).astype(np.float32)
        blk = b2moe.MoEBlock(bank, to_torch(wr, cuda), top_k=2, prepare_prefill=True)
        x = bf16_normal(rng, (T, H))
        out = blk(to_torch_bf16(x, cuda))
        ri, rw = O.topk_softmax(O.router_logits(x, wr), 2)
        assert_bf16_close(from_torch_bf16(out), O.moe_experts(x, ri, rw, nb), what=f"prefill H={H} F={F}")


def test_prefill_bank_rejects_bad_shape(cuda):
    import b2moe

    bank, _ = make_bank(cuda, 2, 512, 160, seed=7)  # ffn 160: not a multiple of 256
    with pytest.raises(ValueError, match="prepare_prefill_bank"):
        b2moe.MoEBlock(bank, to_torch(np.zeros((2, 512), np.float32), cuda), top_k=1, prepare_prefill=True)


def test_prefill_pair_mode_bit_identical(cuda, tmp_path):
    """The opt-in 2-CTA grouped GEMMs (cta_group::2, B2_PREFILL_PAIR=1) give
    the same bits as the single-CTA ones: every output element is the same
    sequence of MMA steps over K.  Run in a child process (the mode is read
    once per process)."""
    import subprocess
    import sys

    import torch

    code = r'''
import sys, numpy as np, torch
sys.path[:0] = sys.argv[2:]
import b2moe
from test_gpu_moe_block import make_bank
dev = torch.device("cuda", 0)
bank, _ = make_bank(dev, 16, 512, 256, seed=77)
g = torch.Generator(device=dev).manual_seed(5)
wr = torch.randn(16, 512, generator=g, device=dev) * 0.02
blk = b2moe.MoEBlock(bank, wr, top_k=4, prepare_prefill=True)
x = torch.randn(300, 512, generator=g, device=dev).to(torch.bfloat16)
np.save(sys.argv[1], blk(x).view(torch.int16).cpu().numpy())
'''
    here = os.path.dirname(os.path.abspath(__file__))
    pkg = os.path.join(os.path.dirname(here), "mlxfast-challenge_senpai_b200")
    outs = []
    for mode in ("0", "1"):
        f = str(tmp_path / f"y{mode}.npy")
        env = dict(os.environ, B2_PREFILL_PAIR=mode)
        r = subprocess.run([sys.executable, "-c", code, f, here, pkg], env=env, capture_output=True, text=True,
                           timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(f))
    assert np.array_equal(outs[0], outs[1])
