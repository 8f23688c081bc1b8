"""GPU parity of the decode step of a decoder stack (b2_decode_step: RMSNorm,
NVFP4 q/k/v and o projections, RoPE, KV-cache append, grouped-query
attention, the MoE block, final RMSNorm) against the checker's restatement
(oracle.decode_step), token after token so the caches build up; bf16 outputs
within max-abs 2e-2 and mean relative 1e-3 for one layer (the contract's
per-op tolerance).  Across two layers every op's last-bit bf16 differences
(summation order of the norms, the attention and the GEMVs) are carried
through six more bf16-rounded ops per layer, so the two-layer checks state
mean relative 3e-3 (max-abs unchanged).  Small shapes (hidden 1024, 8 q /
2 kv heads of 128, 16 experts top-4) keep the checker fast."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from _util import assert_bf16_close, bf16_normal, from_torch_bf16, to_torch, to_torch_bf16

pytestmark = pytest.mark.gpu

H, NQ, NKV, HD, E, F, K, MAXSEQ = 1024, 8, 2, 128, 16, 256, 4, 64
MEAN_REL_STACK = 3e-3  # two layers (see the module docstring)


def _q(rng, shape, scale=0.02):
    return O.fp_quantize((rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float32))


def build(cuda, seed, layers=2):
    import b2moe

    rng = np.random.default_rng(seed)
    attn, moe, nlayers = [], [], []
    for _ in range(layers):
        qkv = _q(rng, ((NQ + 2 * NKV) * HD, H), 0.05)
        o = _q(rng, (H, NQ * HD), 0.03)
        an = O.f32_to_bf16((1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32))
        mn = O.f32_to_bf16((1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32))
        bank_t, bank_n = {}, {}
        for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
            c, s = _q(rng, shp)
            bank_t[nm + "_codes"], bank_t[nm + "_scales"] = to_torch(c.view(np.int32), cuda), to_torch(s, cuda)
            bank_n[nm + "_w"], bank_n[nm + "_s"] = c, s
        wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.05).astype(np.float32)
        attn.append(b2moe.AttentionWeights(
            attn_norm_w=to_torch_bf16(an, cuda), qkv_codes=to_torch(qkv[0].view(np.int32), cuda),
            qkv_scales=to_torch(qkv[1], cuda), o_codes=to_torch(o[0].view(np.int32), cuda),
            o_scales=to_torch(o[1], cuda), mlp_norm_w=to_torch_bf16(mn, cuda)))
        moe.append(b2moe.MoEBlock(b2moe.ExpertBank(**bank_t), to_torch(wr, cuda), top_k=K, prepare_decode=True))
        nlayers.append(dict(attn_norm_w=an, qkv=qkv, o=o, mlp_norm_w=mn, router=wr, bank=bank_n))
    fn = O.f32_to_bf16((1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    stack = b2moe.DecoderStack(attn, moe, to_torch_bf16(fn, cuda), NQ, NKV, MAXSEQ, HD, rope_theta=1e6)
    return stack, nlayers, fn


@pytest.mark.parametrize("layers", [1, 2])
def test_decode_step_matches_oracle_over_positions(cuda, layers):
    stack, nlayers, fn = build(cuda, 4, layers)
    caches = [[np.zeros((NKV, MAXSEQ, HD), np.uint16), np.zeros((NKV, MAXSEQ, HD), np.uint16)]
              for _ in range(layers)]
    rng = np.random.default_rng(44)
    mean_rel = 1e-3 if layers == 1 else MEAN_REL_STACK
    for pos in range(6):
        x = bf16_normal(rng, (1, H))
        got = from_torch_bf16(stack.step(to_torch_bf16(x, cuda), pos))
        ref = O.decode_step(x, nlayers, fn, pos, caches, NQ, NKV, top_k=K)
        assert_bf16_close(got, ref, mean_rel=mean_rel, what=f"decode step ({layers} layers) pos={pos}")
        # the caches the GPU wrote hold the checker's k / v rows
        for li in range(layers):
            assert_bf16_close(from_torch_bf16(stack.k_cache[li])[:, : pos + 1], caches[li][0][:, : pos + 1],
                              what=f"k cache layer {li}")
            assert np.array_equal(from_torch_bf16(stack.v_cache[li])[:, : pos + 1], caches[li][1][:, : pos + 1])


@pytest.mark.parametrize("layers", [1, 2])
def test_decode_step_long_context_attention(cuda, layers):
    """Positions spread over several attention splits: fill the caches with
    seeded rows, then one step at the last position."""
    import torch

    stack, nlayers, fn = build(cuda, 5, layers)
    rng = np.random.default_rng(55)
    pos = MAXSEQ - 1
    caches = []
    for li in range(layers):
        kc = bf16_normal(rng, (NKV, MAXSEQ, HD))
        vc = bf16_normal(rng, (NKV, MAXSEQ, HD))
        stack.k_cache[li].copy_(to_torch_bf16(kc, cuda))
        stack.v_cache[li].copy_(to_torch_bf16(vc, cuda))
        caches.append([kc.copy(), vc.copy()])
    torch.cuda.synchronize()
    x = bf16_normal(rng, (1, H))
    got = from_torch_bf16(stack.step(to_torch_bf16(x, cuda), pos))
    ref = O.decode_step(x, nlayers, fn, pos, caches, NQ, NKV, top_k=K)
    assert_bf16_close(got, ref, mean_rel=1e-3 if layers == 1 else MEAN_REL_STACK,
                      what=f"decode step ({layers} layers) at the last cache position")


def test_decode_step_rejects_position_outside_cache(cuda):
    import torch

    stack, _, _ = build(cuda, 6)
    with pytest.raises(ValueError):
        stack.step(torch.zeros(1, H, dtype=torch.bfloat16, device=cuda), MAXSEQ)
