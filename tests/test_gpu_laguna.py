"""GPU parity of the block in the reference runtime's Laguna mode at the real
model's shapes (E = 256 experts, hidden 2048, expert ffn 512, top-8, bf16
router weight, sigmoid + e_score_correction_bias selection, renormalised
weights, routed scale 2.5, residual; LagunaRuntimeModel.swift:9292-9404 and
:10170-10186, Laguna.swift:149-181) against the CPU checker, with the
library computing the router logits itself.  A bf16 router weight gives bf16
logits (MLX's result type of x.matmul(weight.T), cast to f32 by the gate;
the runtime's fused router stores bfloat(router_result), RM:833-838), so the
checker rounds its logits to bf16 too.  Indices bit-exact on the decode
kernels (both bank layouts) and the prefill grouped GEMMs; bf16 outputs
within max-abs 2e-2, mean relative 1e-3."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from _util import assert_bf16_close, bf16_normal, from_torch_bf16, to_torch, to_torch_bf16
from test_gpu_moe_block import make_bank

pytestmark = pytest.mark.gpu

E, H, F, K = 256, 2048, 512, 8


@pytest.fixture(scope="module")
def laguna(cuda):
    import b2moe

    bank, nbank = make_bank(cuda, E, H, F, seed=256)
    rng = np.random.default_rng(512)
    wr = O.f32_to_bf16((rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32))
    bias = (rng.standard_normal(E, dtype=np.float32) * 0.01).astype(np.float32)
    # the shared expert (LagunaRuntimeMLP, hidden -> 512 -> hidden)
    sh, nsh = {}, {}
    for nm, shp in (("gate", (F, H)), ("up", (F, H)), ("down", (H, F))):
        c_, s_ = O.fp_quantize((rng.standard_normal(shp, dtype=np.float32) * 0.02).astype(np.float32))
        sh[nm + "_codes"], sh[nm + "_scales"] = to_torch(c_.view(np.int32), cuda), to_torch(s_, cuda)
        nsh[nm] = (c_, s_)
    return dict(bank=bank, nbank=nbank, wr=wr, wr_t=to_torch_bf16(wr, cuda), bias=bias,
                bias_t=to_torch(bias, cuda), shared=b2moe.SharedExpert(**sh), nshared=nsh)


def shared_ref(x, nsh):
    """The shared expert on the checker: QuantizedLinear gate / up / down with
    bf16 outputs and the bf16 SwiGLU chain between them."""
    g = O.qmm_bf16(x, *nsh["gate"])
    u = O.qmm_bf16(x, *nsh["up"])
    return O.qmm_bf16(O.swiglu_bf16(g, u), *nsh["down"])


@pytest.mark.parametrize("with_shared", [False, True])
@pytest.mark.parametrize("T,path", [(1, "decode"), (1, "decode_prepared"), (5, "decode_prepared"),
                                    (8, "decode"), (300, "prefill")])
def test_laguna_block_matches_oracle(cuda, laguna, T, path, with_shared):
    import b2moe

    c = laguna
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=K, router_mode=b2moe.ROUTER_SIGMOID_BIAS,
                         router_bias=c["bias_t"], renorm=True, routed_scale=2.5,
                         prepare_decode=path == "decode_prepared", prepare_prefill=path == "prefill",
                         shared=c["shared"] if with_shared else None)
    rng = np.random.default_rng(T * 7 + len(path))
    x = bf16_normal(rng, (T, H))
    res = bf16_normal(rng, (T, H))
    out, inds, wts = blk(to_torch_bf16(x, cuda), residual=to_torch_bf16(res, cuda), return_routing=True)
    logits = O.router_logits(x, O.bf16_to_f32(c["wr"]), bf16_weight=True)
    ri, rw = O.topk_sigmoid_bias(logits, c["bias"], K, renorm=True)
    assert np.array_equal(inds.cpu().numpy().view(np.uint32), ri), "router indices must be bit-exact"
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), rw.view(np.uint32)), "weights must be bit-exact"
    sh = shared_ref(x, c["nshared"]) if with_shared else None
    ref = O.moe_experts(x, ri, rw, c["nbank"], routed_scale=2.5, shared=sh, residual=res)
    assert_bf16_close(from_torch_bf16(out), ref, what=f"laguna {path} T={T} shared={with_shared}")


def test_laguna_shared_expert_through_ep_one_rank(cuda, laguna):
    """The expert-parallel entry point with a shared expert equals the block."""
    import torch
    import b2moe
    import ep

    c = laguna
    T = 64
    blk = b2moe.MoEBlock(c["bank"], c["wr_t"], top_k=K, router_mode=b2moe.ROUTER_SIGMOID_BIAS,
                         router_bias=c["bias_t"], renorm=True, routed_scale=2.5, prepare_prefill=True,
                         shared=c["shared"])
    rng = np.random.default_rng(64)
    x = to_torch_bf16(bf16_normal(rng, (T, H)), cuda)
    res = to_torch_bf16(bf16_normal(rng, (T, H)), cuda)
    ref = blk(x, residual=res)
    e = ep.EPPrefill(c["bank"], c["wr_t"], K, T, router_mode=b2moe.ROUTER_SIGMOID_BIAS, router_bias=c["bias_t"],
                     renorm=True, routed_scale=2.5, shared=c["shared"])
    got = e(x, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    e.close()


def test_laguna_logits_are_bf16_values(cuda, laguna):
    """The library's logits for a bf16 router weight are bf16 values (low 16
    bits zero) equal to the checker's."""
    import b2moe

    c = laguna
    x = bf16_normal(np.random.default_rng(9), (16, H))
    got = b2moe.router_logits(to_torch_bf16(x, cuda), c["wr_t"]).cpu().numpy()
    assert np.all(got.view(np.uint32) & 0xFFFF == 0)
    ref = O.router_logits(x, O.bf16_to_f32(c["wr"]), bf16_weight=True)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
