"""GPU test of b2_moe_block_decode_static, the decode entry point that
allocates nothing.

It serves callers that cannot allocate device memory (a custom-op callback
inside another framework's runtime, whose allocator owns every device buffer,
or a process under a fixed device-memory budget) and therefore cannot pass
b2_moe_block_forward a workspace; its scratch is a static array inside the
library.  The test calls it through the C ABI, twice in a row and
interleaved between blocks of different shapes, with the plain and the
prepared-bank decode kernels, and checks each result against
b2_moe_block_forward with a caller workspace: within the tolerance the other
parity tests use, and in fact bit for bit (same kernel, same inputs).

The file name sorts last so a run that stops at the first failure has run
every other test before this one.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _util import assert_bf16_close, bf16_normal, from_torch_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu


def _bank(cuda, E, H, F, seed):
    import torch
    import b2moe

    gen = torch.Generator(device=cuda).manual_seed(seed)
    t = {}
    for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
        w = torch.randn(shp, generator=gen, device=cuda, dtype=torch.float32) * 0.02
        t[nm + "_codes"], t[nm + "_scales"] = b2moe.quantize(w)
    wr = torch.randn(E, H, generator=gen, device=cuda, dtype=torch.float32) * 0.02
    return b2moe.ExpertBank(**t), wr


def _static_forward(blk, x, T):
    import torch
    import b2moe

    L = b2moe.lib()
    L.b2_moe_block_decode_static.restype = ctypes.c_int
    out = torch.empty_like(x)
    k = blk._blk.top_k
    inds = torch.empty(T, k, dtype=torch.int32, device=x.device)
    wts = torch.empty(T, k, dtype=torch.float32, device=x.device)
    rc = L.b2_moe_block_decode_static(ctypes.byref(blk._blk), ctypes.c_void_p(x.data_ptr()), ctypes.c_int64(T),
                                      None, None, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(inds.data_ptr()),
                                      ctypes.c_void_p(wts.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, L.b2_last_error().decode()
    return out, inds, wts


@pytest.mark.parametrize("prepared", [False, True])
def test_static_scratch_decode_matches_workspace_path_twice(cuda, prepared):
    """Calls through the static scratch, interleaved between two blocks of
    different shapes (and, with prepared banks, the TMA decode kernel), each
    equal bit for bit to the same call with a caller workspace; the first
    block is called twice in a row through the static entry point."""
    import torch
    import b2moe

    bank_a, wr_a = _bank(cuda, 64, 2048, 768, seed=77)
    bank_b, wr_b = _bank(cuda, 32, 1024, 512, seed=78)
    blk_a = b2moe.MoEBlock(bank_a, wr_a, top_k=8, prepare_decode=prepared)
    blk_b = b2moe.MoEBlock(bank_b, wr_b, top_k=4, prepare_decode=prepared)
    rng = np.random.default_rng(5)
    for blk, T in ((blk_a, 1), (blk_a, 4), (blk_b, 4), (blk_a, 2), (blk_b, 1)):
        x = to_torch_bf16(bf16_normal(rng, (T, blk.hidden)), cuda)
        ref, ref_i, ref_w = blk(x, return_routing=True)
        got, got_i, got_w = _static_forward(blk, x, T)
        torch.cuda.synchronize()
        assert torch.equal(got_i, ref_i) and torch.equal(got_w, ref_w)
        assert_bf16_close(from_torch_bf16(got), from_torch_bf16(ref), what=f"static scratch T={T}")
        assert torch.equal(got, ref), f"static scratch T={T}: output differs from the workspace path"
    assert b2moe.device_status() == b2moe.STATUS_OK


def test_static_scratch_rejects_oversized_calls(cuda):
    import torch
    import b2moe

    bank, wr = _bank(cuda, 8, 256, 256, seed=1)
    blk = b2moe.MoEBlock(bank, wr, top_k=4)
    L = b2moe.lib()
    x = torch.zeros(16, 256, dtype=torch.bfloat16, device=cuda)
    out = torch.empty_like(x)
    rc = L.b2_moe_block_decode_static(ctypes.byref(blk._blk), ctypes.c_void_p(x.data_ptr()), ctypes.c_int64(16),
                                      None, None, ctypes.c_void_p(out.data_ptr()), None, None, None)
    assert rc == b2moe.B2_ERR_INVALID_ARGUMENT
    assert "caller workspace" in L.b2_last_error().decode()
