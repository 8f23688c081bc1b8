"""A decode-kernel wait that runs out, driven without any GPU fault: the test
hook b2_testing_set_decode_fault makes one CTA leave its router logits
unwritten (a flag that nothing sets) and shortens the wait bound, so every
CTA's wait for those logits gives up after a few thousand polls.  Checks that
the launch reports B2_STATUS_WAIT_TIMEOUT through b2_device_status and
returns, and that the cross-launch state it leaves behind (in a caller
workspace and in the library's static scratch) is valid: the next calls on
both entry points are bit-identical to calls made before the fault."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _util import bf16_normal, to_torch_bf16

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


def _static(blk, x):
    import torch
    import b2moe

    L = b2moe.lib()
    T = x.shape[0]
    out = torch.empty_like(x)
    inds = torch.empty(T, blk._blk.top_k, dtype=torch.int32, device=x.device)
    wts = torch.empty(T, blk._blk.top_k, dtype=torch.float32, device=x.device)
    rc = L.b2_moe_block_decode_static(ctypes.byref(blk._blk), ctypes.c_void_p(x.data_ptr()), ctypes.c_int64(T),
                                      None, None, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(inds.data_ptr()),
                                      ctypes.c_void_p(wts.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, L.b2_last_error().decode()
    return out, inds, wts


@pytest.mark.parametrize("prepared", [False, True])
def test_decode_wait_timeout_reported_and_next_calls_exact(cuda, prepared):
    import torch
    import b2moe

    L = b2moe.lib()
    L.b2_testing_set_decode_fault.restype = ctypes.c_int
    bank, wr = _bank(cuda, 64, 2048, 768, seed=91)
    blk = b2moe.MoEBlock(bank, wr, top_k=8, prepare_decode=prepared)
    x = to_torch_bf16(bf16_normal(np.random.default_rng(91), (2, 2048)), cuda)
    ref = blk(x, return_routing=True)
    ref_s = _static(blk, x)
    torch.cuda.synchronize()
    assert b2moe.device_status() == b2moe.STATUS_OK
    assert all(torch.equal(a, b) for a, b in zip(ref, ref_s))
    assert L.b2_testing_set_decode_fault(0, 4096) == 0
    try:
        blk(x)
        assert b2moe.device_status() == b2moe.STATUS_WAIT_TIMEOUT
        _static(blk, x)
        assert b2moe.device_status() == b2moe.STATUS_WAIT_TIMEOUT
    finally:
        assert L.b2_testing_set_decode_fault(-1, 0) == 0
    for _ in range(2):
        got = blk(x, return_routing=True)
        got_s = _static(blk, x)
        torch.cuda.synchronize()
        assert b2moe.device_status() == b2moe.STATUS_OK
        assert all(torch.equal(a, b) for a, b in zip(got, ref)), "workspace path after a timed-out launch"
        assert all(torch.equal(a, b) for a, b in zip(got_s, ref)), "static scratch after a timed-out launch"


def test_fault_hook_rejects_bad_cta(cuda):
    import b2moe

    L = b2moe.lib()
    assert L.b2_testing_set_decode_fault(100000, 0) == b2moe.B2_ERR_INVALID_ARGUMENT
    assert L.b2_testing_set_decode_fault(-1, 0) == 0
