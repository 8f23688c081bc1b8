"""GPU tests of SwitchGLU (b2_moe_switch_glu) and the expert-parallel prefill
block: SwitchGLU + ordered combine equals the block forward bit for bit; both
EP implementations -- the NVLink peer-memory path of the C ABI
(b2_moe_ep_prefill, ep.EPPrefill) and the NCCL all-to-all formulation
(ep.EPMoEBlock) -- on one rank and on two GPUs (when present) equal the
single-GPU block on the same tokens bit for bit (the per-row expert
arithmetic does not depend on the rows sharing a tile; the combine order is
the slot order).  Multi-GPU children run with NVLS off (NCCL_NVLS_ENABLE=0)."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from test_gpu_moe_block import make_bank

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "mlxfast-challenge_senpai_b200")
E, H, F, K = 16, 1024, 256, 4


def _block_and_data(dev, T, seed=3):
    import torch
    import b2moe

    bank, _ = make_bank(dev, E, H, F, seed=seed)
    gen = torch.Generator(device=dev).manual_seed(seed)
    wr = torch.randn(E, H, generator=gen, device=dev) * 0.05
    x = torch.randn(T, H, generator=gen, device=dev).to(torch.bfloat16)
    res = torch.randn(T, H, generator=gen, device=dev).to(torch.bfloat16)
    return bank, wr, x, res


def test_switch_glu_plus_combine_is_the_block(cuda):
    import torch
    import b2moe

    bank, wr, x, res = _block_and_data(cuda, 300)
    blk = b2moe.MoEBlock(bank, wr, top_k=K, prepare_prefill=True, routed_scale=2.5)
    out, inds, wts = blk(x, residual=res, return_routing=True)
    y = blk.switch_glu(x, inds)
    assert y.shape == (300, K, H)
    again = b2moe.combine(y.reshape(-1, H), wts, routed_scale=2.5, residual=res)
    assert torch.equal(again, out)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_worker(rank, world, port, T, errq, impl="nccl", placement=False):
    try:
        import torch
        import torch.distributed as dist

        sys.path.insert(0, PKG)
        import b2moe
        import ep

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        bank, wr, x, res = _block_and_data(dev, T * world)
        sl = slice(rank * T, (rank + 1) * T)
        single = b2moe.MoEBlock(bank, wr, top_k=K, prepare_prefill=True, routed_scale=2.5)
        ref, ri, rw = single(x[sl].contiguous(), residual=res[sl].contiguous(), return_routing=True)
        if impl == "peer":
            slot = list(np.random.default_rng(7).permutation(E)) if placement else None
            blk = ep.EPPrefill(bank, wr, K, T, routed_scale=2.5, wait_timeout_ms=5000, expert_slot=slot)
            for it in range(3):  # repeated calls reuse the exchange buffers
                out, inds, wts = blk(x[sl].contiguous(), residual=res[sl].contiguous(), return_routing=True)
                torch.cuda.synchronize()
                assert torch.equal(out, ref), f"rank {rank} call {it}: EP output differs from the single-GPU block"
                assert torch.equal(inds, ri) and torch.equal(wts, rw), f"rank {rank}: routing differs"
            assert b2moe.device_status() == b2moe.STATUS_OK
            blk.close()
        else:
            blk = ep.make_gpu_block(bank, wr, K, routed_scale=2.5)
            out = blk(x[sl].contiguous(), residual=res[sl].contiguous())
            torch.cuda.synchronize()
            assert torch.equal(out, ref), f"rank {rank}: EP output differs from the single-GPU block"
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _run_ep(world, T, impl="nccl", placement=False):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, T, errq, impl, placement)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "an EP rank did not finish"
    assert not errs, "; ".join(errs)
    assert all(p.exitcode == 0 for p in procs)


def test_ep_one_rank_matches_block(cuda):
    _run_ep(1, 200)


def test_ep_two_gpus_matches_block(cuda):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_ep(2, 200)


def test_ep_peer_one_rank_matches_block(cuda):
    """b2_moe_ep_prefill with a single rank (no peers, same kernels and
    barriers) equals the single-GPU block bit for bit, call after call."""
    import torch
    import b2moe
    import ep

    T = 300
    bank, wr, x, res = _block_and_data(cuda, T)
    single = b2moe.MoEBlock(bank, wr, top_k=K, prepare_prefill=True, routed_scale=2.5)
    ref, ri, rw = single(x, residual=res, return_routing=True)
    blk = ep.EPPrefill(bank, wr, K, T, routed_scale=2.5)
    blk.set_phase_timing(True)
    for _ in range(3):
        out, inds, wts = blk(x, residual=res, return_routing=True)
        torch.cuda.synchronize()
        assert torch.equal(out, ref) and torch.equal(inds, ri) and torch.equal(wts, rw)
    ph = blk.phase_times()
    assert set(ph) == set(ep.EP_PHASES) and all(v >= 0 for v in ph.values())
    # given logits (the routerLogits: argument of the reference block)
    logits = b2moe.router_logits(x, wr)
    assert torch.equal(blk(x, residual=res, logits=logits), ref)
    assert b2moe.device_status() == b2moe.STATUS_OK
    with pytest.raises(ValueError):
        blk(x[:10].contiguous())
    blk.close()


@pytest.mark.parametrize("placement", [False, True])
def test_ep_peer_two_gpus_matches_block(cuda, placement):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_ep(2, 200, impl="peer", placement=placement)


@pytest.mark.parametrize("world", [4, 8])
def test_ep_peer_many_gpus_matches_block(cuda, world):
    """Every rank of a 4- or 8-GPU expert-parallel block (balanced-looking
    permuted placement) equals the single-GPU block on its own tokens."""
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_ep(world, 96, impl="peer", placement=True)


def test_ep_peer_one_rank_with_placement_matches_block(cuda):
    """A placement permutes the local expert slots (one rank: all experts
    local, in the permuted order): the output is unchanged."""
    import torch
    import b2moe
    import ep

    T = 256
    bank, wr, x, res = _block_and_data(cuda, T)
    ref = b2moe.MoEBlock(bank, wr, top_k=K, prepare_prefill=True, routed_scale=2.5)(x, residual=res)
    slot = list(np.random.default_rng(11).permutation(E))
    blk = ep.EPPrefill(bank, wr, K, T, routed_scale=2.5, expert_slot=slot)
    assert torch.equal(blk(x, residual=res), ref)
    blk.close()
    with pytest.raises(ValueError):
        ep.EPPrefill(bank, wr, K, T, expert_slot=[0] * E)
