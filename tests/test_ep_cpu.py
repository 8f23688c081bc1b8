"""Expert-parallel exchange logic (ep.EPMoEBlock) on CPU ranks over gloo.

The compute steps come from the checker (router top-k, stable sort, per-row
expert MLP, ordered combine); the test checks that the dispatch by owner
rank, the all_to_all exchanges and the return through the sort's inverse
reproduce the single-process block bit for bit on every rank, with 2 and 4
ranks, a skewed routing (ranks receiving no rows) and the residual/scale
tail."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "mlxfast-challenge_senpai_b200")

E, H, F, K, T_PER_RANK = 8, 128, 64, 3, 10


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().numpy().view(np.uint16)


def _t16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16))


class CpuOps:
    """Checker-backed compute steps with the interface of ep.GpuOps."""

    def __init__(self, bank, rank, n_local):
        self.bank, self.rank, self.El = bank, rank, n_local

    def route(self, x, k, logits):
        inds, w = O.topk_softmax(logits.numpy(), k)
        return torch.from_numpy(inds.view(np.int32)), torch.from_numpy(w)

    def sort_by(self, keys, n_bins):
        order, _, inverse, offsets = O.gather_sort(keys.numpy().astype(np.uint32), n_bins)
        return (torch.from_numpy(order.view(np.int32)), torch.from_numpy(inverse.view(np.int32)),
                torch.from_numpy(offsets.view(np.int32)))

    def gather_rows(self, src, idx):
        return _t16(_u16(src)[idx.numpy().astype(np.int64)])

    def experts(self, rows, local_ids):
        ids = (local_ids.numpy().astype(np.uint32) + self.rank * self.El).reshape(-1, 1)
        ones = np.ones(ids.shape, np.float32)
        return _t16(O.moe_experts(_u16(rows), ids, ones, self.bank))

    def combine(self, y, inverse, weights, routed_scale, residual):
        T, k = weights.shape
        d = _u16(y)[inverse.numpy().astype(np.int64)].reshape(T, k, -1)
        res = None if residual is None else _u16(residual)
        return _t16(O.combine_bf16(d, weights.numpy(), routed_scale=routed_scale, residual=res))


def _data(world, skew):
    rng = np.random.default_rng(123)
    bank = {}
    for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
        w, s = O.fp_quantize((rng.standard_normal(shp, dtype=np.float32) * 0.05).astype(np.float32))
        bank[nm + "_w"], bank[nm + "_s"] = w, s
    T = T_PER_RANK * world
    x = O.f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32))
    res = O.f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32))
    logits = rng.standard_normal((T, E), dtype=np.float32)
    if skew:  # every token prefers experts 0..2: the ranks owning the rest receive nothing
        logits[:, :3] += 8.0
    return bank, x, res, logits


def _worker(rank, world, port, skew, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        sys.path.insert(0, PKG)
        import ep  # noqa: E402

        dist.init_process_group("gloo", rank=rank, world_size=world)
        bank, x, res, logits = _data(world, skew)
        sl = slice(rank * T_PER_RANK, (rank + 1) * T_PER_RANK)
        blk = ep.EPMoEBlock(E, K, CpuOps(bank, rank, E // world), routed_scale=2.5)
        out, inds, w, (ss, rs) = blk(_t16(x[sl]), residual=_t16(res[sl]), logits=torch.from_numpy(logits[sl]),
                                     return_routing=True)
        ri, rw = O.topk_softmax(logits[sl], K)
        want = O.moe_experts(x[sl], ri, rw, bank, routed_scale=2.5, residual=res[sl])
        assert np.array_equal(_u16(out), want), f"rank {rank}: EP output differs from the single-process block"
        assert sum(ss) == T_PER_RANK * K
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,skew", [(2, False), (4, False), (4, True)])
def test_ep_exchange_matches_single_process(world, skew):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, skew, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "an EP rank did not finish"
    assert not errs, "; ".join(errs)
    assert all(p.exitcode == 0 for p in procs)


# ---------------------------------------------------------------------------
# The NVLink peer-memory formulation (b2_moe_ep_prefill) restated on CPU ranks.
# Its device kernels index rows as i = q*T*k + t*k + s (source rank q, token
# t, slot s): every rank reads every rank's expert ids, keys its owned rows
# by local expert id (others go to a discard bin El), sorts them stably, runs
# its experts on the owned rows and stores row i at local row i % (T*k) of
# rank i // (T*k); each rank then combines its own tokens in (t, s) order.
# Here the reads of peer memory are all_gather and the peer stores are an
# exchange of (row, data) lists; the test checks that this index arithmetic
# reproduces the single-process block bit for bit.
def _peer_worker(rank, world, port, skew, errq, placement=False):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        bank, x, res, logits = _data(world, skew)
        T, k, El = T_PER_RANK, K, E // world
        sl = slice(rank * T, (rank + 1) * T)
        my_inds, my_w = O.topk_softmax(logits[sl], k)
        # "peer loads": every rank's ids and tokens
        ids = [torch.empty(T * k, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(ids, torch.from_numpy(my_inds.reshape(-1).astype(np.int64)))
        xs = [torch.empty(T, H // 2, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(xs, _t16(x[sl]).view(torch.int32))  # bf16 pairs as 32-bit words
        all_ids = torch.cat(ids).numpy()
        # expert placement: slot[e] (rank-major); identity = contiguous ranges
        slot = np.random.default_rng(99).permutation(E) if placement else np.arange(E)
        row_slot = slot[all_ids]
        keys = np.where(row_slot // El == rank, row_slot % El, El).astype(np.uint32)
        order, _, _, offsets = O.gather_sort(keys, El + 1)
        owned = order[:offsets[El]].astype(np.int64)
        stores = {q: [] for q in range(world)}
        for i in owned:
            tg = i // k
            q, t = int(tg // T), int(tg % T)
            e = np.array([[all_ids[i]]], np.uint32)
            row = O.moe_experts(xs[q].numpy().view(np.uint16)[t:t + 1], e, np.ones((1, 1), np.float32), bank)
            stores[int(i // (T * k))].append((int(i % (T * k)), row[0]))
        # "peer stores": each rank's rows land in their source rank's buffer
        gathered = [None] * world
        dist.all_gather_object(gathered, stores)
        y = np.zeros((T * k, H), np.uint16)
        written = np.zeros(T * k, bool)
        for src in gathered:
            for r, row in src[rank]:
                assert not written[r], "two ranks stored the same row"
                y[r], written[r] = row, True
        assert written.all(), "a (token, slot) row of this rank was never stored"
        out = O.combine_bf16(y.reshape(T, k, H), my_w, routed_scale=2.5, residual=res[sl])
        want = O.moe_experts(x[sl], my_inds, my_w, bank, routed_scale=2.5, residual=res[sl])
        assert np.array_equal(out, want), f"rank {rank}: peer-exchange output differs from the single-process block"
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,skew,placement", [(2, False, False), (4, True, False), (4, True, True),
                                                  (8, False, True)])
def test_ep_peer_exchange_index_math_matches_single_process(world, skew, placement):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, skew, errq, placement)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "an EP rank did not finish"
    assert not errs, "; ".join(errs)
    assert all(p.exitcode == 0 for p in procs)


def test_balanced_placement_is_a_balanced_permutation():
    sys.path.insert(0, PKG)
    import ep

    rng = np.random.default_rng(3)
    E, world = 128, 8
    loads = (1.0 / np.arange(1, E + 1) ** 1.1)[rng.permutation(E)]
    slot = ep.balanced_placement(loads, world)
    assert sorted(slot) == list(range(E))
    El = E // world
    per_rank = np.zeros(world)
    for e, s_ in enumerate(slot):
        per_rank[s_ // El] += loads[e]
    contiguous = np.array([loads[r * El:(r + 1) * El].sum() for r in range(world)])
    assert per_rank.max() <= contiguous.max()
    assert per_rank.max() - per_rank.min() <= loads.max()
    for r in range(world):
        assert [slot[e] for e in ep.local_experts(slot, world, r)] == list(range(r * El, (r + 1) * El))
