"""Expert-parallel MoE prefill block.

Two implementations of the same block, both bit-identical to the single-GPU
block on every rank's tokens:

* ``EPPrefill`` -- the product path: ``b2_moe_ep_prefill`` from the C ABI.
  Dispatch and return are NVLink peer loads and stores into CUDA-IPC-mapped
  buffers with flag barriers in peer memory, all on the device (no host
  round trip, no counts on the host).  torch.distributed only carries the
  one-time handle exchange.
* ``EPMoEBlock`` -- the NCCL formulation (all_to_all_single dispatch and
  return around the grouped GEMMs), kept as the collective-library baseline
  and as the exchange logic the CPU tests run over gloo.

EPMoEBlock: rank r of P owns experts [r*E/P, (r+1)*E/P) (E divisible by P)
and a shard of the tokens.  One forward:

  1. route the local tokens (router logits and top-k on this rank; the router
     weight is replicated) -> global expert ids and weights [T, k];
  2. order the (token, slot) rows by owning rank with the stable expert sort
     (keys = owner rank), so each destination's rows are contiguous and keep
     token-slot order; gather those rows of x;
  3. exchange per-destination row counts, then the rows and their local
     expert ids (all_to_all_single over NCCL on GPUs);
  4. run the owner's experts on the rows it received (SwitchGLU with one
     expert per row: the prefill grouped GEMMs);
  5. send the per-row expert outputs back (the reverse all_to_all, same
     splits), so each source receives its own rows in the order it sent them;
  6. ordered weighted combine through the inverse of step 2's permutation
     (the row of (t, s) sits at inverse[t*k + s]), + routed scale, +
     residual -- the single-GPU prefill's combine, so the result is the same.

The per-row expert arithmetic does not depend on which other rows share a
tile, and the combine folds the slots in slot order, so the output equals the
single-GPU block's output on the same tokens.  The compute steps are the
methods of an `ops` object (GPU kernels by default) so the exchange logic can
be exercised on CPU ranks with the gloo backend.
"""
from __future__ import annotations

from typing import Optional

import ctypes

import torch
import torch.distributed as dist

import b2moe

EP_MAX_RANKS = 8
EP_HANDLE_BYTES = 128
EP_PHASES = ("route", "barrier_a", "keys_sort_gather", "gate_up_gemm", "down_gemm_peer_stores", "barrier_b",
             "combine")


class _EPConfig(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("tokens_per_rank", ctypes.c_int64),
                ("wait_timeout_ms", ctypes.c_int32), ("expert_slot", ctypes.POINTER(ctypes.c_int32))]


def balanced_placement(loads, world: int):
    """Expert placement that evens the ranks' expected work: experts in
    decreasing load, each to the least-loaded rank that still has one of its
    E/world slots free (longest-processing-time greedy).  Returns slot[e]
    (rank-major: rank = slot // (E/world)) for b2_ep_config.expert_slot."""
    loads = [float(v) for v in loads]
    E = len(loads)
    if E % world:
        raise ValueError(f"[ep_prefill] {E} experts do not divide over {world} ranks")
    El = E // world
    rank_load = [0.0] * world
    used = [0] * world
    slot = [0] * E
    for e in sorted(range(E), key=lambda i: (-loads[i], i)):
        r = min((q for q in range(world) if used[q] < El), key=lambda q: (rank_load[q], q))
        slot[e] = r * El + used[r]
        used[r] += 1
        rank_load[r] += loads[e]
    return slot


def local_experts(slot, world: int, rank: int):
    """Global ids of the experts placed on `rank`, in local-slot order."""
    E = len(slot)
    El = E // world
    local = [0] * El
    for e, s in enumerate(slot):
        if s // El == rank:
            local[s % El] = e
    return local


def _ep_lib():
    L = b2moe.lib()
    if not getattr(L, "_ep_bound", False):
        L.b2_ep_create.restype = ctypes.c_int
        L.b2_ep_create.argtypes = [ctypes.POINTER(b2moe._Block), ctypes.POINTER(_EPConfig),
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        L.b2_ep_connect.restype = ctypes.c_int
        L.b2_ep_connect.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.b2_moe_ep_prefill.restype = ctypes.c_int
        L.b2_moe_ep_prefill.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p]
        L.b2_ep_set_phase_timing.restype = ctypes.c_int
        L.b2_ep_set_phase_timing.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.b2_ep_phase_times.restype = ctypes.c_int
        L.b2_ep_phase_times.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)]
        L.b2_ep_destroy.restype = ctypes.c_int
        L.b2_ep_destroy.argtypes = [ctypes.c_void_p]
        L._ep_bound = True
    return L


class EPPrefill:
    """Expert-parallel prefill block on this rank's GPU (b2_moe_ep_prefill).

    `bank` is the whole block's expert bank (this rank keeps its experts) or,
    with `local_bank=True`, already this rank's E/world experts in local-slot
    order.  `expert_slot` (optional, the same on every rank) places expert e
    on rank slot[e] // (E/world); see balanced_placement.  Every rank
    passes `tokens_per_rank` tokens to every call, and all ranks make the
    same calls.  Construction is collective over `group` (handle exchange)."""

    def __init__(self, bank: "b2moe.ExpertBank", router_w: torch.Tensor, top_k: int, tokens_per_rank: int,
                 group=None, router_mode: int = b2moe.ROUTER_SOFTMAX, router_bias: Optional[torch.Tensor] = None,
                 renorm: bool = True, routed_scale: float = 1.0, local_bank: bool = False,
                 wait_timeout_ms: int = 10000, shared: Optional["b2moe.SharedExpert"] = None,
                 expert_slot: Optional[list] = None):
        self.group = group
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        E = router_w.shape[0]
        if E % world:
            raise ValueError(f"[ep_prefill] {E} experts do not divide over {world} ranks")
        El = E // world
        self.expert_slot = None if expert_slot is None else [int(v) for v in expert_slot]
        if not local_bank:
            ids = (list(range(rank * El, (rank + 1) * El)) if self.expert_slot is None
                   else local_experts(self.expert_slot, world, rank))
            idx = torch.tensor(ids, dtype=torch.long, device=bank.gate_codes.device)
            bank = b2moe.ExpertBank(**{f: getattr(bank, f).index_select(0, idx).contiguous() for f in
                                       ("gate_codes", "gate_scales", "up_codes", "up_scales", "down_codes",
                                        "down_scales")})
        self.bank = bank
        self.router_w = router_w.contiguous()
        self.router_bias = None if router_bias is None else router_bias.contiguous().float()
        self.rank, self.world, self.T, self.k, self.E = rank, world, tokens_per_rank, top_k, E
        self.H = bank.gate_codes.shape[2] * 8
        b = b2moe._Block()
        b.hidden, b.ffn, b.n_experts = self.H, bank.gate_codes.shape[1], E
        b.top_k, b.router_mode, b.renorm = top_k, router_mode, int(renorm)
        b.router_w_dtype = b2moe._DT[self.router_w.dtype]
        b.routed_scale = routed_scale
        b.router_w = self.router_w.data_ptr()
        b.router_bias = None if self.router_bias is None else self.router_bias.data_ptr()
        for nm in ("gate_codes", "gate_scales", "up_codes", "up_scales", "down_codes", "down_scales"):
            setattr(b, nm, getattr(bank, nm).data_ptr())
        self.shared = None
        if shared is not None:  # dense MLP on this rank's tokens, added before the residual
            names = ("gate_codes", "gate_scales", "up_codes", "up_scales", "down_codes", "down_scales")
            self.shared = b2moe.SharedExpert(**{nm: getattr(shared, nm).contiguous() for nm in names})
            b.shared_ffn = self.shared.gate_codes.shape[0]
            for nm in names:
                setattr(b, "shared_" + nm, getattr(self.shared, nm).data_ptr())
        self._blk = b
        self._slot_arr = None
        if self.expert_slot is not None:
            self._slot_arr = (ctypes.c_int32 * E)(*self.expert_slot)
        cfg = _EPConfig(rank, world, tokens_per_rank, wait_timeout_ms,
                        None if self._slot_arr is None else ctypes.cast(self._slot_arr, ctypes.POINTER(ctypes.c_int32)))
        L = _ep_lib()
        ctx = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * EP_HANDLE_BYTES)()
        b2moe._check(L.b2_ep_create(ctypes.byref(b), ctypes.byref(cfg), ctypes.byref(ctx), ctypes.addressof(handle)))
        self._ctx = ctx
        mine = torch.tensor(bytearray(handle), dtype=torch.uint8)
        if world > 1:
            dev_t = mine.to(router_w.device) if dist.get_backend(group) == "nccl" else mine
            allh = [torch.empty_like(dev_t) for _ in range(world)]
            dist.all_gather(allh, dev_t, group=group)
            allb = b"".join(bytes(h.cpu().numpy().tobytes()) for h in allh)
        else:
            allb = bytes(mine.numpy().tobytes())
        buf = (ctypes.c_uint8 * len(allb)).from_buffer_copy(allb)
        b2moe._check(L.b2_ep_connect(ctx, ctypes.addressof(buf)))
        if world > 1:
            dist.barrier(group=group)  # every rank mapped its peers before the first call

    def set_phase_timing(self, enable: bool) -> None:
        b2moe._check(_ep_lib().b2_ep_set_phase_timing(self._ctx, int(enable)))

    def phase_times(self) -> dict:
        """Per-phase device times (ms) of the last call (phase timing on)."""
        ms = (ctypes.c_float * (len(EP_PHASES)))()
        b2moe._check(_ep_lib().b2_ep_phase_times(self._ctx, ms))
        return {nm: float(v) for nm, v in zip(EP_PHASES, ms)}

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 logits: Optional[torch.Tensor] = None, return_routing: bool = False,
                 out: Optional[torch.Tensor] = None):
        if x.shape != (self.T, self.H) or x.dtype != torch.bfloat16:
            raise ValueError(f"[ep_prefill] x must be bf16 [{self.T}, {self.H}] (tokens_per_rank x hidden)")
        x = x.contiguous()
        if out is None:
            out = torch.empty_like(x)
        inds = wts = None
        if return_routing:
            inds = torch.empty(self.T, self.k, dtype=torch.int32, device=x.device)
            wts = torch.empty(self.T, self.k, dtype=torch.float32, device=x.device)
        res = None if residual is None else residual.contiguous()
        lg = None if logits is None else logits.contiguous().float()
        b2moe._check(_ep_lib().b2_moe_ep_prefill(self._ctx, x.data_ptr(), self.T, b2moe._ptr(lg), b2moe._ptr(res),
                                                 out.data_ptr(), b2moe._ptr(inds), b2moe._ptr(wts),
                                                 b2moe._stream(x)))
        return (out, inds, wts) if return_routing else out

    def close(self) -> None:
        """Collective: every rank's calls complete before any rank unmaps."""
        if self._ctx:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            b2moe._check(_ep_lib().b2_ep_destroy(self._ctx))
            self._ctx = None


def _words(t: torch.Tensor) -> torch.Tensor:
    """[n, H] 16-bit rows viewed as [n, H/2] int32 (H even)."""
    return t.view(torch.int32)


class GpuOps:
    """Compute steps on the GPU (libb2moe kernels)."""

    def __init__(self, local_block: "b2moe.MoEBlock", router_w: torch.Tensor, router_mode: int,
                 router_bias: Optional[torch.Tensor], renorm: bool):
        self.local = local_block
        self.router_w = router_w
        self.mode, self.bias, self.renorm = router_mode, router_bias, renorm

    def route(self, x: torch.Tensor, k: int, logits: Optional[torch.Tensor] = None):
        if logits is None:
            logits = b2moe.router_logits(x, self.router_w)
        return b2moe.router_topk(logits, k, self.mode, bias=self.bias, renorm=self.renorm)

    def sort_by(self, keys: torch.Tensor, n_bins: int):
        order, _, inverse, offsets = b2moe.gather_sort(keys, n_bins, multi_cta=keys.numel() > 2048)
        return order, inverse, offsets

    def gather_rows(self, src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        return b2moe.gather_rows(src, idx)

    def experts(self, rows: torch.Tensor, local_ids: torch.Tensor) -> torch.Tensor:
        return self.local.switch_glu(rows, local_ids.reshape(-1, 1)).reshape(rows.shape[0], -1)

    def combine(self, y: torch.Tensor, inverse: torch.Tensor, weights: torch.Tensor, routed_scale: float,
                residual: Optional[torch.Tensor]) -> torch.Tensor:
        return b2moe.combine(y, weights, inverse=inverse, routed_scale=routed_scale, residual=residual)


class EPMoEBlock:
    """MoE block with experts sharded over the ranks of `group`."""

    def __init__(self, n_experts: int, top_k: int, ops, group=None, routed_scale: float = 1.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if n_experts % self.world:
            raise ValueError(f"[ep_moe] {n_experts} experts do not divide over {self.world} ranks")
        self.E, self.k = n_experts, top_k
        self.El = n_experts // self.world
        self.ops = ops
        self.routed_scale = routed_scale

    def owned_experts(self):
        return range(self.rank * self.El, (self.rank + 1) * self.El)

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 logits: Optional[torch.Tensor] = None, return_routing: bool = False):
        T, H = x.shape
        k = self.k
        inds, weights = self.ops.route(x, k, logits)
        flat = inds.reshape(-1).to(torch.int32)
        owner = torch.div(flat, self.El, rounding_mode="floor").to(torch.int32)
        order, inverse, offsets = self.ops.sort_by(owner, self.world)
        send_rows = self.ops.gather_rows(x, torch.div(order, k, rounding_mode="floor").to(torch.int32))
        send_ids = (flat[order.long()] - owner[order.long()] * self.El).to(torch.int32)
        send_counts = (offsets[1:] - offsets[:-1]).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        ss, rs = send_counts.tolist(), recv_counts.tolist()
        n_recv = int(sum(rs))
        # rows travel as 32-bit words (two bf16 values each): the same bytes on
        # every backend
        recv_rows = torch.empty(n_recv, H, dtype=x.dtype, device=x.device)
        recv_ids = torch.empty(n_recv, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(_words(recv_rows), _words(send_rows), rs, ss, group=self.group)
        dist.all_to_all_single(recv_ids, send_ids, rs, ss, group=self.group)
        y_recv = self.ops.experts(recv_rows, recv_ids) if n_recv else recv_rows
        y_back = torch.empty(T * k, H, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(_words(y_back), _words(y_recv.contiguous()), ss, rs, group=self.group)
        out = self.ops.combine(y_back, inverse, weights, self.routed_scale, residual)
        if return_routing:
            return out, inds, weights, (ss, rs)
        return out


def make_gpu_block(bank: "b2moe.ExpertBank", router_w: torch.Tensor, top_k: int, group=None,
                   router_mode: int = b2moe.ROUTER_SOFTMAX, router_bias: Optional[torch.Tensor] = None,
                   renorm: bool = True, routed_scale: float = 1.0) -> EPMoEBlock:
    """EP block on this rank's GPU from the full expert bank (slices out the
    experts this rank owns and prepares their prefill bank)."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    E = bank.gate_codes.shape[0]
    El = E // world
    sl = slice(rank * El, (rank + 1) * El)
    local_bank = b2moe.ExpertBank(**{f: getattr(bank, f)[sl].contiguous() for f in
                                     ("gate_codes", "gate_scales", "up_codes", "up_scales", "down_codes",
                                      "down_scales")})
    # the local block only runs SwitchGLU: its router fields are not used
    local = b2moe.MoEBlock(local_bank, router_w[:El].contiguous(), top_k=1, prepare_prefill=True)
    ops = GpuOps(local, router_w, router_mode, router_bias, renorm)
    return EPMoEBlock(E, top_k, ops, group=group, routed_scale=routed_scale)
