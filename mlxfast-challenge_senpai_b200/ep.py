"""Expert-parallel MoE prefill block over a torch.distributed process group.

Rank r of P owns experts [r*E/P, (r+1)*E/P) (E divisible by P) and a shard of
the tokens.  One forward:

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

import torch
import torch.distributed as dist

import b2moe


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
