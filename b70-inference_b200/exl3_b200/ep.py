"""Expert parallelism over the GPUs of one box: rank r holds experts [r*E/W, (r+1)*E/W) of every MoE layer in its HBM
(the reference's VRAM/RAM/NVMe tiers, glm/xpu/glm_xpu/tier.py:1-20, collapse to this residency), tokens stay
data-parallel, and two NCCL all-to-alls over NVLink move the routed tokens:

  dispatch: every rank sends each peer one chunk of `capacity` rows: its token rows (fp16/bf16) with their routed
            expert ids (already rebased to that peer's expert range, -1 for picks of other ranks' experts) and
            weights; rows past the rank's batch are padding with no picks. Every token row goes to every peer (the
            chunk size is fixed so that the step needs no host synchronisation and can be graph-captured): the
            exchange moves W * capacity rows per rank whatever the routing, and a row without a pick on a peer
            costs that peer nothing but its bytes;
  local:    each rank runs the grouped MoE kernels on the W * capacity received rows (picks of other ranks' experts
            are -1 and skipped), producing one fp32 partial row per received row (decode kernels for small batches,
            the tcgen05 prefill path from PREFILL_MIN_PAIRS picks on);
  combine:  the partial rows go back to their source rank, which sums the W partials in rank order (fixed order:
            bit-reproducible for a given world size) and adds the shared expert of its own rows (every rank holds
            the shared expert; it runs once per token, on the token's rank).

Every rank must call forward with a batch of at most `capacity` rows (the capacity is fixed at construction, or by
the first call); batches may differ between ranks. NCCL's all-to-all is the only data-path collective. The local
step is pluggable so that the exchange logic is tested on CPU gloo ranks with the oracle standing in for the GPU
kernels.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def expert_range(E: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous expert shard of a rank (E must divide evenly)."""
    if E % world:
        raise ValueError(f"expert parallelism: {E} experts do not split over {world} ranks")
    per = E // world
    return rank * per, (rank + 1) * per


def localize_ids(ids: torch.Tensor, e0: int, e1: int) -> torch.Tensor:
    """Global expert ids -> this rank's local ids; picks of other ranks' experts (and invalid ids) become -1."""
    mine = (ids >= e0) & (ids < e1)
    return torch.where(mine, ids - e0, torch.full_like(ids, -1))


PREFILL_MIN_PAIRS = 4096          # received picks from which the local step uses the tcgen05 prefill kernels


class ExpertParallelMoE:
    """One MoE layer's routed experts sharded over a process group.

    local_fn(x_rows [R, H], local_ids int32 [R, k], w fp32 [R, k]) -> fp32 [R, H] computes this rank's routed
    experts' weighted contributions (default: the grouped MoE kernels on `table`, without its shared expert).
    shared_fn(x [B, H]) -> fp32 [B, H] or None: the shared expert of this rank's own tokens (default: the table's
    shared expert, if any)."""

    def __init__(self, E: int, H: int, topk: int, group=None, table=None, act_limit: float = 0.0,
                 local_fn: Callable | None = None, shared_fn: Callable | None = None, capacity: int | None = None):
        self.group = group
        self.capacity = capacity
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.E, self.H, self.topk = E, H, topk
        self.e0, self.e1 = expert_range(E, self.rank, self.world)
        self.table = table
        self.act_limit = act_limit
        if local_fn is None:
            from .moe import moe_forward, moe_prefill

            def local_fn(x, ids, w):
                fn = moe_prefill if ids.numel() >= PREFILL_MIN_PAIRS else moe_forward
                return fn(x, ids, w, self.table, self.act_limit, torch.float32, include_shared=False)
        if shared_fn is None and table is not None and table.shared is not None:
            from .moe import moe_forward, moe_prefill

            def shared_fn(x):
                none = torch.full((x.shape[0], 1), -1, dtype=torch.int32, device=x.device)
                zero = torch.zeros((x.shape[0], 1), dtype=torch.float32, device=x.device)
                fn = moe_prefill if x.shape[0] >= PREFILL_MIN_PAIRS // 8 else moe_forward
                return fn(x, none, zero, self.table, self.act_limit, torch.float32)
        self.local_fn = local_fn
        self.shared_fn = shared_fn

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x [B, H] fp16/bf16 (this rank's tokens, B <= capacity), ids int32 [B, k] global expert ids, w fp32 [B, k]
        -> fp32 [B, H]: the routed sum over all ranks' experts (+ the shared expert)."""
        B, H = x.shape
        W = self.world
        if W == 1:
            out = self.local_fn(x, localize_ids(ids, self.e0, self.e1).to(torch.int32), w)
            if self.shared_fn is not None:
                out += self.shared_fn(x)
            return out
        if self.capacity is None:
            self.capacity = B
        cap = self.capacity
        if B > cap:
            raise ValueError(f"expert parallelism: batch of {B} rows exceeds the capacity {cap} of this layer")
        k = ids.shape[1]
        ids = ids.to(torch.int32)
        if B < cap:                                     # padding rows: no picks anywhere
            x = torch.cat([x, x.new_zeros((cap - B, H))])
            ids = torch.cat([ids, ids.new_full((cap - B, k), -1)])
            w = torch.cat([w.float(), w.new_zeros((cap - B, k), dtype=torch.float32)])
        # ---- dispatch: chunk d = [x | ids rebased to rank d's experts | w] for every row ----
        xb = 2 * H
        per = self.E // W
        send = torch.empty((W, cap, xb + 8 * k), dtype=torch.uint8, device=x.device)
        send[:, :, :xb] = x.contiguous().view(torch.uint8).view(1, cap, xb)
        d0 = (torch.arange(W, device=x.device, dtype=torch.int32) * per).view(W, 1, 1)
        loc = ids.view(1, cap, k) - d0
        loc = torch.where((loc >= 0) & (loc < per), loc, torch.full_like(loc, -1))
        send[:, :, xb:xb + 4 * k] = loc.contiguous().view(torch.uint8).view(W, cap, 4 * k)
        send[:, :, xb + 4 * k:] = w.float().contiguous().view(torch.uint8).view(1, cap, 4 * k)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        recv = recv.view(W * cap, -1)
        xr = recv[:, :xb].contiguous().view(x.dtype)
        rid = recv[:, xb:xb + 4 * k].contiguous().view(torch.int32)
        rw = recv[:, xb + 4 * k:].contiguous().view(torch.float32)
        # ---- local experts on every received row ----
        part = self.local_fn(xr, rid, rw)
        # ---- combine: partial rows back to their source rank, summed in rank order ----
        back = torch.empty((W, cap, H), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(back, part.view(W, cap, H).contiguous(), group=self.group)
        out = back[0, :B].clone()
        for r in range(1, W):
            out += back[r, :B]
        if self.shared_fn is not None:
            out += self.shared_fn(x[:B])
        return out
