"""Expert parallelism over the GPUs of one box: rank r holds experts [r*E/W, (r+1)*E/W) of every MoE layer in its HBM
(the reference's VRAM/RAM/NVMe tiers, glm/xpu/glm_xpu/tier.py:1-20, collapse to this residency), tokens stay
data-parallel, and two NCCL all-to-alls over NVLink move the routed tokens:

  dispatch: every rank sends each peer one fixed-capacity chunk: its B token rows (fp16/bf16) with their routed
            expert ids and weights. Rows go to a peer once, however many of that peer's experts they picked;
  local:    each rank runs the grouped MoE kernels on the B*W received rows, with picks of other ranks' experts
            masked out (id -1), producing one fp32 partial row per received token (decode kernels for small batches,
            the tcgen05 prefill path from PREFILL_MIN_PAIRS picks on);
  combine:  the partial rows go back to their source rank, which sums the W partials in rank order (fixed order:
            bit-reproducible for a given world size) and adds the shared expert of its own rows (every rank holds
            the shared expert; it runs once per token, on the token's rank).

Chunks have fixed capacity (B rows), so no host synchronisation and the step is CUDA-graph capturable; NCCL's
all-to-all is the only data-path collective. The local step is pluggable so that the exchange logic is tested on
CPU gloo ranks with the oracle standing in for the GPU kernels.
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
                 local_fn: Callable | None = None, shared_fn: Callable | None = None):
        self.group = group
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
        """x [B, H] fp16/bf16 (this rank's tokens), ids int32 [B, k] global expert ids, w fp32 [B, k] -> fp32 [B, H]:
        the routed sum over all ranks' experts."""
        B, H = x.shape
        W = self.world
        if W == 1:
            out = self.local_fn(x, localize_ids(ids, self.e0, self.e1).to(torch.int32), w)
            if self.shared_fn is not None:
                out += self.shared_fn(x)
            return out
        k = ids.shape[1]
        # ---- dispatch: one packed byte row per token (x | ids | w), the same chunk to every rank ----
        xb = 2 * H
        row = torch.empty((B, xb + 8 * k), dtype=torch.uint8, device=x.device)
        row[:, :xb] = x.contiguous().view(torch.uint8).view(B, xb)
        row[:, xb:xb + 4 * k] = ids.to(torch.int32).contiguous().view(torch.uint8).view(B, 4 * k)
        row[:, xb + 4 * k:] = w.to(torch.float32).contiguous().view(torch.uint8).view(B, 4 * k)
        send = row.unsqueeze(0).expand(W, B, row.shape[1]).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        recv = recv.view(W * B, -1)
        xr = recv[:, :xb].contiguous().view(x.dtype)
        rid = recv[:, xb:xb + 4 * k].contiguous().view(torch.int32)
        rw = recv[:, xb + 4 * k:].contiguous().view(torch.float32)
        # ---- local experts on every received row ----
        part = self.local_fn(xr, localize_ids(rid, self.e0, self.e1).to(torch.int32), rw)
        # ---- combine: partial rows back to their source rank, summed in rank order ----
        back = torch.empty((W, B, H), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(back, part.view(W, B, H).contiguous(), group=self.group)
        out = back[0].clone()
        for r in range(1, W):
            out += back[r]
        if self.shared_fn is not None:
            out += self.shared_fn(x)
        return out
