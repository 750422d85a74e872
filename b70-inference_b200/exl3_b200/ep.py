"""Expert parallelism over the GPUs of one box: rank r holds experts [r*E/W, (r+1)*E/W) of every MoE layer in its HBM
(the reference's VRAM/RAM/NVMe tiers, glm/xpu/glm_xpu/tier.py:1-20, collapse to this residency), tokens stay
data-parallel, and each layer exchanges the routed rows in three steps:

  dispatch: every rank hands each peer its rows (fp16/bf16) with their routed expert ids rebased to that peer's
            expert range (-1 for picks of other ranks' experts) and weights; rows past the rank's batch are padding
            with no picks;
  local:    each rank runs the grouped MoE kernels on the W * capacity received rows (picks of other ranks' experts
            are -1 and skipped), producing one fp32 partial row per received row (decode kernels for small batches,
            the tcgen05 prefill path from PREFILL_MIN_PAIRS picks on);
  combine:  the partial rows go back to their source rank, which sums them in rank order (fixed order:
            bit-reproducible for a given world size) and adds the shared expert of its own rows (every rank holds
            the shared expert; it runs once per token, on the token's rank).

Two exchanges implement dispatch / combine:
  "p2p" (GPUs, the default there): this package's kernels write straight into the peers' exchange buffers over
        NVLink (exl3_ep_dispatch, then exl3_ep_combine_reduce, or exl3_ep_combine / exl3_ep_reduce as two launches;
        buffers shared once through CUDA IPC handles):
        a row's activations go only to the ranks it picked, a partial row comes back only from the ranks it picked,
        no host synchronisation, no collective launch, graph-capturable (the calls count themselves on the device);
  "nccl": two NCCL (or gloo) all_to_all_single calls per layer on fixed-size chunks (every row to every rank), and
        the summation on the host side's tensors; the path the CPU gloo tests exercise with the oracle as the local
        step.
Every rank must call forward with a batch of at most `capacity` rows (fixed at construction, or by the first call);
batches may differ between ranks; every rank makes the same calls in the same order.
"""
from __future__ import annotations

import ctypes as C
import os
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


class PeerExchange:
    """One exchange buffer per rank for (W, capacity, H, topk), mapped on every peer through CUDA IPC handles
    (exchanged with all_gather_object on the group). Shared by every layer of that shape: layers run one after
    another, and the buffer's device-side call counters keep the ranks in step."""

    _cache: dict = {}

    @classmethod
    def get(cls, group, W: int, rank: int, cap: int, H: int, k: int, device):
        key = (id(group), W, cap, H, k, str(device))
        ex = cls._cache.get(key)
        if ex is None:
            ex = cls._cache[key] = cls(group, W, rank, cap, H, k, device)
        return ex

    def __init__(self, group, W, rank, cap, H, k, device):
        from . import _lib as L
        self.L = L
        lib = L.lib()
        self.W, self.rank, self.cap, self.H, self.k, self.device = W, rank, cap, H, k, device
        nbytes = lib.exl3_ep_buffer_bytes(W, cap, H, k)
        if nbytes == 0:
            raise L.Exl3Error("PeerExchange: unsupported shape")
        with torch.cuda.device(device):
            ptr = C.c_void_p()
            handle = (C.c_ubyte * 64)()
            L.check(lib.exl3_ep_buffer_create(nbytes, C.byref(ptr), handle), "exl3_ep_buffer_create")
            self.ptr = ptr.value
            handles = [None] * W
            dist.all_gather_object(handles, bytes(handle), group=group)
            addrs, self.opened = [], []
            for r, h in enumerate(handles):
                if r == rank:
                    addrs.append(self.ptr)
                    continue
                pp = C.c_void_p()
                hb = (C.c_ubyte * 64).from_buffer_copy(h)
                L.check(lib.exl3_ep_buffer_open(hb, C.byref(pp)), "exl3_ep_buffer_open")
                addrs.append(pp.value)
                self.opened.append(pp.value)
        self.peers = torch.tensor([a if a < (1 << 63) else a - (1 << 64) for a in addrs], dtype=torch.int64,
                                  device=device)
        ox, oi, ow = C.c_size_t(), C.c_size_t(), C.c_size_t()
        L.check(lib.exl3_ep_recv_offsets(W, cap, H, k, C.byref(ox), C.byref(oi), C.byref(ow)), "exl3_ep_recv_offsets")
        self.off = (ox.value, oi.value, ow.value)
        dist.barrier(group=group)

    def recv_views(self, x_dtype):
        """The receive region as tensors: x [W*cap, H], ids int32 [W*cap, k], w fp32 [W*cap, k] (views of the
        library's buffer, valid while this object lives)."""
        W, cap, H, k = self.W, self.cap, self.H, self.k

        def view(off, numel, dt):
            n = numel * torch.tensor([], dtype=dt).element_size()
            return _device_view(self.ptr + off, n, self.device).view(dt)

        return (view(self.off[0], W * cap * H, x_dtype).view(W * cap, H),
                view(self.off[1], W * cap * k, torch.int32).view(W * cap, k),
                view(self.off[2], W * cap * k, torch.float32).view(W * cap, k))

    def close(self):
        lib = self.L.lib()
        for p in self.opened:
            lib.exl3_ep_buffer_close(p)
        self.opened = []
        if self.ptr:
            lib.exl3_ep_buffer_free(self.ptr)
            self.ptr = 0


def _device_view(addr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor over device memory the library owns (no copy; the owner keeps it alive)."""
    class _Arr:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (addr, False), "version": 3,
                                    "strides": None}
    return torch.as_tensor(_Arr(), device=device)


class ExpertParallelMoE:
    """One MoE layer's routed experts sharded over a process group.

    local_fn(x_rows [R, H], local_ids int32 [R, k], w fp32 [R, k]) -> fp32 [R, H] computes this rank's routed
    experts' weighted contributions (default: the grouped MoE kernels on `table`, without its shared expert).
    shared_fn(x [B, H]) -> fp32 [B, H] or None: the shared expert of this rank's own tokens (default: the table's
    shared expert, if any)."""

    def __init__(self, E: int, H: int, topk: int, group=None, table=None, act_limit: float = 0.0,
                 local_fn: Callable | None = None, shared_fn: Callable | None = None, capacity: int | None = None,
                 exchange: str | None = None):
        self.group = group
        self.capacity = capacity
        self.exchange = exchange
        self.fused_reduce = True          # p2p: combine and reduce in one launch (exl3_ep_combine_reduce)
        # p2p: the shared expert on a side stream, overlapping the exchange (EXL3_EP_SHARED_SIDE_STREAM=0: in line)
        self.shared_side_stream = os.environ.get("EXL3_EP_SHARED_SIDE_STREAM", "1") != "0"
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

            def shared_fn(x, workspace_key=None):
                none = torch.full((x.shape[0], 1), -1, dtype=torch.int32, device=x.device)
                zero = torch.zeros((x.shape[0], 1), dtype=torch.float32, device=x.device)
                prefill = x.shape[0] >= PREFILL_MIN_PAIRS // 8
                fn = moe_prefill if prefill else moe_forward
                ws = None
                if workspace_key is not None:                # a call that overlaps the routed experts' own
                    from . import _lib as L
                    lib = L.lib()
                    size = (lib.exl3_moe_prefill_workspace_size if prefill else lib.exl3_moe_workspace_size)(
                        x.shape[0], 1, self.table.E, self.H, self.table.I, 1)
                    ws = L.workspace(x.device, size, workspace_key)
                return fn(x, none, zero, self.table, self.act_limit, torch.float32, workspace=ws)
            shared_fn.own_workspace = True
        self.local_fn = local_fn
        self.shared_fn = shared_fn

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None
                ) -> torch.Tensor:
        """x [B, H] fp16/bf16 (this rank's tokens, B <= capacity), ids int32 [B, k] global expert ids, w fp32 [B, k]
        -> fp32 [B, H]: the routed sum over all ranks' experts (+ the shared expert), written into `out` (fp32,
        contiguous) when given."""
        B, H = x.shape
        W = self.world
        if W == 1:
            res = self.local_fn(x, localize_ids(ids, self.e0, self.e1).to(torch.int32), w)
            if self.shared_fn is not None:
                res += self.shared_fn(x)
            if out is not None:
                out.copy_(res)
                return out
            return res
        if self.capacity is None:
            self.capacity = B
        cap = self.capacity
        if B > cap:
            raise ValueError(f"expert parallelism: batch of {B} rows exceeds the capacity {cap} of this layer")
        exchange = self.exchange or ("p2p" if x.is_cuda else "nccl")
        if exchange == "p2p":
            return self._forward_p2p(x, ids, w, out)
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
        res = back[0, :B].clone()
        for r in range(1, W):
            res += back[r, :B]
        if self.shared_fn is not None:
            res += self.shared_fn(x[:B])
        if out is not None:
            out.copy_(res)
            return out
        return res

    _SIDE: dict = {}

    @classmethod
    def _side_stream(cls, device) -> torch.cuda.Stream:
        """One side stream per device for the shared expert (reused across layers and calls)."""
        key = str(device)
        if key not in cls._SIDE:
            cls._SIDE[key] = torch.cuda.Stream(device=device)
        return cls._SIDE[key]

    def _forward_p2p(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, out=None) -> torch.Tensor:
        """dispatch / local experts / combine / reduce on this package's peer-memory kernels."""
        from . import _lib as L
        B, H = x.shape
        W, cap, k = self.world, self.capacity, ids.shape[1]
        ex = PeerExchange.get(self.group, W, self.rank, cap, H, k, x.device)
        lib = L.lib()
        st = L.stream_of(x)
        xc = x if x.dtype in (torch.float16, torch.bfloat16) else x.half()
        xc = xc.contiguous()
        idc = ids.to(torch.int32).contiguous()
        wc = w.to(torch.float32).contiguous()
        # the shared expert of this rank's own rows needs nothing from the peers: on a side stream (its own
        # workspace), it overlaps the exchange's waits and the routed experts
        shared = None
        side = None
        if (self.shared_fn is not None and self.fused_reduce and self.shared_side_stream
                and getattr(self.shared_fn, "own_workspace", False)):
            cur = torch.cuda.current_stream(x.device)
            side = self._side_stream(x.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                shared = self.shared_fn(xc, workspace_key="moe_ep_shared").contiguous()
        L.check(lib.exl3_ep_dispatch(xc.data_ptr(), L.dtype_code(xc.dtype), xc.stride(0), B, idc.data_ptr(),
                                     wc.data_ptr(), k, self.E, H, W, self.rank, cap, ex.peers.data_ptr(), ex.ptr, st),
                "exl3_ep_dispatch")
        xr, rid, rw = ex.recv_views(xc.dtype)
        part = self.local_fn(xr, rid, rw)
        part = part.contiguous()
        if out is None or out.dtype != torch.float32 or not out.is_contiguous():
            out = torch.empty((B, H), dtype=torch.float32, device=x.device)
        if self.fused_reduce:
            if side is not None:
                torch.cuda.current_stream(x.device).wait_stream(side)
            elif self.shared_fn is not None:
                shared = self.shared_fn(xc).contiguous()
            L.check(lib.exl3_ep_combine_reduce(part.data_ptr(), idc.data_ptr(), B, k, self.E, H, W, self.rank, cap,
                                               L.ptr(shared), ex.peers.data_ptr(), ex.ptr, out.data_ptr(), st),
                    "exl3_ep_combine_reduce")
            return out
        L.check(lib.exl3_ep_combine(part.data_ptr(), k, self.E, H, W, self.rank, cap, ex.peers.data_ptr(), ex.ptr,
                                    st), "exl3_ep_combine")
        shared = self.shared_fn(xc).contiguous() if self.shared_fn is not None else None
        L.check(lib.exl3_ep_reduce(idc.data_ptr(), B, k, self.E, H, W, self.rank, cap, L.ptr(shared), ex.ptr,
                                   out.data_ptr(), st), "exl3_ep_reduce")
        return out
