"""Routed-expert MoE on B200: expert pointer tables, the decode-path moe_forward, and a BlockSparseMLP module with the
reference's load/forward API.

Reference: glm/xpu/glm_xpu/moe_patch.py:15-94 (BlockSparseMLP load/forward = router + routed sum + shared expert),
glm/xpu/csrc/exl3_moe.n128.sycl:1338-1439 (moe_forward over expert pointer tables), dsv41/xpu/dsv_xpu/moe.py:
914-994,1563-1630 (router with residency bias, per-pick expert math, module forward).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L
from .ops import pack, pack_gateup, route, route_hidden

ROUTE_SIGMOID, ROUTE_SOFTMAX, ROUTE_SQRT_SOFTPLUS = L.ROUTE_SIGMOID, L.ROUTE_SOFTMAX, L.ROUTE_SQRT_SOFTPLUS
# Rows from which a MoE layer runs on the tcgen05 grouped GEMMs instead of the decode GEMVs (the decode kernels read a
# picked expert once per 8 rows; a 320-row tensor-core tile pays off once experts see tens of rows each)
PREFILL_MIN_ROWS = 256


@dataclass
class Exl3Matrix:
    """One EXL3 linear's tensors (exllamav3 layout): trellis int16 [k/16, n/16, 16K], suh fp16 [k], svh fp16 [n]."""
    trellis: torch.Tensor
    suh: torch.Tensor
    svh: torch.Tensor
    K: int

    @property
    def k(self) -> int:
        return self.trellis.shape[0] * 16

    @property
    def n(self) -> int:
        return self.trellis.shape[1] * 16

    @classmethod
    def from_bc(cls, bc) -> "Exl3Matrix":
        """From a BC_LinearEXL3-like object (reads trellis/suh/svh/K by name, as exllamav3's BC classes do)."""
        return cls(bc.trellis, bc.suh, bc.svh, int(bc.K))


@dataclass
class Expert:
    gate: Exl3Matrix
    up: Exl3Matrix
    down: Exl3Matrix


class ExpertTable:
    """Device array of exl3_expert descriptors for E routed experts (+ an optional shared expert at index E).

    The table holds references to the tensors, so their device addresses stay valid while it lives
    (the pointer-table convention of glm/xpu/csrc/exl3_moe.n128.sycl:10-13 and exllamav3's BC_BlockSparseMLP)."""

    def __init__(self, experts: list[Expert], shared: Expert | None = None, device=None):
        if not experts:
            raise L.Exl3Error("ExpertTable: no experts")
        self.experts = list(experts)
        self.shared = shared
        e0 = experts[0]
        self.H, self.I = e0.gate.k, e0.gate.n
        allx = self.experts + ([shared] if shared is not None else [])
        for ex in allx:
            for m in (ex.gate, ex.up):
                if (m.k, m.n) != (self.H, self.I) and ex is not shared:
                    raise L.Exl3Error("ExpertTable: routed experts must share H and I")
            if ex.down.k != ex.gate.n or ex.down.n != self.H or ex.up.n != ex.gate.n:
                raise L.Exl3Error("ExpertTable: inconsistent expert shapes")
            for m in (ex.gate, ex.up, ex.down):
                if m.trellis.data_ptr() % 16:
                    raise L.Exl3Error("ExpertTable: trellis tensors must be 16-byte aligned")
                if m.suh.data_ptr() % 8 or m.svh.data_ptr() % 8:
                    raise L.Exl3Error("ExpertTable: suh / svh tensors must be 8-byte aligned")
        if shared is not None and shared.gate.n != self.I:
            raise L.Exl3Error("ExpertTable: the shared expert must have the routed intermediate size "
                              "(run a wider shared expert as its own BC_GatedMLP)")
        self.E = len(self.experts)
        # packed copies the kernels stream: gate|up fused per 128-column block, down column-block-major
        self.packed = []
        arr = (L.Expert * len(allx))()
        for i, ex in enumerate(allx):
            gu = pack_gateup(ex.gate.trellis, ex.up.trellis, ex.gate.K, ex.up.K)
            dn = pack(ex.down.trellis, ex.down.K)
            self.packed.append((gu, dn))
            arr[i].trellis[0] = gu.data_ptr()
            arr[i].trellis[1] = gu.data_ptr()
            arr[i].trellis[2] = dn.data_ptr()
            for j, m in enumerate((ex.gate, ex.up, ex.down)):
                arr[i].suh[j] = m.suh.data_ptr()
                arr[i].svh[j] = m.svh.data_ptr()
                arr[i].K[j] = int(m.K)
        self.max_bits = max(int(m.K) for ex in allx for m in (ex.gate, ex.up, ex.down))
        raw = bytes(C.string_at(C.addressof(arr), C.sizeof(arr)))
        dev = device or self.experts[0].gate.trellis.device
        self.table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev)
        self.device = dev

    def weight_bytes(self, ids: torch.Tensor | None = None) -> int:
        """Trellis + sign-vector bytes of the experts listed in ids (all if None), each counted once."""
        sel = range(self.E) if ids is None else sorted({int(e) for e in ids.reshape(-1).tolist() if 0 <= e < self.E})
        tot = 0
        for e in sel:
            for m in (self.experts[e].gate, self.experts[e].up, self.experts[e].down):
                tot += m.trellis.numel() * 2 + (m.k + m.n) * 2
        return tot


def moe_forward(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, table: ExpertTable,
                act_limit: float = 0.0, out_dtype=torch.float32, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None, n_ctas: int = 0, events: dict | None = None,
                include_shared: bool = True) -> torch.Tensor:
    """Routed MoE sum (+ the table's shared expert, weight 1) for x [M, H] fp16/bf16:
    out[m] = sum_j topk_w[m, j] * expert_{topk_ids[m, j]}(x[m]) + shared(x[m]), fp32 (or fp16) [M, H].
    topk_ids int32 [M, k] (other int types converted; ids < 0 or >= E skipped), topk_w fp32 [M, k].
    The exl3xpu_moe.moe_forward contract (glm/xpu/csrc/exl3_moe.n128.sycl:1338-1341) over ExpertTable descriptors.
    events: if a dict is given, the phases run as separate C-ABI calls and (start, end) CUDA event pairs around the
    gate|up and down GEMV launches are appended to events["gateup"] / events["down"] (benchmark instrumentation;
    events["external"] = True makes them event-record nodes when the call is captured in a CUDA graph).
    include_shared=False leaves out the table's shared expert (expert parallelism adds it once, on the token's rank)."""
    L.require_cuda(x, topk_ids, topk_w)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype not in (torch.float16, torch.bfloat16):
        x2 = x2.half()
    x2 = x2.contiguous()
    M, H = x2.shape
    if H != table.H:
        raise L.Exl3Error(f"moe_forward: hidden {H} != table hidden {table.H}")
    ids = topk_ids.reshape(M, -1).to(torch.int32).contiguous()
    w = topk_w.reshape(M, -1).to(torch.float32).contiguous()
    k = ids.shape[1]
    if out is None:
        out = torch.empty((M, H), dtype=out_dtype, device=x2.device)
    if M == 0:
        return out
    shared = int(table.shared is not None and include_shared)
    lib = L.lib()
    need = lib.exl3_moe_workspace_size(M, k, table.E, H, table.I, shared)
    ws = workspace if workspace is not None else L.workspace(x2.device, need, "moe")
    st = L.stream_of(x2)
    if events is None:
        rc = lib.exl3_moe_decode(x2.data_ptr(), L.dtype_code(x2.dtype), x2.stride(0), M, ids.data_ptr(),
                                 w.data_ptr(), k, table.table.data_ptr(), table.E, shared, H, table.I,
                                 float(act_limit), out.data_ptr(), L.dtype_code(out.dtype), ws.data_ptr(), ws.numel(),
                                 int(n_ctas), st)
        L.check(rc, "moe_forward")
        return out
    # the same launches one phase at a time, with CUDA events around the two GEMV kernels
    L.check(lib.exl3_moe_prepare(x2.data_ptr(), L.dtype_code(x2.dtype), x2.stride(0), M, ids.data_ptr(),
                                 w.data_ptr(), k, table.table.data_ptr(), table.E, shared, H, table.I, ws.data_ptr(),
                                 ws.numel(), st), "moe_forward prepare")
    ext = bool(events.get("external", False))      # event record nodes when captured in a CUDA graph
    e0, e1, e2, e3 = (torch.cuda.Event(enable_timing=True, external=ext) for _ in range(4))
    e0.record()
    L.check(lib.exl3_moe_gateup(M, k, table.table.data_ptr(), table.E, shared, H, table.I, float(act_limit),
                                ws.data_ptr(), ws.numel(), int(n_ctas), st), "moe_forward gate|up")
    e1.record()
    e2.record()
    L.check(lib.exl3_moe_down(M, k, table.table.data_ptr(), table.E, shared, H, table.I, ws.data_ptr(), ws.numel(),
                              int(n_ctas), st), "moe_forward down")
    e3.record()
    L.check(lib.exl3_moe_combine(M, k, table.E, shared, H, table.I, out.data_ptr(), L.dtype_code(out.dtype),
                                 ws.data_ptr(), ws.numel(), st), "moe_forward combine")
    events.setdefault("gateup", []).append((e0, e1))
    events.setdefault("down", []).append((e2, e3))
    return out


def moe_prefill(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, table: ExpertTable,
                act_limit: float = 0.0, out_dtype=torch.float32, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None, include_shared: bool = True) -> torch.Tensor:
    """moe_forward for prefill-sized batches on the tensor cores (C ABI exl3_moe_prefill): the same contract, with
    pairs grouped into items of <= 320 positions per expert and grouped tcgen05 GEMMs for the projections."""
    L.require_cuda(x, topk_ids, topk_w)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype not in (torch.float16, torch.bfloat16):
        x2 = x2.half()
    x2 = x2.contiguous()
    M, H = x2.shape
    if H != table.H:
        raise L.Exl3Error(f"moe_prefill: hidden {H} != table hidden {table.H}")
    ids = topk_ids.reshape(M, -1).to(torch.int32).contiguous()
    w = topk_w.reshape(M, -1).to(torch.float32).contiguous()
    k = ids.shape[1]
    if out is None:
        out = torch.empty((M, H), dtype=out_dtype, device=x2.device)
    if M == 0:
        return out
    shared = int(table.shared is not None and include_shared)
    lib = L.lib()
    need = lib.exl3_moe_prefill_workspace_size(M, k, table.E, H, table.I, shared)
    ws = workspace if workspace is not None else L.workspace(x2.device, need, "moe_prefill")
    rc = lib.exl3_moe_prefill(x2.data_ptr(), L.dtype_code(x2.dtype), x2.stride(0), M, ids.data_ptr(), w.data_ptr(),
                              k, table.table.data_ptr(), table.E, shared, H, table.I, float(act_limit),
                              out.data_ptr(), L.dtype_code(out.dtype), ws.data_ptr(), ws.numel(), L.stream_of(x2))
    L.check(rc, "moe_prefill")
    return out


def moe_align(topk_ids: torch.Tensor, topk_w: torch.Tensor, E: int, shared: bool = False, chunk: int = 8):
    """Alignment tables as tensors (the reference's debug moe_align, glm/xpu/csrc/exl3_moe.n128.sycl:1442-1450):
    dict of n_items, n_valid, item_expert/start/cnt, pair_tok, pair_expert, pair_of, pair_w, pair_src."""
    ids = topk_ids.to(torch.int32).contiguous()
    w = topk_w.to(torch.float32).contiguous()
    M, k = ids.shape
    npairs = M * k
    active = min(npairs, E)
    shared_items = (M + chunk - 1) // chunk if shared else 0
    max_items = (npairs + active * (chunk - 1)) // chunk + shared_items
    p_max = npairs + (M if shared else 0)
    nseg = (npairs + 8191) // 8192                                          # multi-CTA alignment segments
    nbytes = 32 + 4 * (3 * max_items + 4 * p_max + npairs + max_items + nseg * E)   # tables, tickets, counts
    ws = torch.zeros(nbytes + 4096, dtype=torch.uint8, device=ids.device)
    rc = L.lib().exl3_moe_align(ids.data_ptr(), w.data_ptr(), M, k, E, int(shared), chunk, ws.data_ptr(), ws.numel(),
                                L.stream_of(ids))
    L.check(rc, "moe_align")
    wi = ws[:nbytes].view(torch.int32)
    o = 8
    item_expert = wi[o:o + max_items]; o += max_items
    item_start = wi[o:o + max_items]; o += max_items
    item_cnt = wi[o:o + max_items]; o += max_items
    pair_tok = wi[o:o + p_max]; o += p_max
    pair_expert = wi[o:o + p_max]; o += p_max
    pair_of = wi[o:o + npairs]; o += npairs
    pair_w = wi[o:o + p_max].view(torch.float32); o += p_max
    pair_src = wi[o:o + p_max]; o += p_max
    n_items = int(wi[0])
    n_valid = int(wi[1])
    n_pos = n_valid + (M if shared else 0)
    return dict(n_items=n_items, n_valid=n_valid, pair_expert=pair_expert[:n_pos].clone(),
                item_expert=item_expert[:n_items].clone(),
                item_start=item_start[:n_items].clone(), item_cnt=item_cnt[:n_items].clone(),
                pair_tok=pair_tok[:n_valid + (M if shared else 0)].clone(), pair_of=pair_of.clone(),
                pair_w=pair_w[:n_valid + (M if shared else 0)].clone(), pair_src=pair_src[:n_pos].clone())


class BlockSparseMLP:
    """Routed-expert MLP block with the reference's module API (glm/xpu/glm_xpu/moe_patch.py:66-94):
    forward(x, params, out_dtype) = router (with residency bias) -> routed sum on the MoE kernels (the decode GEMVs,
    or the tcgen05 grouped GEMMs from PREFILL_MIN_ROWS rows) + shared expert.

    router_kind: ROUTE_SIGMOID (GLM / DeepSeek-V3 noaux_tc), ROUTE_SOFTMAX (Qwen-Next), ROUTE_SQRT_SOFTPLUS
    (DeepSeek-V4). gate: router weight fp16 [H, E] (exllamav3 stores it in x out). bias: e_score_correction_bias
    (or the cold-tier bias). res: residency bias per expert (0 resident, -margin slower tier, -inf unreadable, or
    +b on a preferred subset), applied to selection only."""

    def __init__(self, experts: list[Expert], gate: torch.Tensor | None, num_experts_per_tok: int,
                 router_kind: int = ROUTE_SIGMOID, e_score_correction_bias: torch.Tensor | None = None,
                 routed_scaling_factor: float = 1.0, renormalize: bool = True, act_limit: float = 0.0,
                 shared: Expert | None = None, res: torch.Tensor | None = None, mul: torch.Tensor | None = None):
        self.table = ExpertTable(experts, shared)
        self.hidden_size = self.table.H
        self.num_experts = self.table.E
        self.num_experts_per_tok = num_experts_per_tok
        self.gate = gate
        self.router_kind = router_kind
        self.bias = e_score_correction_bias
        self.routed_scaling_factor = routed_scaling_factor
        self.renormalize = renormalize
        self.act_limit = act_limit
        self.res = res
        self.mul = mul

    def route_logits(self, logits: torch.Tensor):
        ids, w, _ = route(logits, self.router_kind, self.num_experts_per_tok, bias=self.bias, res=self.res,
                          mul=self.mul, scale=self.routed_scaling_factor, renorm=self.renormalize)
        return ids, w

    def forward(self, x: torch.Tensor, params=None, out_dtype=None, logits: torch.Tensor | None = None):
        y = x.view(-1, self.hidden_size)
        if y.dtype not in (torch.float16, torch.bfloat16):
            y = y.half()
        if logits is None:
            if self.gate is None:
                raise L.Exl3Error("BlockSparseMLP.forward: no router weight; pass logits")
            if getattr(self, "_gate_t", None) is None:
                self._gate_t = self.gate[:, :self.num_experts].t().contiguous().half()
            ids, w, _ = route_hidden(y, self._gate_t, self.router_kind, self.num_experts_per_tok, bias=self.bias,
                                     res=self.res, mul=self.mul, scale=self.routed_scaling_factor,
                                     renorm=self.renormalize)
        else:
            ids, w = self.route_logits(logits)
        fn = moe_prefill if y.shape[0] >= PREFILL_MIN_ROWS else moe_forward
        out = fn(y, ids, w, self.table, self.act_limit, torch.float32)
        out = out.view(x.shape[:-1] + (self.hidden_size,))
        if out_dtype is not None:
            out = out.to(out_dtype)
        return out
