"""The hot entry points as torch custom ops (torch.library), so that torch.compile, torch.export and graph-capturing
runtimes see each call as one opaque node with a known output shape, as the reference registers its linear
(`exl3xpu::linear` with a register_fake, glm/xpu/exl3xpu/ops.py:119-129; the C++ `exl3xpu_C::linear` fake at
:32-36).

    torch.ops.exl3_b200.linear(x, packed, suh, svh, K, fp32_out) -> y [..., n]
    torch.ops.exl3_b200.route(logits, kind, k, bias, res, mul, scale, renorm) -> (ids int32 [R, k], w fp32 [R, k])
    torch.ops.exl3_b200.moe(x, ids, w, table, E, I, shared, act_limit, prefill) -> fp32 [M, H]

Each real implementation calls this package's CUDA library through its C ABI (ops.py / moe.py); each fake returns an
empty tensor of the output's shape and dtype on the input's device. There is no CPU implementation.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import ops as _ops

SMALL_M_MAX = _ops.SMALL_M_MAX


@torch.library.custom_op("exl3_b200::linear", mutates_args=())
def linear(x: torch.Tensor, packed: torch.Tensor, suh: torch.Tensor | None, svh: torch.Tensor, K: int,
           fp32_out: bool) -> torch.Tensor:
    """EXL3 linear y = Had(Had(x * suh) @ W_hat) * svh on packed weights (exl3_pack): rows up to SMALL_M_MAX on the
    fused decode GEMV (8 rows per launch), more on the tcgen05 linear. y fp32 or fp16."""
    k = x.shape[-1]
    n = svh.shape[0]
    x2 = x.reshape(-1, k)
    x2 = x2 if x2.dtype in (torch.float16, torch.bfloat16) else x2.half()
    x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty((M, n), dtype=torch.float32 if fp32_out else torch.float16, device=x.device)
    if M:
        if M <= SMALL_M_MAX:
            for m0 in range(0, M, 8):
                _ops.exl3_gemv(x2[m0:m0 + 8], packed, suh, svh, K, y[m0:m0 + 8])
        else:
            _ops.exl3_gemm_tc(x2, packed, suh, svh, K, y)
    return y.view(*x.shape[:-1], n)


@linear.register_fake
def _(x, packed, suh, svh, K, fp32_out):
    return x.new_empty((*x.shape[:-1], svh.shape[0]), dtype=torch.float32 if fp32_out else torch.float16)


@torch.library.custom_op("exl3_b200::route", mutates_args=())
def route(logits: torch.Tensor, kind: int, k: int, bias: torch.Tensor | None, res: torch.Tensor | None,
          mul: torch.Tensor | None, scale: float, renorm: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k routing with the residency bias (exl3_route): ids int32 [R, k], weights fp32 [R, k]."""
    ids, w, _ = _ops.route(logits, kind, k, bias=bias, res=res, mul=mul, scale=scale, renorm=renorm)
    return ids, w


@route.register_fake
def _(logits, kind, k, bias, res, mul, scale, renorm):
    R = logits.shape[0]
    return (logits.new_empty((R, k), dtype=torch.int32), logits.new_empty((R, k), dtype=torch.float32))


@torch.library.custom_op("exl3_b200::moe", mutates_args=())
def moe(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, table: torch.Tensor, E: int, I: int, shared: bool,
        act_limit: float, prefill: bool) -> torch.Tensor:
    """Routed MoE sum (+ the shared expert at table entry E when `shared`) over a device array of exl3_expert
    descriptors (ExpertTable.table): the decode kernels (exl3_moe_decode) or, with `prefill`, the tcgen05 grouped
    GEMMs (exl3_moe_prefill). x fp16/bf16 [M, H]; ids [M, topk] (< 0 skipped); w [M, topk] -> fp32 [M, H]."""
    x2 = x if x.dtype in (torch.float16, torch.bfloat16) else x.half()
    x2 = x2.contiguous()
    M, H = x2.shape
    idc = ids.to(torch.int32).contiguous()
    wc = w.to(torch.float32).contiguous()
    topk = idc.shape[1]
    out = torch.empty((M, H), dtype=torch.float32, device=x.device)
    if M == 0:
        return out
    lib = L.lib()
    st = L.stream_of(x2)
    if prefill:
        need = lib.exl3_moe_prefill_workspace_size(M, topk, E, H, I, int(shared))
        ws = L.workspace(x2.device, need, "moe_prefill")
        rc = lib.exl3_moe_prefill(x2.data_ptr(), L.dtype_code(x2.dtype), x2.stride(0), M, idc.data_ptr(),
                                  wc.data_ptr(), topk, table.data_ptr(), E, int(shared), H, I, float(act_limit),
                                  out.data_ptr(), L.F32, ws.data_ptr(), ws.numel(), st)
    else:
        need = lib.exl3_moe_workspace_size(M, topk, E, H, I, int(shared))
        ws = L.workspace(x2.device, need, "moe")
        rc = lib.exl3_moe_decode(x2.data_ptr(), L.dtype_code(x2.dtype), x2.stride(0), M, idc.data_ptr(),
                                 wc.data_ptr(), topk, table.data_ptr(), E, int(shared), H, I, float(act_limit),
                                 out.data_ptr(), L.F32, ws.data_ptr(), ws.numel(), 0, st)
    L.check(rc, "exl3_b200::moe")
    return out


@moe.register_fake
def _(x, ids, w, table, E, I, shared, act_limit, prefill):
    return x.new_empty((x.shape[0], x.shape[1]), dtype=torch.float32)
