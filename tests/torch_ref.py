"""A torch (CUDA, fp32/fp64) restatement of the oracle's EXL3 linear and MoE expert math, for parity checks at the
BASELINE configurations' full sizes, where the numpy oracle would take minutes per matrix.

The weights come from exl3_reconstruct (the bit-exact dequantisation, itself checked against the oracle and the
reference's w_hat golden tiles), the rounding points are the oracle's (oracle.had_in / linear_acc / had_out /
silu_mul / expert_forward / moe_forward), and the 128-point Hadamard runs the same butterfly stage order in fp32,
so this reference equals the oracle up to fp64-vs-fp64 summation order of the products. `test_torch_ref_matches_oracle`
pins it to the oracle on the full configuration shapes. Test infrastructure only.
"""
from __future__ import annotations

import numpy as np
import torch

from exl3_b200 import ops

RSQRT128 = 0.08838834764831845


def fwht128(v: torch.Tensor) -> torch.Tensor:
    """Unnormalised FWHT over the last axis in 128-blocks, fp32, stages h = 1, 2, ..., 64 (oracle.fwht128_f32)."""
    shp = v.shape
    v = v.float().reshape(-1, 128).clone()
    h = 1
    while h < 128:
        u = v.view(-1, 128 // (2 * h), 2, h)
        a = u[:, :, 0, :].clone()
        b = u[:, :, 1, :].clone()
        u[:, :, 0, :] = a + b
        u[:, :, 1, :] = a - b
        h *= 2
    return v.reshape(shp)


def had_in(x: torch.Tensor, suh: torch.Tensor | None) -> torch.Tensor:
    """xh = fp16(FWHT(fp16(x * suh)) / sqrt(128)) per 128-block (oracle.had_in)."""
    v = x.float() if suh is None else x.float() * suh.float()
    v = v.half().float()
    return (fwht128(v) * RSQRT128).half()


def had_out(acc: torch.Tensor, svh: torch.Tensor, out_dtype) -> torch.Tensor:
    """fp32: FWHT(acc) r svh; fp16: fp16(fp16(FWHT(acc) r) * svh) (oracle.had_out)."""
    y = fwht128(acc.float()) * RSQRT128
    if out_dtype == torch.float32:
        return y * svh.float()
    return (y.half().float() * svh.float()).half()


def w_hat(trellis: torch.Tensor, K: int) -> torch.Tensor:
    """Decoded weights fp16 [k, n] by exl3_reconstruct (bit-exact with oracle.w_hat)."""
    k, n = trellis.shape[0] * 16, trellis.shape[1] * 16
    W = torch.empty((k, n), dtype=torch.float16, device=trellis.device)
    ops.exl3_reconstruct(trellis.contiguous(), W, 0, int(K))
    return W


def linear(x: torch.Tensor, W: torch.Tensor, suh, svh, out_dtype=torch.float32) -> torch.Tensor:
    """EXL3 linear with the oracle's roundings; the product accumulates in fp64 and rounds once to fp32
    (oracle.linear_acc)."""
    xh = had_in(x, suh)
    acc = (xh.double() @ W.double()).float()
    return had_out(acc, svh, out_dtype)


def silu_mul(g: torch.Tensor, u: torch.Tensor, act_limit: float) -> torch.Tensor:
    """fp16(min(silu(g), L) * clamp(u, -L, L)), fp32 math (oracle.silu_mul)."""
    g32 = g.float()
    s = g32 / (1.0 + torch.exp(-g32))
    v = u.float()
    if act_limit:
        s = torch.clamp(s, max=act_limit)
        v = torch.clamp(v, -act_limit, act_limit)
    return (s * v).half()


class TorchExpert:
    """An expert's three matrices (Exl3Matrix-like: trellis, suh, svh, K), dequantised on first use."""

    def __init__(self, ex):
        self.mats = (ex.gate, ex.up, ex.down)
        self._W = None

    def weights(self):
        if self._W is None:
            self._W = [w_hat(m.trellis, m.K) for m in self.mats]
        return self._W

    def release(self):
        self._W = None

    def forward(self, x: torch.Tensor, act_limit: float) -> torch.Tensor:
        """x fp16/bf16 [r, H] -> fp32 [r, H] (oracle.expert_forward)."""
        Wg, Wu, Wd = self.weights()
        g, u, d = self.mats
        gg = linear(x, Wg, g.suh, g.svh, torch.float16)
        uu = linear(x, Wu, u.suh, u.svh, torch.float16)
        a = silu_mul(gg, uu, act_limit)
        return linear(a, Wd, d.suh, d.svh, torch.float32)


def moe_forward(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, experts: list, act_limit: float,
                shared=None, release: bool = True) -> torch.Tensor:
    """Routed MoE layer, fp32 (oracle.moe_forward): out[m] = sum over slots j in order of w[m, j] * expert(x[m]),
    ids < 0 skipped, + the shared expert. Experts are evaluated on all the rows that picked them at once; with
    `release` each expert's dequantised weights are dropped after use (full-size layers do not fit otherwise)."""
    M, topk = ids.shape
    H = x.shape[-1]
    ids_c = ids.cpu().numpy()
    per_slot = torch.zeros((M, topk, H), dtype=torch.float32, device=x.device)
    for e in sorted({int(v) for v in ids_c.reshape(-1) if v >= 0}):
        rows, slots = np.nonzero(ids_c == e)
        te = experts[e] if isinstance(experts[e], TorchExpert) else TorchExpert(experts[e])
        ri = torch.from_numpy(rows).to(x.device)
        si = torch.from_numpy(slots).to(x.device)
        per_slot[ri, si] = te.forward(x[ri], act_limit)
        if release:
            te.release()
    out = torch.zeros((M, H), dtype=torch.float32, device=x.device)
    for j in range(topk):
        out = out + w[:, j:j + 1].float() * per_slot[:, j]
    if shared is not None:
        te = shared if isinstance(shared, TorchExpert) else TorchExpert(shared)
        out = out + te.forward(x, act_limit)
        if release:
            te.release()
    return out
