"""Drop-in for exllamav3's BlockSparseMLP on B200, the seam the reference patches
(glm/xpu/glm_xpu/moe_patch.py:15-94): install() replaces the class's load() and forward().

  load(device):   exllamav3's own load (router, shared experts, score-correction bias, and the routed experts' EXL3
                  linears, which stay resident in HBM: the reference's VRAM / RAM / NVMe tiers collapse to residency),
                  then an ExpertTable of the routed experts built once from the modules' trellis / suh / svh / K
                  attributes (the attribute contract exllamav3's BC classes read by name); the shared expert joins
                  the table when it has the routed intermediate size.
  forward(x, params, out_dtype=None):
                  routing by the module's own routing_fn(bsz, routing_cfg, y, params), as the reference does; the
                  routed sum on this package's kernels through the torch custom op exl3_b200::moe: the decode
                  kernels below PREFILL_MIN_ROWS rows, the tcgen05 grouped GEMMs from there on (exllamav3 switches to
                  its grouped prefill path above 8 rows, glm/docs/ext-op-inventory.md:1150-1165; the decode kernels
                  here read each picked expert once per 8 rows, which keeps them ahead of a mostly empty 320-row
                  tensor-core tile for small batches); plus the shared expert (in the table, or its own forward).
                  Output fp32 [..., hidden] (or out_dtype).

exllamav3 is not a dependency: install() takes the class to patch, and imports exllamav3's when none is given.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import torch_ops  # noqa: F401  (registers torch.ops.exl3_b200.*)
from .moe import Expert, ExpertTable, Exl3Matrix

PREFILL_MIN_ROWS = 256


def install(cls=None):
    """Patch `cls` (default: exllamav3.modules.block_sparse_mlp.BlockSparseMLP) in place; returns it. Idempotent."""
    if cls is None:
        from exllamav3.modules.block_sparse_mlp import BlockSparseMLP as cls  # noqa: N813
    if getattr(cls, "_exl3_b200_installed", False):
        return cls
    cls._exl3_b200_orig_load = cls.load
    cls.load = _load
    cls.forward = _forward
    cls._exl3_b200_installed = True
    return cls


def _matrix(m) -> Exl3Matrix:
    """An EXL3 linear's tensors from an exllamav3 module: the module itself or its `inner` (exllamav3's Linear wraps
    a LinearEXL3), read by name."""
    inner = m if hasattr(m, "trellis") else getattr(m, "inner", None)
    if inner is None or not hasattr(inner, "trellis"):
        raise L.Exl3Error(f"BlockSparseMLP: expert linear {type(m).__name__} is not an EXL3 linear")
    if getattr(inner, "mcg", False) or not getattr(inner, "mul1", True):
        raise L.Exl3Error("BlockSparseMLP: only the mul1 codebook is supported")
    return Exl3Matrix(inner.trellis, inner.suh, inner.svh, int(inner.K))


def _shared_expert(sh, I: int):
    """The shared expert as a table entry when its gate / up / down are EXL3 linears of the routed intermediate size
    (else None: forward() calls its own forward)."""
    mats = []
    for names in (("gate", "gates"), ("up", "ups"), ("down", "downs")):
        m = None
        for nm in names:
            m = getattr(sh, nm, None)
            if isinstance(m, (list, tuple)):
                m = m[0] if len(m) == 1 else None
            if m is not None:
                break
        if m is None:
            return None
        try:
            mats.append(_matrix(m))
        except L.Exl3Error:
            return None
    g, u, d = mats
    if g.n != I or u.n != I or d.k != I:
        return None
    return Expert(g, u, d)


def _load(self, device, **kwargs):
    type(self)._exl3_b200_orig_load(self, device, **kwargs)
    experts = [Expert(_matrix(g), _matrix(u), _matrix(d)) for g, u, d in zip(self.gates, self.ups, self.downs)]
    sh = getattr(self, "shared_experts", None)
    shared = _shared_expert(sh, experts[0].gate.n) if sh is not None else None
    self._exl3_table = ExpertTable(experts, shared)
    self._exl3_shared_in_table = shared is not None


def _forward(self, x, params, out_dtype=None):
    y = x.view(-1, self.hidden_size)
    if y.dtype not in (torch.float16, torch.bfloat16):
        y = y.half()
    bsz = y.shape[0]
    sel, w = self.routing_fn(bsz, self.routing_cfg, y, params)
    t = self._exl3_table
    out = torch.ops.exl3_b200.moe(y, sel, w, t.table, t.E, t.I, self._exl3_shared_in_table,
                                  float(getattr(self, "act_limit", 0.0) or 0.0), bsz >= PREFILL_MIN_ROWS)
    sh = getattr(self, "shared_experts", None)
    if sh is not None and not self._exl3_shared_in_table:
        out += sh.forward(x, params).view(out.shape).float()
    out = out.view(x.shape[:-1] + (self.hidden_size,))
    if out_dtype is not None:
        out = out.to(out_dtype)
    return out
