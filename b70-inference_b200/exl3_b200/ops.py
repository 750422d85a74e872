"""exllamav3_ext ops of the EXL3 linear path on B200, with the reference's names, arguments and in-place semantics.

Mirrors glm/xpu/glm_xpu/ops.py of horvay/b70-inference (the XPU stand-in for exllamav3's extension): callers hand in
preallocated outputs and read them back, as the CUDA ops do. Every op runs on this package's CUDA library through
its C ABI; none has a CPU path.
"""
from __future__ import annotations

import os
import weakref

import torch

from . import _lib as L

SMALL_M_MAX = int(os.environ.get("EXL3_SMALL_M_MAX", "32"))        # rows up to this: fused decode GEMV (16-row calls)
GEMV_MAX_ROWS = 16                                                  # rows per exl3_gemv call


def _f16(t: torch.Tensor) -> torch.Tensor:
    t = t if t.dtype in (torch.float16, torch.bfloat16) else t.half()
    return t if t.is_contiguous() else t.contiguous()


# ----------------------------------------------------------------------------------------------- EXL3 linear

def pack(trellis: torch.Tensor, K: int) -> torch.Tensor:
    """exllamav3 trellis [k/16, n/16, 16K] int16 -> the GEMV's column-block-major layout (same bytes, permuted)."""
    L.require_cuda(trellis)
    tr = trellis.contiguous()
    k, n = tr.shape[0] * 16, tr.shape[1] * 16
    out = torch.empty(n // 128, k // 16, 8 * 16 * int(K), dtype=torch.int16, device=tr.device)
    L.check(L.lib().exl3_pack(tr.data_ptr(), k, n, int(K), out.data_ptr(), L.stream_of(tr)), "exl3_pack")
    return out


def pack_gateup(gate: torch.Tensor, up: torch.Tensor, Kg: int, Ku: int) -> torch.Tensor:
    """Fused gate|up packing: [I/128, H/16, 8 gate tiles | 8 up tiles] (int16 view)."""
    L.require_cuda(gate, up)
    g, u = gate.contiguous(), up.contiguous()
    H, I = g.shape[0] * 16, g.shape[1] * 16
    if u.shape[0] * 16 != H or u.shape[1] * 16 != I:
        raise L.Exl3Error("pack_gateup: gate and up shapes differ")
    out = torch.empty(I // 128, H // 16, 8 * 16 * (int(Kg) + int(Ku)), dtype=torch.int16, device=g.device)
    L.check(L.lib().exl3_pack_gateup(g.data_ptr(), u.data_ptr(), H, I, int(Kg), int(Ku), out.data_ptr(),
                                     L.stream_of(g)), "exl3_pack_gateup")
    return out


def exl3_gemv(x: torch.Tensor, packed: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
              y: torch.Tensor, n_ctas: int = 0, workspace: torch.Tensor | None = None) -> None:
    """y[M, n] = Had(Had(x * suh) @ W_hat) * svh for M <= 16 rows; packed = pack(trellis, K); y fp16/bf16/fp32
    preallocated (C ABI exl3_gemv). n_ctas: CTAs of the persistent launch (0 = one per SM)."""
    L.require_cuda(x, packed, y)
    M, k = x.shape
    n = svh.shape[0]
    lib = L.lib()
    need = lib.exl3_gemv_workspace_size(M, k, n)
    ws = workspace if workspace is not None else L.workspace(x.device, need, "gemv")
    rc = lib.exl3_gemv(x.data_ptr(), L.dtype_code(x.dtype), x.stride(0), M, packed.data_ptr(), L.ptr(suh),
                       svh.data_ptr(), k, n, int(K), 2, y.data_ptr(), L.dtype_code(y.dtype), y.stride(0),
                       ws.data_ptr(), ws.numel(), int(n_ctas), L.stream_of(x))
    L.check(rc, "exl3_gemv")


def exl3_gemm_tc(x: torch.Tensor, packed: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
                 y: torch.Tensor, workspace: torch.Tensor | None = None) -> None:
    """y[M, n] = Had(Had(x * suh) @ W_hat) * svh for any M on tcgen05 (C ABI exl3_gemm_tc); packed = pack(trellis,
    K); n % 128 == 0; y fp16/bf16/fp32 preallocated."""
    L.require_cuda(x, packed, y)
    M, k = x.shape
    n = svh.shape[0]
    lib = L.lib()
    need = lib.exl3_gemm_tc_workspace_size(M, k)
    ws = workspace if workspace is not None else L.workspace(x.device, need, "gemm_tc")
    rc = lib.exl3_gemm_tc(x.data_ptr(), L.dtype_code(x.dtype), x.stride(0), M, packed.data_ptr(), L.ptr(suh),
                          svh.data_ptr(), k, n, int(K), 2, y.data_ptr(), L.dtype_code(y.dtype), y.stride(0),
                          ws.data_ptr(), ws.numel(), L.stream_of(x))
    L.check(rc, "exl3_gemm_tc")


def exl3_gemv_noalloc(x: torch.Tensor, packed: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
                      y: torch.Tensor) -> None:
    """exl3_gemv with the library's static device scratch instead of a workspace (C ABI exl3_gemv_noalloc):
    M <= 8, k <= 32768, n <= 65536; calls on one device must not overlap."""
    L.require_cuda(x, packed, y)
    M, k = x.shape
    n = svh.shape[0]
    rc = L.lib().exl3_gemv_noalloc(x.data_ptr(), L.dtype_code(x.dtype), x.stride(0), M, packed.data_ptr(),
                                   L.ptr(suh), svh.data_ptr(), k, n, int(K), 2, y.data_ptr(), L.dtype_code(y.dtype),
                                   y.stride(0), L.stream_of(x))
    L.check(rc, "exl3_gemv_noalloc")


def exl3_reconstruct(trellis: torch.Tensor, w: torch.Tensor, n0: int, K: int, cb: int = 2) -> None:
    """w[k, n_slice] (fp16, written) = W_hat[:, n0 : n0 + n_slice] (glm/xpu/csrc/exl3_ops.sycl:539-555)."""
    L.require_cuda(trellis, w)
    k, n = trellis.shape[0] * 16, trellis.shape[1] * 16
    rc = L.lib().exl3_dequant(trellis.data_ptr(), k, n, int(K), int(cb), int(n0), w.shape[1], w.data_ptr(),
                              w.stride(0), L.stream_of(w))
    L.check(rc, "exl3_dequant")


def reconstruct(unpacked: torch.Tensor, packed: torch.Tensor, K, mcg: bool = False, mul1: bool = True) -> None:
    """exllamav3 reconstruct(unpacked, packed, K, mcg, mul1) (glm/docs/ext-op-inventory.md:597-612)."""
    if mcg or not mul1:
        raise L.Exl3Error("reconstruct: only the mul1 codebook is supported")
    exl3_reconstruct(packed, unpacked, 0, int(K))


def reconstruct_slice(unpacked: torch.Tensor, packed: torch.Tensor, K, mcg: bool, mul1: bool, n_offset: int) -> None:
    if mcg or not mul1:
        raise L.Exl3Error("reconstruct_slice: only the mul1 codebook is supported")
    exl3_reconstruct(packed, unpacked, int(n_offset), int(K))


def had_r_128(input: torch.Tensor, output: torch.Tensor, pre_scale, post_scale, scale: float) -> None:
    """Blockwise 128-point Hadamard * scale/sqrt(128); pre_scale wins over post_scale (glm/xpu/glm_xpu/ops.py:
    132-142). fp16 in/out (products rounded to fp16) or fp32 in/out. In place allowed."""
    L.require_cuda(input, output)
    if input.dtype != output.dtype or input.dtype not in (torch.float16, torch.float32):
        raise L.Exl3Error("had_r_128: input/output must both be fp16 or both fp32")
    x = input if input.is_contiguous() else input.contiguous()
    out = output if output.is_contiguous() else torch.empty_like(output)
    cols = x.shape[-1]
    rows = x.numel() // cols
    pre = pre_scale.half().contiguous() if pre_scale is not None else None
    post = post_scale.half().contiguous() if post_scale is not None else None
    rc = L.lib().exl3_had_r_128(x.data_ptr(), out.data_ptr(), L.dtype_code(x.dtype), rows, cols, L.ptr(pre),
                                L.ptr(post), float(scale), L.stream_of(x))
    L.check(rc, "had_r_128")
    if out is not output:
        output.copy_(out)


class BC_LinearEXL3:
    """EXL3 linear y = Had(Had(x * suh) @ W_hat) * svh (glm/xpu/glm_xpu/ops.py:34-88; exllamav3 contract
    glm/docs/ext-op-inventory.md:471-496). Other modules read trellis/suh/svh/K/mcg/mul1 by name.

    run(x, y): x fp16/bf16 [..., k] -> y (fp16/bf16/fp32, preallocated) [..., n].
      rows <= SMALL_M_MAX: the fused decode GEMV, up to 16 rows per launch (weights streamed and decoded once per
      launch, each decoded fragment feeding one MMA per 8 rows);
      larger: the tcgen05 linear (exl3_gemm_tc: trellis decoded into tensor memory, 2-SM MMAs, weights decoded once
      per 320 rows), in place of the reference's dequantise + library GEMM prefill path
      (glm/xpu/csrc/exl3_ops.sycl:651-757)."""

    def __init__(self, trellis, suh, svh, K, bias, mcg, mul1, xh):
        if mcg or not mul1:
            raise L.Exl3Error("BC_LinearEXL3: only the mul1 codebook is supported")
        if float(K) != int(K) or not 1 <= int(K) <= 8:
            raise L.Exl3Error(f"BC_LinearEXL3: K={K} (integer 1..8 supported)")
        self.trellis = trellis
        self.suh = suh
        self.svh = svh
        self.K = K
        self.bias = bias
        self.mcg = mcg
        self.mul1 = mul1
        self.xh = xh
        self.Ki = int(K)
        self.in_features = trellis.shape[0] * 16
        self.out_features = trellis.shape[1] * 16
        if trellis.shape[2] != 16 * self.Ki:
            raise L.Exl3Error(f"BC_LinearEXL3: trellis {tuple(trellis.shape)} does not match K={K}")
        # the decode GEMV reads a column-block-major copy of the trellis (packed once, on first use)
        self._packed = None
        _LINEARS[trellis.data_ptr()] = self          # exl3_mgemm resolves trellis addresses to linears

    def packed(self) -> torch.Tensor:
        if self._packed is None or self._packed.device != self.trellis.device:
            self._packed = pack(self.trellis, self.Ki)
        return self._packed

    def run(self, x: torch.Tensor, y: torch.Tensor) -> None:
        x2 = _f16(x.reshape(-1, self.in_features))
        y2 = y.view(-1, self.out_features)
        M = x2.shape[0]
        if M == 0:
            return
        if M <= SMALL_M_MAX:
            pk = self.packed()
            for m0 in range(0, M, GEMV_MAX_ROWS):
                exl3_gemv(x2[m0:m0 + GEMV_MAX_ROWS], pk, self.suh, self.svh, self.Ki, y2[m0:m0 + GEMV_MAX_ROWS])
        else:
            suh = self.suh if self.suh is None or self.suh.data_ptr() % 8 == 0 else self.suh.clone()
            svh = self.svh if self.svh.data_ptr() % 8 == 0 else self.svh.clone()
            if y2.stride(-1) != 1 or y2.stride(0) % 4 or y2.data_ptr() % 16:
                tmp = torch.empty((M, self.out_features), dtype=y2.dtype, device=y2.device)
                exl3_gemm_tc(x2, self.packed(), suh, svh, self.Ki, tmp)
                y2.copy_(tmp)
            else:
                exl3_gemm_tc(x2, self.packed(), suh, svh, self.Ki, y2)
        if self.bias is not None:
            y2.add_(self.bias)

    def run_alloc(self, x: torch.Tensor, out_features: int, output_fp32: bool) -> torch.Tensor:
        y = torch.empty(x.shape[:-1] + (out_features,), dtype=torch.float if output_fp32 else torch.half,
                        device=x.device)
        if out_features == 0:
            return y
        self.run(x.reshape(-1, x.shape[-1]), y.view(-1, out_features))
        return y


# trellis device address -> the BC_LinearEXL3 that owns it (weak: the registry does not keep linears alive)
_LINEARS: "weakref.WeakValueDictionary[int, BC_LinearEXL3]" = weakref.WeakValueDictionary()
_MG_TABLES: dict = {}


def register_linear(trellis: torch.Tensor, suh: torch.Tensor | None, svh: torch.Tensor, K) -> "BC_LinearEXL3":
    """A BC_LinearEXL3 for tensors created outside one (exl3_mgemm finds matrices by trellis address); keep the
    returned object alive while its address may appear in a pointer table."""
    return BC_LinearEXL3(trellis, suh, svh, K, None, False, True, None)


def _mg_tables(B: torch.Tensor):
    """Packed-trellis address table and bit widths for a table of trellis addresses (cached per table: exllamav3
    builds its pointer tables once; the first call reads the table to the host)."""
    key = (B.data_ptr(), B.numel(), B.device)
    hit = _MG_TABLES.get(key)
    if hit is not None and all(r() is not None for r in hit[2]):
        return hit[0], hit[1]
    addrs = [int(a) for a in B.reshape(-1).tolist()]
    lins = []
    for a in addrs:
        lin = _LINEARS.get(a)
        if lin is None:
            raise L.Exl3Error(f"exl3_mgemm: trellis at 0x{a:x} belongs to no BC_LinearEXL3 (create one, or call "
                              f"register_linear)")
        lins.append(lin)
    packed = torch.tensor([lin.packed().data_ptr() for lin in lins], dtype=torch.int64, device=B.device)
    ks = torch.tensor([lin.Ki for lin in lins], dtype=torch.int32, device=B.device)
    _MG_TABLES[key] = (packed, ks, [weakref.ref(lin) for lin in lins], [lin.packed() for lin in lins])
    return packed, ks


def exl3_mgemm(A, B, C, suh, A_had, svh, indices=None, weights=None, K=None, force_shape_idx=-1, mcg=False,
               mul1=True, min_index=-1, max_index=-1, force_num_sms=0, num_tokens=1, size_n_list=None, c_ptrs=None,
               n_stride_list=None, had_src_list=None, num_had_src=0) -> int:
    """exllamav3 exl3_mgemm(A, B, C, suh, A_had, svh, indices, weights, K, ...) (glm/docs/ext-op-inventory.md:664-688,
    1104-1120) on the C ABI exl3_mgemm: B / suh / svh are int64 device tables of trellis / suh / svh addresses (the
    trellis tensors of BC_LinearEXL3 objects); A fp16/bf16 [a_batches, m, k]; C fp16/bf16/fp32 [c_batches, m, n].
    Slot j: C[j] = lin(A[j or 0], B[indices[j] or j]); with weights, C[t] = sum of token t's weighted slots.
    A_had is not needed (the rotated rows live in the library's workspace). Returns 0."""
    if size_n_list is not None or c_ptrs is not None or n_stride_list is not None or had_src_list is not None:
        raise L.Exl3Error("exl3_mgemm: the sliced mode is not supported")
    if mcg or not mul1:
        raise L.Exl3Error("exl3_mgemm: only the mul1 codebook is supported")
    L.require_cuda(A, B, C, svh)
    A3 = A if A.dim() == 3 else A.reshape(1, *A.shape)
    A3 = _f16(A3)
    a_batches, m, k = A3.shape
    n = C.shape[-1]
    packed, ks = _mg_tables(B)
    n_mats = packed.numel()
    idx = None if indices is None else indices.reshape(-1).to(torch.int32).contiguous()
    slots = n_mats if idx is None else idx.numel()
    w = None if weights is None else weights.reshape(-1).to(torch.float32).contiguous()
    C3 = C.reshape(-1, m, n)
    if C3.stride(-1) != 1 or C3.stride(1) != n or C3.stride(0) != m * n:
        raise L.Exl3Error("exl3_mgemm: C must be contiguous")
    lib = L.lib()
    need = lib.exl3_mgemm_workspace_size(slots, m, k, n, n_mats)
    ws = L.workspace(A3.device, need, "mgemm")
    rc = lib.exl3_mgemm(A3.data_ptr(), L.dtype_code(A3.dtype), a_batches, k, m, k, n, packed.data_ptr(),
                        L.ptr(suh), svh.data_ptr(), ks.data_ptr(), n_mats, L.ptr(idx), slots, L.ptr(w),
                        int(num_tokens), int(min_index), int(max_index), C3.data_ptr(), L.dtype_code(C3.dtype), n,
                        ws.data_ptr(), ws.numel(), L.stream_of(A3))
    L.check(rc, "exl3_mgemm")
    return 0


def exl3_gemm(A, B, C, suh, A_had, svh, force_shape_idx=-1, mcg=False, mul1=True, force_num_sms=0) -> int:
    """exllamav3 exl3_gemm(A, B, C, suh, A_had, svh, ...) (glm/docs/ext-op-inventory.md:498-557): C = lin(A)."""
    K = B.shape[2] // 16
    BC_LinearEXL3(B, suh, svh, K, None, mcg, mul1, A_had).run(A, C)
    return 0


# ----------------------------------------------------------------------------------------------- activation / MLP

def silu_mul(x: torch.Tensor, y: torch.Tensor, z: torch.Tensor, act_limit: float) -> None:
    """z = min(silu(x), L) * clamp(y, -L, L) (L = act_limit, 0 disables), fp32 math, stored to z (fp16)
    (glm/xpu/glm_xpu/ops.py:147-154)."""
    L.require_cuda(x, y, z)
    g = x.half().contiguous()
    u = y.half().contiguous()
    zz = z if (z.dtype == torch.float16 and z.is_contiguous()) else torch.empty_like(g)
    rc = L.lib().exl3_silu_mul(g.data_ptr(), u.data_ptr(), zz.data_ptr(), g.numel(), float(act_limit or 0.0),
                               L.stream_of(g))
    L.check(rc, "silu_mul")
    if zz is not z:
        z.copy_(zz.view(z.shape))


class BC_GatedMLP:
    """Dense / shared-expert gated MLP for rows <= 8: g, u = gate(x), up(x); a = silu_mul(g, u); d = down(a)
    (glm/xpu/glm_xpu/ops.py:157-172)."""

    def __init__(self, guh, gu, a, down_xh, gu_ptrs_trellis, gu_ptrs_suh, gu_ptrs_svh, gu_K, gu_mcg, gu_mul1,
                 act_silu, act_gelu, act_relu2, gate, up, down, act_limit):
        if gate is None or up is None:
            raise L.Exl3Error("BC_GatedMLP: fused gate/up pointer tables are not supported; pass gate and up")
        if not act_silu:
            raise L.Exl3Error("BC_GatedMLP: only SiLU gated MLPs")
        self.gate, self.up, self.down = gate, up, down
        self.act_limit = act_limit

    def run_bszN(self, x: torch.Tensor, d: torch.Tensor) -> None:
        x2 = x.reshape(-1, x.shape[-1])
        g = self.gate.run_alloc(x2, self.gate.out_features, False)
        u = self.up.run_alloc(x2, self.up.out_features, False)
        silu_mul(g, u, u, self.act_limit)
        self.down.run(u, d.view(-1, d.shape[-1]))


# ----------------------------------------------------------------------------------------------- routing

def route(logits: torch.Tensor, kind: int, k: int, bias=None, res=None, mul=None, scale: float = 1.0,
          renorm: bool = True, want: bool = False, ids_dtype=torch.int32):
    """Top-k routing with residency bias on fp32 logits [R, E] -> (ids [R, k], w fp32 [R, k], want or None).
    See exl3_route in include/exl3_b200.h for the exact math."""
    L.require_cuda(logits)
    lg = logits.float().contiguous()
    R, E = lg.shape
    dev = lg.device
    ids = torch.empty((R, k), dtype=ids_dtype, device=dev)
    w = torch.empty((R, k), dtype=torch.float32, device=dev)
    wt = torch.empty((R, k), dtype=ids_dtype, device=dev) if want else None
    b = bias.float().contiguous() if bias is not None else None
    r = res.float().contiguous() if res is not None else None
    m = mul.float().contiguous() if mul is not None else None
    rc = L.lib().exl3_route(lg.data_ptr(), lg.stride(0), R, E, int(kind), int(k), L.ptr(b), L.ptr(r), L.ptr(m),
                            float(scale), int(bool(renorm)), ids.data_ptr(), int(ids_dtype == torch.int64),
                            w.data_ptr(), L.ptr(wt), L.stream_of(lg))
    L.check(rc, "exl3_route")
    return ids, w, wt


ROUTE_HIDDEN_MAX_ROWS = 64


def router_logits(hidden: torch.Tensor, gate_t: torch.Tensor, logits_f16: torch.Tensor | None = None) -> torch.Tensor:
    """logits fp32 [R, E] = fp16(hidden [R, H] @ gate_t [E, H]^T) on the tensor cores (C ABI exl3_router_logits),
    any R; logits_f16 (optional, fp16 [R, E]) receives the same values in fp16."""
    L.require_cuda(hidden, gate_t)
    h = _f16(hidden.reshape(-1, hidden.shape[-1]))
    if h.data_ptr() % 16 or h.stride(0) % 8:
        h = h.clone()
    R, H = h.shape
    g = gate_t.half().contiguous()
    E = g.shape[0]
    out = torch.empty((R, E), dtype=torch.float32, device=h.device)
    lo = logits_f16
    if lo is not None and (lo.dtype != torch.float16 or not lo.is_contiguous() or lo.numel() != R * E):
        raise L.Exl3Error("router_logits: logits_f16 must be a contiguous fp16 [R, E] tensor")
    rc = L.lib().exl3_router_logits(h.data_ptr(), L.dtype_code(h.dtype), h.stride(0), R, H, g.data_ptr(), E,
                                    out.data_ptr(), L.ptr(lo), L.stream_of(h))
    L.check(rc, "exl3_router_logits")
    return out


def route_hidden(hidden: torch.Tensor, gate_t: torch.Tensor, kind: int, k: int, bias=None, res=None, mul=None,
                 scale: float = 1.0, renorm: bool = True, want: bool = False, ids_dtype=torch.int32,
                 logits_out: torch.Tensor | None = None, next_router: dict | None = None):
    """Top-k routing from hidden states [R, H] fp16/bf16 and the router weight transposed gate_t fp16 [E, H]:
    logits = fp16(hidden @ gate_t^T) then `route`. Up to ROUTE_HIDDEN_MAX_ROWS rows: one fused launch (C ABI
    exl3_route_hidden); more rows: the tensor-core router GEMM (exl3_router_logits), then exl3_route. logits_out
    (optional, fp16 [R, E]) receives the logits. Returns (ids, w, want or None).

    next_router: the next layer's router for the layer-ahead prediction, dict(gate_t fp16 [E1, H], kind, k, and
    optionally bias, mul, scale, renorm): its logits come from the same GEMV and its picks from the same launch (C ABI
    exl3_route_hidden_pair); the return value is then (ids, w, want, ids_next, w_next)."""
    L.require_cuda(hidden, gate_t)
    h = _f16(hidden.reshape(-1, hidden.shape[-1]))
    R, H = h.shape
    E = gate_t.shape[0]
    g = gate_t.half().contiguous()
    f32 = lambda t: t.float().contiguous() if t is not None else None     # noqa: E731
    if R > ROUTE_HIDDEN_MAX_ROWS:
        logits = router_logits(h, g, logits_out)
        res_ = route(logits, kind, k, bias, res, mul, scale, renorm, want, ids_dtype)
        if next_router is None:
            return res_
        nr = next_router
        lg1 = router_logits(h, nr["gate_t"])
        ids1, w1, _ = route(lg1, nr["kind"], nr["k"], nr.get("bias"), None, nr.get("mul"), nr.get("scale", 1.0),
                            nr.get("renorm", True), False, ids_dtype)
        return (*res_, ids1, w1)
    dev = h.device
    ids = torch.empty((R, k), dtype=ids_dtype, device=dev)
    w = torch.empty((R, k), dtype=torch.float32, device=dev)
    wt = torch.empty((R, k), dtype=ids_dtype, device=dev) if want else None
    b, r, m = f32(bias), f32(res), f32(mul)
    lo = logits_out
    if lo is not None and (lo.dtype != torch.float16 or not lo.is_contiguous() or lo.numel() != R * E):
        raise L.Exl3Error("route_hidden: logits_out must be a contiguous fp16 [R, E] tensor")
    lib = L.lib()
    i64 = int(ids_dtype == torch.int64)
    if next_router is None:
        ws = L.zeroed_workspace(dev, lib.exl3_route_hidden_workspace_size(R, E), "route_hidden")
        rc = lib.exl3_route_hidden(h.data_ptr(), L.dtype_code(h.dtype), h.stride(0), R, H, g.data_ptr(), E, int(kind),
                                   int(k), L.ptr(b), L.ptr(r), L.ptr(m), float(scale), int(bool(renorm)),
                                   ids.data_ptr(), i64, w.data_ptr(), L.ptr(wt), L.ptr(lo), ws.data_ptr(), ws.numel(),
                                   L.stream_of(h))
        L.check(rc, "exl3_route_hidden")
        return ids, w, wt
    nr = next_router
    g1 = nr["gate_t"].half().contiguous()
    E1, k1 = g1.shape[0], int(nr["k"])
    ids1 = torch.empty((R, k1), dtype=ids_dtype, device=dev)
    w1 = torch.empty((R, k1), dtype=torch.float32, device=dev)
    b1, m1 = f32(nr.get("bias")), f32(nr.get("mul"))
    ws = L.zeroed_workspace(dev, lib.exl3_route_hidden_workspace_size(R, E + E1), "route_hidden")
    rc = lib.exl3_route_hidden_pair(h.data_ptr(), L.dtype_code(h.dtype), h.stride(0), R, H, g.data_ptr(), E,
                                    int(kind), int(k), L.ptr(b), L.ptr(r), L.ptr(m), float(scale), int(bool(renorm)),
                                    ids.data_ptr(), i64, w.data_ptr(), L.ptr(wt), L.ptr(lo), g1.data_ptr(), E1,
                                    int(nr["kind"]), k1, L.ptr(b1), L.ptr(m1), float(nr.get("scale", 1.0)),
                                    int(bool(nr.get("renorm", True))), ids1.data_ptr(), i64, w1.data_ptr(),
                                    ws.data_ptr(), ws.numel(), L.stream_of(h))
    L.check(rc, "exl3_route_hidden_pair")
    return ids, w, wt, ids1, w1


def routing_ds3_nogroup(hidden, gate, scores, bias, topk_indices, topk_weights, scaling_factor, gate_t, act_fn,
                        gate_i8, gate_sb, res=None):
    """Sigmoid / noaux_tc top-k routing (glm/xpu/glm_xpu/ops.py:177-193): logits = hidden @ gate rounded to fp16
    (written to scores; the routing GEMV runs in the router's launch, `route_hidden`); selection by sigmoid + bias (+ residency bias `res`, glm/xpu/glm_xpu/block_graphs.py:
    164-167); weights from the unbiased sigmoid, normalised over the picks and scaled. Writes scores, topk_indices,
    topk_weights in place."""
    if act_fn != 0:
        raise L.Exl3Error("routing_ds3_nogroup: sigmoid routing only (act_fn 0)")
    E = scores.shape[-1]
    k = topk_indices.shape[-1]
    gt = gate_t[:E] if gate_t is not None else gate[:, :E].t()
    lo = torch.empty(scores.shape, dtype=torch.float16, device=scores.device)
    ids, w, _ = route_hidden(hidden, gt, L.ROUTE_SIGMOID, k, bias=bias, res=res, scale=scaling_factor,
                             ids_dtype=torch.int64 if topk_indices.dtype == torch.int64 else torch.int32,
                             logits_out=lo)
    scores.copy_(lo)
    topk_indices.copy_(ids)
    topk_weights.copy_(w)


def det_quant_weight(w, w_i8, w_s) -> None:
    """No-op: only feeds exllamav3's deterministic routing GEMM, which this path does not use
    (glm/xpu/glm_xpu/ops.py:196-197)."""
    return None
