"""CPU oracle for the EXL3 trellis path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's algorithms for the hot path: trellis decode (mul1 codebook),
the blockwise 128-point Hadamard rotations, the EXL3 linear, the three routers with their residency (locality)
bias, token/expert alignment, and the MoE expert math. It exists so that tests, `__graft_entry__.smoke()` and the
`cpu_baseline` leg of `bench.py` can CHECK the CUDA path; the product never imports it.

Parity pinning: the restatement is checked against golden vectors produced by running the reference's own Python
code in the build container (`tests/golden/make_golden.py`, which imports `glm/xpu/tests/units.py` helpers and
`glm_xpu.ops` from the reference tree) and against the known answers the reference states (mul1 constants
0x1EEE / 0xC931, codebook range, expert blob sizes). exllamav3's CUDA kernels are not in the reference mount, so
parity at that boundary rests on the reference's torch restatements (see the golden script).

Reference files cited below are paths inside horvay/b70-inference.
"""
from __future__ import annotations

import math

import numpy as np

# ------------------------------------------------------------------------------------------------ codebook

MUL1 = 0x83DCD12D                     # glm/xpu/tests/units.py:42
K_INV = 0.00676727294921875           # fp16 0x1EEE, dsv41/xpu/dsv_xpu/exl3_tri.py:18,218
K_BIAS = -10.3828125                  # fp16 0xC931, dsv41/xpu/dsv_xpu/exl3_tri.py:19,218
RSQRT128 = 0.08838834764831845        # glm/xpu/csrc/exl3_esimd.h:223

_LUT = None


def mul1_lut() -> np.ndarray:
    """fp16[65536]: 16-bit trellis state -> weight (glm/xpu/tests/units.py:45-52; spec
    glm/docs/ext-op-inventory.md:559-574). x = st*MUL1 mod 2^32; h = 1024 + sum of x's bytes;
    w = fp16(h*K_INV + K_BIAS): exact in fp64/fp32, one rounding to fp16."""
    global _LUT
    if _LUT is None:
        st = np.arange(65536, dtype=np.uint64)
        x = (st * MUL1) & 0xFFFFFFFF
        s = (x & 255) + ((x >> 8) & 255) + ((x >> 16) & 255) + ((x >> 24) & 255)
        _LUT = ((1024.0 + s.astype(np.float64)) * K_INV + K_BIAS).astype(np.float16)
        _LUT.flags.writeable = False
    return _LUT


def decode_mul1_state(st):
    """Same codebook for an array of states (no table), used by known-answer tests."""
    st = np.asarray(st, dtype=np.uint64) & 0xFFFF
    x = (st * MUL1) & 0xFFFFFFFF
    s = (x & 255) + ((x >> 8) & 255) + ((x >> 16) & 255) + ((x >> 24) & 255)
    return ((1024.0 + s.astype(np.float64)) * K_INV + K_BIAS).astype(np.float16)


# ------------------------------------------------------------------------------------------------ tile format

def tile_tables(K: int):
    """Per ring position t (0..255) of a 16x16 tile: the two uint32 words holding its 16-bit window, the right
    shift, and the (row, col) it lands on (glm/xpu/tests/units.py:55-68; layout glm/docs/ext-op-inventory.md:
    698-733; glm/xpu/csrc/exl3_esimd.h:4-8). Window of t = stream bits [(t+1)K-16, (t+1)K), MSB-first, circular
    in the tile's 256K-bit ring; row (input dim) = 8((t>>1)&1) + 2((t>>3)&3) + (t&1), col = (t>>5) + 8((t>>2)&1)."""
    t = np.arange(256, dtype=np.int64)
    e = (t + 1) * K
    ih = (e - 1) // 32
    sh = 32 * (ih + 1) - e
    il = (ih - 1) % (8 * K)
    row = 8 * ((t >> 1) & 1) + 2 * ((t >> 3) & 3) + (t & 1)
    col = (t >> 5) + 8 * ((t >> 2) & 1)
    return il, ih, sh, row, col


def trellis_words(trellis: np.ndarray) -> np.ndarray:
    """int16/uint16 trellis [tk, tn, 16K] -> uint32 words [tk, tn, 8K] (little-endian pairs, as every kernel loads
    them: word[i] = u16[2i] | u16[2i+1] << 16)."""
    tr = np.ascontiguousarray(trellis)
    return tr.view(np.uint32)


def tile_states(trellis: np.ndarray, K: int) -> np.ndarray:
    """uint16 states [tk, tn, 256] in ring-position order: state(t) = ((word[il] << 32 | word[ih]) >> sh) & 0xFFFF,
    evaluated position by position on whole [tk, tn] word planes in uint32 arithmetic (the high word contributes
    word[il] << (32 - sh) when sh > 0 and nothing when sh == 0)."""
    words = trellis_words(trellis)
    il, ih, sh, _, _ = tile_tables(K)
    tk, tn, _ = words.shape
    st = np.empty((tk, tn, 256), dtype=np.uint16)
    for t in range(256):
        s_ = int(sh[t])
        v = words[..., ih[t]] >> np.uint32(s_)
        if s_ > 0:
            v = v | (words[..., il[t]] << np.uint32(32 - s_))
        st[..., t] = (v & np.uint32(0xFFFF)).astype(np.uint16)
    return st


def w_hat(trellis: np.ndarray, K: int) -> np.ndarray:
    """Decoded Hadamard-domain weights fp16 [k, n] (glm/xpu/tests/units.py:55-68 == exllamav3 reconstruct,
    glm/docs/ext-op-inventory.md:597-612)."""
    tk, tn, w16 = trellis.shape
    assert w16 == 16 * K, (trellis.shape, K)
    st = tile_states(trellis, K)
    _, _, _, row, col = tile_tables(K)
    tiles = np.empty((tk, tn, 16, 16), dtype=np.float16)
    tiles[:, :, row, col] = mul1_lut()[st]
    return tiles.transpose(0, 2, 1, 3).reshape(tk * 16, tn * 16)


def w_hat_cols(trellis: np.ndarray, K: int, n0: int, n1: int) -> np.ndarray:
    """Column slice [:, n0:n1] of w_hat (== exllamav3 reconstruct_slice / exl3_reconstruct with n0,
    glm/xpu/csrc/exl3_ops.sycl:539-555)."""
    assert n0 % 16 == 0 and n1 % 16 == 0
    return w_hat(np.ascontiguousarray(trellis[:, n0 // 16:n1 // 16]), K)


# ------------------------------------------------------------------------------------------------ Hadamard

def sylvester128() -> np.ndarray:
    """Natural-order Sylvester H128 (unnormalised), H[i,j] = (-1)^popcount(i&j) (glm/xpu/tests/units.py:71-75)."""
    h = np.ones((1, 1))
    while h.shape[0] < 128:
        h = np.block([[h, h], [h, -h]])
    return h


def fwht128_f32(v: np.ndarray) -> np.ndarray:
    """Unnormalised FWHT over the last axis (length 128) in fp32, stages h = 1, 2, ..., 64 in order, each stage
    (a, b) -> (a + b, a - b) — the butterfly order of glm/xpu/csrc/exl3_esimd.h:210-221 and of exllamav3's
    had_r_128 (4 values per lane then xor shuffles, glm/docs/ext-op-inventory.md:576-595). fp32 adds round
    identically whatever hardware does them, so this is bit-exact with any kernel using the same stage order."""
    v = np.array(v, dtype=np.float32)
    shp = v.shape
    v = v.reshape(-1, 128)
    h = 1
    while h < 128:
        u = v.reshape(-1, 128 // (2 * h), 2, h)
        a = u[:, :, 0, :].copy()
        b = u[:, :, 1, :].copy()
        u[:, :, 0, :] = a + b
        u[:, :, 1, :] = a - b
        v = u.reshape(-1, 128)
        h *= 2
    return v.reshape(shp)


def had_in(x: np.ndarray, suh: np.ndarray) -> np.ndarray:
    """Input rotation, exllamav3 roundings (glm/docs/ext-op-inventory.md:515-529, exl3_esimd.h:283-315):
    xh = fp16( FWHT_fp32( fp16(x * suh) ) * (1/sqrt(128)) ) per 128-block of the last axis."""
    v = (x.astype(np.float32) * suh.astype(np.float32)).astype(np.float16)     # fp16 product (exact then RNE)
    y = fwht128_f32(v.astype(np.float32).reshape(-1, 128)) * np.float32(RSQRT128)
    return y.astype(np.float16).reshape(x.shape)


def had_out(acc: np.ndarray, svh: np.ndarray, out_dtype) -> np.ndarray:
    """Output rotation of the fp32 accumulator (glm/docs/ext-op-inventory.md:524-529; exl3_esimd.h:318-338):
    fp32 out: FWHT(acc) * r * svh (fp32); fp16 out: fp16(FWHT(acc) * r) * svh (fp16 multiply)."""
    y = fwht128_f32(acc.astype(np.float32).reshape(-1, 128)).reshape(acc.shape) * np.float32(RSQRT128)
    if out_dtype == np.float32:
        return (y * svh.astype(np.float32)).astype(np.float32)
    return (y.astype(np.float16).astype(np.float32) * svh.astype(np.float32)).astype(np.float16)


def had_r_128(x: np.ndarray, pre=None, post=None, scale: float = 1.0) -> np.ndarray:
    """exllamav3 had_r_128 semantics (glm/xpu/glm_xpu/ops.py:132-142): pre_scale wins over post_scale; fp16 in/out:
    pre multiply in fp16, butterfly fp32, *scale/sqrt(128) fp32, round, post multiply in fp16."""
    v = x
    if pre is not None:
        v = (v.astype(np.float32) * pre.astype(np.float32)).astype(x.dtype)
    y = fwht128_f32(v.astype(np.float32).reshape(-1, 128)).reshape(x.shape) * np.float32(scale * RSQRT128)
    y = y.astype(x.dtype)
    if pre is None and post is not None:
        y = (y.astype(np.float32) * post.astype(np.float32)).astype(x.dtype)
    return y


# ------------------------------------------------------------------------------------------------ linear

def linear_acc(xh: np.ndarray, trellis: np.ndarray, K: int) -> np.ndarray:
    """acc = xh @ W_hat, fp64-accumulated then rounded to fp32 (the 'fp32-accumulated reference')."""
    W = w_hat(trellis, K).astype(np.float64)
    return (xh.astype(np.float64) @ W).astype(np.float32)


def exl3_linear(x: np.ndarray, trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray, K: int,
                out_dtype=np.float16) -> np.ndarray:
    """EXL3 linear y = Had(Had(x*suh) @ W_hat) * svh with exllamav3's rounding points
    (exl3_linear_ref, glm/docs/ext-op-inventory.md:735-774; math :512-529)."""
    x2 = x.reshape(-1, x.shape[-1])
    xh = had_in(x2, suh)
    acc = linear_acc(xh, trellis, K)
    return had_out(acc, svh, out_dtype).reshape(*x.shape[:-1], -1)


def ref_linear_f64(x, trellis, suh, svh, K) -> np.ndarray:
    """fp64 linear with no intermediate rounding (glm/xpu/tests/units.py:78-85)."""
    H = sylvester128() / math.sqrt(128)
    x2 = x.reshape(-1, x.shape[-1]).astype(np.float64)
    xh = (x2 * suh.astype(np.float64)).reshape(-1, 128) @ H
    acc = xh.reshape(x2.shape[0], -1) @ w_hat(trellis, K).astype(np.float64)
    return ((acc.reshape(-1, 128) @ H).reshape(acc.shape) * svh.astype(np.float64)).reshape(*x.shape[:-1], -1)


# ------------------------------------------------------------------------------------------------ activation

def silu_mul(g: np.ndarray, u: np.ndarray, act_limit: float) -> np.ndarray:
    """a = fp16( min(silu(g), L) * clamp(u, -L, L) ), fp32 math; L = 0 disables the clamps
    (glm/xpu/glm_xpu/ops.py:147-154; clamp after SiLU per glm/xpu/csrc/exl3_moe.n128.sycl:37-44)."""
    g32 = g.astype(np.float32)
    with np.errstate(over="ignore"):
        s = (g32 / (np.float32(1.0) + np.exp(-g32))).astype(np.float32)
    v = u.astype(np.float32)
    if act_limit:
        L = np.float32(act_limit)
        s = np.minimum(s, L)
        v = np.clip(v, -L, L)
    return (s * v).astype(np.float16)


# ------------------------------------------------------------------------------------------------ routers

ROUTE_SIGMOID, ROUTE_SOFTMAX, ROUTE_SQRT_SOFTPLUS = 0, 1, 2


def route_scores(logits: np.ndarray, kind: int) -> np.ndarray:
    """Per-expert score that enters the selection key, fp32. sigmoid (routing_ds3_nogroup,
    glm/xpu/glm_xpu/ops.py:186-189) and sqrt(softplus) with the l > 20 shortcut
    (dsv41/xpu/csrc/dsv_moe_glue.sycl:163-164; dsv41/xpu/dsv_xpu/moe.py:955) are evaluated in fp64 and rounded
    once to fp32, so kernel and oracle agree bit-for-bit; softmax routing ranks on the raw logit
    (trellis-serve.patch:401-411)."""
    l = logits.astype(np.float32)
    if kind == ROUTE_SIGMOID:
        d = l.astype(np.float64)
        with np.errstate(over="ignore"):
            return (1.0 / (1.0 + np.exp(-d))).astype(np.float32)
    if kind == ROUTE_SQRT_SOFTPLUS:
        d = l.astype(np.float64)
        with np.errstate(over="ignore"):
            sp = np.where(d > 20.0, d, np.log1p(np.exp(np.minimum(d, 20.0))))
        return np.sqrt(sp).astype(np.float32)
    if kind == ROUTE_SOFTMAX:
        return l.copy()
    raise ValueError(kind)


def softmax_probs(logits: np.ndarray) -> np.ndarray:
    """softmax over experts in fp64, rounded to fp32 (trellis-serve.patch:399-401)."""
    d = logits.astype(np.float64)
    d = d - d.max(axis=-1, keepdims=True)
    e = np.exp(d)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def topk_lowest_tie(key: np.ndarray, k: int) -> np.ndarray:
    """k argmax passes, ties to the lowest index (dsv41/xpu/csrc/dsv_moe_glue.sycl:170-180). Output slot j holds
    the j-th best expert (descending key). -inf keys are never preferred over finite ones."""
    R, E = key.shape
    order = np.lexsort((np.broadcast_to(np.arange(E), key.shape), -key.astype(np.float64)), axis=-1)
    return order[:, :k].astype(np.int32)


def route(logits: np.ndarray, kind: int, k: int, bias=None, res=None, mul=None, scale: float = 1.0,
          renorm: bool = True, want: bool = False):
    """Top-k routing with a residency (locality) bias.

    key[e] = score[e] * mul[e] + bias[e] + res[e] (fp32, each term optional), where
      * bias is e_score_correction_bias (sigmoid, glm/xpu/glm_xpu/ops.py:188), the DSV gate bias
        (dsv41/xpu/dsv_xpu/moe.py:957-961) or the Qwen-Next cold-tier bias (trellis-serve.patch:404-406);
      * res is the residency bias: 0 resident, -margin for a slower tier, -inf not readable
        (glm/xpu/glm_xpu/block_graphs.py:164-167; dsv41/xpu/csrc/dsv_moe_glue.sycl:168-169), or +b for a resident
        subset; a uniform shift of res does not change the picks;
      * mul is the residency boost multiplier (dsv41/xpu/csrc/dsv_moe_glue.sycl:167).
    Weights come from the unbiased score: sigmoid / sqrt-softplus: w = s[sel] * scale / (sum + 1e-20);
    softmax: w = p[sel] / (sum + 1e-20) when renorm, else p[sel] (trellis-serve.patch:412-415).
    The sum runs over the k picks in slot order, in fp32. want = top-k of score*1 + bias (no res, no mul)."""
    s = route_scores(logits, kind)
    key = s.copy()
    if mul is not None:
        key = (key * mul.astype(np.float32)).astype(np.float32)
    if bias is not None:
        key = (key + bias.astype(np.float32)).astype(np.float32)
    if res is not None:
        key = (key + res.astype(np.float32)).astype(np.float32)
    ids = topk_lowest_tie(key, k)
    if kind == ROUTE_SOFTMAX:
        p = softmax_probs(logits)
        w = np.take_along_axis(p, ids.astype(np.int64), axis=-1).astype(np.float32)
        if renorm:
            tot = np.zeros(w.shape[0], dtype=np.float32)
            for j in range(k):
                tot = (tot + w[:, j]).astype(np.float32)
            w = (w / (tot + np.float32(1e-20))[:, None]).astype(np.float32)
    else:
        w = np.take_along_axis(s, ids.astype(np.int64), axis=-1).astype(np.float32)
        tot = np.zeros(w.shape[0], dtype=np.float32)
        for j in range(k):
            tot = (tot + w[:, j]).astype(np.float32)
        w = (w * np.float32(scale) / (tot + np.float32(1e-20))[:, None]).astype(np.float32)
    wanted = None
    if want:
        k0 = s if bias is None else (s + bias.astype(np.float32)).astype(np.float32)
        wanted = topk_lowest_tie(k0, k)
    return ids, w, wanted


# ------------------------------------------------------------------------------------------------ align

def moe_align(ids: np.ndarray, E: int):
    """Histogram of the (token, pick) pairs by expert (glm/xpu/csrc/exl3_moe.n128.sycl:693-734): active experts in
    ascending id order with their start/count, pairs sorted by expert (stable: ascending pair index within an
    expert), pair_tok[pos] = token of the pair at pos, pair_of[pair] = pos. Invalid ids (< 0 or >= E) are dropped
    (pair_of = -1)."""
    flat = ids.reshape(-1).astype(np.int64)
    topk = ids.shape[-1]
    valid = (flat >= 0) & (flat < E)
    order = np.argsort(np.where(valid, flat, E), kind="stable")
    nvalid = int(valid.sum())
    order = order[:nvalid]
    cnt = np.bincount(flat[valid], minlength=E)
    act = np.nonzero(cnt)[0].astype(np.int32)
    start = np.concatenate([[0], np.cumsum(cnt)])[:-1]
    pair_of = np.full(flat.shape[0], -1, dtype=np.int32)
    pair_of[order] = np.arange(nvalid, dtype=np.int32)
    return dict(act_expert=act, act_start=start[act].astype(np.int32), act_cnt=cnt[act].astype(np.int32),
                n_act=len(act), pair_tok=(order // topk).astype(np.int32), pair_src=order.astype(np.int32),
                pair_of=pair_of)


# ------------------------------------------------------------------------------------------------ MoE

class ExpertW:
    """One expert's three EXL3 linears (gate, up: H -> I; down: I -> H) with per-matrix K."""

    def __init__(self, gate, up, down):
        self.gate, self.up, self.down = gate, up, down       # each (trellis, suh, svh, K)


def expert_forward(x: np.ndarray, ex: ExpertW, act_limit: float) -> np.ndarray:
    """Expert math (glm/docs/ext-op-inventory.md:923-942; per-pick torch path dsv41/xpu/dsv_xpu/moe.py:967-994):
    g, u = lin(x, gate), lin(x, up) as fp16; a = fp16(min(silu(g), L) * clamp(u, +-L)); d = lin(a, down) fp32."""
    g = exl3_linear(x, *ex.gate, out_dtype=np.float16)
    u = exl3_linear(x, *ex.up, out_dtype=np.float16)
    a = silu_mul(g, u, act_limit)
    return exl3_linear(a, *ex.down, out_dtype=np.float32)


def moe_forward(x: np.ndarray, ids: np.ndarray, w: np.ndarray, experts: list, act_limit: float,
                shared: ExpertW | None = None) -> np.ndarray:
    """Routed MoE layer, fp32 output: out[m] = sum_k w[m,k] * expert_{ids[m,k]}(x[m]) in slot order k = 0..topk-1
    (fixed order, glm/xpu/csrc/exl3_moe.n128.sycl:387-410) + shared expert (glm/xpu/glm_xpu/moe_patch.py:88-89).
    Picks with id < 0 contribute nothing."""
    M, topk = ids.shape
    H = x.shape[-1]
    out = np.zeros((M, H), dtype=np.float32)
    cache = {}
    for m in range(M):
        for j in range(topk):
            e = int(ids[m, j])
            if e < 0:
                continue
            key = (m, e)
            if key not in cache:
                cache[key] = expert_forward(x[m:m + 1], experts[e], act_limit)[0]
            out[m] = (out[m] + np.float32(w[m, j]) * cache[key]).astype(np.float32)
    if shared is not None:
        out = (out + expert_forward(x, shared, act_limit)).astype(np.float32)
    return out


# ------------------------------------------------------------------------------------------------ blob packing

def blob_bytes(H: int, I: int, K: int) -> int:
    """Per-expert blob size of the reference's pointer-table MoE format (glm/xpu/csrc/exl3_moe.n128.sycl:56-68):
    gate|up trellis [H/16][2I/16][8K] u32 + down [I/16][H/16][8K] u32 + six fp16 sign vectors."""
    gu = (H // 16) * (2 * I // 16) * 8 * K * 4
    d = (I // 16) * (H // 16) * 8 * K * 4
    return gu + d + 2 * (2 * H + 2 * I + I + H)


# ------------------------------------------------------------------------------------------------ synthetic inputs

def random_trellis(rng: np.random.Generator, k: int, n: int, K: int) -> np.ndarray:
    """Uniform uint16 trellis [k/16, n/16, 16K] (uniform random packed bitstreams)."""
    return rng.integers(0, 65536, size=(k // 16, n // 16, 16 * K), dtype=np.uint16)


def random_signs(rng: np.random.Generator, n: int) -> np.ndarray:
    return np.where(rng.integers(0, 2, size=n) == 1, 1.0, -1.0).astype(np.float16)
