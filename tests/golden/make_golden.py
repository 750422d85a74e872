"""Generate the golden fixtures in this directory by running the REFERENCE's own Python code on CPU.

Run in a container where the reference tree is mounted (default /root/reference, or $B70_REFERENCE):

    python tests/golden/make_golden.py            # every fixture
    python tests/golden/make_golden.py softmax    # only route_softmax.npz
    python tests/golden/make_golden.py stores     # only the expert blob / piece store / checkpoint fixtures

What runs (all from horvay/b70-inference, unmodified, imported or exec'd from its files):
  * glm/xpu/tests/units.py:42-89  -- mul1_lut, w_hat, H128, ref_linear (the reference's own torch restatement of
    the EXL3 linear, fp64); the module body needs an XPU, so only that line range is exec'd;
  * glm/xpu/glm_xpu/ops.py        -- routing_ds3_nogroup (sigmoid router), silu_mul, had_r_128;
  * dsv41/xpu/dsv_xpu/moe.py      -- route() (sqrt-softplus router with the residency bias), its torch path;
  * trellis-serve.patch            -- fused_xpu.py's Triton `_router_kernel` / `router` (the Qwen-Next softmax router
    with the cold-tier bias and the RAM margin), cut out of the patch text and run on CPU under Triton's interpreter
    (TRITON_INTERPRET=1);
  * glm/xpu/exl3xpu/moe_offload.py -- pack_expert / planar4 (the GLM / Qwen-Next expert blob), cross-checked against
    the record permutation blob_perm of glm/xpu/pack_store.py;
  * dsv41/xpu/dsv_xpu/pack_store.py -- main(): the DeepSeek-V4 piece store written from a small EXL3 safetensors
    checkpoint (its module constants H, I set to the fixture's sizes).
The outputs are small .npz files with seeded inputs and the reference's outputs; tests compare the oracle and the
CUDA path against them. Nothing here runs at test time.
"""
from __future__ import annotations

import json
import os
import sys
import types

# the softmax router is a Triton kernel: run it with Triton's CPU interpreter (must be set before triton loads)
os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

REF = os.environ.get("B70_REFERENCE", "/root/reference")
HERE = os.path.dirname(os.path.abspath(__file__))


def load_units_slice():
    """exec glm/xpu/tests/units.py lines 42-89 (MUL1 .. ref_linear) in a fresh namespace."""
    path = os.path.join(REF, "glm/xpu/tests/units.py")
    lines = open(path).read().splitlines()
    src = "\n".join(lines[41:89])
    assert "def mul1_lut" in src and "def ref_linear" in src and "def w_hat" in src, "units.py layout changed"
    ns = {"torch": torch, "math": __import__("math")}
    exec(compile(src, path, "exec"), ns)
    return ns


def load_fused_router():
    """The reference's softmax router: trellis-serve.patch adds xpu/exl3xpu/fused_xpu.py as a new file; its
    `_router_kernel` (Triton) and `router` wrapper are cut out of the patch text (lines starting with '+') and exec'd
    with their own imports. Nothing of them is changed."""
    path = os.path.join(REF, "trellis-serve.patch")
    lines = open(path).read().splitlines()
    start = next(i for i, l in enumerate(lines) if l.startswith("+++ ") and l.endswith("xpu/exl3xpu/fused_xpu.py"))
    end = next(i for i in range(start + 1, len(lines)) if lines[i].startswith("diff --git"))
    src = "\n".join(l[1:] for l in lines[start + 1:end] if l.startswith("+"))
    i0 = src.index("@triton.jit\ndef _router_kernel")
    i1 = src.index("@triton.jit", i0 + 10)
    body = src[i0:i1]
    assert "def router(logits" in body and "tl.argmax" in body, "fused_xpu.py layout changed"
    ns = {}
    exec(compile("import os\nimport torch\nimport triton\nimport triton.language as tl\n" + body, path, "exec"), ns)
    return ns["router"]


def make_softmax():
    """route_softmax.npz: the reference's fused softmax router (Triton, CPU interpreter) on seeded logits, with and
    without the cold-tier bias / RAM margin, with and without renormalisation, on tie-heavy logits and on an expert
    count that is not a power of two."""
    router = load_fused_router()
    rng = np.random.default_rng(20261202)
    cases = {}
    # (R, E, k, renorm, bias?, margin?, quantised logits for ties?)
    specs = [("plain", 8, 512, 10, True, False, False, False),
             ("cold_margin", 8, 512, 10, True, True, True, False),
             ("cold_only", 4, 512, 10, True, True, False, False),
             ("norenorm", 4, 512, 10, False, True, True, False),
             ("ties", 6, 512, 10, True, True, True, True),
             ("e160", 4, 160, 8, True, True, True, False)]
    for name, R, E, k, renorm, has_cold, has_margin, ties in specs:
        lg = rng.standard_normal((R, E)).astype(np.float32)
        if ties:
            lg = (np.round(lg * 4) / 4).astype(np.float32)          # many equal logits
        cold = slot = margin = None
        if has_cold:
            cold = np.zeros(E, dtype=np.float32)
            cold[rng.random(E) < 0.15] = -1e4                       # NVMe-only experts
        if has_margin:
            slot = np.where(rng.random(E) < 0.6, np.arange(E), -1).astype(np.int32)   # -1: not in a VRAM slot
            margin = np.array([0.5], dtype=np.float32)
        w, ids = router(torch.from_numpy(lg), k, renorm,
                        cold=None if cold is None else torch.from_numpy(cold),
                        slot_of=None if slot is None else torch.from_numpy(slot),
                        margin=None if margin is None else torch.from_numpy(margin))
        d = {"logits": lg, "k": k, "renorm": int(renorm), "ids": ids.numpy(), "w": w.numpy()}
        if cold is not None:
            d["cold"] = cold
        if slot is not None:
            d["slot_of"] = slot
            d["margin"] = margin
        for kk, v in d.items():
            cases[f"{name}__{kk}"] = np.asarray(v)
    np.savez_compressed(os.path.join(HERE, "route_softmax.npz"), **cases)


def make_stores():
    """expert_blob.npz: experts (H 256, I 128; K 3, 4, 5) and their blobs by the reference's pack_expert, which must
    agree with its record permutation blob_perm. dsv_store/: an EXL3 checkpoint of two MoE layers x 4 experts (K 1-3
    per projection, DeepSeek-V4 key names) and the piece store the reference's pack_store.main writes from it."""
    import importlib
    import shutil
    import tempfile
    from safetensors.torch import save_file
    sys.path.insert(0, os.path.join(REF, "glm/xpu"))
    mo = importlib.import_module("exl3xpu.moe_offload")
    ps = importlib.import_module("pack_store")
    rng = np.random.default_rng(20261203)
    H, I = 256, 128
    blobs = {}
    for K in (3, 4, 5):
        mats = {}
        for nm, (k, n) in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
            mats[nm] = {"trellis": torch.from_numpy(rng.integers(-32768, 32768, (k // 16, n // 16, 16 * K),
                                                                 dtype=np.int16)),
                        "suh": torch.from_numpy(np.where(rng.random(k) < 0.5, 1.0, -1.0).astype(np.float16)),
                        "svh": torch.from_numpy((rng.standard_normal(n) * 0.1).astype(np.float16))}
        blob = mo.pack_expert(mats["gate"], mats["up"], mats["down"], K).numpy()
        # the same bytes through blob_perm: the raw record is gate | up | down trellis words, then g_suh g_svh u_suh
        # u_svh d_suh d_svh as fp16 pairs
        raw = np.concatenate([mats[m]["trellis"].numpy().view(np.uint32).reshape(-1) for m in ("gate", "up", "down")]
                             + [np.ascontiguousarray(mats[m][v].numpy()).view(np.uint32)
                                for m, v in (("gate", "suh"), ("gate", "svh"), ("up", "suh"), ("up", "svh"),
                                             ("down", "suh"), ("down", "svh"))])
        perm = ps.blob_perm(H, I, K)
        assert np.array_equal(raw[perm].view(np.uint8), blob), f"pack_expert and blob_perm disagree at K={K}"
        blobs[f"K{K}_blob"] = blob
        for m in mats:
            for v in mats[m]:
                blobs[f"K{K}_{m}_{v}"] = mats[m][v].numpy()
    np.savez_compressed(os.path.join(HERE, "expert_blob.npz"), H=H, I=I, **blobs)

    # DeepSeek-V4 piece store from a small checkpoint
    sys.path.insert(0, os.path.join(REF, "dsv41/xpu"))
    dps = importlib.import_module("dsv_xpu.pack_store")
    dps.H, dps.I = H, I
    dps.UNIT = H * I // 8
    dps.VEC = 2 * H + 2 * I + I + H
    out = os.path.join(HERE, "dsv_store")
    shutil.rmtree(out, ignore_errors=True)
    with tempfile.TemporaryDirectory() as ck:
        tens = {}
        for L in range(2):
            for e in range(4):
                for p, (k, n) in (("w1", (H, I)), ("w3", (H, I)), ("w2", (I, H))):
                    K = int(rng.integers(1, 4))
                    key = f"layers.{L}.ffn.experts.{e}.{p}"
                    tens[f"{key}.trellis"] = torch.from_numpy(
                        rng.integers(-32768, 32768, (k // 16, n // 16, 16 * K), dtype=np.int16))
                    tens[f"{key}.suh"] = torch.from_numpy(np.where(rng.random(k) < 0.5, 1.0, -1.0).astype(np.float16))
                    tens[f"{key}.svh"] = torch.from_numpy((rng.standard_normal(n) * 0.1).astype(np.float16))
        save_file(tens, os.path.join(ck, "model-00001-of-00001.safetensors"))
        with open(os.path.join(ck, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": {k: "model-00001-of-00001.safetensors" for k in tens}}, f)
        dps.main(ck, out, n_layers=2, n_experts=4)
        os.makedirs(out, exist_ok=True)
        shutil.copy(os.path.join(ck, "model-00001-of-00001.safetensors"), os.path.join(out, "checkpoint.safetensors"))


def main():
    if sys.argv[1:] == ["softmax"]:
        make_softmax()
        print("route_softmax.npz written to", HERE)
        return
    if sys.argv[1:] == ["stores"]:
        make_stores()
        print("expert_blob.npz and dsv_store/ written to", HERE)
        return
    sys.path.insert(0, os.path.join(REF, "glm/xpu"))
    sys.path.insert(0, os.path.join(REF, "dsv41/xpu"))
    from glm_xpu import ops as glm_ops            # noqa: E402
    from dsv_xpu import moe as dsv_moe            # noqa: E402
    U = load_units_slice()
    rng = np.random.default_rng(20261201)
    torch.manual_seed(1234)
    meta = {}

    # 1. codebook known answers (units.py mul1_lut)
    lut = U["LUT"].numpy()
    bits = lut.view(np.uint16).astype(np.uint64)
    meta["lut"] = {"first8_bits": [int(b) for b in bits[:8]], "checksum_u64": int(bits.sum()),
                   "weighted_checksum": int((bits * np.arange(65536, dtype=np.uint64)).sum() % (1 << 61)),
                   "min": float(lut.astype(np.float32).min()), "max": float(lut.astype(np.float32).max()),
                   "std": float(lut.astype(np.float64).std())}

    # 2. decoded tiles for every K = 1..8 (units.py w_hat)
    for K in range(1, 9):
        tr = rng.integers(0, 65536, size=(2, 3, 16 * K), dtype=np.uint16)
        w = U["w_hat"](torch.from_numpy(tr.view(np.int16).copy()), K).numpy()
        np.savez_compressed(os.path.join(HERE, f"w_hat_K{K}.npz"), trellis=tr, w_hat=w)

    # 3. EXL3 linear, fp64 reference (units.py ref_linear), k = n = 256
    for K in (2, 3, 4, 5, 6):
        k, n, M = 256, 384, 4
        tr = rng.integers(0, 65536, size=(k // 16, n // 16, 16 * K), dtype=np.uint16)
        suh = np.where(rng.integers(0, 2, k) == 1, 1.0, -1.0).astype(np.float16)
        svh = (np.where(rng.integers(0, 2, n) == 1, 1.0, -1.0) * rng.uniform(0.5, 1.5, n)).astype(np.float16)
        x = rng.standard_normal((M, k)).astype(np.float16)
        y = U["ref_linear"](torch.from_numpy(x), torch.from_numpy(tr.view(np.int16).copy()), torch.from_numpy(suh),
                            torch.from_numpy(svh), K).numpy()
        np.savez_compressed(os.path.join(HERE, f"linear_K{K}.npz"), trellis=tr, suh=suh, svh=svh, x=x, y=y)

    # 4. sigmoid router with e_score_correction_bias (glm_xpu.ops.routing_ds3_nogroup)
    R, H, E, k = 16, 256, 160, 8
    hidden = torch.from_numpy(rng.standard_normal((R, H)).astype(np.float16))
    gate = torch.from_numpy((rng.standard_normal((H, E)) * 0.1).astype(np.float16))
    bias = torch.from_numpy((rng.standard_normal(E) * 0.05).astype(np.float32))
    scores = torch.empty((R, E), dtype=torch.half)
    ids = torch.empty((R, k), dtype=torch.int64)
    wts = torch.empty((R, k), dtype=torch.float32)
    glm_ops.routing_ds3_nogroup(hidden, gate, scores, bias, ids, wts, 2.5, None, 0, None, None)
    np.savez_compressed(os.path.join(HERE, "route_sigmoid.npz"), logits=scores.float().numpy(), bias=bias.numpy(),
                        ids=ids.numpy(), w=wts.numpy(), k=k, scale=2.5)

    # 5. sqrt-softplus router with residency bias (dsv_xpu.moe.route, torch path), exact and no-sync
    R, H, E, k = 16, 256, 256, 8
    y = torch.from_numpy(rng.standard_normal((R, H)).astype(np.float16))
    gate_t = torch.from_numpy((rng.standard_normal((H, E)) * 0.1).astype(np.float16))
    dbias = torch.from_numpy((rng.standard_normal(E) * 0.05).astype(np.float32))
    res = np.zeros(E, dtype=np.float32)
    res[rng.random(E) < 0.5] = -0.2                   # slower tier: -margin
    res[rng.random(E) < 0.1] = -np.inf                # not readable
    mod = types.SimpleNamespace(_gate_t=gate_t, num_experts_per_tok=k, routed_scaling_factor=1.5, _bias=dbias, _li=0)
    dsv_moe.TIER = types.SimpleNamespace(nosync=False, res_pin=[torch.from_numpy(res)], res=[torch.from_numpy(res)])
    dsv_moe.IN_PREFILL[0] = False
    ids0, w0, _ = dsv_moe.route(mod, y, nosync=False)
    ids1, w1, want1 = dsv_moe.route(mod, y, nosync=True)
    logits = torch.matmul(y, gate_t).float().numpy()
    np.savez_compressed(os.path.join(HERE, "route_sqrt_softplus.npz"), logits=logits, bias=dbias.numpy(), res=res,
                        ids_exact=ids0.numpy(), w_exact=w0.numpy(), ids_nosync=ids1.numpy(), w_nosync=w1.numpy(),
                        want_nosync=want1.numpy(), k=k, scale=1.5)

    # 6. silu_mul (glm_xpu.ops.silu_mul) with and without the clamp
    g = torch.from_numpy((rng.standard_normal(4096) * 6).astype(np.float16))
    u = torch.from_numpy((rng.standard_normal(4096) * 6).astype(np.float16))
    z10 = torch.empty_like(g)
    z0 = torch.empty_like(g)
    glm_ops.silu_mul(g, u, z10, 10.0)
    glm_ops.silu_mul(g, u, z0, 0.0)
    np.savez_compressed(os.path.join(HERE, "silu_mul.npz"), g=g.numpy(), u=u.numpy(), z10=z10.numpy(), z0=z0.numpy())

    # 7. had_r_128 (glm_xpu.ops.had_r_128): pre-scaled fp16, post-scaled fp32
    x16 = torch.from_numpy(rng.standard_normal((4, 512)).astype(np.float16))
    pre = torch.from_numpy(np.where(rng.integers(0, 2, 512) == 1, 1.0, -1.0).astype(np.float16))
    o16 = torch.empty_like(x16)
    glm_ops.had_r_128(x16, o16, pre, None, 1.0)
    x32 = torch.from_numpy(rng.standard_normal((4, 512)).astype(np.float32))
    post = torch.from_numpy(rng.uniform(-2, 2, 512).astype(np.float32))
    o32 = torch.empty_like(x32)
    glm_ops.had_r_128(x32, o32, None, post, 1.0)
    np.savez_compressed(os.path.join(HERE, "had_r_128.npz"), x16=x16.numpy(), pre=pre.numpy(), o16=o16.numpy(),
                        x32=x32.numpy(), post=post.numpy(), o32=o32.numpy())

    # 8. MoE expert math from reference pieces (units.py ref_linear + glm_xpu.ops.silu_mul), as units.py:140-157 does
    H, I, E, M, topk, L = 256, 128, 4, 3, 2, 10.0
    Ks = [2, 3, 4, 3]
    ex = {}
    for e in range(E):
        K = Ks[e]
        for nm, (kk, nn) in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
            ex[f"{e}_{nm}_tr"] = rng.integers(0, 65536, size=(kk // 16, nn // 16, 16 * K), dtype=np.uint16)
            ex[f"{e}_{nm}_suh"] = np.where(rng.integers(0, 2, kk) == 1, 1.0, -1.0).astype(np.float16)
            ex[f"{e}_{nm}_svh"] = np.where(rng.integers(0, 2, nn) == 1, 1.0, -1.0).astype(np.float16)
    x = rng.standard_normal((M, H)).astype(np.float16)
    sel = np.stack([rng.permutation(E)[:topk] for _ in range(M)]).astype(np.int32)
    wsel = rng.random((M, topk)).astype(np.float32)

    def lin(xx, e, nm):
        return U["ref_linear"](torch.from_numpy(xx), torch.from_numpy(ex[f"{e}_{nm}_tr"].view(np.int16).copy()),
                               torch.from_numpy(ex[f"{e}_{nm}_suh"]), torch.from_numpy(ex[f"{e}_{nm}_svh"]), Ks[e])

    out = np.zeros((M, H), dtype=np.float64)
    for m in range(M):
        for j in range(topk):
            e = int(sel[m, j])
            gg = lin(x[m:m + 1], e, "gate").half()
            uu = lin(x[m:m + 1], e, "up").half()
            glm_ops.silu_mul(gg, uu, uu, L)
            d = lin(uu.numpy(), e, "down").numpy()[0]
            out[m] += float(wsel[m, j]) * d
    np.savez_compressed(os.path.join(HERE, "moe_expert.npz"), x=x, sel=sel, w=wsel, out=out, Ks=np.array(Ks),
                        H=H, I=I, act_limit=L, **ex)

    make_softmax()
    make_stores()

    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
