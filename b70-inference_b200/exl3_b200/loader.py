"""Expert weights from the reference's on-disk and in-memory formats into ExpertTables (weights resident in HBM).

* Expert blobs of the GLM / Qwen-Next store (glm/xpu/exl3xpu/moe_offload.py:66-94 pack_expert / planar4, the record
  word order of glm/xpu/pack_store.py:35-70 blob_perm; layout glm/xpu/csrc/exl3_moe.n128.sycl:1-13):
      gate|up trellis u32 [H/16][2I/16][8K] | down trellis u32 [I/16][H/16][8K]     (PLANAR4 word order)
      | suh_g[H] suh_u[H] svh_g[I] svh_u[I] suh_d[I] svh_d[H]                      (fp16)
  PLANAR4: in every k-row the tiles are grouped by 4 along n, and each group's 4 * 8K words are stored plane-major:
  word (tile t, period g, plane i) at [i][t][g] instead of [t][D g + i], with D = K / gcd(K, 32) words per period
  and G = 8K / D periods per tile (the identity for D = 1, i.e. K = 1, 2, 4, 8).
* The DeepSeek-V4 piece store (dsv41/xpu/dsv_xpu/pack_store.py:1-120): experts.bin holds per expert gate | up | down
  trellis, each K_p units of H * I / 8 bytes in exllamav3's own [k/16][n/16][16K] int16 layout; vectors [L][E][VEC]
  fp16 = suh_g suh_u svh_g svh_u suh_d svh_d; store.json gives per layer and expert [Kg, Ku, Kd, unit offset].
* exllamav3 / EXL3 safetensors checkpoints: `{prefix}.{e}.{proj}.trellis | suh | svh` per expert (int16 trellis
  [k/16][n/16][16K], fp16 vectors), read straight from the file (8-byte header length, JSON header, raw data).

Everything here is load-time host code; the kernels only ever see the ExpertTable's packed copies.
"""
from __future__ import annotations

import json
import math
import os
import struct

import numpy as np
import torch

from .moe import Expert, ExpertTable, Exl3Matrix


# ------------------------------------------------------------------------------------------------ expert blobs

def blob_bytes(H: int, I: int, K: int) -> int:
    """Size of one expert blob (glm/xpu/csrc/exl3_moe.n128.sycl:56-68)."""
    gu = (H // 16) * (2 * I // 16) * 8 * K * 4
    d = (I // 16) * (H // 16) * 8 * K * 4
    return gu + d + 2 * (2 * H + 2 * I + I + H)


def _planar_dims(K: int):
    D = K // math.gcd(K, 32)
    return D, 8 * K // D


def unplanar4(words: torch.Tensor, rows: int, n_tiles: int, K: int) -> torch.Tensor:
    """PLANAR4 u32 words of a [rows][n_tiles] tile grid -> exllamav3 int16 trellis [rows][n_tiles][16K]."""
    D, G = _planar_dims(K)
    w = words.reshape(rows, n_tiles // 4, D, 4, G)                 # [row, group, plane i, tile t, period g]
    w = w.permute(0, 1, 3, 4, 2).contiguous().reshape(-1)          # [row, group, tile, g, i] = word D g + i
    return w.view(torch.int16).reshape(rows, n_tiles, 16 * K)


def planar4(trellis: torch.Tensor, K: int) -> torch.Tensor:
    """exllamav3 int16 trellis [rows][n_tiles][16K] -> PLANAR4 u32 words (the inverse of unplanar4)."""
    rows, n_tiles, _ = trellis.shape
    D, G = _planar_dims(K)
    w = trellis.contiguous().reshape(-1).view(torch.int32).reshape(rows, n_tiles // 4, 4, G, D)
    return w.permute(0, 1, 4, 2, 3).contiguous().reshape(-1)


def expert_from_blob(blob: torch.Tensor, H: int, I: int, K: int) -> Expert:
    """One expert blob (uint8, any device) -> an Expert of exllamav3-layout tensors on the blob's device."""
    if blob.dtype != torch.uint8 or blob.numel() != blob_bytes(H, I, K):
        raise ValueError(f"expert blob: {blob.numel()} bytes, expected {blob_bytes(H, I, K)} (H={H}, I={I}, K={K})")
    if (I // 16) % 2 or (H // 16) % 4 or (2 * I // 16) % 4:
        raise ValueError("expert blob: tile counts must be multiples of 4 (PLANAR4 groups)")
    b = blob.contiguous()
    gu_b = (H // 16) * (2 * I // 16) * 8 * K * 4
    d_b = (I // 16) * (H // 16) * 8 * K * 4
    gu = unplanar4(b[:gu_b].view(torch.int32), H // 16, 2 * I // 16, K)
    dn = unplanar4(b[gu_b:gu_b + d_b].view(torch.int32), I // 16, H // 16, K)
    v = b[gu_b + d_b:].view(torch.float16)
    o = 0
    vec = {}
    for name, n in (("suh_g", H), ("suh_u", H), ("svh_g", I), ("svh_u", I), ("suh_d", I), ("svh_d", H)):
        vec[name] = v[o:o + n].clone()
        o += n
    it = I // 16
    gate = Exl3Matrix(gu[:, :it].contiguous(), vec["suh_g"], vec["svh_g"], K)
    up = Exl3Matrix(gu[:, it:].contiguous(), vec["suh_u"], vec["svh_u"], K)
    down = Exl3Matrix(dn, vec["suh_d"], vec["svh_d"], K)
    return Expert(gate, up, down)


def blob_from_expert(ex: Expert) -> torch.Tensor:
    """An Expert (one K for its three matrices) -> its blob (uint8, on the expert's device)."""
    K = int(ex.gate.K)
    if int(ex.up.K) != K or int(ex.down.K) != K:
        raise ValueError("expert blob: one K per expert")
    gu = torch.cat([ex.gate.trellis, ex.up.trellis], dim=1)
    parts = [planar4(gu, K), planar4(ex.down.trellis, K)]
    parts = [p.view(torch.uint8) for p in parts]
    for t in (ex.gate.suh, ex.up.suh, ex.gate.svh, ex.up.svh, ex.down.suh, ex.down.svh):
        parts.append(t.half().contiguous().view(torch.uint8))
    return torch.cat(parts)


def table_from_blobs(blobs: torch.Tensor, H: int, I: int, K: int, shared: Expert | None = None,
                     device=None) -> ExpertTable:
    """ExpertTable from a layer's blobs uint8 [E][blob_bytes] (host or device): each blob is moved to the device,
    un-planarised and packed for the kernels."""
    dev = torch.device(device) if device is not None else (blobs.device if blobs.is_cuda else torch.device("cuda"))
    experts = [expert_from_blob(blobs[e].to(dev), H, I, K) for e in range(blobs.shape[0])]
    return ExpertTable(experts, shared, dev)


# ------------------------------------------------------------------------------------------------ DSV piece store

DSV_VEC_FIELDS = ("suh_g", "suh_u", "svh_g", "svh_u", "suh_d", "svh_d")


def expert_from_pieces(data: torch.Tensor, vec: torch.Tensor, H: int, I: int, Ks) -> Expert:
    """One expert of the DSV piece store: data uint8 = gate | up | down trellis (K_p units of H*I/8 bytes each,
    exllamav3 layout), vec fp16 [2H + 3I + H] = suh_g suh_u svh_g svh_u suh_d svh_d."""
    unit = H * I // 8
    Kg, Ku, Kd = (int(k) for k in Ks)
    if data.numel() != (Kg + Ku + Kd) * unit:
        raise ValueError(f"piece record: {data.numel()} bytes, expected {(Kg + Ku + Kd) * unit}")
    d = data.contiguous()
    o = 0
    mats = []
    for K, (k, n) in zip((Kg, Ku, Kd), ((H, I), (H, I), (I, H))):
        tr = d[o:o + K * unit].view(torch.int16).reshape(k // 16, n // 16, 16 * K)
        mats.append(tr)
        o += K * unit
    v = vec.contiguous().view(torch.float16)
    offs = {}
    o = 0
    for name, n in zip(DSV_VEC_FIELDS, (H, H, I, I, I, H)):
        offs[name] = v[o:o + n].clone()
        o += n
    return Expert(Exl3Matrix(mats[0], offs["suh_g"], offs["svh_g"], Kg),
                  Exl3Matrix(mats[1], offs["suh_u"], offs["svh_u"], Ku),
                  Exl3Matrix(mats[2], offs["suh_d"], offs["svh_d"], Kd))


def table_from_piece_store(store_dir: str, layer: int, device="cuda", name: str = "experts",
                           shared: Expert | None = None) -> ExpertTable:
    """ExpertTable of one layer of a DSV piece store directory (store.json = {name}.json, {name}.bin,
    {name}_vectors.bin.npy). Experts with K = 0 (empty rows) are not allowed in a routed table."""
    meta = json.load(open(os.path.join(store_dir, f"{name}.json")))
    H, I, unit = int(meta["H"]), int(meta["I"]), int(meta["unit"])
    vec = np.load(os.path.join(store_dir, f"{name}_vectors.bin.npy"), mmap_mode="r")
    experts = []
    with open(os.path.join(store_dir, f"{name}.bin"), "rb") as f:
        for e, (Kg, Ku, Kd, off) in enumerate(meta["layers"][layer]):
            n = (Kg + Ku + Kd) * unit
            f.seek(off * unit)
            raw = torch.frombuffer(bytearray(f.read(n)), dtype=torch.uint8).to(device)
            v = torch.from_numpy(np.array(vec[layer, e])).to(device)
            experts.append(expert_from_pieces(raw, v, H, I, (Kg, Ku, Kd)))
    return ExpertTable(experts, shared, torch.device(device))


# ------------------------------------------------------------------------------------------------ safetensors

_ST_DTYPES = {"I16": torch.int16, "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32,
              "U8": torch.uint8, "I32": torch.int32, "I64": torch.int64, "BOOL": torch.bool}


def safetensors_header(path: str):
    """(data start offset, {name: {dtype, shape, data_offsets}}) of a .safetensors file."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        h = json.loads(f.read(n))
    h.pop("__metadata__", None)
    return 8 + n, h


class SafetensorsDir:
    """Tensor reader over one .safetensors file or a checkpoint directory (model.safetensors.index.json or every
    *.safetensors file in it)."""

    def __init__(self, path: str):
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                files = sorted(set(json.load(open(idx))["weight_map"].values()))
            else:
                files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
            files = [os.path.join(path, f) for f in files]
        else:
            files = [path]
        self.loc = {}
        for fn in files:
            base, h = safetensors_header(fn)
            for k, v in h.items():
                self.loc[k] = (fn, base, v)

    def keys(self):
        return self.loc.keys()

    def get(self, key: str, device="cpu") -> torch.Tensor:
        fn, base, v = self.loc[key]
        a, b = v["data_offsets"]
        with open(fn, "rb") as f:
            f.seek(base + a)
            buf = bytearray(f.read(b - a))
        t = torch.frombuffer(buf, dtype=_ST_DTYPES[v["dtype"]]) if b > a else torch.empty(0, dtype=_ST_DTYPES[v["dtype"]])
        return t.reshape(v["shape"]).to(device)


def load_linear(st: SafetensorsDir, key: str, device="cuda") -> Exl3Matrix:
    """An EXL3 linear `{key}.trellis / .suh / .svh` (K from the trellis shape [k/16][n/16][16K])."""
    tr = st.get(f"{key}.trellis", device)
    K = tr.shape[-1] // 16
    suh = st.get(f"{key}.suh", device).half() if f"{key}.suh" in st.loc else None
    svh = st.get(f"{key}.svh", device).half()
    return Exl3Matrix(tr.view(torch.int16), suh, svh, K)


def table_from_safetensors(path: str, prefix: str, n_experts: int, device="cuda",
                           proj=("gate_proj", "up_proj", "down_proj"), shared_prefix: str | None = None
                           ) -> ExpertTable:
    """ExpertTable of one MoE layer of an EXL3 checkpoint: experts `{prefix}.{e}.{proj}` (e.g. prefix
    "model.layers.3.mlp.experts", proj gate_proj/up_proj/down_proj; DeepSeek-V4 names w1/w3/w2), and optionally the
    shared expert `{shared_prefix}.{proj}`."""
    st = SafetensorsDir(path)
    experts = [Expert(*(load_linear(st, f"{prefix}.{e}.{p}", device) for p in proj)) for e in range(n_experts)]
    shared = None
    if shared_prefix is not None:
        shared = Expert(*(load_linear(st, f"{shared_prefix}.{p}", device) for p in proj))
    return ExpertTable(experts, shared, torch.device(device))


def save_safetensors(path: str, tensors: dict) -> None:
    """Write tensors (CPU) as a .safetensors file (for tests and conversions)."""
    rev = {v: k for k, v in _ST_DTYPES.items()}
    header, off, blobs = {}, 0, []
    for k, t in tensors.items():
        b = t.contiguous().cpu().view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[k] = {"dtype": rev[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
