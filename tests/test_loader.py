"""Expert weights from the reference's formats: GLM / Qwen-Next expert blobs (PLANAR4, written by the reference's own
pack_expert in tests/golden/make_golden.py), the DeepSeek-V4 piece store (written by the reference's own
pack_store.main from a small EXL3 safetensors checkpoint), and the checkpoint itself. CPU: every format decodes to
the checkpoint's tensors bit for bit. GPU: ExpertTables built from each format give the per-tensor table's MoE output
bit for bit, and the oracle's within tolerance."""
import json
import os

import numpy as np
import pytest
import torch

from exl3_b200 import loader, moe
from oracle import oracle as O
from tests.tolerance import assert_close

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
STORE = os.path.join(G, "dsv_store")
DEV = "cuda:0"


def blob_case(K):
    d = np.load(os.path.join(G, "expert_blob.npz"))
    mats = {m: {v: torch.from_numpy(d[f"K{K}_{m}_{v}"]) for v in ("trellis", "suh", "svh")}
            for m in ("gate", "up", "down")}
    return int(d["H"]), int(d["I"]), torch.from_numpy(d[f"K{K}_blob"]), mats


@pytest.mark.parametrize("K", [3, 4, 5])
def test_blob_unpacks_to_the_checkpoint_tensors(K):
    H, I, blob, mats = blob_case(K)
    assert blob.numel() == loader.blob_bytes(H, I, K) == O.blob_bytes(H, I, K)
    ex = loader.expert_from_blob(blob, H, I, K)
    for nm, m in (("gate", ex.gate), ("up", ex.up), ("down", ex.down)):
        assert torch.equal(m.trellis, mats[nm]["trellis"]), nm
        assert torch.equal(m.suh.view(torch.int16), mats[nm]["suh"].view(torch.int16)), nm
        assert torch.equal(m.svh.view(torch.int16), mats[nm]["svh"].view(torch.int16)), nm
        assert m.K == K
    assert torch.equal(loader.blob_from_expert(ex), blob)          # and back: the reference's bytes


def test_planar4_is_a_permutation_for_every_K():
    for K in range(1, 9):
        tr = torch.arange(2 * 8 * 8 * K, dtype=torch.int32).view(torch.int16).reshape(2, 8, 16 * K)
        w = loader.planar4(tr, K)
        assert torch.equal(torch.sort(w.view(torch.int32))[0], torch.sort(tr.reshape(-1).view(torch.int32))[0])
        assert torch.equal(loader.unplanar4(w, 2, 8, K), tr)


def test_blob_size_is_checked():
    with pytest.raises(ValueError):
        loader.expert_from_blob(torch.zeros(100, dtype=torch.uint8), 256, 128, 3)


def test_piece_store_matches_the_checkpoint():
    meta = json.load(open(os.path.join(STORE, "experts.json")))
    st = loader.SafetensorsDir(os.path.join(STORE, "checkpoint.safetensors"))
    vec = np.load(os.path.join(STORE, "experts_vectors.bin.npy"))
    raw = open(os.path.join(STORE, "experts.bin"), "rb").read()
    H, I, unit = meta["H"], meta["I"], meta["unit"]
    for L in range(meta["n_layers"]):
        for e, (Kg, Ku, Kd, off) in enumerate(meta["layers"][L]):
            data = torch.frombuffer(bytearray(raw[off * unit:(off + Kg + Ku + Kd) * unit]), dtype=torch.uint8)
            ex = loader.expert_from_pieces(data, torch.from_numpy(vec[L, e].copy()), H, I, (Kg, Ku, Kd))
            for p, m in zip(("w1", "w3", "w2"), (ex.gate, ex.up, ex.down)):
                ref = loader.load_linear(st, f"layers.{L}.ffn.experts.{e}.{p}", "cpu")
                assert m.K == ref.K
                assert torch.equal(m.trellis, ref.trellis)
                assert torch.equal(m.suh.view(torch.int16), ref.suh.view(torch.int16))
                assert torch.equal(m.svh.view(torch.int16), ref.svh.view(torch.int16))


def test_safetensors_round_trip(tmp_path):
    t = {"a.trellis": torch.arange(-50, 46, dtype=torch.int16).reshape(2, 3, 16), "a.svh": torch.ones(48).half(),
         "b": torch.zeros(0, dtype=torch.float32)}
    p = str(tmp_path / "x.safetensors")
    loader.save_safetensors(p, t)
    st = loader.SafetensorsDir(p)
    assert set(st.keys()) == set(t)
    for k, v in t.items():
        assert torch.equal(st.get(k), v)


# ------------------------------------------------------------------------------------------------ GPU

def run_layer(table, x, ids, w):
    return moe.moe_forward(x, ids, w, table, 10.0)


@pytest.mark.gpu
@pytest.mark.parametrize("K", [3, 4, 5])
def test_table_from_blobs_equals_per_tensor_table(K):
    H, I, blob, mats = blob_case(K)
    blobs = torch.stack([blob] * 3)                                  # three experts sharing the reference's blob
    t_blob = loader.table_from_blobs(blobs, H, I, K, device=DEV)
    per = [moe.Expert(*(moe.Exl3Matrix(mats[m]["trellis"].to(DEV), mats[m]["suh"].to(DEV), mats[m]["svh"].to(DEV), K)
                        for m in ("gate", "up", "down")))] * 3
    t_ref = moe.ExpertTable(per)
    g = torch.Generator(device=DEV).manual_seed(K)
    x = torch.randn((4, H), device=DEV, generator=g).half()
    ids = torch.tensor([[0, 1], [2, 0], [1, 2], [2, 1]], dtype=torch.int32, device=DEV)
    w = torch.rand((4, 2), device=DEV, generator=g)
    assert torch.equal(run_layer(t_blob, x, ids, w), run_layer(t_ref, x, ids, w))


@pytest.mark.gpu
def test_tables_from_piece_store_and_checkpoint():
    meta = json.load(open(os.path.join(STORE, "experts.json")))
    H, I = meta["H"], meta["I"]
    ckpt = os.path.join(STORE, "checkpoint.safetensors")
    g = torch.Generator(device=DEV).manual_seed(3)
    for L in range(meta["n_layers"]):
        t_store = loader.table_from_piece_store(STORE, L, DEV)
        t_ckpt = loader.table_from_safetensors(ckpt, f"layers.{L}.ffn.experts", 4, DEV, proj=("w1", "w3", "w2"))
        x = torch.randn((3, H), device=DEV, generator=g).half()
        ids = torch.tensor([[0, 3], [1, 2], [3, 1]], dtype=torch.int32, device=DEV)
        w = torch.rand((3, 2), device=DEV, generator=g)
        a, b = run_layer(t_store, x, ids, w), run_layer(t_ckpt, x, ids, w)
        assert torch.equal(a, b)
        st = loader.SafetensorsDir(ckpt)
        np_exp = []
        for e in range(4):
            mats = []
            for p in ("w1", "w3", "w2"):
                m = loader.load_linear(st, f"layers.{L}.ffn.experts.{e}.{p}", "cpu")
                mats.append((m.trellis.numpy().view(np.uint16), m.suh.numpy(), m.svh.numpy(), m.K))
            np_exp.append(O.ExpertW(*mats))
        ref = O.moe_forward(x.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), np_exp, 10.0)
        assert_close(a.cpu().numpy(), ref, what=f"piece store layer {L}")
