"""The CPU oracle against the reference's own outputs (tests/golden/*, produced by make_golden.py from the reference's
Python code) and against the known answers the reference states. CPU only."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.tolerance import assert_close

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(G, name))


def test_mul1_constants():
    # dsv41/xpu/dsv_xpu/exl3_tri.py:18-19,218: the affine constants are the fp16 bit patterns 0x1EEE and 0xC931
    assert np.float16(O.K_INV).view(np.uint16) == 0x1EEE
    assert np.float16(O.K_BIAS).view(np.uint16) == 0xC931
    assert float(np.float16(O.K_INV)) == O.K_INV and float(np.float16(O.K_BIAS)) == O.K_BIAS


def test_codebook_known_answers():
    ka = json.load(open(os.path.join(G, "known_answers.json")))["lut"]
    lut = O.mul1_lut()
    bits = lut.view(np.uint16).astype(np.uint64)
    assert [int(b) for b in bits[:8]] == ka["first8_bits"]
    assert int(bits.sum()) == ka["checksum_u64"]
    assert int((bits * np.arange(65536, dtype=np.uint64)).sum() % (1 << 61)) == ka["weighted_checksum"]
    # glm/docs/ext-op-inventory.md:571: values lie in [-3.453, 3.348], std about 1.0
    assert float(lut.min()) == -3.453125 and float(lut.max()) == 3.34765625
    assert abs(float(lut.astype(np.float64).std()) - 1.0) < 1e-3
    # the table equals the formula evaluated state by state
    st = np.arange(0, 65536, 97)
    assert np.array_equal(O.decode_mul1_state(st).view(np.uint16), lut[st].view(np.uint16))


@pytest.mark.parametrize("K", range(1, 9))
def test_w_hat_matches_reference(K):
    d = load(f"w_hat_K{K}.npz")
    w = O.w_hat(d["trellis"], K)
    assert np.array_equal(w.view(np.uint16), d["w_hat"].view(np.uint16))


def test_tile_position_map_is_a_permutation():
    for K in (1, 3, 8):
        _, _, _, row, col = O.tile_tables(K)
        assert len({(int(r), int(c)) for r, c in zip(row, col)}) == 256


@pytest.mark.parametrize("K", [2, 3, 4, 5, 6])
def test_linear_matches_reference(K):
    d = load(f"linear_K{K}.npz")
    y64 = O.ref_linear_f64(d["x"], d["trellis"], d["suh"], d["svh"], K)
    assert np.array_equal(y64, d["y"])                        # same fp64 math as units.py ref_linear
    # the exllamav3-rounded linear (fp16 x*suh, fp16 xh) stays inside the reference's own tolerance
    # (glm/xpu/tests/units.py:104: rel < 5e-3)
    y = O.exl3_linear(d["x"], d["trellis"], d["suh"], d["svh"], K, np.float32)
    rel = np.linalg.norm(y - d["y"]) / np.linalg.norm(d["y"])
    assert rel < 5e-3


def test_sigmoid_router_matches_reference():
    d = load("route_sigmoid.npz")
    ids, w, _ = O.route(d["logits"], O.ROUTE_SIGMOID, int(d["k"]), bias=d["bias"], scale=float(d["scale"]))
    assert np.array_equal(ids, d["ids"])
    np.testing.assert_allclose(w, d["w"], rtol=1e-6, atol=1e-7)


def test_sqrt_softplus_router_matches_reference():
    d = load("route_sqrt_softplus.npz")
    k, sc = int(d["k"]), float(d["scale"])
    ids, w, _ = O.route(d["logits"], O.ROUTE_SQRT_SOFTPLUS, k, bias=d["bias"], scale=sc)
    # the reference's torch.topk(sorted=False) returns an unordered set: compare sets and per-expert weights
    assert np.array_equal(np.sort(ids, 1), np.sort(d["ids_exact"], 1))
    ids2, w2, want = O.route(d["logits"], O.ROUTE_SQRT_SOFTPLUS, k, bias=d["bias"], res=d["res"], scale=sc,
                             want=True)
    assert np.array_equal(np.sort(ids2, 1), np.sort(d["ids_nosync"], 1))
    assert np.array_equal(np.sort(want, 1), np.sort(d["want_nosync"], 1))
    a = np.take_along_axis(w2, np.argsort(ids2, 1), 1)
    b = np.take_along_axis(d["w_nosync"], np.argsort(d["ids_nosync"], 1), 1)
    np.testing.assert_allclose(a, b, rtol=1e-6, atol=1e-7)
    # non-readable experts (-inf residency bias) are never picked when enough readable ones exist
    assert np.isfinite(d["res"][ids2]).all()


def test_softmax_router_semantics():
    # trellis-serve.patch:394-441: rank on logits + bias, weights = softmax of the unbiased logits, renormalised
    rng = np.random.default_rng(3)
    lg = rng.standard_normal((5, 512)).astype(np.float32)
    cold = np.where(rng.random(512) < 0.1, -1e4, 0.0).astype(np.float32)
    ids, w, _ = O.route(lg, O.ROUTE_SOFTMAX, 10, bias=cold)
    p = np.exp(lg.astype(np.float64) - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    key = lg + cold
    for r in range(5):
        exp_ids = np.argsort(-key[r], kind="stable")[:10]
        assert list(ids[r]) == list(exp_ids)
        pw = p[r, exp_ids]
        np.testing.assert_allclose(w[r], pw / pw.sum(), rtol=1e-6)


SOFTMAX_CASES = ["plain", "cold_margin", "cold_only", "norenorm", "ties", "e160"]


def softmax_case(name):
    """One case of route_softmax.npz (the reference's Triton router run under the CPU interpreter) as exl3_route
    arguments: the cold-tier bias is the key bias, the RAM margin becomes the residency bias -margin on experts
    without a device slot (trellis-serve.patch:404-407)."""
    d = load("route_softmax.npz")
    g = {kk.split("__", 1)[1]: d[kk] for kk in d.files if kk.startswith(name + "__")}
    bias = g.get("cold")
    res = None
    if "slot_of" in g:
        res = np.where(g["slot_of"] < 0, -np.float32(g["margin"][0]), np.float32(0.0)).astype(np.float32)
    return g["logits"], int(g["k"]), bool(g["renorm"]), bias, res, g["ids"], g["w"]


@pytest.mark.parametrize("name", SOFTMAX_CASES)
def test_softmax_router_matches_reference(name):
    lg, k, renorm, bias, res, ids_ref, w_ref = softmax_case(name)
    ids, w, _ = O.route(lg, O.ROUTE_SOFTMAX, k, bias=bias, res=res, renorm=renorm)
    assert np.array_equal(ids, ids_ref.astype(ids.dtype))
    # the reference evaluates the softmax in fp32 (exp, sum, divide); the oracle in fp64 rounded once
    np.testing.assert_allclose(w, w_ref, rtol=2e-6, atol=1e-9)


def test_router_ties_go_to_lowest_index():
    lg = np.zeros((2, 64), dtype=np.float32)
    ids, _, _ = O.route(lg, O.ROUTE_SOFTMAX, 4)
    assert ids.tolist() == [[0, 1, 2, 3], [0, 1, 2, 3]]


def test_silu_mul_matches_reference():
    d = load("silu_mul.npz")
    assert np.array_equal(O.silu_mul(d["g"], d["u"], 10.0).view(np.uint16), d["z10"].view(np.uint16))
    assert np.array_equal(O.silu_mul(d["g"], d["u"], 0.0).view(np.uint16), d["z0"].view(np.uint16))


def test_had_r_128_matches_reference():
    d = load("had_r_128.npz")
    o16 = O.had_r_128(d["x16"], pre=d["pre"])
    diff = np.abs(o16.view(np.int16).astype(np.int32) - d["o16"].view(np.int16).astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 0.01       # butterfly vs matmul order: at most 1 fp16 ulp
    o32 = O.had_r_128(d["x32"], post=d["post"])
    np.testing.assert_allclose(o32, d["o32"], rtol=1e-5, atol=1e-5)


def test_moe_expert_math_matches_reference():
    d = load("moe_expert.npz")
    H, I, L = int(d["H"]), int(d["I"]), float(d["act_limit"])
    Ks = [int(k) for k in d["Ks"]]
    experts = []
    for e in range(len(Ks)):
        mats = [(d[f"{e}_{nm}_tr"], d[f"{e}_{nm}_suh"], d[f"{e}_{nm}_svh"], Ks[e]) for nm in ("gate", "up", "down")]
        experts.append(O.ExpertW(*mats))
    out = O.moe_forward(d["x"], d["sel"], d["w"], experts, L)
    assert_close(out, d["out"], rel_tol=5e-3, what="oracle MoE vs reference pieces")


def test_blob_sizes_known_answers():
    # glm/xpu/csrc/exl3_moe.n128.sycl:7 (H=2560, I=640, K=3) and glm/xpu/glm_xpu/tier.py:3 (H=4096, I=2048, K=3)
    assert O.blob_bytes(2560, 640, 3) == 1_862_400
    assert O.blob_bytes(4096, 2048, 3) == 9_474_048


def test_align_is_stable_and_complete():
    rng = np.random.default_rng(7)
    ids = rng.integers(-1, 20, size=(6, 4)).astype(np.int32)
    a = O.moe_align(ids, 20)
    flat = ids.reshape(-1)
    valid = np.nonzero((flat >= 0) & (flat < 20))[0]
    assert sorted(a["pair_src"].tolist()) == valid.tolist()
    # sorted by expert, then by pair index
    keys = [(int(flat[i]), int(i)) for i in a["pair_src"]]
    assert keys == sorted(keys)
    assert (a["pair_of"][flat < 0] == -1).all()
