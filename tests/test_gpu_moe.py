"""GPU parity of the router (residency bias), the alignment tables and the grouped MoE decode against the oracle and
the reference's golden vectors. Routed ids and alignment tables bit-exact; layer outputs within tolerance."""
import os

import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import moe, ops
from oracle import oracle as O
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda:0"


def to_dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if t.dtype == torch.uint16:
        t = t.view(torch.int16)
    return t.to(DEV)


def poisoned(nbytes):
    """A workspace of 0xFF bytes (NaN as fp32, -1 as int32): nothing may depend on its previous contents."""
    return torch.full((nbytes,), 255, dtype=torch.uint8, device=DEV)


@pytest.fixture(autouse=True)
def _status_clean():
    L.lib().exl3_device_status(1)
    yield
    torch.cuda.synchronize()
    assert L.lib().exl3_device_status(0) == 0


# ------------------------------------------------------------------------------------------------ router

@pytest.mark.parametrize("kind", [O.ROUTE_SIGMOID, O.ROUTE_SOFTMAX, O.ROUTE_SQRT_SOFTPLUS])
@pytest.mark.parametrize("R,E,k", [(1, 160, 8), (4, 512, 10), (37, 256, 8), (3, 1024, 32), (5, 100, 7)])
@pytest.mark.parametrize("ties", [False, True])
def test_route_bitexact(kind, R, E, k, ties):
    rng = np.random.default_rng(R * E + kind)
    lg = rng.standard_normal((R, E)).astype(np.float32) * 3
    if ties:                                             # many equal scores: the lowest expert index wins a tie
        lg = np.round(lg * 2).astype(np.float32) / 2
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    res = np.zeros(E, dtype=np.float32)
    res[rng.random(E) < 0.25] = 0.1                      # resident subset preferred
    res[rng.random(E) < 0.05] = -np.inf                  # unreadable
    mul = np.where(rng.random(E) < 0.3, 1.3, 1.0).astype(np.float32)
    for b, r, m in ((None, None, None), (bias, res, None), (bias, res, mul)):
        ids, w, want = ops.route(to_dev(lg), kind, k, bias=None if b is None else to_dev(b),
                                 res=None if r is None else to_dev(r), mul=None if m is None else to_dev(m),
                                 scale=2.5, want=True)
        rid, rw, rwant = O.route(lg, kind, k, bias=b, res=r, mul=m, scale=2.5, want=True)
        assert np.array_equal(ids.cpu().numpy(), rid), "routed ids must be bit-exact"
        assert np.array_equal(want.cpu().numpy(), rwant)
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("kind", [O.ROUTE_SIGMOID, O.ROUTE_SOFTMAX, O.ROUTE_SQRT_SOFTPLUS])
@pytest.mark.parametrize("R,H,E,k,dt", [(1, 2048, 512, 10, torch.float16), (4, 6144, 160, 8, torch.bfloat16),
                                        (37, 256, 1024, 32, torch.float16), (64, 512, 9, 3, torch.float16),
                                        (65, 512, 130, 4, torch.float16), (300, 7168, 256, 8, torch.bfloat16),
                                        (1000, 2048, 512, 10, torch.float16)])
def test_route_hidden_fused(kind, R, H, E, k, dt):
    """The router GEMV fused into the routing launch (up to 64 rows) or the tensor-core router GEMM (more rows): fp16
    logits within one ulp of the fp32 product, then ids bit-exact and weights as the oracle router gives for those
    logits; repeated calls reuse the zeroed ticket."""
    rng = np.random.default_rng(R + H + E + kind)
    hid = torch.from_numpy(rng.standard_normal((R, H)).astype(np.float32)).to(DEV, dt)
    gate_t = torch.from_numpy((rng.standard_normal((E, H)) / np.sqrt(H) * 3).astype(np.float16)).to(DEV)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    res = np.zeros(E, dtype=np.float32)
    res[rng.random(E) < 0.25] = 0.1
    for _ in range(2):
        lo = torch.empty((R, E), dtype=torch.float16, device=DEV)
        ids, w, want = ops.route_hidden(hid, gate_t, kind, k, bias=to_dev(bias), res=to_dev(res), scale=2.5,
                                        want=True, logits_out=lo)
        # faithful fp16 rounding of the exact (fp64) product: one of its two fp16 neighbours (an fp32 sum in any
        # order may land on either side of a rounding midpoint, as the reference's own GEMV may)
        # plus the fp32 accumulation error, which dominates for logits that cancel to near zero
        hd, gd = hid.double().cpu().numpy(), gate_t.double().cpu().numpy()
        exact = hd @ gd.T
        mag = np.abs(hd) @ np.abs(gd).T
        got = lo.cpu().numpy().astype(np.float64)
        ulp = np.abs(np.spacing(np.abs(exact).astype(np.float16))).astype(np.float64)
        assert np.all(np.abs(got - exact) <= ulp + 64 * 2.0 ** -24 * mag), "logits are not a faithful fp16 rounding"
        rid, rw, rwant = O.route(got, kind, k, bias=bias, res=res, scale=2.5, want=True)
        assert np.array_equal(ids.cpu().numpy(), rid), "routed ids must be bit-exact"
        assert np.array_equal(want.cpu().numpy(), rwant)
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("R", [1, 4, 64, 200])
def test_route_hidden_pair_predicts_the_next_layer(R):
    """This layer's and the next layer's routers in one launch (exl3_route_hidden_pair): both layers' picks equal
    the separate routers' on the same hidden states, bit for bit."""
    rng = np.random.default_rng(900 + R)
    H, E0, E1 = 1024, 160, 256
    hid = to_dev(rng.standard_normal((R, H)).astype(np.float16))
    g0 = to_dev((rng.standard_normal((E0, H)) / np.sqrt(H) * 3).astype(np.float16))
    g1 = to_dev((rng.standard_normal((E1, H)) / np.sqrt(H) * 3).astype(np.float16))
    b0 = to_dev((rng.standard_normal(E0) * 0.1).astype(np.float32))
    b1 = to_dev((rng.standard_normal(E1) * 0.1).astype(np.float32))
    res = to_dev(np.where(rng.random(E0) < 0.25, 0.1, 0.0).astype(np.float32))
    lo = torch.empty((R, E0), dtype=torch.float16, device=DEV)
    ids, w, want, ids1, w1 = ops.route_hidden(hid, g0, O.ROUTE_SIGMOID, 8, bias=b0, res=res, scale=2.5, want=True,
                                              logits_out=lo, next_router=dict(gate_t=g1, kind=O.ROUTE_SQRT_SOFTPLUS,
                                                                              k=6, bias=b1, scale=1.5))
    lo_ref = torch.empty((R, E0), dtype=torch.float16, device=DEV)
    rid, rw, rwant = ops.route_hidden(hid, g0, O.ROUTE_SIGMOID, 8, bias=b0, res=res, scale=2.5, want=True,
                                      logits_out=lo_ref)
    rid1, rw1, _ = ops.route_hidden(hid, g1, O.ROUTE_SQRT_SOFTPLUS, 6, bias=b1, scale=1.5)
    assert torch.equal(lo, lo_ref)
    assert torch.equal(ids, rid) and torch.equal(w, rw) and torch.equal(want, rwant)
    assert torch.equal(ids1, rid1) and torch.equal(w1, rw1)


def test_route_prefill_rows_and_int64():
    rng = np.random.default_rng(11)
    lg = rng.standard_normal((8192, 256)).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.05).astype(np.float32)
    ids, w, _ = ops.route(to_dev(lg), O.ROUTE_SQRT_SOFTPLUS, 8, bias=to_dev(bias), scale=2.5, ids_dtype=torch.int64)
    rid, rw, _ = O.route(lg, O.ROUTE_SQRT_SOFTPLUS, 8, bias=bias, scale=2.5)
    assert ids.dtype == torch.int64
    assert np.array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


def test_route_golden_sigmoid():
    d = np.load(os.path.join(G, "route_sigmoid.npz"))
    ids, w, _ = ops.route(to_dev(d["logits"]), O.ROUTE_SIGMOID, int(d["k"]), bias=to_dev(d["bias"]),
                          scale=float(d["scale"]), ids_dtype=torch.int64)
    assert np.array_equal(ids.cpu().numpy(), d["ids"])
    np.testing.assert_allclose(w.cpu().numpy(), d["w"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("name", ["plain", "cold_margin", "cold_only", "norenorm", "ties", "e160"])
def test_route_golden_softmax(name):
    # the reference's own softmax router (trellis-serve.patch:394-441, run by make_golden.py under Triton's CPU
    # interpreter): cold-tier bias as the key bias, the RAM margin as the residency bias on slotless experts
    from tests.test_oracle_golden import softmax_case
    lg, k, renorm, bias, res, ids_ref, w_ref = softmax_case(name)
    ids, w, _ = ops.route(to_dev(lg), O.ROUTE_SOFTMAX, k, bias=None if bias is None else to_dev(bias),
                          res=None if res is None else to_dev(res), renorm=renorm)
    assert np.array_equal(ids.cpu().numpy(), ids_ref.astype(np.int32)), "routed ids must be bit-exact"
    np.testing.assert_allclose(w.cpu().numpy(), w_ref, rtol=2e-6, atol=1e-9)


def test_routing_ds3_nogroup_api():
    """The reference op's signature: logits from hidden @ gate (fp16), outputs written in place."""
    rng = np.random.default_rng(4)
    R, H, E, k = 4, 256, 160, 8
    hidden = to_dev(rng.standard_normal((R, H)).astype(np.float16))
    gate = to_dev((rng.standard_normal((H, E)) * 0.1).astype(np.float16))
    bias = to_dev((rng.standard_normal(E) * 0.05).astype(np.float32))
    scores = torch.empty((R, E), dtype=torch.half, device=DEV)
    idx = torch.empty((R, k), dtype=torch.int64, device=DEV)
    wts = torch.empty((R, k), dtype=torch.float32, device=DEV)
    ops.routing_ds3_nogroup(hidden, gate, scores, bias, idx, wts, 2.5, None, 0, None, None)
    rid, rw, _ = O.route(scores.float().cpu().numpy(), O.ROUTE_SIGMOID, k, bias=bias.cpu().numpy(), scale=2.5)
    assert np.array_equal(idx.cpu().numpy(), rid)
    np.testing.assert_allclose(wts.cpu().numpy(), rw, rtol=2e-6)


def test_route_golden_sqrt_softplus():
    d = np.load(os.path.join(G, "route_sqrt_softplus.npz"))
    ids, w, want = ops.route(to_dev(d["logits"]), O.ROUTE_SQRT_SOFTPLUS, int(d["k"]), bias=to_dev(d["bias"]),
                             res=to_dev(d["res"]), scale=float(d["scale"]), want=True)
    assert np.array_equal(np.sort(ids.cpu().numpy(), 1), np.sort(d["ids_nosync"], 1))
    assert np.array_equal(np.sort(want.cpu().numpy(), 1), np.sort(d["want_nosync"], 1))


# ------------------------------------------------------------------------------------------------ align

@pytest.mark.parametrize("M,k,E", [(1, 10, 512), (4, 8, 160), (64, 8, 256), (8192, 8, 256)])
@pytest.mark.parametrize("shared", [False, True])
def test_align_matches_oracle(M, k, E, shared):
    rng = np.random.default_rng(M + E)
    ids = rng.integers(0, E, size=(M, k)).astype(np.int32)
    ids[rng.random((M, k)) < 0.02] = -1                 # dropped picks
    if M >= 64:
        ids[: M // 2, 0] = 3                            # a hot expert with many rows (several items)
    w = rng.random((M, k)).astype(np.float32)
    a = moe.moe_align(to_dev(ids), to_dev(w), E, shared=shared, chunk=8)
    ref = O.moe_align(ids, E)
    nv = len(ref["pair_src"])
    assert a["n_valid"] == nv
    assert np.array_equal(a["pair_of"].cpu().numpy(), ref["pair_of"])
    assert np.array_equal(a["pair_tok"].cpu().numpy()[:nv], ref["pair_tok"])
    assert np.array_equal(a["pair_w"].cpu().numpy()[:nv], w.reshape(-1)[ref["pair_src"]])
    assert np.array_equal(a["pair_src"].cpu().numpy()[:nv], ref["pair_src"])
    if shared:
        assert np.array_equal(a["pair_src"].cpu().numpy()[nv:], M * k + np.arange(M))
    # items: ceil(count / 8) per active expert, in expert order
    exp_items = []
    for e, s0, c in zip(ref["act_expert"], ref["act_start"], ref["act_cnt"]):
        for j in range(0, int(c), 8):
            exp_items.append((int(e), int(s0) + j, min(8, int(c) - j)))
    if shared:
        for j in range(0, M, 8):
            exp_items.append((E, nv + j, min(8, M - j)))
        assert np.array_equal(a["pair_tok"].cpu().numpy()[nv:], np.arange(M))
    got = list(zip(a["item_expert"].tolist(), a["item_start"].tolist(), a["item_cnt"].tolist()))
    assert got == exp_items


@pytest.mark.parametrize("M,k,E,chunk", [(8, 8, 40, 3), (3, 7, 20, 2), (1, 1, 4, 1)])
@pytest.mark.parametrize("shared", [False, True])
def test_align_warp_path_hot_expert(M, k, E, chunk, shared):
    """Decode-sized alignments (<= 64 pairs, one warp): several items per expert, dropped picks, shared rows."""
    rng = np.random.default_rng(M * k + E + chunk)
    ids = rng.integers(0, E, size=(M, k)).astype(np.int32)
    ids[:, 0] = 3                                       # a hot expert picked by every token
    ids[rng.random((M, k)) < 0.1] = -1
    ids[0, -1] = E + 5                                  # out of range: dropped as well
    w = rng.random((M, k)).astype(np.float32)
    a = moe.moe_align(to_dev(ids), to_dev(w), E, shared=shared, chunk=chunk)
    ref = O.moe_align(np.where((ids >= 0) & (ids < E), ids, -1), E)
    nv = len(ref["pair_src"])
    assert a["n_valid"] == nv
    assert np.array_equal(a["pair_of"].cpu().numpy(), ref["pair_of"])
    assert np.array_equal(a["pair_tok"].cpu().numpy()[:nv], ref["pair_tok"])
    assert np.array_equal(a["pair_src"].cpu().numpy()[:nv], ref["pair_src"])
    assert np.array_equal(a["pair_w"].cpu().numpy()[:nv], w.reshape(-1)[ref["pair_src"]])
    exp_items = []
    for e, s0, c in zip(ref["act_expert"], ref["act_start"], ref["act_cnt"]):
        for j in range(0, int(c), chunk):
            exp_items.append((int(e), int(s0) + j, min(chunk, int(c) - j)))
    if shared:
        for j in range(0, M, chunk):
            exp_items.append((E, nv + j, min(chunk, M - j)))
        assert np.array_equal(a["pair_src"].cpu().numpy()[nv:], M * k + np.arange(M))
    got = list(zip(a["item_expert"].tolist(), a["item_start"].tolist(), a["item_cnt"].tolist()))
    assert got == exp_items


# ------------------------------------------------------------------------------------------------ MoE decode

def make_experts(rng, E, H, I, Ks, shared_K=None):
    np_exp, dev_exp = [], []

    def mat(k, n, K):
        tr = O.random_trellis(rng, k, n, K)
        suh = O.random_signs(rng, k)
        svh = O.random_signs(rng, n)
        return (tr, suh, svh, K), moe.Exl3Matrix(to_dev(tr), to_dev(suh), to_dev(svh), K)

    for e in range(E):
        kg, ku, kd = Ks[e]
        g, gd = mat(H, I, kg)
        u, ud = mat(H, I, ku)
        d, dd = mat(I, H, kd)
        np_exp.append(O.ExpertW(g, u, d))
        dev_exp.append(moe.Expert(gd, ud, dd))
    sh_np = sh_dev = None
    if shared_K:
        g, gd = mat(H, I, shared_K)
        u, ud = mat(H, I, shared_K)
        d, dd = mat(I, H, shared_K)
        sh_np, sh_dev = O.ExpertW(g, u, d), moe.Expert(gd, ud, dd)
    return np_exp, dev_exp, sh_np, sh_dev


@pytest.mark.parametrize("M", [1, 2, 4, 8, 19])
@pytest.mark.parametrize("shared", [False, True])
def test_moe_decode_matches_oracle(M, shared):
    rng = np.random.default_rng(50 + M + 7 * shared)
    E, H, I, topk, Lc = 12, 256, 256, 4, 10.0
    Ks = [tuple(int(v) for v in rng.integers(1, 5, size=3)) for _ in range(E)]   # mixed K per projection
    np_exp, dev_exp, sh_np, sh_dev = make_experts(rng, E, H, I, Ks, 4 if shared else None)
    table = moe.ExpertTable(dev_exp, sh_dev)
    x = rng.standard_normal((M, H)).astype(np.float16)
    ids = np.stack([rng.permutation(E)[:topk] for _ in range(M)]).astype(np.int32)
    if M > 2:
        ids[1, 2] = -1                                  # a dropped pick
    w = rng.random((M, topk)).astype(np.float32)
    out = moe.moe_forward(to_dev(x), to_dev(ids), to_dev(w), table, Lc)
    ref = O.moe_forward(x, ids, w, np_exp, Lc, sh_np)
    assert_close(out.cpu().numpy(), ref, what=f"moe M={M} shared={shared}")
    out2 = moe.moe_forward(to_dev(x), to_dev(ids), to_dev(w), table, Lc)
    assert torch.equal(out, out2), "MoE decode must be deterministic"
    # the phase-by-phase launches compute the same thing; any k-group count matches the oracle
    need = L.lib().exl3_moe_workspace_size(M, topk, E, H, I, int(shared))
    out3 = moe.moe_forward(to_dev(x), to_dev(ids), to_dev(w), table, Lc, events={}, workspace=poisoned(need))
    assert torch.equal(out, out3)
    for groups in (1, 3, 11):
        og = moe.moe_forward(to_dev(x), to_dev(ids), to_dev(w), table, Lc, n_ctas=groups, workspace=poisoned(need))
        assert_close(og.cpu().numpy(), ref, what=f"moe M={M} ctas={groups}")
        # split units handed to the ticket (finisher wait 0): the same bits
        assert L.lib().exl3_set_finisher_wait(0) == 0
        try:
            oh = moe.moe_forward(to_dev(x), to_dev(ids), to_dev(w), table, Lc, n_ctas=groups,
                                 workspace=poisoned(need))
            torch.cuda.synchronize()
        finally:
            L.lib().exl3_set_finisher_wait(20000)
        assert torch.equal(og, oh), f"moe M={M} ctas={groups}: hand-off path differs"


def test_moe_decode_no_clamp_and_bf16_input():
    rng = np.random.default_rng(8)
    E, H, I, topk = 6, 512, 128, 2
    np_exp, dev_exp, _, _ = make_experts(rng, E, H, I, [(3, 3, 3)] * E)
    table = moe.ExpertTable(dev_exp)
    xb = torch.randn((3, H), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    ids = np.array([[0, 5], [5, 0], [2, 2]], dtype=np.int32)        # duplicate pick in one row
    w = rng.random((3, topk)).astype(np.float32)
    out = moe.moe_forward(xb.to(DEV), to_dev(ids), to_dev(w), table, 0.0)
    ref = O.moe_forward(xb.float().numpy(), ids, w, np_exp, 0.0)
    assert_close(out.cpu().numpy(), ref, what="bf16 no clamp")


def test_moe_decode_benchmark_shape():
    """The benchmark's layer shape (H 2048, I 512, top-10 of many experts, 4 tokens): every GEMV unit is split over
    several CTAs, so the ticketed reduction carries the whole result."""
    rng = np.random.default_rng(123)
    E, H, I, topk, M = 48, 2048, 512, 10, 4
    np_exp, dev_exp, _, _ = make_experts(rng, E, H, I, [(3, 3, 3)] * E)
    table = moe.ExpertTable(dev_exp)
    x = rng.standard_normal((M, H)).astype(np.float16)
    ids = np.stack([rng.permutation(E)[:topk] for _ in range(M)]).astype(np.int32)
    w = rng.random((M, topk)).astype(np.float32)
    need = L.lib().exl3_moe_workspace_size(M, topk, E, H, I, 0)
    out = moe.moe_forward(to_dev(x), to_dev(ids), to_dev(w), table, 0.0, workspace=poisoned(need))
    ref = O.moe_forward(x, ids, w, np_exp, 0.0)
    assert_close(out.cpu().numpy(), ref, what="moe benchmark shape")


@pytest.mark.parametrize("shared", [False, True])
def test_moe_decode_token_without_picks(shared):
    """A token whose picks are all dropped gets zeros (or only the shared expert), from a poisoned workspace."""
    rng = np.random.default_rng(31)
    E, H, I, topk, M = 8, 256, 128, 3, 3
    np_exp, dev_exp, sh_np, sh_dev = make_experts(rng, E, H, I, [(3, 3, 3)] * E, 3 if shared else None)
    table = moe.ExpertTable(dev_exp, sh_dev)
    x = rng.standard_normal((M, H)).astype(np.float16)
    ids = np.array([[1, 4, 6], [-1, -1, -1], [6, 1, 2]], dtype=np.int32)
    w = rng.random((M, topk)).astype(np.float32)
    need = L.lib().exl3_moe_workspace_size(M, topk, E, H, I, int(shared))
    out = torch.full((M, H), float("nan"), device=DEV)
    moe.moe_forward(to_dev(x), to_dev(ids), to_dev(w), table, 0.0, out=out, workspace=poisoned(need))
    ref = O.moe_forward(x, ids, w, np_exp, 0.0, sh_np)
    assert_close(out.cpu().numpy(), ref, what=f"dropped token shared={shared}")
    if not shared:
        assert (out[1] == 0).all()


def test_moe_golden_expert_math():
    d = np.load(os.path.join(G, "moe_expert.npz"))
    H, I, Lc = int(d["H"]), int(d["I"]), float(d["act_limit"])
    Ks = [int(k) for k in d["Ks"]]
    dev_exp = []
    for e in range(len(Ks)):
        mats = [moe.Exl3Matrix(to_dev(d[f"{e}_{nm}_tr"]), to_dev(d[f"{e}_{nm}_suh"]), to_dev(d[f"{e}_{nm}_svh"]), Ks[e])
                for nm in ("gate", "up", "down")]
        dev_exp.append(moe.Expert(*mats))
    table = moe.ExpertTable(dev_exp)
    out = moe.moe_forward(to_dev(d["x"]), to_dev(d["sel"]), to_dev(d["w"]), table, Lc)
    assert_close(out.cpu().numpy(), d["out"], rel_tol=5e-3, what="golden MoE (reference pieces, fp64)")


def test_block_sparse_mlp_forward():
    """Module API: router (sigmoid + bias + residency) -> routed experts + shared expert, against the oracle."""
    rng = np.random.default_rng(21)
    E, H, I, topk = 16, 256, 128, 4
    np_exp, dev_exp, sh_np, sh_dev = make_experts(rng, E, H, I, [(2, 3, 3)] * E, 4)
    gate = (rng.standard_normal((H, E)) * 0.2).astype(np.float16)
    bias = (rng.standard_normal(E) * 0.05).astype(np.float32)
    res = np.where(rng.random(E) < 0.25, 0.1, 0.0).astype(np.float32)
    mlp = moe.BlockSparseMLP(dev_exp, to_dev(gate), topk, moe.ROUTE_SIGMOID, to_dev(bias), 2.5, act_limit=10.0,
                             shared=sh_dev, res=to_dev(res))
    x = rng.standard_normal((2, 3, H)).astype(np.float16)
    out = mlp.forward(to_dev(x))
    assert out.shape == (2, 3, H) and out.dtype == torch.float32
    logits = torch.matmul(to_dev(x).view(-1, H), to_dev(gate)).float().cpu().numpy()
    ids, w, _ = O.route(logits, O.ROUTE_SIGMOID, topk, bias=bias, res=res, scale=2.5)
    ref = O.moe_forward(x.reshape(-1, H), ids, w, np_exp, 10.0, sh_np)
    assert_close(out.view(-1, H).cpu().numpy(), ref, what="BlockSparseMLP")


def test_decode_step_graph_replay_matches_oracle():
    """A two-layer decode step (router with residency bias -> moe_forward per layer) captured in one CUDA graph and
    replayed twice with new inputs copied into its static buffers, as a serving loop does (the reference captures
    per-block graphs, glm/xpu/glm_xpu/block_graphs.py:275-312): each replay equals the oracle."""
    rng = np.random.default_rng(77)
    E, H, I, topk, M, Lc, layers = 16, 256, 128, 4, 3, 10.0, 2
    nets = [make_experts(rng, E, H, I, [(2, 3, 3)] * E, 3) for _ in range(layers)]
    tables = [moe.ExpertTable(n[1], n[3]) for n in nets]
    res = np.where(rng.random(E) < 0.25, 0.1, 0.0).astype(np.float32)
    res_d = to_dev(res)
    x = torch.zeros((layers, M, H), dtype=torch.half, device=DEV)
    lg = torch.zeros((layers, M, E), dtype=torch.float32, device=DEV)
    out = torch.zeros((layers, M, H), dtype=torch.float32, device=DEV)

    def step():
        for l in range(layers):
            ids, w, _ = ops.route(lg[l], O.ROUTE_SIGMOID, topk, res=res_d, scale=2.5)
            moe.moe_forward(x[l], ids, w, tables[l], Lc, out=out[l])

    step()                                               # eager warm-up: attributes, workspaces
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for rep in range(2):
        xn = rng.standard_normal((layers, M, H)).astype(np.float16)
        ln = rng.standard_normal((layers, M, E)).astype(np.float32)
        x.copy_(to_dev(xn))
        lg.copy_(to_dev(ln))
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for l in range(layers):
            rid, rw, _ = O.route(ln[l], O.ROUTE_SIGMOID, topk, res=res, scale=2.5)
            ref = O.moe_forward(xn[l], rid, rw, nets[l][0], Lc, nets[l][2])
            assert_close(out[l].cpu().numpy(), ref, what=f"graph replay {rep} layer {l}")
    del graph
