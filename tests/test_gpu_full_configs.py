"""Parity at the BASELINE configurations' full sizes, through the C ABI:

* config 3 (GLM-like MoE decode layer): H 6144, 160 routed experts + a shared expert (K 4), I 1536, expert K 2 / 3
  (2.5 bits average), top-8 sigmoid router with +0.1 on a seeded resident 25 % subset, scale 2.5, act_limit 10;
* config 5 (DeepSeek-V4-like MoE prefill): 8192 tokens, H 7168, 256 routed experts + a shared expert, I 2048,
  K 1 / 2 per projection with P(2) = 0.62, top-8 sqrt-softplus router with a gate bias, bf16 activations;
* config 2's dense shapes at K 2..5 and batch 1 / 2 / 4, with unit-rms outputs checked at the literal 1e-2 max-abs.

Routed ids are compared bit for bit with the oracle's router. Layer outputs are compared with tests/torch_ref.py:
the oracle's rounding points in torch on the bit-exact dequantised weights (every token), which is itself pinned to
the numpy oracle on the same shapes (test_torch_ref_matches_oracle). Measured errors are appended, one JSON object
per line, to the file named by $EXL3_PARITY_LOG when it is set."""
import json
import os

import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import moe, ops
from oracle import oracle as O
from tests import torch_ref as T
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
PARITY_LOG = os.environ.get("EXL3_PARITY_LOG")


@pytest.fixture(autouse=True)
def _status_clean():
    L.lib().exl3_device_status(1)
    yield
    torch.cuda.synchronize()
    assert L.lib().exl3_device_status(0) == 0, "a device-side wait timed out"


def record(what, out, ref):
    """Relative L2 error, max |err| and reference rms of one comparison (for the parity record)."""
    o = out.double()
    r = ref.double()
    rel = float((o - r).norm() / max(float(r.norm()), 1e-30))
    mx = float((o - r).abs().max())
    rms = float(r.pow(2).mean().sqrt())
    if PARITY_LOG:
        with open(PARITY_LOG, "a") as f:
            f.write(json.dumps({"what": what, "rel_l2": rel, "max_abs": mx, "ref_rms": rms}) + "\n")
    return rel, mx, rms


def mat(gen, k, n, K, svh_scale=1.0):
    tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=DEV, generator=gen)
    s1 = (torch.randint(0, 2, (k,), device=DEV, generator=gen) * 2 - 1).half()
    s2 = ((torch.randint(0, 2, (n,), device=DEV, generator=gen) * 2 - 1) * svh_scale).half()
    return moe.Exl3Matrix(tr, s1, s2, K)


def to_np_mat(m: moe.Exl3Matrix):
    return (m.trellis.cpu().numpy().view(np.uint16), m.suh.cpu().numpy(), m.svh.cpu().numpy(), int(m.K))


# ------------------------------------------------------------------------------------------------ the torch reference

@pytest.mark.parametrize("H,I,Ks", [(6144, 1536, (2, 3, 3)), (7168, 2048, (2, 1, 2))])
def test_torch_ref_matches_oracle(H, I, Ks):
    """tests/torch_ref.py against the numpy oracle on one expert of config 3 / config 5 (two tokens)."""
    g = torch.Generator(device=DEV).manual_seed(H + I)
    ex = moe.Expert(mat(g, H, I, Ks[0]), mat(g, H, I, Ks[1]), mat(g, I, H, Ks[2]))
    x = torch.randn((2, H), device=DEV, generator=g).half()
    ref_t = T.TorchExpert(ex).forward(x, 10.0)
    ref_o = O.expert_forward(x.cpu().numpy(), O.ExpertW(*(to_np_mat(m) for m in (ex.gate, ex.up, ex.down))), 10.0)
    rel, mx, rms = record(f"torch_ref vs oracle H{H} I{I}", ref_t, torch.from_numpy(ref_o).to(DEV))
    assert rel < 1e-5, rel


# ------------------------------------------------------------------------------------------------ config 3

def glm_layer(unit_rms: bool):
    """The config-3 layer: 160 experts with K 2 / 3 per expert (alternating, 2.5 bits average), shared expert K 4.
    unit_rms scales every svh by 1/sqrt(k) so that each linear's output has about unit rms."""
    H, E, I = 6144, 160, 1536
    g = torch.Generator(device=DEV).manual_seed(3)
    sg, sd = (1 / np.sqrt(H), 1 / np.sqrt(I)) if unit_rms else (1.0, 1.0)
    experts = []
    for e in range(E):
        K = (2, 3)[e % 2]
        experts.append(moe.Expert(mat(g, H, I, K, sg), mat(g, H, I, K, sg), mat(g, I, H, K, sd)))
    shared = moe.Expert(mat(g, H, I, 4, sg), mat(g, H, I, 4, sg), mat(g, I, H, 4, sd))
    return H, E, I, experts, shared, g


@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("unit_rms", [False, True])
def test_glm_decode_layer_config3(M, unit_rms):
    H, E, I, experts, shared, g = glm_layer(unit_rms)
    table = moe.ExpertTable(experts, shared)
    logits = torch.randn((M, E), device=DEV, generator=g)
    res = torch.where(torch.rand(E, device=DEV, generator=g) < 0.25, 0.1, 0.0).float()
    bias = torch.randn(E, device=DEV, generator=g) * 0.05
    ids, w, _ = ops.route(logits, L.ROUTE_SIGMOID, 8, bias=bias, res=res, scale=2.5)
    rid, rw, _ = O.route(logits.cpu().numpy(), O.ROUTE_SIGMOID, 8, bias=bias.cpu().numpy(), res=res.cpu().numpy(),
                         scale=2.5)
    assert np.array_equal(ids.cpu().numpy(), rid), "routed ids must be bit-exact"
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    x = torch.randn((M, H), device=DEV, generator=g).half()
    need = L.lib().exl3_moe_workspace_size(M, 8, E, H, I, 1)
    ws = torch.full((need,), 255, dtype=torch.uint8, device=DEV)
    out = moe.moe_forward(x, ids, w, table, 10.0, workspace=ws)
    ref = T.moe_forward(x, ids, w, experts, 10.0, shared)
    rel, mx, rms = record(f"glm config3 M{M} unit_rms={unit_rms}", out, ref)
    assert_close(out.cpu().numpy(), ref.cpu().numpy(), what=f"glm layer M={M}")
    if unit_rms:
        assert 0.1 < rms < 10, rms
        assert mx <= 1e-2, f"max abs error {mx:.3e} > 1e-2 on unit-rms outputs"
    out2 = moe.moe_forward(x, ids, w, table, 10.0, workspace=ws)
    assert torch.equal(out, out2)


# ------------------------------------------------------------------------------------------------ config 5

def test_dsv4_prefill_config5():
    H, E, I, topk, T_ = 7168, 256, 2048, 8, 8192
    g = torch.Generator(device=DEV).manual_seed(5)
    experts = []
    for e in range(E):
        rng = np.random.default_rng(1000 + e)
        Ks = [2 if rng.random() < 0.62 else 1 for _ in range(3)]
        experts.append(moe.Expert(mat(g, H, I, Ks[0]), mat(g, H, I, Ks[1]), mat(g, I, H, Ks[2])))
    shared = moe.Expert(mat(g, H, I, 2), mat(g, H, I, 2), mat(g, I, H, 2))
    table = moe.ExpertTable(experts, shared)
    x = torch.randn((T_, H), device=DEV, generator=g).to(torch.bfloat16)
    logits = torch.randn((T_, E), device=DEV, generator=g)
    bias = torch.randn(E, device=DEV, generator=g) * 0.1
    ids, w, _ = ops.route(logits, L.ROUTE_SQRT_SOFTPLUS, topk, bias=bias, scale=2.5)
    rid, rw, _ = O.route(logits.cpu().numpy(), O.ROUTE_SQRT_SOFTPLUS, topk, bias=bias.cpu().numpy(), scale=2.5)
    assert np.array_equal(ids.cpu().numpy(), rid), "routed ids must be bit-exact"
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    need = L.lib().exl3_moe_prefill_workspace_size(T_, topk, E, H, I, 1)
    ws = torch.full((need,), 255, dtype=torch.uint8, device=DEV)
    out = moe.moe_prefill(x, ids, w, table, 10.0, workspace=ws)
    del ws
    ref = T.moe_forward(x, ids, w, experts, 10.0, shared)
    rel, mx, rms = record("dsv4 config5 prefill 8192 tokens", out, ref)
    assert_close(out.cpu().numpy(), ref.cpu().numpy(), what="config-5 prefill")
    # per token as well: no token may carry a large error hidden by the layer-wide norm
    tok_rel = ((out - ref).norm(dim=1) / ref.norm(dim=1).clamp_min(1e-30)).max().item()
    assert tok_rel < 2e-3, tok_rel


# ------------------------------------------------------------------------------------------------ config 2

@pytest.mark.parametrize("k,n", [(5120, 25600), (25600, 5120), (5120, 5120)])
@pytest.mark.parametrize("K", [2, 3, 4, 5])
def test_dense_config2_unit_rms(k, n, K):
    """Dense decode GEMV at config 2's shapes, batch 1 / 2 / 4, svh = +-1/sqrt(k): unit-rms outputs, literal
    2e-3 relative and 1e-2 max-abs against the torch reference on the dequantised weights."""
    g = torch.Generator(device=DEV).manual_seed(k + n + K)
    m = mat(g, k, n, K, 1 / np.sqrt(k))
    W = T.w_hat(m.trellis, K)
    bc = ops.BC_LinearEXL3(m.trellis, m.suh, m.svh, K, None, False, True, None)
    for M in (1, 2, 4):
        x = torch.randn((M, k), device=DEV, generator=g).half()
        y = bc.run_alloc(x, n, True)
        ref = T.linear(x, W, m.suh, m.svh, torch.float32)
        rel, mx, rms = record(f"dense {k}x{n} K{K} M{M}", y, ref)
        assert rel <= 2e-3 and mx <= 1e-2, (rel, mx, rms)
