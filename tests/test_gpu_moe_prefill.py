"""GPU parity of the tcgen05 MoE prefill (exl3_moe_prefill): against the CPU oracle on a small batch and against
the oracle-checked decode path (exl3_moe_decode) at prefill sizes; mixed bit widths per projection, shared expert,
dropped picks, experts split into several 320-row items."""
import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import moe
from oracle import oracle as O
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def to_dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return (t.view(torch.int16) if t.dtype == torch.uint16 else t).to(DEV)


@pytest.fixture(autouse=True)
def _status_clean():
    L.lib().exl3_device_status(1)
    yield
    torch.cuda.synchronize()
    assert L.lib().exl3_device_status(0) == 0, "a device-side wait timed out"


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


@pytest.mark.parametrize("shared", [False, True])
def test_moe_prefill_matches_oracle(shared):
    rng = np.random.default_rng(70 + shared)
    E, H, I, topk, M, Lc = 6, 256, 128, 3, 24, 10.0
    Ks = [tuple(int(v) for v in rng.integers(1, 5, size=3)) for _ in range(E)]
    np_exp, dev_exp, sh_np, sh_dev = make_experts(rng, E, H, I, Ks, 3 if shared else None)
    table = moe.ExpertTable(dev_exp, sh_dev)
    x = rng.standard_normal((M, H)).astype(np.float16)
    ids = np.stack([rng.permutation(E)[:topk] for _ in range(M)]).astype(np.int32)
    ids[2, 1] = -1
    w = rng.random((M, topk)).astype(np.float32)
    out = moe.moe_prefill(to_dev(x), to_dev(ids), to_dev(w), table, Lc)
    ref = O.moe_forward(x, ids, w, np_exp, Lc, sh_np)
    assert_close(out.cpu().numpy(), ref, what=f"moe prefill shared={shared}")


@pytest.mark.parametrize("M,E,topk,shared", [(600, 8, 4, True), (1100, 16, 8, False)])
def test_moe_prefill_matches_decode_path(M, E, topk, shared):
    """Hundreds of rows per expert (several 320-row items), against the decode kernels on the same inputs."""
    rng = np.random.default_rng(M + E)
    H, I, Lc = 512, 256, 10.0
    Ks = [(2, 3, 2) if e % 2 else (3, 2, 4) for e in range(E)]
    _, dev_exp, _, sh_dev = make_experts(rng, E, H, I, Ks, 4 if shared else None)
    table = moe.ExpertTable(dev_exp, sh_dev)
    x = torch.randn((M, H), generator=torch.Generator().manual_seed(M)).to(torch.bfloat16).to(DEV)
    ids = torch.from_numpy(np.stack([rng.permutation(E)[:topk] for _ in range(M)]).astype(np.int32)).to(DEV)
    ids[::7, 0] = 1                                      # a hot expert
    w = torch.rand((M, topk), generator=torch.Generator().manual_seed(1)).to(DEV)
    need = L.lib().exl3_moe_prefill_workspace_size(M, topk, E, H, I, int(shared))
    ws = torch.full((need,), 255, dtype=torch.uint8, device=DEV)          # poisoned: nothing may depend on it
    out = moe.moe_prefill(x, ids, w, table, Lc, workspace=ws)
    ref = torch.cat([moe.moe_forward(x[i:i + 8], ids[i:i + 8], w[i:i + 8], table, Lc) for i in range(0, M, 8)])
    assert_close(out.cpu().numpy(), ref.cpu().numpy(), what=f"moe prefill vs decode M={M}")
    out2 = moe.moe_prefill(x, ids, w, table, Lc, workspace=ws)
    assert torch.equal(out, out2)
