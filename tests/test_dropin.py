"""The drop-in boundary: exllamav3's BlockSparseMLP patched by exl3_b200.install() (the seam of
glm/xpu/glm_xpu/moe_patch.py:15-94), and the torch custom ops (torch.ops.exl3_b200.*) with their fake (meta)
implementations, as the reference registers its linear (glm/xpu/exl3xpu/ops.py:119-129).

exllamav3 is not installed here: a stand-in class carries its attribute contract (gates / ups / downs as Linear
modules wrapping an EXL3 inner with trellis / suh / svh / K / mcg / mul1, routing_fn(bsz, routing_cfg, y, params),
shared_experts, hidden_size, act_limit, load(device)). The GPU tests run its forward at a decode batch (4 rows, the
decode kernels) and a prefill batch (600 rows, the tcgen05 kernels) against the oracle."""
import numpy as np
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import exl3_b200
from exl3_b200 import _lib as L
from exl3_b200 import exllama_patch, ops
from oracle import oracle as O
from tests.tolerance import assert_close

DEV = "cuda:0"


class Exl3Inner:
    """exllamav3 LinearEXL3's attributes, read by name."""

    def __init__(self, trellis, suh, svh, K, mcg=False, mul1=True):
        self.trellis, self.suh, self.svh, self.K, self.mcg, self.mul1 = trellis, suh, svh, K, mcg, mul1


class Linear:
    def __init__(self, inner):
        self.inner = inner


class GatedMLP:
    def __init__(self, gate, up, down):
        self.gate, self.up, self.down = gate, up, down

    def forward(self, x, params):
        raise AssertionError("the shared expert runs inside the table")


class RoutingCfg:
    def __init__(self, gate_tensor, bias, topk, scale):
        self.gate_tensor, self.e_score_correction_bias, self.top_k, self.routed_scaling_factor = (
            gate_tensor, bias, topk, scale)


class BlockSparseMLP:
    """Stand-in for exllamav3.modules.block_sparse_mlp.BlockSparseMLP (its attribute contract, no kernels)."""

    def __init__(self, gates, ups, downs, shared, routing_cfg, hidden_size, act_limit):
        self.gates, self.ups, self.downs = gates, ups, downs
        self.shared_experts = shared
        self.routing_cfg = routing_cfg
        self.hidden_size = hidden_size
        self.num_experts = len(gates)
        self.num_experts_per_tok = routing_cfg.top_k
        self.act_limit = act_limit
        self.loaded_on = None
        self.last_routing = None

        def routing_fn(bsz, cfg, y, params):
            # exllamav3's routing returns int64 ids and fp16 weights; the routing GEMV + top-k is this package's
            ids, w, _ = ops.route_hidden(y, cfg.gate_tensor.t().contiguous(), L.ROUTE_SIGMOID, cfg.top_k,
                                         bias=cfg.e_score_correction_bias, scale=cfg.routed_scaling_factor,
                                         ids_dtype=torch.int64)
            self.last_routing = (ids, w.half())
            return ids, w.half()

        self.routing_fn = routing_fn

    def load(self, device, **kwargs):
        self.loaded_on = device

    def forward(self, x, params, out_dtype=None):
        raise AssertionError("exllamav3's own forward must be replaced")


def test_install_patches_the_class_once():
    class Cls(BlockSparseMLP):
        pass

    orig_load = Cls.load
    out = exl3_b200.install(Cls)
    assert out is Cls and Cls._exl3_b200_installed
    assert Cls.load is not orig_load and Cls._exl3_b200_orig_load is orig_load
    assert Cls.forward is exllama_patch._forward
    exl3_b200.install(Cls)                                      # idempotent
    assert Cls._exl3_b200_orig_load is orig_load


def test_expert_linears_are_read_by_name():
    t = torch.zeros((16, 8, 48), dtype=torch.int16)
    m = exllama_patch._matrix(Linear(Exl3Inner(t, None, torch.zeros(128), 3)))
    assert (m.k, m.n, m.K) == (256, 128, 3)
    with pytest.raises(L.Exl3Error):
        exllama_patch._matrix(Linear(Exl3Inner(t, None, torch.zeros(128), 3, mcg=True)))
    with pytest.raises(L.Exl3Error):
        exllama_patch._matrix(object())


def test_custom_op_fakes_give_output_shapes():
    with FakeTensorMode():
        x = torch.empty(5, 2048, dtype=torch.half, device="cuda")
        y = torch.ops.exl3_b200.linear(x, torch.empty(4, 128, 384, dtype=torch.int16, device="cuda"), None,
                                       torch.empty(512, dtype=torch.half, device="cuda"), 3, False)
        assert y.shape == (5, 512) and y.dtype == torch.float16
        ids, w = torch.ops.exl3_b200.route(torch.empty(5, 160, device="cuda"), 0, 8, None, None, None, 2.5, True)
        assert ids.shape == (5, 8) and ids.dtype == torch.int32 and w.dtype == torch.float32
        o = torch.ops.exl3_b200.moe(x, ids, w, torch.empty(64, dtype=torch.uint8, device="cuda"), 160, 512, True,
                                    10.0, False)
        assert o.shape == (5, 2048) and o.dtype == torch.float32


# ------------------------------------------------------------------------------------------------ GPU

def to_dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return (t.view(torch.int16) if t.dtype == torch.uint16 else t).to(DEV)


def make_module(rng, E, H, I, topk, cls):
    np_exp, mods = [], []

    def lin(k, n, K):
        tr, s1, s2 = O.random_trellis(rng, k, n, K), O.random_signs(rng, k), O.random_signs(rng, n)
        return (tr, s1, s2, K), Linear(Exl3Inner(to_dev(tr), to_dev(s1), to_dev(s2), K))

    for e in range(E):
        K = 2 + e % 2
        (g, gm), (u, um), (d, dm) = lin(H, I, K), lin(H, I, K), lin(I, H, 3)
        np_exp.append(O.ExpertW(g, u, d))
        mods.append((gm, um, dm))
    (g, gm), (u, um), (d, dm) = lin(H, I, 4), lin(H, I, 4), lin(I, H, 4)
    sh_np, sh = O.ExpertW(g, u, d), GatedMLP(gm, um, dm)
    gate = to_dev((rng.standard_normal((H, E)) * 0.2).astype(np.float16))
    bias = to_dev((rng.standard_normal(E) * 0.05).astype(np.float32))
    mod = cls([m[0] for m in mods], [m[1] for m in mods], [m[2] for m in mods], sh, RoutingCfg(gate, bias, topk, 2.5),
              H, 10.0)
    return mod, np_exp, sh_np


@pytest.mark.gpu
@pytest.mark.parametrize("bsz", [4, 600])
def test_patched_block_sparse_mlp_matches_oracle(bsz):
    class Cls(BlockSparseMLP):
        pass

    exl3_b200.install(Cls)
    rng = np.random.default_rng(bsz)
    E, H, I, topk = 16, 256, 128, 4
    mod, np_exp, sh_np = make_module(rng, E, H, I, topk, Cls)
    mod.load(DEV)
    assert mod.loaded_on == DEV and mod._exl3_shared_in_table
    x = rng.standard_normal((1, bsz, H)).astype(np.float16)
    out = mod.forward(to_dev(x), {})
    assert out.shape == (1, bsz, H) and out.dtype == torch.float32
    ids, w = mod.last_routing
    ref = O.moe_forward(x.reshape(bsz, H), ids.cpu().numpy().astype(np.int32), w.float().cpu().numpy(), np_exp, 10.0,
                        sh_np)
    assert_close(out.view(bsz, H).cpu().numpy(), ref, what=f"patched BlockSparseMLP bsz={bsz}")
    assert L.lib().exl3_device_status(0) == 0


@pytest.mark.gpu
def test_custom_ops_trace_under_torch_compile():
    """The ops are single opaque nodes: a fullgraph torch.compile (aot_eager backend, no code generation) traces them
    through their fakes and gives the eager results bit for bit."""
    g = torch.Generator(device=DEV).manual_seed(9)
    k, n, K = 512, 256, 3
    tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=DEV, generator=g)
    pk = ops.pack(tr, K)
    suh = (torch.randint(0, 2, (k,), device=DEV, generator=g) * 2 - 1).half()
    svh = (torch.randint(0, 2, (n,), device=DEV, generator=g) * 2 - 1).half()
    x = torch.randn((3, k), device=DEV, generator=g).half()

    def fn(x):
        y = torch.ops.exl3_b200.linear(x, pk, suh, svh, K, True)
        ids, w = torch.ops.exl3_b200.route(y[:, :64].contiguous(), L.ROUTE_SOFTMAX, 4, None, None, None, 1.0, True)
        return y * 2.0, ids, w

    eager = fn(x)
    comp = torch.compile(fn, backend="aot_eager", fullgraph=True)(x)
    for a, b in zip(eager, comp):
        assert torch.equal(a, b)
    bc = ops.BC_LinearEXL3(tr, suh, svh, K, None, False, True, None)
    assert torch.equal(eager[0] / 2.0, bc.run_alloc(x, n, True))
