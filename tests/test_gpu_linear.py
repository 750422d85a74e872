"""GPU parity of the dense EXL3 path (dequant, Hadamard, fused GEMV, BC_LinearEXL3) against the CPU oracle and the
reference's golden vectors. Decoded weights must be bit-exact; linear outputs within the BASELINE tolerance."""
import os

import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import ops
from oracle import oracle as O
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda:0"


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if t.dtype == torch.uint16:
        t = t.view(torch.int16)
    return t.to(DEV) if dtype is None else t.to(DEV, dtype)


def rand_linear(rng, k, n, K):
    tr = O.random_trellis(rng, k, n, K)
    suh = O.random_signs(rng, k)
    svh = (O.random_signs(rng, n).astype(np.float32) * rng.uniform(0.5, 1.5, n)).astype(np.float16)
    return tr, suh, svh


def poisoned_workspace(nbytes):
    """A workspace of 0xFF bytes (NaN as fp32, -1 as int32): nothing may depend on its previous contents."""
    return torch.full((nbytes,), 255, dtype=torch.uint8, device=DEV)


@pytest.fixture(autouse=True)
def _status_clean():
    L.lib().exl3_device_status(1)
    yield
    torch.cuda.synchronize()
    assert L.lib().exl3_device_status(0) == 0, "a device-side wait timed out"


@pytest.mark.parametrize("K", range(1, 9))
def test_dequant_bitexact(K):
    rng = np.random.default_rng(100 + K)
    k, n = 256, 384
    tr = O.random_trellis(rng, k, n, K)
    ref = O.w_hat(tr, K)
    w = torch.empty((k, n), dtype=torch.half, device=DEV)
    ops.exl3_reconstruct(to_dev(tr), w, 0, K)
    assert np.array_equal(w.cpu().numpy().view(np.uint16), ref.view(np.uint16))
    # column slice (reconstruct_slice semantics), written into a wider buffer
    wbuf = torch.zeros((k, 256), dtype=torch.half, device=DEV)
    ops.exl3_reconstruct(to_dev(tr), wbuf[:, :128], 128, K)
    assert np.array_equal(wbuf[:, :128].cpu().numpy().view(np.uint16), ref[:, 128:256].view(np.uint16))
    assert (wbuf[:, 128:] == 0).all()


@pytest.mark.parametrize("K", [1, 3, 8])
def test_pack_is_the_column_block_permutation(K):
    rng = np.random.default_rng(K)
    k, n = 64, 384
    tr = O.random_trellis(rng, k, n, K)
    pk = ops.pack(to_dev(tr), K).cpu().numpy().view(np.uint16)
    exp = tr.reshape(k // 16, n // 128, 8 * 16 * K).transpose(1, 0, 2)
    assert np.array_equal(pk.reshape(exp.shape), exp)
    tr2 = O.random_trellis(rng, k, n, 2)
    gu = ops.pack_gateup(to_dev(tr), to_dev(tr2), K, 2).cpu().numpy().view(np.uint16)
    exp2 = np.concatenate([exp, tr2.reshape(k // 16, n // 128, 8 * 32).transpose(1, 0, 2)], axis=2)
    assert np.array_equal(gu.reshape(exp2.shape), exp2)


@pytest.mark.parametrize("K", range(1, 9))
def test_dequant_golden(K):
    d = np.load(os.path.join(G, f"w_hat_K{K}.npz"))
    tr = d["trellis"]
    k, n = tr.shape[0] * 16, tr.shape[1] * 16
    w = torch.empty((k, n), dtype=torch.half, device=DEV)
    ops.exl3_reconstruct(to_dev(tr), w, 0, K)
    assert np.array_equal(w.cpu().numpy().view(np.uint16), d["w_hat"].view(np.uint16))


def test_had_r_128_bitexact():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((6, 512)).astype(np.float16)
    pre = O.random_signs(rng, 512)
    post = rng.uniform(-2, 2, 512).astype(np.float16)
    out = torch.empty((6, 512), dtype=torch.half, device=DEV)
    ops.had_r_128(to_dev(x), out, to_dev(pre), None, 1.0)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), O.had_r_128(x, pre=pre).view(np.uint16))
    ops.had_r_128(to_dev(x), out, None, to_dev(post), 1.0)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), O.had_r_128(x, post=post).view(np.uint16))
    x32 = rng.standard_normal((3, 256)).astype(np.float32)
    o32 = torch.empty((3, 256), dtype=torch.float32, device=DEV)
    ops.had_r_128(to_dev(x32), o32, None, to_dev(post[:256]), 1.0)
    assert np.array_equal(o32.cpu().numpy(), O.had_r_128(x32, post=post[:256]))
    # golden: reference had_r_128 outputs (matmul order): within one fp16 ulp
    d = np.load(os.path.join(G, "had_r_128.npz"))
    o16 = torch.empty(d["x16"].shape, dtype=torch.half, device=DEV)
    ops.had_r_128(to_dev(d["x16"]), o16, to_dev(d["pre"]), None, 1.0)
    diff = np.abs(o16.cpu().numpy().view(np.int16).astype(np.int32) - d["o16"].view(np.int16).astype(np.int32))
    assert diff.max() <= 1


@pytest.mark.parametrize("K", range(1, 9))
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
def test_gemv_matches_oracle(K, M):
    rng = np.random.default_rng(1000 * K + M)
    k, n = 512, 384
    tr, suh, svh = rand_linear(rng, k, n, K)
    x = rng.standard_normal((M, k)).astype(np.float16)
    for y_dt, np_dt in ((torch.float32, np.float32), (torch.float16, np.float16)):
        y = torch.full((M, n), float("nan"), dtype=y_dt, device=DEV)
        ops.exl3_gemv(to_dev(x), ops.pack(to_dev(tr), K), to_dev(suh), to_dev(svh), K, y)
        ref = O.exl3_linear(x, tr, suh, svh, K, np_dt)
        assert_close(y.float().cpu().numpy(), ref.astype(np.float32), what=f"gemv K={K} M={M} {y_dt}")


@pytest.mark.parametrize("M", [4, 13])
@pytest.mark.parametrize("groups", [1, 2, 3, 7, 64, 0])
def test_gemv_cta_counts_are_consistent(groups, M):
    """Any CTA count (1 = every unit whole in one CTA; many = units split over CTAs and reduced through the tickets)
    gives the oracle's result, bit-identically from call to call; also with two row groups (13 rows)."""
    rng = np.random.default_rng(77)
    k, n, K = 1024, 256, 3
    tr, suh, svh = rand_linear(rng, k, n, K)
    x = rng.standard_normal((M, k)).astype(np.float16)
    y = torch.full((M, n), float("nan"), dtype=torch.float32, device=DEV)
    pk = ops.pack(to_dev(tr), K)
    ws = poisoned_workspace(L.lib().exl3_gemv_workspace_size(M, k, n))
    ops.exl3_gemv(to_dev(x), pk, to_dev(suh), to_dev(svh), K, y, n_ctas=groups, workspace=ws)
    assert_close(y.cpu().numpy(), O.exl3_linear(x, tr, suh, svh, K, np.float32), what=f"groups {groups}")
    y2 = torch.full_like(y, float("nan"))
    ops.exl3_gemv(to_dev(x), pk, to_dev(suh), to_dev(svh), K, y2, n_ctas=groups, workspace=ws)
    assert torch.equal(y, y2), "fixed-order split-unit reduction must be deterministic"


@pytest.mark.parametrize("groups", [3, 7, 64, 0])
def test_gemv_finisher_hand_off_gives_the_same_bits(groups):
    """Split units finished by the ticket hand-off (finisher wait 0: the first contributor never waits for the
    others) give bit for bit the result of the default path, for the linear and the MoE decode GEMVs."""
    rng = np.random.default_rng(78)
    k, n, K, M = 1024, 384, 3, 5
    tr, suh, svh = rand_linear(rng, k, n, K)
    x = to_dev(rng.standard_normal((M, k)).astype(np.float16))
    pk = ops.pack(to_dev(tr), K)
    outs = []
    for wait in (20000, 0):
        assert L.lib().exl3_set_finisher_wait(wait) == 0
        try:
            y = torch.full((M, n), float("nan"), dtype=torch.float32, device=DEV)
            ops.exl3_gemv(x, pk, to_dev(suh), to_dev(svh), K, y, n_ctas=groups)
            torch.cuda.synchronize()
            outs.append(y)
        finally:
            L.lib().exl3_set_finisher_wait(20000)
    assert torch.equal(outs[0], outs[1])
    assert_close(outs[1].cpu().numpy(), O.exl3_linear(x.cpu().numpy(), tr, suh, svh, K, np.float32), what="hand-off")
    assert L.lib().exl3_device_status(0) == 0


def test_gemv_bf16_input_and_output():
    rng = np.random.default_rng(9)
    k, n, K, M = 256, 256, 4, 2
    tr, suh, svh = rand_linear(rng, k, n, K)
    xb = torch.randn((M, k), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    y = torch.empty((M, n), dtype=torch.bfloat16, device=DEV)
    ops.exl3_gemv(xb.to(DEV), ops.pack(to_dev(tr), K), to_dev(suh), to_dev(svh), K, y)
    ref = O.exl3_linear(xb.float().numpy(), tr, suh, svh, K, np.float32)
    assert_close(y.float().cpu().numpy(), ref, rel_tol=5e-3, what="bf16")     # bf16 output rounding (8 bits)


@pytest.mark.parametrize("K", [2, 3, 4, 5, 6])
def test_linear_golden(K):
    """The reference's units.py ref_linear outputs (fp64) through the CUDA path, at the reference's tolerance."""
    d = np.load(os.path.join(G, f"linear_K{K}.npz"))
    bc = ops.BC_LinearEXL3(to_dev(d["trellis"]), to_dev(d["suh"]), to_dev(d["svh"]), K, None, False, True, None)
    y = bc.run_alloc(to_dev(d["x"]), bc.out_features, True)
    rel = np.linalg.norm(y.cpu().numpy() - d["y"]) / np.linalg.norm(d["y"])
    assert rel < 5e-3          # glm/xpu/tests/units.py:104


@pytest.mark.parametrize("M", [1, 5, 12, 20, 32, 100])
def test_bc_linear_paths(M):
    rng = np.random.default_rng(M)
    k, n, K = 256, 640, 4
    tr, suh, svh = rand_linear(rng, k, n, K)
    bc = ops.BC_LinearEXL3(to_dev(tr), to_dev(suh), to_dev(svh), K, None, False, True, None)
    x = rng.standard_normal((M, k)).astype(np.float16)
    y32 = bc.run_alloc(to_dev(x), n, True)
    assert_close(y32.cpu().numpy(), O.exl3_linear(x, tr, suh, svh, K, np.float32), what=f"fp32 M={M}")
    y16 = bc.run_alloc(to_dev(x), n, False)
    assert y16.dtype == torch.float16
    assert_close(y16.float().cpu().numpy(), O.exl3_linear(x, tr, suh, svh, K, np.float16).astype(np.float32),
                 rel_tol=3e-3, what=f"fp16 M={M}")


def test_silu_mul_golden():
    d = np.load(os.path.join(G, "silu_mul.npz"))
    g, u = to_dev(d["g"]), to_dev(d["u"])
    for L_, key in ((10.0, "z10"), (0.0, "z0")):
        z = torch.empty_like(g)
        ops.silu_mul(g, u, z, L_)
        got = z.cpu().numpy().view(np.uint16).astype(np.int32)
        exp = d[key].view(np.uint16).astype(np.int32)
        assert np.abs(got - exp).max() <= 1 and (got != exp).mean() < 0.01   # expf vs libm: last-bit at most


@pytest.mark.parametrize("k,n,K", [(5120, 25600, 2), (25600, 5120, 3), (5120, 5120, 5)])
def test_gemv_full_size_against_torch(k, n, K):
    """BASELINE dense shapes: the GEMV against a torch fp32 matmul of the (bit-exact) GPU-dequantised weights and the
    GPU-rotated input; plus a decode checksum of one slice against the oracle."""
    g = torch.Generator(device=DEV).manual_seed(k + n + K)
    tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=DEV, generator=g)
    suh = (torch.randint(0, 2, (k,), device=DEV, generator=g) * 2 - 1).half()
    svh = (torch.randint(0, 2, (n,), device=DEV, generator=g) * 2 - 1).half()
    x = torch.randn((4, k), device=DEV, generator=g).half()
    y = torch.full((4, n), float("nan"), dtype=torch.float32, device=DEV)
    ops.exl3_gemv(x, ops.pack(tr, K), suh, svh, K, y)
    W = torch.empty((k, n), dtype=torch.half, device=DEV)
    ops.exl3_reconstruct(tr, W, 0, K)
    xh = torch.empty_like(x)
    ops.had_r_128(x, xh, suh, None, 1.0)
    acc = xh.float() @ W.float()
    ref = torch.empty_like(acc)
    ops.had_r_128(acc, ref, None, svh.float(), 1.0)
    assert_close(y.cpu().numpy(), ref.cpu().numpy(), what=f"{k}x{n} K={K}")
    # bit-exact decode of a 256-column slice at full k
    sl = O.w_hat_cols(tr.cpu().numpy().view(np.uint16), K, 256, 512)
    assert np.array_equal(W[:, 256:512].cpu().numpy().view(np.uint16), sl.view(np.uint16))
