"""GPU parity of the tcgen05 prefill linear (exl3_gemm_tc) against the CPU oracle and, at BASELINE sizes, against a
torch fp32 product of the bit-exact GPU-dequantised weights and the GPU-rotated input."""
import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import ops
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


@pytest.mark.parametrize("M,k,n,K", [(256, 512, 256, 3), (300, 1024, 512, 2), (77, 256, 128, 4), (520, 384, 768, 1), (1100, 256, 384, 2),
                                     (256, 640, 256, 8), (1, 128, 256, 5)])
def test_gemm_tc_matches_oracle(M, k, n, K):
    rng = np.random.default_rng(M * 7 + k + n + K)
    tr = O.random_trellis(rng, k, n, K)
    suh = O.random_signs(rng, k)
    svh = (O.random_signs(rng, n).astype(np.float32) * rng.uniform(0.5, 1.5, n)).astype(np.float16)
    x = rng.standard_normal((M, k)).astype(np.float16)
    pk = ops.pack(to_dev(tr), K)
    for y_dt, np_dt in ((torch.float32, np.float32), (torch.float16, np.float16)):
        y = torch.full((M, n), float("nan"), dtype=y_dt, device=DEV)
        ops.exl3_gemm_tc(to_dev(x), pk, to_dev(suh), to_dev(svh), K, y)
        ref = O.exl3_linear(x, tr, suh, svh, K, np_dt)
        assert_close(y.float().cpu().numpy(), ref.astype(np.float32), rel_tol=2e-3 if np_dt == np.float32 else 3e-3,
                     what=f"gemm_tc M={M} k={k} n={n} K={K} {y_dt}")


def test_gemm_tc_bf16_input_and_repeatable():
    rng = np.random.default_rng(3)
    M, k, n, K = 384, 768, 512, 3
    tr = O.random_trellis(rng, k, n, K)
    suh = O.random_signs(rng, k)
    svh = O.random_signs(rng, n)
    xb = torch.randn((M, k), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    pk = ops.pack(to_dev(tr), K)
    y = torch.full((M, n), float("nan"), dtype=torch.float32, device=DEV)
    ops.exl3_gemm_tc(xb.to(DEV), pk, to_dev(suh), to_dev(svh), K, y)
    ref = O.exl3_linear(xb.float().numpy(), tr, suh, svh, K, np.float32)
    assert_close(y.cpu().numpy(), ref, what="gemm_tc bf16 input")
    y2 = torch.full_like(y, float("nan"))
    ops.exl3_gemm_tc(xb.to(DEV), pk, to_dev(suh), to_dev(svh), K, y2)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("M,k,n,K", [(8192, 7168, 2048, 2), (2048, 2048, 7168, 1), (1000, 5120, 5120, 4), (700, 1024, 384, 3)])
def test_gemm_tc_full_size_against_torch(M, k, n, K):
    g = torch.Generator(device=DEV).manual_seed(M + k + n + K)
    tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=DEV, generator=g)
    suh = (torch.randint(0, 2, (k,), device=DEV, generator=g) * 2 - 1).half()
    svh = (torch.randint(0, 2, (n,), device=DEV, generator=g) * 2 - 1).half()
    x = torch.randn((M, k), device=DEV, generator=g).half()
    y = torch.full((M, n), float("nan"), dtype=torch.float32, device=DEV)
    ops.exl3_gemm_tc(x, ops.pack(tr, K), suh, svh, K, y)
    W = torch.empty((k, n), dtype=torch.half, device=DEV)
    ops.exl3_reconstruct(tr, W, 0, K)
    xh = torch.empty_like(x)
    ops.had_r_128(x, xh, suh, None, 1.0)
    acc = xh.float() @ W.float()
    ref = torch.empty_like(acc)
    ops.had_r_128(acc, ref, None, svh.float(), 1.0)
    assert_close(y.cpu().numpy(), ref.cpu().numpy(), what=f"gemm_tc {M}x{k}x{n} K={K}")
