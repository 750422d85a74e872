"""exl3_gemv_noalloc (static device scratch, no workspace) against exl3_gemv: identical results, two calls in a
row, from this file alone or after every other test (the file is collected last)."""
import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import ops
from oracle import oracle as O
from tests.tolerance import assert_close

DEV = "cuda:0"


def test_noalloc_rejects_oversize_and_bad_arguments():
    """Host-side checks, before any device work (no GPU needed)."""
    lib = L.lib()

    def call(M=1, k=128, n=128, K=3, cb=2, x=16, y=16):
        return lib.exl3_gemv_noalloc(x, 0, k, M, 16, 16, 16, k, n, K, cb, y, 0, n, None)

    assert call(k=32768 + 128) == L.EXL3_ERR_UNSUPPORTED
    assert b"static scratch" in lib.exl3_last_error()
    assert call(n=65536 + 128) == L.EXL3_ERR_UNSUPPORTED
    assert call(M=9) == L.EXL3_ERR_ARG
    assert call(cb=1) == L.EXL3_ERR_UNSUPPORTED
    assert call(M=0) == L.EXL3_OK


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,K,M", [(512, 384, 3, 1), (2048, 1024, 2, 4), (5120, 5120, 4, 8), (32768, 256, 3, 2)])
def test_noalloc_matches_workspace_gemv(k, n, K, M):
    L.lib().exl3_device_status(1)
    g = torch.Generator(device=DEV).manual_seed(k + n + K + M)
    tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=DEV, generator=g)
    pk = ops.pack(tr, K)
    suh = (torch.randint(0, 2, (k,), device=DEV, generator=g) * 2 - 1).half()
    svh = (torch.randint(0, 2, (n,), device=DEV, generator=g) * 2 - 1).half()
    ref = torch.full((M, n), float("nan"), dtype=torch.float32, device=DEV)
    ops.exl3_gemv(torch.randn(1, k, device=DEV).half(), pk, suh, svh, K, ref[:1])   # unrelated call first
    outs = []
    for _ in range(2):                                   # two calls in a row on the same static scratch
        x = torch.randn((M, k), device=DEV, generator=g).half()
        ops.exl3_gemv(x, pk, suh, svh, K, ref)
        y = torch.full((M, n), float("nan"), dtype=torch.float32, device=DEV)
        ops.exl3_gemv_noalloc(x, pk, suh, svh, K, y)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), "no-alloc GEMV must equal the workspace GEMV bit for bit"
        outs.append(y)
    assert not torch.equal(outs[0], outs[1])
    assert L.lib().exl3_device_status(0) == 0


@pytest.mark.gpu
def test_noalloc_against_oracle_fp16_out():
    rng = np.random.default_rng(12)
    k, n, K, M = 1024, 512, 3, 3
    tr = O.random_trellis(rng, k, n, K)
    suh = O.random_signs(rng, k)
    svh = O.random_signs(rng, n)
    x = rng.standard_normal((M, k)).astype(np.float16)

    def t(a):
        v = torch.from_numpy(np.ascontiguousarray(a))
        return (v.view(torch.int16) if v.dtype == torch.uint16 else v).to(DEV)

    y = torch.full((M, n), float("nan"), dtype=torch.half, device=DEV)
    ops.exl3_gemv_noalloc(t(x), ops.pack(t(tr), K), t(suh), t(svh), K, y)
    ref = O.exl3_linear(x, tr, suh, svh, K, np.float16)
    assert_close(y.float().cpu().numpy(), ref.astype(np.float32), rel_tol=3e-3, what="no-alloc fp16")
