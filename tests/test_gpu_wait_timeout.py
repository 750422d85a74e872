"""The bounded device waits give up with a status instead of hanging: exl3_wait_probe waits, with the library's own
wait and a short limit, on an mbarrier that nothing completes. The wait runs out, EXL3_ERR_TIMEOUT lands in the
device status word, and the context stays usable for the next call. No GPU fault is involved."""
import time

import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import ops

DEV = "cuda:0"


def test_wait_probe_rejects_bad_limits():
    lib = L.lib()
    assert lib.exl3_wait_probe(0, None) == L.EXL3_ERR_ARG
    assert lib.exl3_wait_probe(10 ** 9, None) == L.EXL3_ERR_ARG      # above the library's 100 ms limit
    assert b"exl3_wait_probe" in lib.exl3_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("limit_ms", [1, 20])
def test_wait_that_nothing_completes_times_out(limit_ms):
    lib = L.lib()
    torch.cuda.synchronize()
    assert lib.exl3_device_status(1) in (0, L.EXL3_ERR_TIMEOUT)
    assert lib.exl3_device_status(0) == 0
    t0 = time.perf_counter()
    L.check(lib.exl3_wait_probe(limit_ms * 1_000_000, torch.cuda.current_stream().cuda_stream), "wait probe")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert lib.exl3_device_status(0) == L.EXL3_ERR_TIMEOUT
    assert limit_ms * 1e-3 * 0.9 <= dt < 5.0, dt                    # it waited its limit, then returned
    assert lib.exl3_device_status(1) == L.EXL3_ERR_TIMEOUT            # read and clear
    assert lib.exl3_device_status(0) == 0
    # the context is still good: a GEMV afterwards runs and leaves the status clean
    g = torch.Generator(device=DEV).manual_seed(5)
    k, n, K = 256, 128, 3
    tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=DEV, generator=g)
    suh = torch.ones(k, dtype=torch.half, device=DEV)
    svh = torch.ones(n, dtype=torch.half, device=DEV)
    y = torch.empty((1, n), dtype=torch.float32, device=DEV)
    ops.exl3_gemv(torch.randn((1, k), device=DEV, generator=g).half(), ops.pack(tr, K), suh, svh, K, y)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    assert lib.exl3_device_status(0) == 0
