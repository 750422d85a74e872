"""GPU parity of exl3_mgemm (several EXL3 linears over pointer tables, exllamav3's contract) against the CPU oracle:
plain slots with a broadcast or per-slot A, indices with skipped and filtered slots, and weighted per-token sums."""
import numpy as np
import pytest
import torch

from exl3_b200 import _lib as L
from exl3_b200 import ops
from oracle import oracle as O
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
k, n = 256, 384


def to_dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if t.dtype == torch.uint16:
        t = t.view(torch.int16)
    return t.to(DEV)


@pytest.fixture(autouse=True)
def _status_clean():
    L.lib().exl3_device_status(1)
    yield
    torch.cuda.synchronize()
    assert L.lib().exl3_device_status(0) == 0, "a device-side wait timed out"


def make_mats(rng, Ks):
    host, lins = [], []
    for K in Ks:
        tr = O.random_trellis(rng, k, n, K)
        suh = O.random_signs(rng, k)
        svh = (O.random_signs(rng, n).astype(np.float32) * rng.uniform(0.5, 1.5, n)).astype(np.float16)
        host.append((tr, suh, svh, K))
        lins.append(ops.BC_LinearEXL3(to_dev(tr), to_dev(suh), to_dev(svh), K, None, False, True, None))
    tables = [torch.tensor([getattr(l, a).data_ptr() for l in lins], dtype=torch.int64, device=DEV)
              for a in ("trellis", "suh", "svh")]
    return host, lins, tables


@pytest.mark.parametrize("a_batches", [1, 3])
@pytest.mark.parametrize("m", [1, 5, 11])
def test_mgemm_slots_match_oracle(a_batches, m):
    rng = np.random.default_rng(10 * a_batches + m)
    host, lins, (B, S, V) = make_mats(rng, [2, 3, 4])
    A = rng.standard_normal((a_batches, m, k)).astype(np.float16)
    C = torch.full((3, m, n), float("nan"), dtype=torch.float16, device=DEV)
    ops.exl3_mgemm(to_dev(A), B, C, S, None, V)
    for j, (tr, suh, svh, K) in enumerate(host):
        ref = O.exl3_linear(A[0 if a_batches == 1 else j], tr, suh, svh, K, np.float16)
        assert_close(C[j].float().cpu().numpy(), ref.astype(np.float32), what=f"slot {j}")


def test_mgemm_indices_skip_and_filter():
    rng = np.random.default_rng(7)
    host, lins, (B, S, V) = make_mats(rng, [2, 3, 1, 4])
    m = 4
    A = rng.standard_normal((1, m, k)).astype(np.float16)
    idx = torch.tensor([3, -1, 1, 0, 2], dtype=torch.int64, device=DEV)
    C = torch.full((5, m, n), 7.0, dtype=torch.float32, device=DEV)
    ops.exl3_mgemm(to_dev(A), B, C, S, None, V, indices=idx)
    for j, q in enumerate([3, -1, 1, 0, 2]):
        if q < 0:
            assert (C[j] == 7.0).all(), "a skipped slot must stay untouched"
            continue
        tr, suh, svh, K = host[q]
        assert_close(C[j].cpu().numpy(), O.exl3_linear(A[0], tr, suh, svh, K, np.float32), what=f"slot {j}")
    # min/max filter: keep matrices [1, 3), rebased to 0, 1 of a table that starts at matrix 1
    B2, S2, V2 = (t[1:3].contiguous() for t in (B, S, V))
    C2 = torch.full((5, m, n), 7.0, dtype=torch.float32, device=DEV)
    ops.exl3_mgemm(to_dev(A), B2, C2, S2, None, V2, indices=idx, min_index=1, max_index=3)
    for j, q in enumerate([3, -1, 1, 0, 2]):
        if not 1 <= q < 3:
            assert (C2[j] == 7.0).all()
            continue
        tr, suh, svh, K = host[q]
        assert_close(C2[j].cpu().numpy(), O.exl3_linear(A[0], tr, suh, svh, K, np.float32), what=f"filtered {j}")


def test_mgemm_weighted_token_sums():
    rng = np.random.default_rng(11)
    host, lins, (B, S, V) = make_mats(rng, [2, 3, 2, 4, 3, 1])
    m, tokens, per = 3, 2, 4                                  # 8 slots: 4 per token
    A = rng.standard_normal((tokens * per, m, k)).astype(np.float16)
    ids = np.array([0, 5, 2, -1, 1, 3, 4, 0], dtype=np.int64)
    w = rng.uniform(0.1, 1.0, tokens * per).astype(np.float16)
    C = torch.full((tokens, m, n), float("nan"), dtype=torch.float32, device=DEV)
    ops.exl3_mgemm(to_dev(A), B, C, S, None, V, indices=to_dev(ids), weights=to_dev(w), num_tokens=tokens)
    for t in range(tokens):
        ref = np.zeros((m, n), dtype=np.float32)
        for j in range(t * per, (t + 1) * per):
            q = int(ids[j])
            if q < 0:
                continue
            tr, suh, svh, K = host[q]
            y = O.exl3_linear(A[j], tr, suh, svh, K, np.float32)
            ref = (ref + np.float32(w[j]) * y).astype(np.float32)
        assert_close(C[t].cpu().numpy(), ref, what=f"token {t}")


def test_mgemm_unregistered_table_raises():
    bogus = torch.tensor([12345678], dtype=torch.int64, device=DEV)
    C = torch.empty((1, 1, n), dtype=torch.float16, device=DEV)
    with pytest.raises(L.Exl3Error):
        ops.exl3_mgemm(torch.zeros((1, 1, k), dtype=torch.float16, device=DEV), bogus, C, bogus, None, bogus)
