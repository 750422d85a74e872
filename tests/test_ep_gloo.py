"""Expert-parallel dispatch/combine on CPU gloo ranks (world sizes 2 and 4), with the oracle as each rank's local expert
compute, against the single-process oracle; and a rank that fails before the exchange surfaces as an error on its
peer (short process-group timeout) instead of a hang. No GPU involved."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as tmp

E, H, I, TOPK, B = 8, 128, 128, 3, 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _experts(n=E, seed=42):
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    ex = []
    for e in range(n):
        K = 2 + e % 3
        mats = [(O.random_trellis(rng, kk, nn, K), O.random_signs(rng, kk), O.random_signs(rng, nn), K)
                for kk, nn in ((H, I), (H, I), (I, H))]
        ex.append(O.ExpertW(*mats))
    return ex


def _tokens(rank, b=B):
    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((b, H)).astype(np.float16)
    ids = np.stack([rng.permutation(E)[:TOPK] for _ in range(b)]).astype(np.int32)
    w = rng.random((b, TOPK)).astype(np.float32)
    return x, ids, w


def _worker(rank, world, port, mode, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "b70-inference_b200")]
    from datetime import timedelta
    from oracle import oracle as O
    from exl3_b200 import ep
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=10))
        experts = _experts()
        e0, e1 = ep.expert_range(E, rank, world)

        def local_fn(x, ids, w):
            xs, ii, ww = x.numpy(), ids.numpy(), w.numpy()
            out = np.zeros((xs.shape[0], H), dtype=np.float32)
            for r in range(xs.shape[0]):
                for j in range(ii.shape[1]):
                    if ii[r, j] >= 0:
                        d = O.expert_forward(xs[r:r + 1], experts[e0 + ii[r, j]], 10.0)[0]
                        out[r] = (out[r] + np.float32(ww[r, j]) * d).astype(np.float32)
            return torch.from_numpy(out)

        shared_fn = None
        if mode == "shared":
            shared = _experts(1, seed=7)[0]

            def shared_fn(x):
                return torch.from_numpy(O.expert_forward(x.numpy(), shared, 10.0).astype(np.float32))

        cap = 4 if mode == "uneven" else None
        m = ep.ExpertParallelMoE(E, H, TOPK, local_fn=local_fn, shared_fn=shared_fn, capacity=cap)
        x, ids, w = _tokens(rank, _batch(mode, rank))
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the dispatch")
        out = m.forward(torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(w))
        if mode == "uneven":                     # a second call with a smaller batch on the same layer
            x2, ids2, w2 = _tokens(rank + 10, 1)
            out2 = m.forward(torch.from_numpy(x2), torch.from_numpy(ids2), torch.from_numpy(w2))
            try:
                x3, ids3, w3 = _tokens(rank, 5)
                m.forward(torch.from_numpy(x3), torch.from_numpy(ids3), torch.from_numpy(w3))
                over = "no error"
            except ValueError as exc:            # raised before any collective: the ranks stay in step
                over = str(exc)
            q.put((rank, "ok", (out.numpy(), out2.numpy(), over)))
            return
        q.put((rank, "ok", out.numpy()))
    except Exception as exc:      # reported to the parent, which decides pass/fail
        q.put((rank, "error", repr(exc)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _batch(mode, rank):
    """Rows per rank: B everywhere, or uneven batches below the capacity of 4."""
    return (3, 2, 4, 1)[rank] if mode == "uneven" else B


def _run(mode, world=2):
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, st, v = q.get(timeout=180)
        res[r] = (st, v)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_ep_dispatch_combine_matches_oracle():
    from oracle import oracle as O
    from tests.tolerance import assert_close
    res = _run("ok")
    experts = _experts()
    for r in range(2):
        st, out = res[r]
        assert st == "ok", out
        x, ids, w = _tokens(r)
        ref = O.moe_forward(x, ids, w, experts, 10.0)
        assert_close(out, ref, what=f"EP rank {r}")


def test_ep_shared_expert_counted_once():
    """A shared expert runs once per token, on the token's own rank (not on every rank that received the row)."""
    from oracle import oracle as O
    from tests.tolerance import assert_close
    res = _run("shared")
    experts = _experts()
    shared = _experts(1, seed=7)[0]
    for r in range(2):
        st, out = res[r]
        assert st == "ok", out
        x, ids, w = _tokens(r)
        ref = O.moe_forward(x, ids, w, experts, 10.0, shared=shared)
        assert_close(out, ref, what=f"EP rank {r} with shared expert")


def test_ep_four_ranks_with_shared_expert():
    """Four ranks (two experts each): every token's picks reach the owners of their experts and come back summed in
    slot order, the shared expert once per token: the exchange pattern of the 4- and 8-GPU runs."""
    from oracle import oracle as O
    from tests.tolerance import assert_close
    res = _run("shared", world=4)
    experts = _experts()
    shared = _experts(1, seed=7)[0]
    for r in range(4):
        st, out = res[r]
        assert st == "ok", out
        x, ids, w = _tokens(r)
        ref = O.moe_forward(x, ids, w, experts, 10.0, shared=shared)
        assert_close(out, ref, what=f"EP rank {r} of 4")


def test_ep_uneven_batches_under_a_fixed_capacity():
    """Ranks with different batch sizes (3, 2, 4, 1 rows) under one capacity (4): padding rows carry no picks, each
    rank gets its own rows' routed sums; a second call with one row reuses the layer; a batch above the capacity
    raises before any collective."""
    from oracle import oracle as O
    from tests.tolerance import assert_close
    res = _run("uneven", world=4)
    experts = _experts()
    for r in range(4):
        st, v = res[r]
        assert st == "ok", v
        out, out2, over = v
        x, ids, w = _tokens(r, _batch("uneven", r))
        assert out.shape == (x.shape[0], H)
        assert_close(out, O.moe_forward(x, ids, w, experts, 10.0), what=f"EP uneven rank {r}")
        x2, ids2, w2 = _tokens(r + 10, 1)
        assert_close(out2, O.moe_forward(x2, ids2, w2, experts, 10.0), what=f"EP second call rank {r}")
        assert "exceeds the capacity" in over


def test_ep_rank_failure_is_reported_not_hung():
    res = _run("fail")
    assert res[1][0] == "error" and "rank 1 fails" in res[1][1]
    assert res[0][0] == "error", "the surviving rank must see an error from the collective, not hang"


def test_expert_range_and_localize():
    from exl3_b200 import ep
    assert ep.expert_range(512, 3, 8) == (192, 256)
    with pytest.raises(ValueError):
        ep.expert_range(10, 0, 4)
    ids = torch.tensor([[0, 63, 64, 127, -1, 200]], dtype=torch.int32)
    assert ep.localize_ids(ids, 64, 128).tolist() == [[-1, -1, 0, 63, -1, -1]]
