"""Expert parallelism on two GPUs with the peer-memory exchange (exl3_ep_dispatch / combine / reduce, and the fused
combine + reduce, bit for bit): each rank's output equals moe_forward / moe_prefill on the full expert table for the
same tokens; uneven batches under one capacity; the exchange captured in a CUDA graph and replayed; and a rank that
skips a dispatch makes its peer's wait run out with EXL3_ERR_TIMEOUT instead of hanging (no GPU fault involved: the
absent rank stays alive, its buffer mapped, until the waiting rank has finished). Child processes, one per GPU, NCCL for the plumbing with NVLS off.
Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as tmp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "b70-inference_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from datetime import timedelta

    import torch.distributed as dist

    from exl3_b200 import _lib as L
    from exl3_b200 import ep, moe, ops
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    try:
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        L.lib().exl3_device_status(1)
        E, H, I, topk = 8 * world, 512, 256, 4
        g = torch.Generator(device=dev).manual_seed(77)             # the same experts on every rank

        def mat(k, n, K):
            tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=dev, generator=g)
            s1 = (torch.randint(0, 2, (k,), device=dev, generator=g) * 2 - 1).half()
            s2 = (torch.randint(0, 2, (n,), device=dev, generator=g) * 2 - 1).half()
            return moe.Exl3Matrix(tr, s1, s2, K)

        full = [moe.Expert(mat(H, I, 2 + e % 2), mat(H, I, 3), mat(I, H, 2)) for e in range(E)]
        shared = moe.Expert(mat(H, I, 3), mat(H, I, 3), mat(I, H, 3))
        e0, e1 = ep.expert_range(E, rank, world)
        local_tab = moe.ExpertTable(full[e0:e1], shared)
        full_tab = moe.ExpertTable(full, shared)
        res = {}
        tg = torch.Generator(device=dev).manual_seed(1000 + rank)
        if mode == "fail":
            epm = ep.ExpertParallelMoE(E, H, topk, None, local_tab, 10.0, capacity=4, exchange="p2p")
            x = torch.randn((4, H), device=dev, generator=tg).half()
            ids, w, _ = ops.route(torch.randn((4, E), device=dev, generator=tg), L.ROUTE_SOFTMAX, topk)
            epm.forward(x, ids, w)                                   # one good exchange first
            torch.cuda.synchronize()
            if rank == 0:                                             # rank 1 skips the next call
                ex = ep.PeerExchange.get(None, world, rank, 4, H, topk, dev)
                xc, idc, wc = x.contiguous(), ids.contiguous(), w.contiguous()
                L.check(L.lib().exl3_ep_dispatch(xc.data_ptr(), 0, H, 4, idc.data_ptr(), wc.data_ptr(), topk, E, H,
                                                 world, rank, 4, ex.peers.data_ptr(), ex.ptr,
                                                 torch.cuda.current_stream().cuda_stream), "dispatch")
                torch.cuda.synchronize()
                res["status"] = L.lib().exl3_device_status(1)
            dist.barrier()                                            # rank 1 leaves only after rank 0's wait ended
            q.put((rank, "ok", res))
            return
        for B, cap in ((4, 4), (3 - rank, 4), (700, 700)):
            x = torch.randn((B, H), device=dev, generator=tg).half()
            ids, w, _ = ops.route(torch.randn((B, E), device=dev, generator=tg), L.ROUTE_SOFTMAX, topk)
            epm = ep.ExpertParallelMoE(E, H, topk, None, local_tab, 10.0, capacity=cap, exchange="p2p")
            got = epm.forward(x, ids, w)
            epm.fused_reduce = False                                  # combine and reduce as two launches
            got2 = epm.forward(x, ids, w)
            epm.fused_reduce = True
            res[f"fused_equal_B{B}"] = bool(torch.equal(got, got2))
            fn = moe.moe_prefill if B * topk >= ep.PREFILL_MIN_PAIRS else moe.moe_forward
            ref = fn(x, ids, w, full_tab, 10.0)
            torch.cuda.synchronize()
            d = (got.double() - ref.double())
            res[f"B{B}"] = (float(d.norm() / ref.double().norm()), float(d.abs().max()),
                            float(ref.double().pow(2).mean().sqrt()))
        # graph capture of the exchange: two replays with new inputs
        B = 4
        epm = ep.ExpertParallelMoE(E, H, topk, None, local_tab, 10.0, capacity=B, exchange="p2p")
        x = torch.randn((B, H), device=dev, generator=tg).half()
        lg = torch.randn((B, E), device=dev, generator=tg)
        out = torch.empty((B, H), device=dev)

        def step():
            ids, w, _ = ops.route(lg, L.ROUTE_SOFTMAX, topk)
            out.copy_(epm.forward(x, ids, w))

        step()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for rep in range(2):
            x.copy_(torch.randn((B, H), device=dev, generator=tg).half())
            lg.copy_(torch.randn((B, E), device=dev, generator=tg))
            dist.barrier()
            graph.replay()
            torch.cuda.synchronize()
            ids, w, _ = ops.route(lg, L.ROUTE_SOFTMAX, topk)
            ref = moe.moe_forward(x, ids, w, full_tab, 10.0)
            d = (out.double() - ref.double())
            res[f"graph{rep}"] = (float(d.norm() / ref.double().norm()), float(d.abs().max()),
                                  float(ref.double().pow(2).mean().sqrt()))
        del graph
        res["status"] = L.lib().exl3_device_status(0)
        dist.barrier()
        q.put((rank, "ok", res))
    except Exception as exc:
        q.put((rank, "error", repr(exc)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2):
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        r, st, v = q.get(timeout=600)
        out[r] = (st, v)
    for p in ps:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_expert_parallel_matches_full_table():
    res = _run("ok")
    for r in range(2):
        st, v = res[r]
        assert st == "ok", v
        assert v["status"] == 0
        for key, t in v.items():
            if key == "status":
                continue
            if key.startswith("fused_equal"):
                assert t, (r, key)                                    # one launch or two: the same bits
                continue
            rel, mx, rms = t
            assert rel <= 2e-3 and mx <= 1e-2 * max(1.0, rms), (r, key, rel, mx, rms)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_missing_peer_times_out():
    res = _run("fail")
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    assert res[0][1]["status"] == 5, res[0][1]          # EXL3_ERR_TIMEOUT, and the context is still usable
