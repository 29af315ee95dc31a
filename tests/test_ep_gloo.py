"""CPU, world_size 2 and 4 (gloo): the expert-parallel prefill exchange (exl3b200.ep.EPPrefill) with host stand-ins
for the device steps.  Every rank's output equals the one-device prefill of its tokens (oracle, same picks) within the
layer tolerance; a rank with no tokens and a rank whose tokens all stay local are covered."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case, q):
    import sys
    sys.path[:0] = [os.path.join(ROOT, "qwen38-flash-next-b70-offload_b200"), os.path.join(ROOT, "oracle"),
                    os.path.join(ROOT, "tests")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import oracle as O
        from ep_host import HostEPKernels
        from exl3b200 import synth
        from exl3b200.ep import EPPrefill
        from helpers import assert_close_layer
        E, H, I, K, topk = 8, 256, 128, 3, 3
        per = E // world
        blobs = [synth.make_blob(11, e, H, I, K).numpy() for e in range(E)]
        T = case["T"][rank]
        g = torch.Generator().manual_seed(100 + rank)
        if case.get("local_only") and rank == 0:
            ids = torch.stack([torch.randperm(per, generator=g)[:topk] for _ in range(T)]).to(torch.int32)
        else:
            ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).to(torch.int32) if T else \
                torch.zeros((0, topk), dtype=torch.int32)
        w = torch.rand(T, topk, generator=g)
        w = (w / w.sum(1, keepdim=True)).float() if T else torch.zeros((0, topk))
        x = synth.activations(T, H, 200 + rank) if T else torch.zeros((0, H), dtype=torch.bfloat16)
        k = HostEPKernels(blobs[rank * per:(rank + 1) * per], H, I, K)
        ep = EPPrefill(dist.group.WORLD, E, H, I, K, torch.zeros(per, dtype=torch.int64), kernels=k,
                       max_tokens=case.get("max_tokens"), chunks=case.get("chunks", 1))
        out = ep.forward(x, ids, w)
        if T:
            xb = x.view(torch.int16).numpy().view(np.uint16)
            ref = O.moe_layer_fast(xb, ids.numpy(), w.numpy(), blobs, H, I, K, y_half=True, threads=2)
            assert_close_layer(out.view(torch.int16).numpy().view(np.uint16), ref)
        q.put((rank, "ok", ep.stats()))
    except Exception as e:   # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}", None))
    finally:
        dist.destroy_process_group()


def _run(case, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    for rank, status, _ in res:
        assert status == "ok", f"rank {rank}: {status}"
    return {r: last for r, _, last in res}


def test_ep_exchange_two_ranks():
    last = _run({"T": [7, 5]})
    assert last[0]["send_rows"] > 0 and last[1]["recv_rows"] > 0
    assert last[0]["cap"] == last[1]["cap"] == 7   # agreed by the ranks: the largest token count


def test_ep_exchange_fixed_capacity():
    """A capacity given to every rank (max_tokens) instead of agreed per call: the same exchange, no host read."""
    last = _run({"T": [7, 5], "max_tokens": 9})
    assert last[0]["cap"] == last[1]["cap"] == 9
    assert [last[d]["recv_counts"][0] for d in range(2)] == last[0]["send_counts"]


def test_ep_exchange_in_chunks():
    """The batch split into 3 token ranges whose exchanges are pipelined with the experts (async all-to-alls): the
    same outputs, and the per-rank counts add up over the chunks; a rank with fewer tokens than a chunk's capacity
    sends empty chunks."""
    last = _run({"T": [7, 2], "chunks": 3})
    assert last[0]["cap"] == last[1]["cap"] == 3
    assert [last[d]["recv_counts"][0] for d in range(2)] == last[0]["send_counts"]
    assert [last[d]["recv_counts"][1] for d in range(2)] == last[1]["send_counts"]


def test_ep_rank_without_tokens():
    _run({"T": [6, 0]})


def test_ep_tokens_all_local():
    last = _run({"T": [5, 4], "local_only": True})
    assert last[0]["send_counts"][1] == 0


def test_ep_exchange_four_ranks():
    """Four ranks (two experts each), one of them without tokens: every rank sends to and receives from the others
    in rank order."""
    last = _run({"T": [5, 0, 7, 3]}, world=4)
    assert last[1]["send_rows"] == 0
    assert sum(last[r]["recv_rows"] for r in range(4)) == sum(last[r]["send_rows"] for r in range(4))
    for r in range(4):
        assert [last[d]["recv_counts"][r] for d in range(4)] == last[r]["send_counts"]


def _fail_worker(rank, world, port, q):
    """Rank 1 leaves right after joining the group (no collective); rank 0 runs a layer and must get an error."""
    import sys
    sys.path[:0] = [os.path.join(ROOT, "qwen38-flash-next-b70-offload_b200"), os.path.join(ROOT, "oracle"),
                    os.path.join(ROOT, "tests")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    def report(msg):   # flush the queue's feeder thread before the hard exit
        q.put((rank, msg))
        q.close()
        q.join_thread()

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        report("left")
        os._exit(0)
    try:
        from ep_host import HostEPKernels
        from exl3b200 import synth
        from exl3b200.ep import EPPrefill
        E, H, I, K, topk, T = 8, 256, 128, 3, 3, 4
        blobs = [synth.make_blob(11, e, H, I, K).numpy() for e in range(E)]
        g = torch.Generator().manual_seed(5)
        ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).to(torch.int32)
        w = torch.full((T, topk), 1.0 / topk)
        x = synth.activations(T, H, 9)
        ep = EPPrefill(dist.group.WORLD, E, H, I, K, torch.zeros(E // world, dtype=torch.int64),
                       kernels=HostEPKernels(blobs[:E // world], H, I, K))
        ep.forward(x, ids, w)
        report("no error")
    except RuntimeError as e:
        report("raised: " + str(e)[:300])
    except Exception as e:
        report(f"other {type(e).__name__}: {e}")
    os._exit(0)   # no teardown against the departed peer


def test_ep_peer_failure_raises():
    """A rank that stops ends the other rank's next layer with a RuntimeError naming the exchange (bounded by the
    group's 10 s timeout), not a hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_fail_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("raised:") and "EPPrefill" in res[0], res[0]
