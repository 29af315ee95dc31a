"""GPU: the expert-parallel device steps (exl3b_ep_plan / _pack / _combine, and the exchange EPPrefill runs:
exl3b_ep_dispatch / _combine_h, with the local grouped prefill).

On one GPU a single source serves G virtual ranks: the plan tables equal the host reference bit for bit, and the
layer output equals the one-device prefill and the oracle within the layer tolerance.  With two or more GPUs the
full NCCL exchange (EPPrefill on a 2-rank group) is checked against the one-device prefill as well."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle as O
from ep_host import HostEPKernels
from exl3b200 import _lib, synth
from exl3b200 import ops as X
from exl3b200.ep import CudaEPKernels
from helpers import assert_close_f32, assert_close_layer, bits, make_layer

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def _status():
    X.register()
    yield
    st = np.zeros(1, np.int32)
    _lib.check(_lib.lib().exl3b_device_status(st.ctypes.data, 1, None))
    assert st[0] == 0, f"device status word {st[0]}"


def _route(T, E, topk, seed, s=1.1):
    g = torch.Generator().manual_seed(seed)
    p = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** s
    ids = torch.multinomial(p.expand(T, E), topk, replacement=False, generator=g).to(torch.int32)
    w = torch.rand(T, topk, generator=g)
    return ids, (w / w.sum(1, keepdim=True)).float()


@pytest.mark.parametrize("G,T", [(2, 300), (4, 520), (8, 64)])
def test_ep_device_steps_single_source(G, T):
    H, I, E, topk, K = 256, 256, 16, 4, 3
    arena, ptrs, views = make_layer(E, H, I, K, seed=40 + G)
    x = synth.activations(T, H, 41 + G)
    ids, w = _route(T, E, topk, 42 + G)
    xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
    k = CudaEPKernels()
    p = k.plan(idd, wd, E, G)
    ref = HostEPKernels([], H, I, K).plan(ids, w, E, G)
    for key in ("counts", "offs", "pos"):
        assert np.array_equal(p[key].cpu().numpy()[: ref[key].shape[0]], ref[key].numpy()), key
    n = int(p["offs"][G].item())
    for key in ("send_src", "send_ids", "send_w"):
        assert np.array_equal(p[key][:n].cpu().numpy(), ref[key][:n].numpy()), key
    send_x = k.pack(xd, p["send_src"], n)
    assert torch.equal(send_x.cpu(), x[ref["send_src"][:n].long()])
    per = E // G
    offs = p["offs"].cpu().tolist()
    parts = []
    for d in range(G):
        r0, r1 = offs[d], offs[d + 1]
        parts.append(k.local(send_x[r0:r1], p["send_ids"][r0:r1].contiguous(), p["send_w"][r0:r1].contiguous(),
                             ptrs[d * per:(d + 1) * per].contiguous(), None, I, K, per))
    part = torch.cat(parts) if n else torch.zeros((0, H), dtype=torch.float32, device=DEV)
    out = k.combine(part, p["pos"], T, G, H, torch.float32)
    torch.cuda.synchronize()
    blobs = [views[e].cpu().numpy() for e in range(E)]
    semantics_prefill = T >= X.G.prefill_min_m
    ref32 = O.moe_layer_fast(bits(x), ids.numpy(), w.numpy(), blobs, H, I, K, out_f32=True, y_half=True)
    # rows routed through the decode kernels (fewer than prefill_min_m at a rank) keep fp32 pick outputs: both
    # semantics are within the layer tolerance of each other
    assert_close_f32(out.cpu().numpy(), ref32)
    if semantics_prefill:
        one = X.moe_prefill(xd, idd, wd, ptrs, I, K, E, out=torch.empty(T, H, dtype=torch.float32, device=DEV))
        assert_close_f32(out.cpu().numpy(), one.cpu().numpy())


@pytest.mark.parametrize("G,T,cap", [(2, 300, 300), (4, 520, 600), (8, 64, 64)])
def test_ep_dispatch_records_and_fp16_combine(G, T, cap):
    """The exchange EPPrefill runs, on one GPU with one source serving G virtual ranks: the send records (fixed-capacity
    blocks, unused rows with no picks) equal the host contract byte for byte on every row a receiver reads, each
    destination's MoE over its whole block returns fp16 partial sums, and their combine equals the one-device prefill
    and the oracle within the layer tolerance."""
    from exl3b200.ep import unpack_records
    H, I, E, topk, K = 256, 256, 16, 4, 3
    arena, ptrs, views = make_layer(E, H, I, K, seed=50 + G)
    x = synth.activations(T, H, 51 + G)
    ids, w = _route(T, E, topk, 52 + G)
    xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
    k = CudaEPKernels()
    p = k.dispatch(xd, idd, wd, E, G, cap)
    ref = HostEPKernels([], H, I, K).dispatch(x, ids, w, E, G, cap)
    assert np.array_equal(p["pos"].cpu().numpy()[:T], ref["pos"].numpy()[:T])
    assert np.array_equal(p["counts"].cpu().numpy(), ref["counts"].numpy())
    sd, sr = p["send"].cpu().numpy(), ref["send"].numpy()
    assert sd.shape == sr.shape
    assert np.array_equal(sd[:, 2 * H:], sr[:, 2 * H:])                     # ids and weights of every row
    counts = ref["counts"].numpy()
    for d in range(G):                                                     # rows of x where they are used
        r0 = d * cap
        assert np.array_equal(sd[r0:r0 + counts[d], :2 * H], sr[r0:r0 + counts[d], :2 * H])
    per = E // G
    blocks = []
    for d in range(G):
        xr, idr, wr = unpack_records(p["send"][d * cap:(d + 1) * cap], H, topk, xd.dtype)
        blocks.append(k.local(xr, idr, wr, ptrs[d * per:(d + 1) * per].contiguous(), None, I, K, per,
                              dtype=torch.float16))
    out = k.combine_h(torch.cat(blocks), p["pos"], T, G, H, torch.float32)
    torch.cuda.synchronize()
    blobs = [views[e].cpu().numpy() for e in range(E)]
    ref32 = O.moe_layer_fast(bits(x), ids.numpy(), w.numpy(), blobs, H, I, K, out_f32=True, y_half=True)
    assert_close_f32(out.cpu().numpy(), ref32)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, q):
    import sys
    sys.path[:0] = [os.path.join(ROOT, "qwen38-flash-next-b70-offload_b200"), os.path.join(ROOT, "tests"),
                    os.path.join(ROOT, "oracle")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from exl3b200 import ops as X2, synth as S2
        from exl3b200.ep import EPPrefill
        from helpers import assert_close_f32 as close, make_layer as mk
        X2.register()
        H, I, E, topk, K, T = 256, 256, 16, 4, 3, 400
        arena, ptrs, _ = mk(E, H, I, K, seed=55, device=f"cuda:{rank}")
        per = E // world
        x = S2.activations(T, H, 60 + rank).to(rank)
        g = torch.Generator().manual_seed(70 + rank)
        ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).to(torch.int32).to(rank)
        w = torch.softmax(torch.rand(T, topk, generator=g), 1).float().to(rank)
        ep = EPPrefill(dist.group.WORLD, E, H, I, K, ptrs[rank * per:(rank + 1) * per].contiguous())
        x32 = torch.empty(T, H, dtype=torch.float32, device=rank)
        out = ep.forward(x, ids, w)
        one = X2.moe_prefill(x, ids, w, ptrs, I, K, E, out=x32)
        torch.cuda.synchronize()
        close(out.float().cpu().numpy(), one.cpu().numpy(), atol=2e-2, rl2=2e-3)
        # the batch in 3 pipelined chunks (async all-to-alls on NCCL's stream beside the expert GEMMs): each chunk
        # runs its experts through the decode kernels or the prefill GEMMs by its own row count
        ep3 = EPPrefill(dist.group.WORLD, E, H, I, K, ptrs[rank * per:(rank + 1) * per].contiguous(), max_tokens=T,
                        chunks=3)
        out3 = ep3.forward(x, ids, w)
        torch.cuda.synchronize()
        close(out3.float().cpu().numpy(), one.cpu().numpy(), atol=2e-2, rl2=2e-3)
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_nccl_two_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, status in res:
        assert status == "ok", f"rank {rank}: {status}"
