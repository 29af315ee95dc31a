"""GPU parity: the CUDA path (through the C ABI / torch ops) against the CPU oracle on seeded inputs.

Bit-exact: decoded fp16 weights, router ids, align tables, cache state.  Layer outputs: max-abs 2e-2, rel-L2 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle as O
from exl3b200 import ExpertStore, ops as exops, synth
from exl3b200 import ops as X
from helpers import assert_close_f32, assert_close_layer, bits, make_layer, oracle_blobs

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status():
    X.register()
    yield
    st = np.zeros(1, np.int32)
    from exl3b200 import _lib
    _lib.check(_lib.lib().exl3b_device_status(st.ctypes.data, 1, None))
    assert st[0] == 0, f"device status word {st[0]}"


# ------------------------------------------------------------------------------------------------ dequant
@pytest.mark.parametrize("K", [2, 3, 4, 5])
@pytest.mark.parametrize("planar", [True, False])
def test_dequant_bit_exact(K, planar):
    rows16, ntiles = 6, 12
    rs = ntiles * 8 * K + 8 * K * 4   # padded row stride
    words = synth.stream_u32(5, 50 + K, rows16 * rs, "cpu").to(torch.int64).numpy().astype(np.uint32)
    tile0 = 4
    ref = O.dequant(words[: rows16 * rs].reshape(-1), rows16, rs, tile0, ntiles - 4, K, planar)
    wd = torch.from_numpy(words.view(np.int32)).to(DEV)
    got = X.dequant(wd, rows16, rs, tile0, ntiles - 4, K, planar)
    torch.cuda.synchronize()
    assert np.array_equal(bits(got), ref)


@pytest.mark.parametrize("K", [3])
def test_blob_dequant_full_shape(K):
    H, I = 2048, 768
    blob = synth.make_blob(0, 3, H, I, K, device=DEV)
    cpu = blob.cpu().numpy()
    for proj in (0, 1, 2):
        got = X.blob_dequant(blob, H, I, K, K, K, proj)
        ref = O.blob_dequant(cpu, H, I, K, K, K, proj)
        assert np.array_equal(bits(got), ref), proj


def test_blob_dequant_mixed_k():
    H, I, ks = 256, 128, (2, 5, 4)
    blob = synth.make_blob(1, 9, H, I, *ks, device=DEV)
    cpu = blob.cpu().numpy()
    for proj in (0, 1, 2):
        assert np.array_equal(bits(X.blob_dequant(blob, H, I, *ks, proj)), O.blob_dequant(cpu, H, I, *ks, proj))


# ------------------------------------------------------------------------------------------------ router
@pytest.mark.parametrize("T", [1, 3, 4, 5, 8, 33, 200])
@pytest.mark.parametrize("with_bias", [False, True])
def test_router_bit_exact(T, with_bias):
    H, E, topk = 2048, 512, 10
    x = synth.activations(T, H, 100 + T)
    wr = synth.router_weight(E, H, 0.02, 7)
    bias = synth.zipf_bias(E, 3, 7) if with_bias else None
    ids, w = X.router_topk(x.to(DEV), wr.to(DEV), bias.to(DEV) if bias is not None else None, topk)
    rid, rw, _ = O.router(bits(x), bits(wr), bias.numpy() if bias is not None else None, topk)
    assert np.array_equal(ids.cpu().numpy(), rid)
    assert np.allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("T", [128, 333])
@pytest.mark.parametrize("H", [2048, 256])
def test_router_logits_bit_exact_tiled(T, H):
    """Token counts of the tiled logits kernel (partial 64-token tiles, a short chunk length at H=256): the logits
    themselves match the oracle bit for bit, then the picks."""
    E, topk = 512, 10
    x = synth.activations(T, H, 700 + T)
    wr = synth.router_weight(E, H, 0.02, 11)
    bias = synth.zipf_bias(E, 3, 11)
    xd, wd, bd = x.to(DEV), wr.to(DEV), bias.to(DEV)
    ids = torch.empty((T, topk), dtype=torch.int32, device=DEV)
    w = torch.empty((T, topk), dtype=torch.float32, device=DEV)
    logits = torch.empty((T, E), dtype=torch.float32, device=DEV)
    from exl3b200._lib import lib, check, stream
    check(lib().exl3b_router_topk(xd.data_ptr(), xd.stride(0), wd.data_ptr(), bd.data_ptr(), T, H, E, topk,
                                  ids.data_ptr(), w.data_ptr(), logits.data_ptr(), None, stream(xd.device)), "router")
    torch.cuda.synchronize()
    rid, rw, rl = O.router(bits(x), bits(wr), bias.numpy(), topk)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), np.asarray(rl, dtype=np.float32).view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), rid)
    assert np.allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("case", ["all_equal", "four_levels", "e64_top32", "e96_top10", "mostly_neg_inf"])
@pytest.mark.parametrize("T", [1, 5, 40])
def test_router_degenerate_logits(case, T):
    """Selections the threshold top-k (candidates at or above the top-k-th lane maximum) must get exactly right or
    hand to the argmax rounds: every logit equal (512 candidates), logits on four levels (ties across lanes), top-32
    of 64 experts, a small expert count, and five finite logits among -inf (the selection ends in -inf ties)."""
    H = 2048
    E, topk = {"e64_top32": (64, 32), "e96_top10": (96, 10)}.get(case, (512, 10))
    x = synth.activations(T, H, 900 + T)
    wr = synth.router_weight(E, H, 0.02, 21)
    bias = None
    if case in ("all_equal", "four_levels", "mostly_neg_inf"):
        x = torch.zeros_like(x)   # logits = bias exactly
        g = torch.Generator().manual_seed(5)
        bias = {"all_equal": torch.zeros(E),
                "four_levels": torch.randint(0, 4, (E,), generator=g).float() * 0.5,
                "mostly_neg_inf": torch.full((E,), float("-inf")).index_put_(
                    (torch.randperm(E, generator=g)[:5],), torch.randn(5, generator=g))}[case]
    ids, w = X.router_topk(x.to(DEV), wr.to(DEV), bias.to(DEV) if bias is not None else None, topk)
    rid, rw, _ = O.router(bits(x), bits(wr), bias.numpy() if bias is not None else None, topk)
    assert np.array_equal(ids.cpu().numpy(), rid)
    assert np.allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)
    if case == "all_equal":
        assert np.array_equal(ids.cpu().numpy(), np.tile(np.arange(topk, dtype=np.int32), (T, 1)))


@pytest.mark.parametrize("T", [1, 6, 12, 150])
def test_router_ties_to_lower_id(T):
    """Duplicated router rows give exactly equal logits: the lower expert id is selected first."""
    H, E, topk = 2048, 512, 10
    x = synth.activations(T, H, 300 + T)
    wr = synth.router_weight(E, H, 0.02, 9)
    wr[256:] = wr[:256]
    ids, w = X.router_topk(x.to(DEV), wr.to(DEV), None, topk)
    rid, rw, _ = O.router(bits(x), bits(wr), None, topk)
    assert np.array_equal(ids.cpu().numpy(), rid)
    assert np.allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)
    idn = ids.cpu().numpy()
    for row in idn:   # every pair (e, e + 256) appears with the lower id first
        pos = {int(e): i for i, e in enumerate(row)}
        for e in pos:
            if e < 256 and e + 256 in pos:
                assert pos[e] < pos[e + 256]


# ------------------------------------------------------------------------------------------------ decode layer
def check_decode(x, ids, w, ptrs, views, H, I, K, E, kinfo=None):
    """bf16 product output and fp32 layer output of the CUDA decode path against the oracle."""
    xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
    kd = kinfo.to(DEV) if kinfo is not None else None
    out = X.moe_decode(xd, idd, wd, ptrs, I, K, E, kinfo=kd)
    o32 = X.moe_decode(xd, idd, wd, ptrs, I, K, E, kinfo=kd,
                       out=torch.empty(x.shape[0], H, dtype=torch.float32, device=DEV))
    ki = kinfo.numpy() if kinfo is not None else None
    blobs = oracle_blobs(views, ids.numpy())
    ref = O.moe_layer(bits(x), ids.numpy(), w.numpy(), blobs, H, I, K or 3, kinfo=ki)
    ref32 = O.moe_layer(bits(x), ids.numpy(), w.numpy(), blobs, H, I, K or 3, kinfo=ki, out_f32=True)
    assert_close_f32(o32.cpu().numpy(), ref32)
    return assert_close_layer(bits(out), ref)


def _route(T, E, topk, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, topk, generator=g)
    w = (w / w.sum(1, keepdim=True)).float()
    return ids, w


@pytest.mark.parametrize("T", [1, 3, 8, 11])
def test_decode_layer_small(T):
    H, I, E, topk, K = 256, 256, 16, 4, 3
    blobs, ptrs, views = make_layer(E, H, I, K, seed=21)
    x = synth.activations(T, H, 5 + T)
    ids, w = _route(T, E, topk, T)
    check_decode(x, ids, w, ptrs, views, H, I, K, E)


@pytest.mark.parametrize("T", [4, 6, 7])
def test_decode_layer_top10_shared_experts(T):
    """Top-10 of 16 experts: 40 / 60 picks go through the small-batch grouping (two picks per lane, most experts
    shared by several tokens), 70 through the grouped path."""
    H, I, E, topk, K = 256, 128, 16, 10, 3
    blobs, ptrs, views = make_layer(E, H, I, K, seed=23)
    x = synth.activations(T, H, 40 + T)
    ids, w = _route(T, E, topk, 60 + T)
    check_decode(x, ids, w, ptrs, views, H, I, K, E)


@pytest.mark.parametrize("T", [1, 4])
def test_decode_layer_full_shape(T):
    """Config 1 (T=1) and the bs-4 decode shape: H=2048, I=768, 512 experts, top-10, K=3, router in the loop."""
    H, I, E, topk, K = 2048, 768, 512, 10, 3
    blobs, ptrs, views = make_layer(E, H, I, K, seed=0)
    x = synth.activations(T, H, 0)
    wr = synth.router_weight(E, H, 0.02, 0)
    ids, w = X.router_topk(x.to(DEV), wr.to(DEV), None, topk)
    rid, rw, _ = O.router(bits(x), bits(wr), None, topk)
    assert np.array_equal(ids.cpu().numpy(), rid)
    check_decode(x, torch.from_numpy(rid), torch.from_numpy(rw), ptrs, views, H, I, K, E)


def test_decode_mixed_k():
    H, I, E, topk, T = 256, 256, 8, 4, 3
    kinfo = [synth.mixed_k(7, e) for e in range(E)]
    arena, ptrs, views = make_layer(E, H, I, 0, seed=7, kinfo=kinfo)
    ki = torch.tensor([synth.kinfo_pack(*k) for k in kinfo], dtype=torch.int32)
    x = synth.activations(T, H, 9)
    ids, w = _route(T, E, topk, 4)
    check_decode(x, ids, w, ptrs, views, H, I, 0, E, kinfo=ki)


def test_zero_weight_picks_and_duplicates():
    """Weight-0 picks (tier-masked) are skipped: same output as computing them; all-masked token -> zeros."""
    H, I, E, topk, K, T = 256, 128, 8, 4, 3, 3
    blobs, ptrs, views = make_layer(E, H, I, K, seed=3)
    x = synth.activations(T, H, 1)
    ids = torch.tensor([[1, 2, 0, 0], [3, 3, 3, 3], [5, 6, 7, 1]], dtype=torch.int32)
    w = torch.tensor([[0.5, 0.5, 0.0, 0.0], [0.0, 0.0, 0.0, 0.0], [0.1, 0.2, 0.3, 0.4]], dtype=torch.float32)
    check_decode(x, ids, w, ptrs, views, H, I, K, E)
    out = X.moe_decode(x.to(DEV), ids.to(DEV), w.to(DEV), ptrs, I, K, E)
    assert torch.all(out[1].float() == 0)


def test_small_batch_expert_with_more_than_eight_picks():
    """One expert picked 10 times in a small batch (repeated within tokens): its picks span two entries of at most
    8 tokens each, as in the grouped path."""
    H, I, E, topk, K, T = 256, 128, 8, 4, 3, 3
    blobs, ptrs, views = make_layer(E, H, I, K, seed=5)
    x = synth.activations(T, H, 3)
    ids = torch.tensor([[2, 2, 2, 2], [2, 2, 2, 2], [2, 4, 2, 6]], dtype=torch.int32)
    w = torch.rand(T, topk, generator=torch.Generator().manual_seed(8)).float()
    check_decode(x, ids, w, ptrs, views, H, I, K, E)


def test_fp16_activations():
    H, I, E, topk, K, T = 256, 128, 8, 2, 3, 2
    blobs, ptrs, views = make_layer(E, H, I, K, seed=4)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(2)).half()
    ids, w = _route(T, E, topk, 5)
    out = X.moe_decode(x.to(DEV), ids.to(DEV), w.to(DEV), ptrs, I, K, E)
    ref = np.empty((T, H), np.uint16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    r = O.moe_layer(xb, ids.numpy(), w.numpy(), oracle_blobs(views, ids.numpy()), H, I, K, x_is_bf16=False)
    # oracle writes bf16; compare in fp32 with the same tolerance
    got = out.float().cpu().numpy()
    ref = (r.astype(np.uint32) << 16).view(np.float32)
    assert np.abs(got - ref).max() <= 2e-2
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 2e-3


# ------------------------------------------------------------------------------------------------ align
@pytest.mark.parametrize("P_tok", [1, 37, 300])
def test_align_bit_exact(P_tok):
    E, topk, pad = 64, 8, 32
    ids, w = _route(P_tok, E, topk, P_tok)
    ib, fb = X.align(ids.to(DEV), w.to(DEV), E, pad)
    r = O.align(ids.numpy(), w.numpy(), E, pad)
    P = ids.numel()
    A = min(P, E)
    ib = ib.cpu().numpy()
    na = int(ib[4 * A])
    assert na == len(r["act_expert"])
    assert np.array_equal(ib[:na], r["act_expert"])
    assert np.array_equal(ib[A:A + na], r["act_start"])
    assert np.array_equal(ib[2 * A:2 * A + na], r["act_cnt"])
    assert np.array_equal(ib[3 * A:3 * A + na], r["act_pstart"])
    o = 4 * A + 1
    assert np.array_equal(ib[o:o + P], r["pair_tok"])
    assert np.array_equal(ib[o + P:o + 2 * P], r["pair_of"])
    mxb = (P + pad - 1) // pad + A
    nb = int(ib[o + 2 * P + 16 + mxb])
    assert nb == r["n_blk"]
    assert np.array_equal(ib[o + 2 * P + 16:o + 2 * P + 16 + nb], r["blk_a"])
    assert np.array_equal(fb.cpu().numpy()[:P], r["pair_w"])


# ------------------------------------------------------------------------------------------------ cache
def _store(H, I, K, E, S, L, seed):
    st = ExpertStore(H, I, K, E, S, device=DEV, max_layers=L)
    for li in range(L):
        h = st.add_layer(f"model.layers.{li}.mlp")
        tmp = torch.empty(E, st.blob, dtype=torch.uint8, device=DEV)
        for e in range(E):
            synth.fill_blob(tmp[e], seed, li * E + e, H, I, K)
        h.copy_(tmp.cpu())
    torch.cuda.synchronize()
    return st


def _oracle_state(st: ExpertStore) -> O.CacheState:
    hb = st.host_base.cpu().numpy()
    cs = O.CacheState(st.max_layers, st.E, st.n_slots, hb, st.slot_base, st.blob)
    cs.ptrs_all[:] = st.ptrs_all.cpu().numpy()
    cs.slot_of[:] = st.slot_of_dev.cpu().numpy()
    cs.slot_key[:] = st.slot_key.cpu().numpy()
    cs.slot_last[:] = st.slot_last.cpu().numpy()
    cs.tick[:] = st.tick.cpu().numpy()
    cs.fill_all[:] = st.fill_all.cpu().numpy()
    return cs


def _assert_state(st, cs):
    assert np.array_equal(st.slot_of_dev.cpu().numpy(), cs.slot_of)
    assert np.array_equal(st.slot_key.cpu().numpy(), cs.slot_key)
    assert np.array_equal(st.slot_last.cpu().numpy(), cs.slot_last)
    assert np.array_equal(st.ptrs_all.cpu().numpy(), cs.ptrs_all)
    assert np.array_equal(st.tick.cpu().numpy(), cs.tick)
    assert np.array_equal(st.fill_all.cpu().numpy(), cs.fill_all)


def test_forward_cached_matches_forward_and_oracle_state():
    """The reference's own invariant (n111_test.py:207-211): cached output == all-resident output, bitwise; plus the
    cache state after every call equals the oracle's deterministic LRU."""
    H, I, K, E, S, L, topk = 256, 128, 3, 32, 12, 3, 4
    st = _store(H, I, K, E, S, L, seed=13)
    keys = list(st.layer_index)
    gold = {k: torch.tensor(st._host_ptr[k].tolist(), dtype=torch.int64, device=DEV) for k in keys}
    cs = _oracle_state(st)
    for step in range(12):
        li = step % L
        T = 1 + step % 3
        x = synth.activations(T, H, 200 + step).to(DEV)
        ids, w = _route(T, E, topk, 300 + step)
        idd, wd = ids.to(DEV), w.to(DEV)
        y = st.forward_cached(keys[li], x, idd, wd, max_fill=3 if step % 4 == 3 else None)
        yr = exops.moe_decode(x, idd, wd, gold[keys[li]], I, K, E)
        torch.cuda.synchronize()
        assert torch.equal(y, yr), step
        ni, nw = ids.numpy().copy(), w.numpy().copy()
        cs.ensure(ni, nw, li, max_fill=3 if step % 4 == 3 else E)
        cs.commit(li)
        _assert_state(st, cs)
    # slots hold exactly the blobs of their owners
    sk = st.slot_key.cpu().numpy()
    for s, key in enumerate(sk):
        if key >= 0:
            li, e = divmod(int(key), E)
            assert torch.equal(st.slots[s].cpu(), st.host[keys[li]][e])


def test_forward_prefill_staged_matches_host_pointers():
    """Staged prefill (moe_offload.py:348-437): each layer's non-resident experts are copied to a device staging
    buffer on a side stream, double-buffered across layers; the outputs equal the same layers read through host
    pointers, bitwise, over two passes of the layers."""
    H, I, K, E, S, L, topk, T = 256, 128, 3, 32, 12, 3, 4, 300
    st = _store(H, I, K, E, S, L, seed=29)
    keys = list(st.layer_index)
    for li, key in enumerate(keys):
        st.make_resident(key, list(range(li, E, 8)))   # four experts per layer in VRAM, the rest staged
    torch.cuda.synchronize()
    gold = {k: torch.tensor(st._host_ptr[k].tolist(), dtype=torch.int64, device=DEV) for k in keys}
    for rep in range(2):
        for li, key in enumerate(keys):
            x = synth.activations(T, H, 900 + 10 * rep + li).to(DEV)
            ids, w = _route(T, E, topk, 950 + 10 * rep + li)
            idd, wd = ids.to(DEV), w.to(DEV)
            y = st.forward_prefill_staged(key, x, idd, wd)
            yr = st.forward(key, x, idd, wd, ptrs=gold[key])
            torch.cuda.synchronize()
            assert torch.equal(y, yr), (rep, li)


@pytest.mark.parametrize("T,topk", [(2, 4), (6, 10)])
def test_tier_mask_ring_and_safe(T, topk):
    H, I, K, E, S, L = 256, 128, 3, 16, 6, 2
    st = _store(H, I, K, E, S, L, seed=17)
    keys = list(st.layer_index)
    ram_res = torch.zeros(L * E, dtype=torch.uint8, device=DEV)
    ram_res[[0, 1, 2, 16, 17]] = 1            # layer 0: experts 0-2 RAM-resident; layer 1: 0-1
    ring = torch.zeros(1 + 8, dtype=torch.int32, device=DEV)
    safe = torch.zeros(L, dtype=torch.int32, device=DEV)
    X.moe_set_tier(ram_res, ring, safe)
    try:
        cs = _oracle_state(st)
        rr, rg = ram_res.cpu().numpy(), ring.cpu().numpy()
        sf = safe.cpu().numpy()
        for step in range(6):
            li = step % L
            x = synth.activations(T, H, 400 + step).to(DEV)
            ids, w = _route(T, E, topk, 500 + step)
            idd, wd = ids.to(DEV), w.to(DEV)
            y = st.forward_cached(keys[li], x, idd, wd)
            ni, nw = ids.numpy().copy(), w.numpy().copy()
            cs.ensure(ni, nw, li, max_fill=E, ram_res=rr, ring=rg, safe=sf)
            cs.commit(li)
            torch.cuda.synchronize()
            assert np.array_equal(idd.cpu().numpy(), ni) and np.array_equal(wd.cpu().numpy(), nw)
            assert np.array_equal(ring.cpu().numpy(), rg)
            _assert_state(st, cs)
            views = [st.host[keys[li]][e] for e in range(E)]
            ref = O.moe_layer(bits(x.cpu()), ni, nw, oracle_blobs(views, ni), H, I, K)
            assert_close_layer(bits(y), ref)
    finally:
        X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.int32))


def test_victim_write_back_restores_dropped_host_copies():
    """Victim write-back (VictimCopyKernel, exl3_moe.a8.sycl:1168-1189, with the RAM-flag rule of the victim list
    :1010-1018): an evicted slot whose expert the RAM tier no longer holds is copied back to the expert's host
    address and flagged resident again; a victim the tier still holds is skipped (-1 in the list)."""
    H, I, K, E, S, L = 256, 128, 3, 16, 4, 1
    st = _store(H, I, K, E, S, L, seed=23)
    key = list(st.layer_index)[0]
    blobs = st.host[key].clone()
    gold = torch.tensor(st._host_ptr[key].tolist(), dtype=torch.int64, device=DEV)
    ram_res = torch.zeros(L * E, dtype=torch.uint8, device=DEV)
    ram_res[:8] = 1
    ring = torch.zeros(1 + 8, dtype=torch.int32, device=DEV)
    safe = torch.zeros(L, dtype=torch.int32, device=DEV)
    vict = torch.zeros(1 + 2 * E, dtype=torch.int32, device=DEV)
    X.moe_set_tier(ram_res, ring, safe)
    X.moe_set_victims(vict)
    try:
        cs = _oracle_state(st)
        rr, rg, sf = ram_res.cpu().numpy(), ring.cpu().numpy(), safe.cpu().numpy()
        vo = np.zeros(1 + 2 * E, np.int32)

        def step(picks, seed):
            x = synth.activations(1, H, seed).to(DEV)
            ids = torch.tensor([picks], dtype=torch.int32)
            w = torch.full((1, len(picks)), 1.0 / len(picks))
            y = st.forward_cached(key, x, ids.to(DEV), w.to(DEV))
            yr = X.moe_decode(x, ids.to(DEV), w.to(DEV), gold, I, K, E)
            torch.cuda.synchronize()
            assert torch.equal(y, yr), picks
            cs.ensure(ids.numpy().copy(), w.numpy().copy(), 0, max_fill=E, ram_res=rr, ring=rg, safe=sf, vict=vo)
            cs.commit(0)
            _assert_state(st, cs)
            assert np.array_equal(vict.cpu().numpy()[:1 + 2 * len(picks)], vo[:1 + 2 * len(picks)])

        step([0, 1, 2, 3], 61)                     # four fills into empty slots: no write-back
        ram_res[[0, 1]] = 0                        # the RAM tier drops experts 0 and 1 while they sit in VRAM
        rr[[0, 1]] = 0
        st.host[key][0].zero_()
        st.host[key][1].zero_()
        torch.cuda.synchronize()
        step([4, 5, 6, 7], 62)                     # all four slots evicted
        v = vict.cpu().numpy()
        assert int(v[0]) == 4 and sorted(int(v[1 + 2 * i]) for i in range(4)) == [-1, -1, 0, 1]
        assert torch.equal(st.host[key][0], blobs[0]) and torch.equal(st.host[key][1], blobs[1])
        assert ram_res[:4].tolist() == [1, 1, 1, 1]
    finally:
        X.moe_set_victims(torch.zeros(0, dtype=torch.int32))
        X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.int32))


def test_tier_host_loop_admits_missed_experts():
    """The RAM tier's host loop (exl3b200.tier.TierHost) against the decode kernels: picks in neither VRAM nor RAM
    are masked and logged; the loop fetches them (host copies are always valid here, so fetch completes at once) and
    uploads their flags; the next call reads them unmasked, bitwise equal to the all-host-pointer layer."""
    from exl3b200.tier import TierHost
    H, I, K, E, S, L = 256, 128, 3, 16, 4, 1
    st = _store(H, I, K, E, S, L, seed=31)
    key = list(st.layer_index)[0]
    gold = torch.tensor(st._host_ptr[key].tolist(), dtype=torch.int64, device=DEV)
    ram_res = torch.zeros(L * E, dtype=torch.uint8, device=DEV)
    ram_res[0] = 1                             # the safe expert
    ring = torch.zeros(1 + 16, dtype=torch.int32, device=DEV)
    safe = torch.zeros(L, dtype=torch.int32, device=DEV)
    pinned = np.zeros(L * E, dtype=bool)
    pinned[0] = True
    X.moe_set_tier(ram_res, ring, safe)
    try:
        tier = TierHost(ram_res, ring, st.slot_of_dev, budget=L * E, fetch=lambda k: tier.fill_done(k),
                        pinned=pinned)
        ids = torch.tensor([[5, 6, 7, 8], [9, 10, 11, 12]], dtype=torch.int32)
        w = torch.full((2, 4), 0.25)
        x = synth.activations(2, H, 77).to(DEV)
        idd, wd = ids.to(DEV), w.to(DEV)
        st.forward_cached(key, x, idd, wd)     # every pick masked (VRAM and RAM hold none of them) and logged
        torch.cuda.synchronize()
        assert torch.all(wd == 0) and int(ring[0]) == 8
        for _ in range(3):                     # snapshot, fetch, flag upload
            tier.step()
        torch.cuda.synchronize()
        assert ram_res[5:13].cpu().tolist() == [1] * 8 and tier.stats["fetches"] == 8
        idd, wd = ids.to(DEV), w.to(DEV)
        y = st.forward_cached(key, x, idd, wd)
        yr = exops.moe_decode(x, ids.to(DEV), w.to(DEV), gold, I, K, E)
        torch.cuda.synchronize()
        assert torch.equal(idd.cpu(), ids) and torch.equal(wd.cpu(), w)   # nothing masked any more
        assert torch.equal(y, yr)
    finally:
        X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.int32))


def test_prefetch_claims_and_copies():
    H, I, K, E, S, L = 256, 128, 3, 16, 5, 1
    st = _store(H, I, K, E, S, L, seed=19)
    key = next(iter(st.layer_index))
    cs = _oracle_state(st)
    ids = torch.tensor([3, 9, 3, 1], dtype=torch.int32)
    st.prefetch(key, ids.to(DEV), max_fill=8)
    torch.cuda.synchronize()
    ni = ids.numpy().copy()
    cs.ensure(ni, np.ones(4, np.float32), 0, max_fill=min(8, E), prefetch=True)
    p = cs.ptrs_all[:E].copy()
    for i in range(cs.fill_list[0]):
        p[cs.fill_list[1 + i]] = cs.slot_base + int(cs.pf_slot[i]) * cs.blob
    cs.ptrs_all[:E] = p
    _assert_state(st, cs)
    for e in (1, 3, 9):
        s = int(st.slot_of_dev[e])
        assert s >= 0 and torch.equal(st.slots[s].cpu(), st.host[key][e])


def test_zero_copy_host_reads():
    """n_slots = 0: every expert is read from pinned host memory through the pointer table."""
    H, I, K, E, topk, T = 256, 128, 3, 8, 3, 2
    st = _store(H, I, K, E, 0, 1, seed=23)
    key = next(iter(st.layer_index))
    x = synth.activations(T, H, 3)
    ids, w = _route(T, E, topk, 8)
    y = st.forward(key, x.to(DEV), ids.to(DEV), w.to(DEV))
    views = [st.host[key][e] for e in range(E)]
    ref = O.moe_layer(bits(x), ids.numpy(), w.numpy(), oracle_blobs(views, ids.numpy()), H, I, K)
    assert_close_layer(bits(y), ref)


def test_graph_capture_forward_cached():
    H, I, K, E, S, L, topk = 256, 128, 3, 16, 8, 1, 4
    st = _store(H, I, K, E, S, L, seed=29)
    key = next(iter(st.layer_index))
    x = synth.activations(1, H, 3).to(DEV)
    ids0, w0 = _route(1, E, topk, 1)
    idd, wd = ids0.to(DEV), w0.to(DEV)
    st.forward_cached(key, x, idd.clone(), wd.clone())   # warm
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    ib, wb = idd.clone(), wd.clone()
    with torch.cuda.graph(g):
        yg = st.forward_cached(key, x, ib, wb)
    for step in range(4):
        ids, w = _route(1, E, topk, 50 + step)
        ib.copy_(ids.to(DEV))
        wb.copy_(w.to(DEV))
        g.replay()
        torch.cuda.synchronize()
        views = [st.host[key][e] for e in range(E)]
        ref = O.moe_layer(bits(x.cpu()), ids.numpy(), w.numpy(), oracle_blobs(views, ids.numpy()), H, I, K)
        assert_close_layer(bits(yg), ref)
