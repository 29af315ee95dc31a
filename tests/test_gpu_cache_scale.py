"""The device cache step at the decode stack's scale, bit for bit against the oracle.

configs[1] sizes the cache: 48 layers x 512 experts (24,576 keys) over 8,000 slots, top-10 of Zipf(1.1)-skewed logits,
decode batches of 1 and 4 tokens.  The cache starts full (each layer's hottest Zipf ranks resident, every slot stamped 0,
so the first victims are chosen by the tie rule), half of the keys are flagged RAM-resident (their misses fill and evict
an LRU slot) and the rest are tier-masked (logged in the miss ring, rewritten to the layer's safe expert with weight 0).
After every call the slot map, slot owners, LRU stamps, pointer table, tick, fill state, fill list, miss ring and the
in-place id / weight rewrite equal the oracle's restatement of launch_ensure (exl3_moe.a8.sycl:837-1040) with the
deterministic tie rule: misses in ascending expert id, victims in ascending (slot_last + 1, slot).

The expert width is small (H = I = 128): the cache step reads no weights, and small blobs keep the 24,576 host copies
in a few hundred MB of pinned memory.  The layer outputs of the same calls are checked elsewhere.
"""
import numpy as np
import pytest
import torch

import oracle as O
from exl3b200 import ExpertStore, synth
from exl3b200 import ops as X

pytestmark = pytest.mark.gpu
DEV = "cuda"
L, E, S, TOPK = 48, 512, 8000, 10


def _zipf_ids(T: int, layer: int, rng: np.random.Generator) -> np.ndarray:
    """Top-10 of -1.1 ln(rank) + Gumbel noise per token: a Zipf(1.1) sample without replacement."""
    rank = np.empty(E, np.float64)
    rank[synth.zipf_rank(E, layer, 1).numpy()] = np.arange(1, E + 1)
    logits = -1.1 * np.log(rank)[None, :] + rng.gumbel(size=(T, E))
    return np.argsort(-logits, axis=1, kind="stable")[:, :TOPK].astype(np.int32)


def test_cache_step_at_decode_stack_scale():
    X.register()
    H = I = 128
    K = 3
    st = ExpertStore(H, I, K, E, S, device=DEV, max_layers=L)
    for li in range(L):
        st.add_layer(f"model.layers.{li}.mlp").zero_()
    keys = list(st.layer_index)
    per = [S // L + (1 if li < S % L else 0) for li in range(L)]
    for li, key in enumerate(keys):   # the cache starts full: each layer's hottest ranks
        st.make_resident(key, synth.zipf_rank(E, li, 1)[:per[li]].tolist())
    torch.cuda.synchronize()
    assert st.resident_count() == S

    rng = np.random.default_rng(11)
    ram_res = torch.from_numpy((rng.random(L * E) < 0.5).astype(np.uint8))
    safe = torch.tensor([int(synth.zipf_rank(E, li, 1)[0]) for li in range(L)], dtype=torch.int32)
    ram_res[torch.arange(L) * E + safe.long()] = 1
    ring_cap = 64
    ram_d, ring_d, safe_d = ram_res.to(DEV), torch.zeros(1 + ring_cap, dtype=torch.int32, device=DEV), safe.to(DEV)
    X.moe_set_tier(ram_d, ring_d, safe_d)
    try:
        hb = st.host_base.cpu().numpy()
        cs = O.CacheState(L, E, S, hb, st.slot_base, st.blob)
        cs.ptrs_all[:] = st.ptrs_all.cpu().numpy()
        cs.slot_of[:] = st.slot_of_dev.cpu().numpy()
        cs.slot_key[:] = st.slot_key.cpu().numpy()
        cs.slot_last[:] = st.slot_last.cpu().numpy()
        cs.tick[:] = st.tick.cpu().numpy()
        cs.fill_all[:] = st.fill_all.cpu().numpy()
        rr, rg, sf = ram_res.numpy().copy(), ring_d.cpu().numpy(), safe.numpy().copy()
        fills = masked = 0
        for step in range(96):
            li = int(rng.integers(L))
            T = 1 if step % 2 == 0 else 4
            ids = _zipf_ids(T, li, rng)
            w = rng.random((T, TOPK)).astype(np.float32)
            w /= w.sum(1, keepdims=True)
            x = synth.activations(T, H, 5000 + step).to(DEV)
            idd, wd = torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV)
            st.forward_cached(keys[li], x, idd, wd)
            ni, nw = ids.copy(), w.copy()
            n = cs.ensure(ni, nw, li, max_fill=E, ram_res=rr, ring=rg, safe=sf)
            fl = cs.fill_list[:1 + n].copy()
            cs.commit(li)
            torch.cuda.synchronize()
            fills += n
            masked += int(((ni == sf[li]) & (nw == 0)).sum())
            where = f"step {step} (layer {li}, T={T})"
            assert np.array_equal(idd.cpu().numpy(), ni), where
            assert np.array_equal(wd.cpu().numpy(), nw), where
            assert np.array_equal(st.fill_list.cpu().numpy()[:1 + n], fl), where
            assert np.array_equal(ring_d.cpu().numpy(), rg), where
            assert np.array_equal(st.slot_of_dev.cpu().numpy(), cs.slot_of), where
            assert np.array_equal(st.slot_key.cpu().numpy(), cs.slot_key), where
            assert np.array_equal(st.slot_last.cpu().numpy(), cs.slot_last), where
            assert np.array_equal(st.ptrs_all.cpu().numpy(), cs.ptrs_all), where
            assert np.array_equal(st.tick.cpu().numpy(), cs.tick), where
            assert np.array_equal(st.fill_all.cpu().numpy(), cs.fill_all), where
        # the run exercised what it is for: fills that evicted LRU slots, and masked picks logged in the ring
        assert fills >= 50 and masked >= 50, (fills, masked)
        assert int(rg[0]) == masked
    finally:
        X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.int32))
