"""The routed cached decode (router + forward_cached in one call; small batches select the picks inside the decode
kernels) against router_topk followed by forward_cached, on two stores built the same way: outputs, picks, weights,
the cache state and the miss ring agree bit for bit after every call.  The cache has fewer slots than experts and half
of the keys are RAM-resident, so calls hit, fill (evicting LRU slots) and mask; batch sizes cover the in-kernel
selection (M topk <= 32) and the two-call fallback."""
import numpy as np
import pytest
import torch

from exl3b200 import ExpertStore, synth
from exl3b200 import ops as X

pytestmark = pytest.mark.gpu
DEV = "cuda"
L, E, S, H, I, K, TOPK = 3, 64, 40, 256, 256, 3, 8


def _store():
    st = ExpertStore(H, I, K, E, S, device=DEV, max_layers=L)
    for li in range(L):
        blobs = torch.stack([synth.make_blob(17, li * E + e, H, I, K) for e in range(E)])
        st.add_layer(f"model.layers.{li}.mlp", blobs)
    for li, key in enumerate(st.layer_index):
        st.make_resident(key, list(range(li, li + 12)))
    torch.cuda.synchronize()
    return st


def _tier():
    g = torch.Generator().manual_seed(3)
    ram_res = (torch.rand(L * E, generator=g) < 0.5).to(torch.uint8)
    safe = torch.tensor([li for li in range(L)], dtype=torch.int32)   # resident by construction
    ram_res[torch.arange(L) * E + safe.long()] = 1
    ring = torch.zeros(1 + 32, dtype=torch.int32, device=DEV)
    X.moe_set_tier(ram_res.to(DEV), ring, safe.to(DEV))
    return ring


def _where(st, addrs):
    """Table addresses as store-independent codes: slot index for a slot address, -1 for the key's own host copy,
    -2 for anything else (0 included)."""
    a = addrs.cpu().numpy().astype(np.int64)
    k = np.arange(a.size)
    hb = st.host_base.cpu().numpy().astype(np.int64)[k // E] + (k % E) * st.blob   # the key's host copy
    base, n = int(st.slot_base), int(st.n_slots)
    in_slot = (a >= base) & (a < base + n * st.blob)
    return np.where(in_slot, (a - base) // st.blob, np.where(a == hb, -1, -2))


def _state(st, ring):
    return [t.cpu().numpy().copy() for t in (st.slot_of_dev, st.slot_key, st.slot_last, st.tick, ring)] + \
        [_where(st, st.ptrs_all), _where(st, st.fill_all)]


def test_routed_decode_matches_router_then_cached():
    X.register()
    routers = [(synth.router_weight(E, H, 0.05, 40 + li).to(DEV), synth.normal_bias(E, 1.0, 50 + li).to(DEV))
               for li in range(L)]
    calls = [(li % L, m) for li, m in enumerate([1, 1, 2, 3, 4, 1, 8, 2, 1, 3, 1, 5])]
    xs = [synth.activations(m, H, 900 + n).to(DEV) for n, (_, m) in enumerate(calls)]
    runs = []
    try:
        for routed in (False, True):
            st, ring = _store(), _tier()
            keys = list(st.layer_index)
            rec = []
            for n, (li, m) in enumerate(calls):
                wr, b = routers[li]
                out = torch.empty(m, H, dtype=torch.float32, device=DEV)
                if routed:
                    _, ids, w = st.forward_cached_routed(keys[li], xs[n], wr, b, TOPK, out=out)
                else:
                    ids, w = X.router_topk(xs[n], wr, b, TOPK)
                    st.forward_cached(keys[li], xs[n], ids, w, out=out)
                torch.cuda.synchronize()
                rec.append([out.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()] + _state(st, ring))
            runs.append(rec)
            del st
    finally:
        X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.int32))
    names = ["out", "ids", "w", "slot_of", "slot_key", "slot_last", "tick", "ring", "ptrs_all", "fill_all"]
    for n, (a, b) in enumerate(zip(*runs)):
        for nm, u, v in zip(names, a, b):
            assert np.array_equal(u.view(np.uint8), v.view(np.uint8)), f"call {n} {calls[n]}: {nm} differs"
    # the run exercised fills and masks
    assert runs[0][-1][7][0] > 0, "no masked pick was logged"
