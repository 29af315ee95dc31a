"""CPU: the RAM tier end to end, after the reference harness's "sim" phase (experimental/n111-victim-ring/
n111_test.py:8, 255-300): small VRAM and RAM tiers, so many evictions, every read checked against the golden data,
periodic audits of every flagged page.

The device is played by the oracle's cache step (oracle.CacheState.ensure: tier mask, miss ring, LRU slots, victim
list) over real memory: a slot arena and a RAM-tier arena whose addresses sit in the pointer table.  Fills, victim
write-backs and reads go through those addresses, as the kernels' copies do.  The host side is the product's own:
exl3b200.tier.TierHost steps once per decode step, its fetch() is a pack_store.StoreFetcher reading records from a
store file on reader threads, and its release() zeroes the key's RAM row (the reference punches the page out).

Invariants checked at every call or audit:
  * every pick, after the mask, reads its own expert's record through the table;
  * a pick is masked exactly when its expert is in neither VRAM nor RAM;
  * every key flagged in ram_res has its record in its RAM row, every slot holds its owner's record;
  * release() is never called for a key whose flag is set.
"""
import ctypes
import mmap
import time

import numpy as np
import pytest
import torch

import oracle as O
from exl3b200 import pack_store as P
from exl3b200.ops import tier_prefetch_ids
from exl3b200.tier import TierHost

L, E, S, TOPK, T = 3, 16, 6, 4, 2
BLOB = 8192 + 320                # not a page multiple: records carry padding
RING = 16


def _record(layer, e):
    return np.random.default_rng(1000 * layer + e).integers(0, 256, BLOB, dtype=np.uint8)


def _aligned(nbytes):
    return np.frombuffer(mmap.mmap(-1, nbytes), dtype=np.uint8)


def _route(rng):
    """Zipf-skewed picks, distinct per token."""
    p = 1.0 / np.arange(1, E + 1) ** 1.1
    perm = rng.permutation(E)
    return np.stack([perm[rng.choice(E, TOPK, replace=False, p=p / p.sum())] for _ in range(T)]).astype(np.int32)


@pytest.mark.parametrize("prefetch,ring", [(False, False), (True, False), (False, True), (True, True)])
def test_tier_end_to_end(tmp_path, prefetch, ring):
    """prefetch: after each call the next layer's predicted experts are planned for copy-engine prefetch (filtered by
    tier_prefetch_ids, claimed and pinned by the oracle's plan step); an emulated copy engine lands each plan after a
    random delay, reading the host rows then, and every call first commits what has landed, as the op does.
    ring: victims go to a 3-slot victim ring (oracle.vring_claim) instead of to their rows, unflagged; the host loop
    drains the ring into the rows and flags them."""
    meta = P.StoreMeta.for_blob(L, E, 3, BLOB, 0, 0)
    P.pack(str(tmp_path), meta, lambda layer, e: _record(layer, e).tobytes())
    gold = np.stack([_record(k // E, k % E) for k in range(L * E)])
    rec = meta.rec

    ram = _aligned(L * E * rec).reshape(L * E, rec)              # the RAM tier: one record-sized row per key
    slots = _aligned(S * BLOB).reshape(S, BLOB)                  # VRAM slots
    ram_base = ram.ctypes.data
    host_base = np.array([ram_base + layer * E * rec for layer in range(L)], np.int64)
    cs = O.CacheState(L, E, S, host_base, slots.ctypes.data, BLOB, hstride=rec)

    ram_res_t = torch.zeros(L * E, dtype=torch.uint8)
    ring_t = torch.zeros(1 + RING, dtype=torch.int32)
    rr, rg = ram_res_t.numpy(), ring_t.numpy()
    safe = np.zeros(L, np.int32)                                 # expert 0 of every layer stays in RAM
    pinned = np.zeros(L * E, bool)
    for layer in range(L):
        key = layer * E
        ram[key, :BLOB] = gold[key]
        rr[key] = 1
        pinned[key] = True

    released, bad_release = [], []

    def release(key):
        if rr[key]:
            bad_release.append(key)
        ram[key] = 0
        released.append(key)

    def read(addr):
        return np.frombuffer(ctypes.string_at(int(addr), BLOB), dtype=np.uint8)

    def audit():
        for key in np.flatnonzero(rr).tolist():
            assert np.array_equal(ram[key, :BLOB], gold[key]), ("ram row", key)
        for s in range(S):
            owner = int(cs.slot_key[s])
            if owner >= 0 and int(cs.slot_last[s]) != 0x7FFFFFFF:   # a pinned slot's copy may not have landed
                assert np.array_equal(slots[s], gold[owner]), ("slot", s, owner)

    reader = P.StoreReader(str(tmp_path))
    rng = np.random.default_rng(3)
    vict = np.zeros(1 + 2 * E, np.int32)
    n_masked = n_victims = n_planned = 0
    cs.cepf_reset()
    done = np.zeros(L, np.int32)
    in_flight = []                                             # plans published, not landed: (layer, seq, pairs)
    safe_t = torch.from_numpy(safe)

    K_RING = 3
    meta_t = torch.full((4 + 2 * K_RING,), -1, dtype=torch.int32)
    meta_t[:4] = torch.tensor([0, 0, 0, K_RING], dtype=torch.int32)
    meta_t[4 + K_RING:] = 0
    ring_buf = torch.zeros(K_RING, BLOB, dtype=torch.uint8)
    sel = np.zeros(E, np.int32)
    vring = (meta_t, ring_buf, lambda key: torch.from_numpy(ram[key])) if ring else None

    def copy_engine(all_of_them=False):
        while in_flight and (all_of_them or rng.random() < 0.4):
            layer, seq, pairs = in_flight.pop(0)
            for e, s in pairs:
                slots[s] = ram[layer * E + e, :BLOB]
            done[layer] = seq
    with P.StoreFetcher(reader, dest=lambda key: torch.from_numpy(ram[key]), done=lambda key: tier.fill_done(key),
                        threads=3) as fetcher:
        tier = TierHost(ram_res_t, ring_t, torch.from_numpy(cs.slot_of), budget=20, fetch=fetcher.fetch,
                        release=release, pinned=pinned, min_age=2, max_inflight=6, vring=vring,
                        slot_last=torch.from_numpy(cs.slot_last))
        hot = [layer * E + e for e in (1, 2) for layer in range(L)]
        assert tier.warm(hot, timeout=10) == len(hot)             # start-up fill of the hottest experts
        assert all(rr[k] == 1 and np.array_equal(ram[k, :BLOB], gold[k]) for k in hot)
        for step in range(80):
            for layer in range(L):
                ids = _route(rng)
                w = np.full(ids.shape, 1.0 / TOPK, np.float32)
                keys = layer * E + ids
                if prefetch:
                    copy_engine()
                    cs.cepf_commit(done)
                expect_masked = (cs.slot_of[keys] < 0) & (rr[keys] == 0)
                cs.ensure(ids, w, layer, max_fill=E, ram_res=rr, ring=rg, safe=safe, vict=vict)
                assert np.array_equal(ids[expect_masked], np.full(expect_masked.sum(), safe[layer]))
                assert (w[expect_masked] == 0).all() and (w[~expect_masked] > 0).all()
                n_masked += int(expect_masked.sum())
                if ring:                                       # victims into the ring, unflagged
                    O.vring_claim(vict, meta_t.numpy(), sel)
                for i in range(int(vict[0])):                  # victim write-back precedes the fills
                    old, s = int(vict[1 + 2 * i]), int(vict[2 + 2 * i])
                    if old >= 0 and not ring:
                        ram[old, :BLOB] = slots[s]
                        rr[old] = 1
                        n_victims += 1
                    elif old >= 0 and sel[i] >= 0:
                        ring_buf[sel[i]] = torch.from_numpy(slots[s])
                        n_victims += 1
                for i in range(int(cs.fill_list[0])):          # fills read the host copy the table points at
                    key = layer * E + int(cs.fill_list[1 + i])
                    slot = (int(cs.fill_all[key]) - slots.ctypes.data) // BLOB
                    slots[slot] = read(cs.ptrs_all[key])
                cs.commit(layer)
                for e in ids.reshape(-1).tolist():             # every read, through the table
                    assert np.array_equal(read(cs.ptrs_all[layer * E + e]), gold[layer * E + e]), (step, layer, e)
                if prefetch:                                   # predictions for the next layer
                    nxt = (layer + 1) % L
                    pred = tier_prefetch_ids(torch.from_numpy(_route(rng).reshape(-1)), nxt, E,
                                             torch.from_numpy(cs.slot_of), ram_res_t, safe_t).numpy()
                    r = cs.cepf_plan(pred, nxt, 4, done)
                    if r is not None and r[1]:
                        in_flight.append((nxt, r[0], r[1]))
                        n_planned += len(r[1])
            tier.step()
            if step % 10 == 7:                                 # an eager prefill call below the staging threshold
                layer = int(rng.integers(L))
                picks = rng.integers(0, E, 24).astype(np.int32)
                tier.ensure_for_prefill(layer, torch.from_numpy(picks), E, timeout=10)
                for e in np.unique(picks).tolist():             # the prefill kernels read through the table
                    k = layer * E + e
                    assert rr[k] == 1 or cs.slot_of[k] >= 0, ("not resident for prefill", k)
                    assert np.array_equal(read(cs.ptrs_all[k]), gold[k]), ("prefill read", step, k)
            if step % 5 == 4:
                audit()
            time.sleep(0.002)                                  # lets the reader threads land some fetches
        for _ in range(500):                                   # no more decode: every fetch and drain completes
            tier.step()
            if not (tier.state == 1).any():
                break
            time.sleep(0.005)
        assert not (tier.state == 1).any(), np.flatnonzero(tier.state == 1)   # nothing left "fetching"
    reader.close()
    if prefetch:
        copy_engine(all_of_them=True)
        cs.cepf_commit(done)
        assert not cs.pend and n_planned > 0
    audit()
    assert not bad_release
    st = tier.stats
    assert n_masked > 0 and st["fetches"] > 0 and st["dropped"] > 0 and len(released) > 0 and n_victims > 0, \
        (n_masked, dict(st), len(released), n_victims)
    if ring:
        assert st["ring_drained"] > 0 and int(meta_t[2]) > 0, (dict(st), meta_t.tolist())   # drained, and full at times
