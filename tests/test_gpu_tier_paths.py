"""GPU tests of the victim ring (ops.moe_set_victim_ring in the decode chain, TierHost's drain) and StoreStager
(prefill streamed from the pack store).  Both paths are also checked on the CPU (tests/test_tier_sim.py,
tests/test_stage.py)."""
import numpy as np
import pytest
import torch

import oracle as O
from exl3b200 import ops as X
from exl3b200 import pack_store as P, synth
from exl3b200.stage import StoreStager
from exl3b200.tier import TierHost
from test_gpu_parity import DEV, _assert_state, _oracle_state, _route, _store

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status():
    X.register()
    yield
    st = np.zeros(1, np.int32)
    from exl3b200 import _lib
    _lib.check(_lib.lib().exl3b_device_status(st.ctypes.data, 1, None))
    assert st[0] == 0, f"device status word {st[0]}"


def test_victim_ring_claims_copies_and_drains():
    """Victims needing a write-back go to a 2-slot ring (claims bit-exact against oracle.vring_claim, ram_res left
    clear, ring slots hold the evicted blobs); a third needs a slot the ring lacks and is dropped; the host loop
    drains the ring into the rows, flags them and frees the slots."""
    H, I, K, E, S, L = 256, 128, 3, 16, 4, 1
    st = _store(H, I, K, E, S, L, seed=37)
    key = list(st.layer_index)[0]
    blobs = st.host[key].clone()
    gold = torch.tensor(st._host_ptr[key].tolist(), dtype=torch.int64, device=DEV)
    ram_res = torch.zeros(L * E, dtype=torch.uint8, device=DEV)
    ram_res[:8] = 1
    ring = torch.zeros(1 + 8, dtype=torch.int32, device=DEV)
    safe = torch.zeros(L, dtype=torch.int32, device=DEV)
    vict = torch.zeros(1 + 2 * E, dtype=torch.int32, device=DEV)
    KR = 2
    meta = torch.full((4 + 2 * KR,), -1, dtype=torch.int32, device=DEV)
    meta[:4] = torch.tensor([0, 0, 0, KR], dtype=torch.int32)
    meta[4 + KR:] = 0
    sel = torch.zeros(E, dtype=torch.int32, device=DEV)
    buf = torch.zeros(KR, st.blob, dtype=torch.uint8, device=DEV)
    X.moe_set_tier(ram_res, ring, safe)
    X.moe_set_victims(vict)
    X.moe_set_victim_ring(meta, sel, buf)
    try:
        cs = _oracle_state(st)
        rr, rg, sf = ram_res.cpu().numpy(), ring.cpu().numpy(), safe.cpu().numpy()
        vo, mo, so = np.zeros(1 + 2 * E, np.int32), meta.cpu().numpy(), np.zeros(E, np.int32)

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
            O.vring_claim(vo, mo, so)
            assert np.array_equal(meta.cpu().numpy(), mo) and np.array_equal(sel.cpu().numpy()[:vo[0]], so[:vo[0]])

        step([0, 1, 2, 3], 71)
        ram_res[[0, 1, 2]] = 0                     # the tier drops three experts that sit in VRAM
        rr[[0, 1, 2]] = 0
        for e in (0, 1, 2):
            st.host[key][e].zero_()
        torch.cuda.synchronize()
        step([4, 5, 6, 7], 72)                     # evicts 0-3: 0 and 1 take the ring, 2 is dropped, 3 is in RAM
        assert int(meta[2]) == 1 and ram_res[:3].tolist() == [0, 0, 0]
        for r in range(KR):
            k = int(meta[4 + r])
            assert torch.equal(buf[r].cpu(), blobs[k]), (r, k)
        row = lambda k: st.host[key][k]
        tier = TierHost(ram_res, ring, st.slot_of_dev, budget=L * E, fetch=lambda k: None,
                        pinned=np.arange(L * E) == 0, vring=(meta, buf, row), slot_last=st.slot_last)
        for _ in range(4):
            tier.step()
        torch.cuda.synchronize()
        assert torch.equal(st.host[key][0], blobs[0]) and torch.equal(st.host[key][1], blobs[1])
        assert ram_res[:2].tolist() == [1, 1] and meta[4:4 + KR].tolist() == [-1, -1]
        assert tier.stats["ring_drained"] == 2
    finally:
        X.moe_set_victim_ring(torch.zeros(0, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                              torch.zeros(0, dtype=torch.uint8))
        X.moe_set_victims(torch.zeros(0, dtype=torch.int32))
        X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.int32))


def test_store_stager_matches_host_pointers(tmp_path):
    """Prefill with the non-VRAM experts streamed from a pack-store file equals the same layers read through host
    pointers, bitwise, over two passes of three layers."""
    H, I, K, E, S, L, topk, T = 256, 128, 3, 32, 12, 3, 4, 300
    st = _store(H, I, K, E, S, L, seed=47)
    keys = list(st.layer_index)
    host = {k: st.host[k].clone() for k in keys}
    P.pack(str(tmp_path), P.StoreMeta.for_blob(L, E, K, st.blob, H, I),
           lambda layer, e: host[keys[layer]][e].numpy().tobytes())
    for li, key in enumerate(keys):
        st.make_resident(key, list(range(li, E, 8)))
    torch.cuda.synchronize()
    gold = {k: torch.tensor(st._host_ptr[k].tolist(), dtype=torch.int64, device=DEV) for k in keys}
    reader = P.StoreReader(str(tmp_path))
    stager = StoreStager(st, reader, read_ahead=1, threads=4)
    try:
        for rep in range(2):
            for li, key in enumerate(keys):
                x = synth.activations(T, H, 700 + 10 * rep + li).to(DEV)
                ids, w = _route(T, E, topk, 750 + 10 * rep + li)
                y = stager.stage_forward(key, x, ids.to(DEV), w.to(DEV))
                yr = st.forward(key, x, ids.to(DEV), w.to(DEV), ptrs=gold[key])
                torch.cuda.synchronize()
                assert torch.equal(y, yr), (rep, li)
    finally:
        stager.close()
        reader.close()
