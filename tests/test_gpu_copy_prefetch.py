"""GPU: copy-engine expert prefetch (ExpertStore.start_copy_prefetch / plan_prefetch / stop_copy_prefetch, the
reference's moe_offload.py:264-302 over exl3_moe.a8.sycl:874-1142) against the oracle's plan / commit restatement.

The first test plays the copy engine itself, so plan, skip, commit and every cache state in between are deterministic
and compared with the oracle bit for bit.  The second runs the real host worker, whose timing decides when plans
land: there the outputs must still equal the all-host-pointer layer at every call, and after the stop every plan is
committed, nothing stays pinned and every slot holds its owner's blob."""
import numpy as np
import pytest
import torch

from exl3b200 import ops as X
from test_gpu_parity import DEV, _assert_state, _oracle_state, _route, _store

pytestmark = pytest.mark.gpu
PINNED = 0x7FFFFFFF


@pytest.fixture(autouse=True)
def _status():
    X.register()
    yield
    st = np.zeros(1, np.int32)
    from exl3b200 import _lib
    _lib.check(_lib.lib().exl3b_device_status(st.ctypes.data, 1, None))
    assert st[0] == 0, f"device status word {st[0]}"


def _gold(st):
    return {k: torch.tensor(st._host_ptr[k].tolist(), dtype=torch.int64, device=DEV) for k in st.layer_index}


def _assert_pend(st, cs):
    pend = st.pend.cpu().numpy()
    for li in range(st.done_seq.numel()):
        row = pend[li * 35:(li + 1) * 35]
        if li in cs.pend:
            seq, T, pairs = cs.pend[li]
            assert row[0] == len(pairs) and row[1] == seq and row[2] == T, (li, row[:3])
            assert [(int(row[3 + 2 * i]), int(row[4 + 2 * i])) for i in range(len(pairs))] == pairs
        else:
            assert row[0] == 0, li


def test_plan_and_commit_match_the_oracle():
    H, I, K, E, S, L = 256, 128, 3, 16, 8, 2
    st = _store(H, I, K, E, S, L, seed=41)
    keys = list(st.layer_index)
    gold = _gold(st)
    plans = X.host_alloc(L * (4 + 2 * E) * 4)
    plans.zero_()
    rec = plans.view(torch.int32).view(L, 4 + 2 * E)
    plan_seq = torch.zeros(L, dtype=torch.int32, device=DEV)
    st.done_seq = torch.zeros(L, dtype=torch.int32, device=DEV)   # copy prefetch state, the worker played below
    st.pend.zero_()
    cs = _oracle_state(st)
    cs.cepf_reset()

    def plan(li, ids, mf=8):
        X.OPS.moe_prefetch_plan(torch.tensor(ids, dtype=torch.int32, device=DEV), st.ptrs_all, li, st.slot_of_dev,
                                st.slot_key, st.slot_last, st.tick, st.host_base, st.slot_base, st.pf_list,
                                st.pf_slot, plans, plan_seq, st.pend, st.done_seq, mf, E, st.blob)
        torch.cuda.synchronize()
        r = cs.cepf_plan(np.array(ids, np.int32), li, mf, st.done_seq.cpu().numpy())
        _assert_state(st, cs)
        _assert_pend(st, cs)
        return r

    def copy_engine(li):
        seq, n = int(rec[li, 0]), int(rec[li, 1])
        for i in range(n):
            e, s = int(rec[li, 4 + 2 * i]), int(rec[li, 5 + 2 * i])
            st.slots[s].copy_(st.host[keys[li]][e].to(DEV))
        st.done_seq[li] = seq
        torch.cuda.synchronize()

    def cached(li, ids, seed):
        x = torch.randn(len(ids), H, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16).to(DEV)
        idt = torch.tensor(ids, dtype=torch.int32)
        w = torch.full(idt.shape, 1.0 / idt.shape[1])
        y = st.forward_cached(keys[li], x, idt.to(DEV), w.to(DEV))
        yr = X.moe_decode(x, idt.to(DEV), w.to(DEV), gold[keys[li]], I, K, E)
        torch.cuda.synchronize()
        assert torch.equal(y, yr), (li, ids)
        cs.cepf_commit(st.done_seq.cpu().numpy())
        cs.ensure(idt.numpy().copy(), w.numpy().copy(), li, max_fill=E)
        cs.commit(li)
        _assert_state(st, cs)
        _assert_pend(st, cs)

    seq, pairs = plan(0, [3, 5, 7, 5])
    assert seq == 1 and [e for e, _ in pairs] == [3, 5, 7]
    assert rec[0, :4].tolist() == [1, 3, int(st.tick[0]), 0]
    assert all(int(st.slot_last[s]) == PINNED for _, s in pairs)
    assert plan(0, [9]) is None and rec[0, 0] == 1              # in flight: dropped, nothing published
    cached(0, [[3, 9], [5, 1]], 1)                                # pending experts read from host, pins kept
    copy_engine(0)
    cached(1, [[2, 4]], 2)                                        # any cached call commits the landed plan
    assert all(int(st.ptrs_all[e]) == st.slot_ptr(s) for e, s in pairs)
    cached(0, [[3, 5], [7, 9]], 3)                                # now read from the slots
    seq, pairs = plan(1, [2, 4, 6, 8, 10], mf=2)                  # 2, 4 resident: two claims for 6, 8, 10
    assert seq == 1 and len(pairs) == 2
    cached(1, [[6, 8], [10, 2]], 4)
    copy_engine(1)
    seq, pairs = plan(0, [11, 12])                                # the plan call commits layer 1 first
    cached(0, [[11, 3], [12, 5]], 5)
    copy_engine(0)
    cached(1, [[6, 8]], 6)
    assert not cs.pend and int(st.pend.cpu()[0::35][:L].sum()) == 0
    st.done_seq = torch.zeros(0, dtype=torch.int32, device=DEV)


def test_worker_copies_and_commits():
    H, I, K, E, S, L, topk = 256, 128, 3, 32, 12, 3, 4
    st = _store(H, I, K, E, S, L, seed=43)
    keys = list(st.layer_index)
    gold = _gold(st)
    st.start_copy_prefetch()
    with pytest.raises(RuntimeError, match="stop_copy_prefetch first"):
        st.make_resident(keys[0], [1])
    try:
        for step in range(10):
            for li, key in enumerate(keys):
                T = 1 + (step + li) % 3
                x = torch.randn(T, H, generator=torch.Generator().manual_seed(step * 10 + li)).to(torch.bfloat16)
                ids, w = _route(T, E, topk, 500 + step * 10 + li)
                y = st.forward_cached(key, x.to(DEV), ids.to(DEV), w.to(DEV))
                yr = X.moe_decode(x.to(DEV), ids.to(DEV), w.to(DEV), gold[key], I, K, E)
                nxt = (li + 1) % L
                pred, _ = _route(1, E, 6, 900 + step * 10 + li)
                st.plan_prefetch(keys[nxt], pred.flatten().to(DEV), max_fill=4)
                torch.cuda.synchronize()
                assert torch.equal(y, yr), (step, li)
    finally:
        plans, copies = st.stop_copy_prefetch()
    assert plans >= 1 and copies >= 1
    assert X.OPS.moe_prefetch_worker_stop() == [0, 0]             # stopped
    last = st.slot_last.cpu().numpy()
    assert (last != PINNED).all() and int(st.pend.cpu()[0::35][:L].sum()) == 0
    sk = st.slot_key.cpu().numpy()
    sod = st.slot_of_dev.cpu().numpy()
    ptrs = st.ptrs_all.cpu().numpy()
    for s, code in enumerate(sk):
        if code >= 0:
            li, e = divmod(int(code), E)
            assert sod[code] == s and ptrs[code] == st.slot_ptr(s)
            assert torch.equal(st.slots[s].cpu(), st.host[keys[li]][e]), (s, li, e)
    for code in range(L * E):
        if sod[code] < 0:
            li, e = divmod(code, E)
            assert ptrs[code] == int(st._host_ptr[keys[li]][e])
