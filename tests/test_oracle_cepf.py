"""CPU: the oracle's restatement of copy-engine prefetch (oracle.CacheState.cepf_plan / cepf_commit; the plan and
commit modes of launch_ensure, exl3_moe.a8.sycl:874-905, 898-1036) on hand-worked cases.  The GPU test
tests/test_gpu_copy_prefetch.py compares the CUDA path with these functions state by state."""
import numpy as np

import oracle as O

E, S, L, BLOB = 16, 4, 2, 4096
PINNED = 0x7FFFFFFF


def _state():
    cs = O.CacheState(L, E, S, np.array([1 << 30, 1 << 31], np.int64), 1 << 34, BLOB)
    cs.cepf_reset()
    return cs


def _decode(cs, layer, ids):
    ids = np.array([ids], np.int32)
    cs.ensure(ids, np.full(ids.shape, 0.5, np.float32), layer, max_fill=E)
    cs.commit(layer)


def test_plan_pins_claims_and_leaves_the_table_at_host():
    cs = _state()
    host = cs.ptrs_all.copy()
    seq, pairs = cs.cepf_plan(np.array([7, 3, 5, 3], np.int32), 0, 8, np.zeros(L, np.int32))
    assert seq == 1 and pairs == [(3, 0), (5, 1), (7, 2)]          # misses ascending, empty slots in order
    assert cs.tick[0] == 0                                          # a plan does not advance the tick
    assert [int(cs.slot_last[s]) for s in range(3)] == [PINNED] * 3
    assert np.array_equal(cs.ptrs_all, host)                        # read from host until the commit
    assert [int(cs.slot_of[e]) for e in (3, 5, 7)] == [0, 1, 2]
    assert cs.pend == {0: (1, 0, [(3, 0), (5, 1), (7, 2)])}


def test_in_flight_plan_drops_the_next_and_pins_survive_decode():
    cs = _state()
    cs.cepf_plan(np.array([3, 5, 7], np.int32), 0, 8, np.zeros(L, np.int32))
    assert cs.cepf_plan(np.array([9], np.int32), 0, 8, np.zeros(L, np.int32)) is None
    assert cs.plan_seq[0] == 1                                      # nothing published
    _decode(cs, 0, [3, 9])                                          # 3 is a hit on a pinned slot: the pin stays
    assert int(cs.slot_last[0]) == PINNED and int(cs.slot_of[9]) == 3
    _decode(cs, 1, [1, 2])                                          # the only unpinned slot goes; pinned never
    assert int(cs.slot_key[3]) == E + 1 and int(cs.slot_of[9]) == -1
    assert [int(cs.slot_key[s]) for s in range(3)] == [3, 5, 7]
    assert cs.cepf_plan(np.array([11], np.int32), 1, 8, np.zeros(L, np.int32)) == (1, [])   # nothing claimable


def test_commit_points_the_table_at_the_slots_once_landed():
    cs = _state()
    cs.cepf_plan(np.array([3, 5], np.int32), 0, 8, np.zeros(L, np.int32))
    _decode(cs, 1, [2, 4])
    cs.cepf_commit(np.array([0, 0], np.int32))                      # not landed: nothing changes
    assert 0 in cs.pend and int(cs.ptrs_all[3]) == 1 << 30 | 3 * BLOB
    cs.cepf_commit(np.array([1, 0], np.int32))
    assert not cs.pend
    assert int(cs.ptrs_all[3]) == (1 << 34) + 0 * BLOB and int(cs.ptrs_all[5]) == (1 << 34) + BLOB
    assert int(cs.slot_last[0]) == 0 and int(cs.slot_last[1]) == 0   # unpinned at the plan's tick
    seq, pairs = cs.cepf_plan(np.array([6], np.int32), 0, 8, np.array([1, 0], np.int32))
    assert seq == 2 and pairs == [(6, 0)]                           # the layer plans again; LRU slot 0 reused
    assert int(cs.slot_of[3]) == -1 and int(cs.ptrs_all[3]) == 1 << 30 | 3 * BLOB


def test_max_fill_caps_a_plan_at_sixteen():
    cs = O.CacheState(1, 64, 32, np.array([1 << 30], np.int64), 1 << 34, BLOB)
    cs.cepf_reset()
    seq, pairs = cs.cepf_plan(np.arange(40, dtype=np.int32), 0, 64, np.zeros(1, np.int32))
    assert len(pairs) == 16 and [e for e, _ in pairs] == list(range(16))


def test_victim_ring_claim_rule_matches_the_device_source():
    """The ring claim rule of csrc/exl3b_vring.cu (its one source compiled for the host, exl3b_vring_claim_host)
    against oracle.vring_claim on random victim lists and ring states."""
    import ctypes
    from exl3b200 import _lib
    L = _lib.lib()
    fn = L.exl3b_vring_claim_host
    fn.restype = None
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int]
    rng = np.random.default_rng(11)
    for trial in range(300):
        K = int(rng.integers(1, 9))
        n = int(rng.integers(0, 12))
        vict = np.zeros(1 + 2 * 16, np.int32)
        vict[0] = n
        vict[1:1 + 2 * n:2] = np.where(rng.random(n) < 0.3, -1, rng.integers(0, 500, n))
        vict[2:2 + 2 * n:2] = rng.integers(0, 64, n)
        meta = np.zeros(4 + 2 * K, np.int32)
        meta[0], meta[1], meta[2], meta[3] = rng.integers(0, K), rng.integers(0, 100), rng.integers(0, 5), K
        meta[4:4 + K] = np.where(rng.random(K) < 0.5, -1, rng.integers(0, 500, K))
        meta[4 + K:] = rng.integers(0, 100, K)
        m_dev, s_dev = meta.copy(), np.full(16, 7, np.int32)
        m_ora, s_ora = meta.copy(), np.full(16, 7, np.int32)
        fn(vict.ctypes.data, m_dev.ctypes.data, s_dev.ctypes.data, K)
        O.vring_claim(vict, m_ora, s_ora)
        assert np.array_equal(m_dev, m_ora) and np.array_equal(s_dev, s_ora), trial
