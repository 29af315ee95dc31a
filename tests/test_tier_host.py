"""CPU: exl3b200.tier.TierHost, the per-step host loop of the RAM tier, against fakes of the device state.

The device side is plain CPU tensors written the way the decode kernels write them: masked picks log their keys to
the miss ring (ring[0] counts, key n at ring[1 + n % cap]), the victim write-back sets ram_res[key].  The host loop
consumes each snapshot one step later, so a key logged before step t is fetched by step t + 1.
"""
import numpy as np
import torch

from exl3b200.tier import TierHost


class FakeDevice:
    def __init__(self, n_keys=16, cap=8):
        self.ram_res = torch.zeros(n_keys, dtype=torch.uint8)
        self.ring = torch.zeros(1 + cap, dtype=torch.int32)
        self.slot_of = torch.full((n_keys,), -1, dtype=torch.int32)
        self.cap = cap

    def log_misses(self, keys):   # what a decode step does for its masked picks
        for key in keys:
            n = int(self.ring[0])
            self.ring[1 + n % self.cap] = key
            self.ring[0] = n + 1

    def victim_writeback(self, key):
        self.ram_res[key] = 1


def _tier(dev, **kw):
    fetched, released = [], []
    kw.setdefault("budget", 8)
    t = TierHost(dev.ram_res, dev.ring, dev.slot_of, fetch=fetched.append, release=released.append, **kw)
    return t, fetched, released


def test_misses_are_fetched_then_flagged():
    dev = FakeDevice()
    t, fetched, _ = _tier(dev)
    assert t.step() == 0                    # first snapshot: nothing to consume
    dev.log_misses([3, 5, 3])
    t.step()                                # consumes the snapshot taken before the misses
    assert fetched == []
    assert t.step() == 3
    assert fetched == [3, 5]                # most-logged first
    t.fill_done(3)
    t.fill_done(5)
    t.step()
    assert dev.ram_res[3] == 1 and dev.ram_res[5] == 1 and t.resident() == 2
    dev.log_misses([3])                     # resident or already fetched: not fetched again
    t.step()
    t.step()
    assert fetched == [3, 5]


def test_budget_drops_vram_copies_first_then_oldest():
    dev = FakeDevice()
    t, fetched, released = _tier(dev, budget=3)
    t.step()
    for key in [1, 2, 4]:                   # resident at steps 2, 3, 4
        dev.log_misses([key])
        t.step()
        t.step()
        t.fill_done(key)
    t.step()
    assert sorted(np.nonzero(t.res)[0].tolist()) == [1, 2, 4]
    dev.slot_of[4] = 0                      # key 4 also sits in VRAM now
    dev.log_misses([7, 9])                  # two wanted keys need two places
    t.step()
    t.step()
    assert fetched[-2:] == [7, 9]
    assert t.res[4] == 0 and t.res[1] == 0 and t.res[2] == 1   # the VRAM copy, then the oldest
    assert dev.ram_res[4] == 0 and dev.ram_res[1] == 0
    assert released == []                   # released only after the device ran a step past the clear
    t.step()
    t.step()
    assert released == [1]                  # 4 is held while its expert sits in VRAM (it may be written back)
    t.step()
    assert released == [1]
    dev.slot_of[4] = -1                     # evicted without a write-back (no victim buffer)
    t.step()
    t.step()
    assert sorted(released) == [1, 4]


def test_a_dropped_vram_copy_written_back_on_eviction_is_kept():
    """The race a release must not lose: the RAM copy of a VRAM-resident key is dropped; several steps later its slot
    is evicted and the victim write-back restores the row and sets the flag.  The row must not be released after
    that write-back, whenever it lands."""
    dev = FakeDevice()
    t, fetched, released = _tier(dev, budget=2)
    t.step()
    for key in [3, 5]:
        dev.log_misses([key])
        t.step()
        t.step()
        t.fill_done(key)
    t.step()
    dev.slot_of[3] = 1                      # 3 also sits in VRAM: its RAM copy goes first
    dev.log_misses([7])
    t.step()
    t.step()
    assert t.res[3] == 0 and fetched[-1] == 7
    for _ in range(4):                      # held: still in VRAM
        t.step()
    assert released == []
    dev.slot_of[3] = -1                     # evicted during a decode step, written back in the same call
    dev.victim_writeback(3)
    t.step()
    t.step()
    assert released == [] and t.res[3] == 1 and t.stats["release_rescued"] == 1


def test_victim_writeback_becomes_resident_and_rescues_a_drop():
    dev = FakeDevice()
    t, fetched, released = _tier(dev, budget=2)
    t.step()
    dev.victim_writeback(6)                 # the kernel copied an evicted VRAM expert to its host slot
    t.step()
    dev.victim_writeback(5)
    t.step()
    t.step()
    assert t.res[6] == 1 and t.res[5] == 1 and t.stats["victims_kept"] == 2
    dev.log_misses([2])                     # over budget: the oldest (6) is dropped for 2
    t.step()
    t.step()
    assert t.res[6] == 0 and t.res[5] == 1 and fetched == [2]
    dev.victim_writeback(6)                 # the next step wrote 6 back before its host copy was released
    t.step()
    t.step()
    assert 6 not in released and t.stats["release_rescued"] == 1
    assert t.res[6] == 1 and t.res[5] == 0  # 6 is resident again (youngest); 5 made room


def test_a_dropped_key_fetched_again_keeps_its_host_copy():
    """A key dropped and wanted again before its release point is being fetched into the same host copy: release()
    must not free it."""
    dev = FakeDevice()
    t, fetched, released = _tier(dev, budget=2)
    t.step()
    for key in [1, 3]:                      # resident at steps 4 and 6
        dev.log_misses([key])
        t.step()
        t.step()
        t.fill_done(key)
    t.step()
    dev.log_misses([2])
    t.step()
    dev.log_misses([1])                     # logged before the drop below is read: it reaches the host one step later
    t.step()                                # 2 wanted: 1 (oldest) dropped, 2 fetched
    assert fetched[-1] == 2 and t.res[1] == 0
    t.step()                                # 1 wanted again: 3 dropped, 1 fetched
    assert fetched[-1] == 1
    for _ in range(3):
        t.step()
    assert 1 not in released and released == [3] and t.stats["release_rescued"] == 1


def test_pinned_keys_are_never_dropped():
    dev = FakeDevice()
    pinned = np.zeros(16, dtype=bool)
    pinned[0] = True
    dev.ram_res[0] = 1
    t, fetched, released = _tier(dev, budget=1, pinned=pinned)
    t.step()
    dev.log_misses([5])
    t.step()
    t.step()
    assert t.res[0] == 1 and fetched == [] and t.stats["admit_deferred"] == 1


def test_ring_overflow_keeps_the_last_cap_keys():
    dev = FakeDevice(cap=8)
    t, fetched, _ = _tier(dev, budget=16)
    t.step()
    dev.log_misses(list(range(12)))         # 12 keys through an 8-entry ring: 0-3 were overwritten
    t.step()
    assert t.step() == 8
    assert t.stats["ring_overflow"] == 4
    assert sorted(fetched) == list(range(4, 12))


def test_admission_limits_keys_in_flight():
    dev = FakeDevice()
    t, fetched, _ = _tier(dev, budget=16, max_inflight=2)
    t.step()
    dev.log_misses([9, 8, 8, 7, 7, 7])
    t.step()
    t.step()
    assert fetched == [7, 8] and t.stats["admit_deferred"] == 1   # most-logged first; 9 stays masked
    t.fill_done(7)
    t.fill_done(8)
    dev.log_misses([9])                     # re-logged on its next miss
    t.step()
    t.step()
    assert fetched == [7, 8, 9]


def test_min_age_protects_fresh_fills():
    dev = FakeDevice()
    t, fetched, _ = _tier(dev, budget=1, min_age=3)
    t.step()
    dev.log_misses([1])
    t.step()
    t.step()
    t.fill_done(1)
    t.step()                                # 1 resident at this step
    dev.log_misses([2])
    t.step()
    t.step()                                # 1 is younger than 3 steps: 2 waits
    assert t.res[1] == 1 and fetched == [1]
    for _ in range(3):
        dev.log_misses([2])
        t.step()
    assert fetched == [1, 2] and t.res[1] == 0


def test_drop_choice_matches_a_full_sort():
    """The budget's drop choice (selected in linear time) equals taking the first keys of a full sort by (not in VRAM,
    resident since, key), over random states with many ties."""
    rng = np.random.default_rng(5)
    for trial in range(200):
        n = int(rng.integers(8, 300))
        dev = FakeDevice(n_keys=n, cap=8)
        t, _, _ = _tier(dev, budget=n, min_age=int(rng.integers(0, 4)))
        t.tick = 20
        t.state[:] = rng.choice([0, 1, 2], size=n, p=[0.3, 0.1, 0.6])
        t.since[:] = rng.integers(0, 20, size=n)
        t.pinned[:] = rng.random(n) < 0.1
        in_vram = rng.random(n) < 0.3
        droppable = (t.state == 2) & ~t.pinned & (in_vram | (t.since <= t.tick - t.min_age))
        want = sorted(np.flatnonzero(droppable).tolist(), key=lambda k: (not in_vram[k], t.since[k], k))
        n_want = int(rng.integers(0, n))
        excess = int(np.count_nonzero(t.state != 0)) + n_want - t.budget
        drop = t._make_room(n_want, in_vram)
        assert drop.tolist() == want[:max(0, excess)], trial


def test_prefetch_ids_skip_experts_in_neither_tier():
    """With the RAM tier on, prefetch must not copy an expert whose host row may be released: predictions in neither
    VRAM nor RAM become the layer's safe expert (exl3b200.ops.tier_prefetch_ids)."""
    from exl3b200.ops import tier_prefetch_ids
    E = 8
    ram_res = torch.zeros(2 * E, dtype=torch.uint8)
    ram_res[[E + 0, E + 3]] = 1                                    # layer 1: experts 0 (safe) and 3 in RAM
    slot_of = torch.full((2 * E,), -1, dtype=torch.int32)
    slot_of[E + 5] = 2                                             # layer 1: expert 5 in VRAM
    safe = torch.tensor([0, 0], dtype=torch.int32)
    ids = torch.tensor([3, 5, 6, 1, 9, -1], dtype=torch.int32)     # 9 and -1 are out of range: left to the cache step
    got = tier_prefetch_ids(ids, 1, E, slot_of, ram_res, safe)
    assert got.tolist() == [3, 5, 0, 0, 9, -1] and got.dtype == torch.int32
    assert tier_prefetch_ids(ids, 1, E, slot_of, None, safe) is ids   # tier off: unchanged


def test_ring_claims_pending_at_start_are_drained():
    """A victim-ring slot claimed before the host loop started is drained like any other: the row receives the
    ring slot's bytes, the key becomes resident and the slot is freed."""
    dev = FakeDevice(n_keys=16)
    K = 2
    meta = torch.tensor([1, 1, 0, K, 9, -1, 1, 0], dtype=torch.int32)   # slot 0 claimed by key 9 (claim 1)
    buf = torch.arange(2 * 64, dtype=torch.uint8).view(2, 64)
    rows = torch.zeros(16, 64, dtype=torch.uint8)
    t, _, _ = _tier(dev, vring=(meta, buf, lambda key: rows[key]))
    t.step()
    t.step()                                # drained (synchronous on the CPU)
    assert torch.equal(rows[9], buf[0]) and t.state[9] == 1
    t.step()                                # the drain has completed: resident, slot freed
    assert t.res[9] == 1 and dev.ram_res[9] == 1 and meta[4:6].tolist() == [-1, -1]


class _Logger:
    def __init__(self):
        self.lines = []

    def info(self, fmt, *args):
        self.lines.append(fmt % args)


def test_ensure_for_prefill_fills_within_budget_and_keeps_protocol():
    """Eager prefill: the picked experts of the layer become resident and flagged now; room is made from other
    layers' keys (a VRAM copy first), never this layer's; the next steps neither resurrect the dropped keys nor
    release a row that is still needed."""
    E = 4
    dev = FakeDevice(n_keys=3 * E)
    fetched = []
    t = TierHost(dev.ram_res, dev.ring, dev.slot_of, budget=4, fetch=lambda k: (fetched.append(k), t.fill_done(k)),
                 release=(released := []).append)
    t.step()
    assert t.warm([5]) == 1                                              # 5 (layer 1) is the oldest resident key
    t.step()
    assert t.warm([0, 1, 5, 9, 10]) == 3 and fetched == [5, 0, 1, 9]     # the budget bounds the warm fill
    assert dev.ram_res.tolist()[:10] == [1, 1, 0, 0, 0, 1, 0, 0, 0, 1]
    dev.slot_of[9] = 3                                                   # 9 also sits in VRAM
    n = t.ensure_for_prefill(1, torch.tensor([[0, 1], [2, 0]]), E)    # layer 1's experts 0-2: keys 4-6
    assert n == 2 and fetched[-2:] == [4, 6]
    assert dev.ram_res[[4, 5, 6]].tolist() == [1, 1, 1]                 # this layer's picks: resident, flagged
    assert t.res[9] == 0 and dev.ram_res[9] == 0                          # the VRAM copy went first ...
    assert sorted(np.flatnonzero(t.res).tolist()) == [1, 4, 5, 6]        # ... then the oldest of other layers (0)
    assert released == [0]                                                # 9 is held while in VRAM
    for _ in range(3):
        t.step()
    assert t.res[0] == 0 and t.res[9] == 0 and t.stats["victims_kept"] == 0   # not resurrected
    dev.slot_of[9] = -1
    t.step()
    t.step()
    assert sorted(released) == [0, 9]
    log = _Logger()
    t.log_stats(log, every=1)
    assert log.lines and "resident 4 of budget 4" in log.lines[0]


def test_a_key_dropped_twice_is_released_once():
    """A key dropped by step() awaits its release there; an eager prefill fetches it again and a later one drops it
    (released at once).  The pending release of the first drop is void: every drop releases the row exactly once."""
    E = 4
    dev = FakeDevice(n_keys=3 * E)
    t = TierHost(dev.ram_res, dev.ring, dev.slot_of, budget=1, fetch=lambda k: t.fill_done(k),
                 release=(released := []).append)
    t.step()
    assert t.warm([0]) == 1
    dev.log_misses([2])
    t.step()
    t.step()                                  # 0 dropped (its release pending), 2 fetched
    t.step()
    assert t.res.tolist()[:3] == [0, 0, 1] and released == []
    t.ensure_for_prefill(0, torch.tensor([0]), E)   # 0 fetched again: 2 dropped and released at once
    t.ensure_for_prefill(1, torch.tensor([0]), E)   # key 4 needs the room: 0 dropped and released at once
    assert released == [2, 0]
    for _ in range(4):
        t.step()
    assert sorted(released) == [0, 2]


def test_ring_claim_of_a_key_being_fetched_is_not_copied():
    """A victim-ring claim for a key whose store fetch is in flight frees its ring slot without a second copy into
    the row the fetch is writing."""
    dev = FakeDevice(n_keys=16)
    K = 2
    meta = torch.tensor([0, 0, 0, K, -1, -1, 0, 0], dtype=torch.int32)
    buf = torch.full((2, 64), 7, dtype=torch.uint8)
    rows = torch.zeros(16, 64, dtype=torch.uint8)
    t, fetched, _ = _tier(dev, vring=(meta, buf, lambda key: rows[key]))
    t.step()
    dev.log_misses([9])
    t.step()
    t.step()
    assert fetched == [9] and t.state[9] == 1          # fetching, not complete
    meta[4], meta[4 + K] = 9, 1                       # slot 0 claimed by key 9
    t.step()
    t.step()                                          # the snapshot that shows the claim
    assert torch.count_nonzero(rows[9]) == 0 and meta[4].item() == -1 and t.stats["ring_drained"] == 0
    t.fill_done(9)
    t.step()
    assert t.res[9] == 1
