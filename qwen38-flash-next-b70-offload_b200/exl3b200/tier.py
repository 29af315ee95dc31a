"""Host side of the RAM tier: the per-decode-step loop that keeps the tier's contract with the decode kernels.

The reference runs this loop as NvTierAsync.step and its admission-controlled variant (plugin/exl3xpu/nvtier.py:
297-386, 708-806), with an NVMe reader pool behind it.  The contract with the kernels (exl3_moe.a8.sycl:762-788):

  * ram_res[key] (uint8, one per (layer, expert) key) is 1 only while the expert's host copy is valid; a pick whose
    expert is in neither VRAM (slot_of[key] >= 0) nor RAM is masked to (safe expert, weight 0);
  * every masked pick's key is logged to the miss ring: ring[0] counts the keys logged so far and the n-th key
    lands at ring[1 + n % cap];
  * the victim write-back (exl3b_victim_copy) copies an evicted VRAM expert to its host slot and sets ram_res[key].

The host keeps one state per key (absent, fetching, resident since step t) and a pinned snapshot of the device's
ram_res, ring and slot_of.  The snapshot is queued at the end of every step(), behind that step's own flag writes, and
read at the start of the next one, after the next decode step has been queued: reading it waits for the previous
decode step only, and it never predates the host's own writes, so a flag that differs from the host's state was set
by the device.  step(), once per decode step after the step's kernels are queued:

  1. absorbs what happened since: keys the device flagged (victim write-backs) and keys whose fetch reported
     fill_done become resident at this step;
  2. releases dropped keys once a snapshot taken after a whole decode step past their flag clear has been read.
     Without a victim ring the snapshot must also show the key out of VRAM: a key whose expert sits in VRAM is written
     back to its row by the device (flag set) when its slot is evicted, at any later step; the snapshot that shows the
     eviction also shows that flag, and the key is resident again instead of released.  Out of VRAM and unflagged, a
     key cannot come back into VRAM (a fill needs the flag), so nothing writes its row after the release; RAM use is
     bounded by budget + VRAM slots.  With a victim ring (vring) the device never writes rows: evicted victims wait in
     the ring until this loop drains them, so dropped rows are released at once and RAM use stays within the budget;
  3. reads the keys logged to the miss ring since the previous snapshot (the last cap of them when more were logged);
     the absent ones are wanted, most-logged first, lower key first on ties;
  4. makes room for them, resident + fetching + wanted <= budget, by dropping resident keys that are not pinned:
     those whose expert also sits in VRAM first, then those resident for at least min_age steps, oldest first in each
     group;
  5. hands wanted keys to fetch(key) while the budget has room and fewer than max_inflight are fetching; the rest stay
     masked and come back through the ring on their next miss;
  6. writes the flags that differ from the snapshot (index_copy_ on the current stream), then queues the next snapshot.

fetch(key) starts making the key's host copy valid (the caller's storage: a file read, a copy from another tier) and
reports completion with fill_done(key), from any thread.  The device tensors may be CPU tensors (tests): copies are
then synchronous.
"""
from __future__ import annotations

import collections
import queue
import time

import numpy as np
import torch

ABSENT, FETCHING, RESIDENT = 0, 1, 2
PINNED_SLOT = 0x7FFFFFFF   # slot_last of a slot claimed by a copy-engine prefetch plan until its copy committed


class _Snapshot:
    """One pinned host copy of the device's (ram_res, ring, slot_of), queued behind an event."""

    def __init__(self, ram_res: torch.Tensor, ring: torch.Tensor, slot_of: torch.Tensor, n: int, extras=None):
        self.cuda = ram_res.device.type == "cuda"
        self.names = list(extras or {})
        self.src = (ram_res[:n], ring, slot_of[:n]) + tuple((extras or {})[k] for k in self.names)
        self.host = tuple(torch.empty(t.numel(), dtype=t.dtype, pin_memory=self.cuda) for t in self.src)
        self.ready = None       # None before the first queue(); then an event, or True on the CPU

    def queue(self) -> None:
        for dst, src in zip(self.host, self.src):
            dst.copy_(src, non_blocking=self.cuda)
        if self.cuda:
            self.ready = torch.cuda.Event()
            self.ready.record(torch.cuda.current_stream(self.src[0].device))
        else:
            self.ready = True

    def read(self):
        """(flags, ring, slot_of, {name: extra}) as numpy views of the host copy, valid until the next queue(); None
        before any."""
        if self.ready is None:
            return None
        if self.cuda:
            self.ready.synchronize()
        flags, ring, slot = (t.numpy() for t in self.host[:3])
        return flags != 0, ring, slot, {k: t.numpy() for k, t in zip(self.names, self.host[3:])}


class TierHost:
    def __init__(self, ram_res: torch.Tensor, ring: torch.Tensor, slot_of: torch.Tensor, budget: int, fetch,
                 release=None, pinned=None, min_age: int = 0, max_inflight: int | None = None, vring=None,
                 slot_last=None):
        """vring: (meta, buf, dest) when the decode kernels write victims to a victim ring (ops.moe_set_victim_ring)
        instead of to host rows: meta / buf are the ring's device tensors, dest(key) the key's host row (uint8, >=
        blob bytes).  Each step then drains the ring's new claims to their rows on a copy stream; a drained key
        becomes resident once its copy completed, and its ring slot is freed (key -1 written on the current stream).
        slot_last: the cache's slot_last tensor.  With a ring, dropped rows are released while their expert sits in
        VRAM, except a slot pinned by a copy-engine prefetch plan whose copy (which reads the row) has not committed;
        given slot_last, exactly those are held, else every key still in VRAM is."""
        if ram_res.dtype != torch.uint8 or ring.dtype != torch.int32 or slot_of.dtype != torch.int32:
            raise RuntimeError("exl3b200 TierHost: uint8 ram_res, int32 ring, int32 slot_of")
        if ring.numel() < 2 or slot_of.numel() < ram_res.numel():
            raise RuntimeError("exl3b200 TierHost: the ring needs >= 1 entry and slot_of one entry per key")
        self.ram_res = ram_res
        self.n = ram_res.numel()
        self.cap = ring.numel() - 1
        self.budget = int(budget)
        self.fetch = fetch
        self.release = release if release is not None else (lambda key: None)
        self.pinned = np.zeros(self.n, dtype=bool) if pinned is None else np.asarray(pinned, dtype=bool).copy()
        self.min_age = int(min_age)
        self.max_inflight = max_inflight
        self.state = np.where(ram_res.cpu().numpy() != 0, RESIDENT, ABSENT).astype(np.int8)
        self.since = np.zeros(self.n, dtype=np.int64)     # step at which a resident key became resident
        self._key_bits = max(1, (self.n - 1).bit_length())  # key field of the packed drop order
        self.tick = 0
        self.ring_seen = int(ring[0].item())
        self._vr = None
        if vring is not None:
            meta, buf, dest = vring
            K = (meta.numel() - 4) // 2
            if meta.dtype != torch.int32 or meta.numel() != 4 + 2 * K or buf.dim() != 2 or buf.shape[0] != K:
                raise RuntimeError("exl3b200 TierHost: vring = (int32 meta [4 + 2K], buf [K, blob], dest)")
            # claim numbers start at 1: every slot already claimed when the loop starts is drained too
            self._vr = {"meta": meta, "buf": buf, "dest": dest, "K": K, "fly": [],
                        "seen": np.zeros(K, dtype=np.int32),
                        "stream": torch.cuda.Stream(meta.device) if meta.is_cuda else None}
        extras = {}
        if vring is not None:
            extras["meta"] = vring[0]
        if slot_last is not None:
            extras["slot_last"] = slot_last
        self._snap = _Snapshot(ram_res, ring, slot_of, self.n, extras=extras)
        self._drop_tick = np.full(self.n, -1, dtype=np.int64)   # step of a drop whose row awaits release, else -1
        self._done = queue.SimpleQueue()
        self.stats = collections.Counter()

    @property
    def res(self) -> np.ndarray:
        """The host's resident flags (uint8 per key), what it last wrote to ram_res."""
        return (self.state == RESIDENT).astype(np.uint8)

    # ---------------------------------------------------------------- outside the decode loop
    def _sync_device(self) -> None:
        if self.ram_res.is_cuda:
            torch.cuda.synchronize(self.ram_res.device)

    def _upload(self, keys, value: int) -> None:
        keys = np.asarray(keys, dtype=np.int64)
        if keys.size:
            idx = torch.from_numpy(keys)
            if self.ram_res.is_cuda:
                idx = idx.pin_memory().to(self.ram_res.device, non_blocking=True)
            self.ram_res.index_fill_(0, idx, value)

    def _wait_fills(self, keys, timeout: float) -> None:
        """Block until every key of `keys` is resident, taking fill completions as they arrive (a completion may also
        have been taken already, by a snapshot's absorb: the key's state is what counts)."""
        keys = np.asarray(keys, dtype=np.int64)
        deadline = time.monotonic() + timeout
        while True:
            pending = int(np.count_nonzero(self.state[keys] != RESIDENT))
            if not pending:
                return
            try:
                key = self._done.get(timeout=max(0.0, deadline - time.monotonic()))
            except queue.Empty:
                raise RuntimeError(f"exl3b200 TierHost: {pending} fills did not complete within {timeout} s")
            self._become_resident([key])

    def _make_room_now(self, n_need: int, keep: np.ndarray) -> None:
        """Drop resident keys (not pinned, not in `keep`) until n_need more fit in the budget, with the device idle: a
        fresh snapshot first (victims written back since become resident), flags cleared, rows released at once
        unless the release rule holds them (then they wait in the release list like any drop)."""
        excess = int(np.count_nonzero(self.state != ABSENT)) + n_need - self.budget
        if excess <= 0:
            return
        self._sync_device()
        self._snap.queue()                                  # the device is idle: this snapshot is exact
        flags, _, slot, extras = self._snap.read()
        self._absorb(flags)
        excess = int(np.count_nonzero(self.state != ABSENT)) + n_need - self.budget
        in_vram = slot >= 0
        protect = self.pinned.copy()
        protect[keep] = True
        saved, self.pinned = self.pinned, protect
        try:
            drop = self._make_room(n_need, in_vram)
        finally:
            self.pinned = saved
        if not drop.size:
            self.stats["prefill_over_budget"] += max(0, excess)
            return
        self._upload(drop, 0)
        self._sync_device()
        held = self._held(drop, slot, extras.get("slot_last"))
        # a key dropped by an earlier step() may still await its release there; this drop supersedes it (released
        # below, or re-queued as held), so step() must not release it a second time
        self._drop_tick[drop] = -1
        for key in drop[~held].tolist():
            self.release(key)
            self.stats["released"] += 1
        if held.any():
            self._drop_tick[drop[held]] = self.tick - 2        # due now; released once the rule allows
        self.stats["prefill_dropped"] += drop.size

    def ensure_for_prefill(self, layer: int, ids, n_experts: int, timeout: float = 120.0) -> int:
        """Eager prefill below the staging threshold (the reference's NvTier.ensure_for_prefill, nvtier.py:389-457):
        make every expert that `ids` picks in `layer` RAM-resident now (fetched and waited for), within the budget,
        and flag it on the device, so the prefill kernels read it from host memory.  When room is needed the device
        is synchronised first.  Not for use inside CUDA graph capture.  Returns the number of experts fetched."""
        ids_np = ids.reshape(-1).to("cpu", torch.int64).numpy() if isinstance(ids, torch.Tensor) else np.asarray(ids)
        ids_np = ids_np[(ids_np >= 0) & (ids_np < n_experts)]
        keys = np.unique(ids_np) + layer * n_experts
        self._finish_drains()             # keys being drained from the victim ring complete here, not via fill_done
        need = keys[self.state[keys] == ABSENT]
        wait = keys[self.state[keys] == FETCHING]
        self._make_room_now(need.size, keys)
        for key in need.tolist():
            self.state[key] = FETCHING
            self.stats["prefill_fetches"] += 1
            self.fetch(key)
        self._wait_fills(np.concatenate([need, wait]), timeout)
        self._upload(keys, 1)
        self._snap.queue()        # the next step() must read a snapshot taken after these flag writes
        return int(need.size)

    def warm(self, keys, max_keys: int | None = None, timeout: float = 600.0) -> int:
        """Fill the RAM tier with `keys` (hottest first) while the budget (or max_keys) has room, and wait for the
        fills (the reference's NvTier.warm, nvtier.py:492-509).  Returns the number fetched."""
        room = self.budget - int(np.count_nonzero(self.state != ABSENT))
        if max_keys is not None:
            room = min(room, int(max_keys))
        todo = []
        for key in dict.fromkeys(int(k) for k in keys):
            if len(todo) >= room:
                break
            if 0 <= key < self.n and self.state[key] == ABSENT:
                todo.append(key)
        for key in todo:
            self.state[key] = FETCHING
            self.fetch(key)
        self._wait_fills(todo, timeout)
        self._upload(todo, 1)
        self._snap.queue()        # the next step() must read a snapshot taken after these flag writes
        return len(todo)

    def log_stats(self, logger, every: int = 200) -> None:
        """Every `every` steps, log the counters' change since the last report (the reference's NvTier.log_stats)."""
        steps = self.stats["steps"]
        if not steps or steps % every:
            return
        last = getattr(self, "_logged", collections.Counter())
        d = {k: v - last.get(k, 0) for k, v in self.stats.items()}
        n = max(1, d.get("steps", 0))
        logger.info("exl3b200 tier: last %d steps: masked/step %.2f fetches/step %.2f dropped/step %.2f released %d "
                    "rescued %d victims kept %d ring drained %d, resident %d of budget %d", n, d.get("masked", 0) / n,
                    d.get("fetches", 0) / n, d.get("dropped", 0) / n, d.get("released", 0),
                    d.get("release_rescued", 0), d.get("victims_kept", 0), d.get("ring_drained", 0), self.resident(),
                    self.budget)
        self._logged = collections.Counter(self.stats)

    def resident(self) -> int:
        return int(np.count_nonzero(self.state == RESIDENT))

    def fill_done(self, key: int) -> None:
        """The host copy of key is valid (thread-safe)."""
        self._done.put(int(key))

    # ---------------------------------------------------------------- per step
    def step(self) -> int:
        """One decode step's bookkeeping (see the module docstring).  Returns the number of misses logged in the
        snapshot it read."""
        self.tick += 1
        snap = self._snap.read()
        logged = 0
        if snap is not None:
            flags, ring, slot, extras = snap
            in_vram = slot >= 0
            self._absorb(flags)
            if self._vr is not None:
                self._drain_ring(extras["meta"])
            self._release_dropped(slot, extras.get("slot_last"))
            want, logged = self._wanted(ring)
            dropped = self._make_room(len(want), in_vram)
            self._admit(want)
            self._write_flags(flags)
            self._drop_tick[dropped] = self.tick
        self._snap.queue()
        self.stats["steps"] += 1
        return logged

    def _become_resident(self, keys) -> None:
        self.state[keys] = RESIDENT
        self.since[keys] = self.tick

    def _absorb(self, flags: np.ndarray) -> None:
        flagged = np.flatnonzero(flags & (self.state != RESIDENT))     # victim write-backs
        self._become_resident(flagged)
        self.stats["victims_kept"] += flagged.size
        filled = []
        while True:
            try:
                filled.append(self._done.get_nowait())
            except queue.Empty:
                break
        if filled:
            self._become_resident(np.asarray(filled, dtype=np.int64))

    def _drain_ring(self, meta: np.ndarray) -> None:
        """Victim ring: finished drains make their keys resident and free their slots; new claims are drained."""
        vr = self._vr
        K = vr["K"]
        keys, seqs = meta[4:4 + K], meta[4 + K:4 + 2 * K]
        free, flying = [], []
        for ev, r, key in vr["fly"]:
            if ev is None or ev.query():
                if self.state[key] != RESIDENT:
                    self._become_resident([key])
                self.stats["ring_drained"] += 1
                free.append(r)
            else:
                flying.append((ev, r, key))
        vr["fly"] = flying
        self._free_ring_slots(free)
        free = []
        for r in np.flatnonzero((keys >= 0) & (seqs != vr["seen"])).tolist():
            vr["seen"][r] = seqs[r]
            key = int(keys[r])
            # nothing to drain: the row is valid already, or a fetch (or an earlier drain) is writing the same bytes
            if not 0 <= key < self.n or self.state[key] != ABSENT:
                free.append(r)
                continue
            self.state[key] = FETCHING                                  # not fetched again, not released
            dst = vr["dest"](key)[: vr["buf"].shape[1]]
            if vr["stream"] is not None:   # the snapshot just read waited for the decode step that wrote the slot
                with torch.cuda.stream(vr["stream"]):
                    dst.copy_(vr["buf"][r], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(vr["stream"])
            else:
                dst.copy_(vr["buf"][r])
                ev = None
            vr["fly"].append((ev, r, key))
        self._free_ring_slots(free)

    def _free_ring_slots(self, slots) -> None:
        if slots:
            meta = self._vr["meta"]
            idx = torch.tensor([4 + r for r in slots], dtype=torch.int64)
            if meta.is_cuda:
                idx = idx.pin_memory().to(meta.device, non_blocking=True)
            meta.index_fill_(0, idx, -1)

    def _finish_drains(self) -> None:
        """Wait for every ring drain in flight; their keys become resident and their slots free."""
        vr = self._vr
        if vr is None or not vr["fly"]:
            return
        if vr["stream"] is not None:
            vr["stream"].synchronize()
        for _, _, key in vr["fly"]:
            if self.state[key] != RESIDENT:
                self._become_resident([key])
            self.stats["ring_drained"] += 1
        self._free_ring_slots([r for _, r, _ in vr["fly"]])
        vr["fly"] = []

    def _held(self, keys: np.ndarray, slot: np.ndarray, slot_last) -> np.ndarray:
        """Dropped keys whose row must stay (see the module docstring, step 2)."""
        s = slot[keys]
        if self._vr is None or slot_last is None:
            return s >= 0
        pinned = np.zeros(len(keys), dtype=bool)
        inside = (s >= 0) & (s < len(slot_last))
        pinned[inside] = slot_last[s[inside]] == PINNED_SLOT
        return pinned

    def _release_dropped(self, slot: np.ndarray, slot_last) -> None:
        # due: the snapshot read now was queued at the end of step tick - 1, after decode step tick - 1 >= drop + 1
        due = np.flatnonzero((self._drop_tick >= 0) & (self._drop_tick <= self.tick - 2))
        if not due.size:
            return
        back = self.state[due] != ABSENT
        self.stats["release_rescued"] += int(back.sum())
        self._drop_tick[due[back]] = -1
        rest = due[~back]
        # without a victim ring, a key still in VRAM is written back to its row by the device whenever its slot is
        # evicted, so its row is released only once a snapshot shows it out of VRAM: the same snapshot then shows the
        # write-back's flag (rescued above).  With a ring the device never writes rows (the host drains the ring
        # itself, marking the key fetching first), so the row goes now and the drain brings it back
        go = rest[~self._held(rest, slot, slot_last)]
        self._drop_tick[go] = -1
        for key in go.tolist():
            self.release(key)
            self.stats["released"] += 1

    def _wanted(self, ring: np.ndarray):
        count = int(ring[0])
        new = count - self.ring_seen
        self.ring_seen = count
        if new > self.cap:
            self.stats["ring_overflow"] += new - self.cap
            new = self.cap
        if new <= 0:
            return np.zeros(0, dtype=np.int64), 0
        self.stats["masked"] += new
        logged = ring[1 + np.arange(count - new, count) % self.cap].astype(np.int64)
        keys, hits = np.unique(logged[(logged >= 0) & (logged < self.n)], return_counts=True)
        absent = self.state[keys] == ABSENT
        keys, hits = keys[absent], hits[absent]
        return keys[np.lexsort((keys, -hits))], new

    def _make_room(self, n_want: int, in_vram: np.ndarray) -> np.ndarray:
        excess = int(np.count_nonzero(self.state != ABSENT)) + n_want - self.budget
        if excess <= 0:
            return np.zeros(0, dtype=np.int64)
        droppable = (self.state == RESIDENT) & ~self.pinned & (in_vram | (self.since <= self.tick - self.min_age))
        cand = np.flatnonzero(droppable)
        # order (not in VRAM, resident since, key) packed into one int64: the first `excess` of ~10^4 candidates are
        # selected in linear time, and only they are sorted
        order = (~in_vram[cand]).astype(np.int64) << 62 | self.since[cand] << self._key_bits | cand
        if excess < cand.size:
            part = np.argpartition(order, excess - 1)[:excess]
            drop = cand[part[np.argsort(order[part])]]
        else:
            drop = cand[np.argsort(order)]
        self.state[drop] = ABSENT
        self.stats["dropped"] += drop.size
        return drop

    def _admit(self, want: np.ndarray) -> None:
        room = self.budget - int(np.count_nonzero(self.state != ABSENT))
        if self.max_inflight is not None:
            room = min(room, self.max_inflight - int(np.count_nonzero(self.state == FETCHING)))
        take = want[:max(0, room)]
        self.stats["admit_deferred"] += len(want) - len(take)
        for key in take.tolist():
            self.state[key] = FETCHING
            self.stats["fetches"] += 1
            self.fetch(key)

    def _write_flags(self, flags: np.ndarray) -> None:
        mine = self.state == RESIDENT
        keys = np.flatnonzero(mine != flags)
        if not keys.size:
            return
        idx = torch.from_numpy(keys)
        val = torch.from_numpy(mine[keys].astype(np.uint8))
        if self.ram_res.is_cuda:
            idx = idx.pin_memory().to(self.ram_res.device, non_blocking=True)
            val = val.pin_memory().to(self.ram_res.device, non_blocking=True)
        self.ram_res.index_copy_(0, idx, val)
