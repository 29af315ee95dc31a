"""Host side of the RAM tier: the per-decode-step loop that keeps the tier's contract with the decode kernels.

The reference runs this loop as NvTierAsync.step and its admission-controlled variant (plugin/exl3xpu/nvtier.py:
297-386, 708-806), with an NVMe reader pool behind it.  The contract with the kernels (exl3_moe.a8.sycl:762-788):

  * ram_res[key] (uint8, one per (layer, expert) key) is 1 only while the expert's host copy is valid; a pick whose
    expert is in neither VRAM (slot_of[key] >= 0) nor RAM is masked to (safe expert, weight 0);
  * every masked pick's key is logged to the miss ring: ring[0] counts the keys logged so far and the n-th key
    lands at ring[1 + n % cap];
  * the victim write-back (exl3b_victim_copy) copies an evicted VRAM expert to its host slot and sets ram_res[key].

TierHost.step() runs once per decode step, after the step has been queued:

  1. snapshot: the device's ram_res, ring and slot_of are copied to host buffers (pinned on a GPU) behind an event,
     and used one step later, so the step itself is never synchronised;
  2. flags: keys the device flagged since (victim write-back) and fills reported complete (fill_done) become
     resident, aged with the current step;
  3. misses: the keys logged since the previous snapshot (the last cap of them when more were logged) that are
     neither resident nor being fetched are the wanted keys, most-logged first;
  4. budget (resident + in flight + wanted <= budget): resident keys are dropped -- first those that also sit in
     VRAM, then the others resident for at least min_age steps, oldest first; pinned keys never;
  5. admission: wanted keys are handed to fetch(key) while the budget has room and fewer than max_inflight are in
     flight; the rest stay masked and come back through the ring on their next miss;
  6. upload: the flags that changed are written to the device (index_copy_ on the current stream); a dropped key's
     host copy goes to release(key) once the device has run a whole step after that flag clear (so a snapshot
     shows any victim write-back of the key in that step) -- unless the device flagged the key again or the key
     was wanted and fetched again meanwhile.

fetch(key) starts making the key's host copy valid (the caller's storage: a file read, a copy from another tier) and
reports completion with fill_done(key), from any thread.  Device tensors may also be CPU tensors (tests): copies are
then synchronous and events complete at once.
"""
from __future__ import annotations

import collections
import queue

import numpy as np
import torch


class _Complete:
    """Event stand-in for CPU tensors: their copies are synchronous."""

    def query(self) -> bool:
        return True

    def synchronize(self) -> None:
        pass


class TierHost:
    def __init__(self, ram_res: torch.Tensor, ring: torch.Tensor, slot_of: torch.Tensor, budget: int, fetch,
                 release=None, pinned=None, min_age: int = 0, max_inflight: int | None = None):
        if ram_res.dtype != torch.uint8 or ring.dtype != torch.int32 or slot_of.dtype != torch.int32:
            raise RuntimeError("exl3b200 TierHost: uint8 ram_res, int32 ring, int32 slot_of")
        if ring.numel() < 2 or slot_of.numel() < ram_res.numel():
            raise RuntimeError("exl3b200 TierHost: the ring needs >= 1 entry and slot_of one entry per key")
        self.ram_res, self.ring, self.slot_of = ram_res, ring, slot_of
        self.dev = ram_res.device
        self.n = ram_res.numel()
        self.cap = ring.numel() - 1
        self.budget = int(budget)
        self.fetch = fetch
        self.release = release if release is not None else (lambda key: None)
        self.pinned = np.zeros(self.n, dtype=bool) if pinned is None else np.asarray(pinned, dtype=bool).copy()
        self.min_age = int(min_age)
        self.max_inflight = max_inflight
        self.res = ram_res.cpu().numpy().astype(np.uint8)          # the host's flags (what it last uploaded)
        self.age = np.zeros(self.n, dtype=np.int64)
        self.inflight = np.zeros(self.n, dtype=bool)
        self.tick = 0
        self.ring_seen = int(ring[0].item())
        pin = self.dev.type == "cuda"
        self._snap = [{"res": torch.empty(self.n, dtype=torch.uint8, pin_memory=pin),
                       "ring": torch.empty(ring.numel(), dtype=torch.int32, pin_memory=pin),
                       "slot": torch.empty(self.n, dtype=torch.int32, pin_memory=pin)} for _ in range(2)]
        self._snap_ev = [None, None]
        self._k = 0
        self._last_diff = None      # (keys, values) uploaded by the previous step
        self._clears = []           # [(event, tick, keys)] dropped keys awaiting release
        self._done = queue.SimpleQueue()
        self.stats = collections.Counter()

    # ---------------------------------------------------------------- storage side
    def fill_done(self, key: int) -> None:
        """The host copy of key is valid (thread-safe)."""
        self._done.put(int(key))

    # ---------------------------------------------------------------- per step
    def _event(self):
        if self.dev.type == "cuda":
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.dev))
            return ev
        return _Complete()

    def _upload(self, keys: np.ndarray, vals: np.ndarray) -> None:
        pin = self.dev.type == "cuda"
        idx = torch.from_numpy(keys.astype(np.int64))
        val = torch.from_numpy(vals.astype(np.uint8))
        if pin:
            idx, val = idx.pin_memory(), val.pin_memory()
        self.ram_res.index_copy_(0, idx.to(self.dev, non_blocking=True), val.to(self.dev, non_blocking=True))

    def step(self) -> int:
        """One decode step's bookkeeping (see the module docstring).  Returns the number of misses logged in the
        snapshot it consumed."""
        self.tick += 1
        k = self._k
        self._k ^= 1
        snap = self._snap[k]
        snap["res"].copy_(self.ram_res[: self.n], non_blocking=True)
        snap["ring"].copy_(self.ring, non_blocking=True)
        snap["slot"].copy_(self.slot_of[: self.n], non_blocking=True)
        self._snap_ev[k] = self._event()
        j = k ^ 1
        if self._snap_ev[j] is None:   # first step: nothing to consume yet
            self.stats["steps"] += 1
            return 0
        self._snap_ev[j].synchronize()   # queued before this step's work: normally complete already
        res_d = self._snap[j]["res"].numpy().copy()
        if self._last_diff is not None:   # the device as of the previous upload
            dk, dv = self._last_diff
            res_d[dk] = dv
        ring = self._snap[j]["ring"].numpy()
        vram = self._snap[j]["slot"].numpy() >= 0

        # dropped keys: the snapshot consumed now was taken a step after their clear was queued (tick + 1), so it
        # shows a victim write-back of the key in that step; release the host copy unless the key is back
        pending = []
        for ev, tq, keys in self._clears:
            if self.tick < tq + 2 or not ev.query():
                pending.append((ev, tq, keys))
                continue
            for key in keys.tolist():
                if res_d[key] or self.res[key] or self.inflight[key]:
                    self.stats["release_rescued"] += 1
                else:
                    self.release(key)
                    self.stats["released"] += 1
        self._clears = pending

        res = self.res.copy()
        flagged = (res_d == 1) & (res == 0)   # victim write-back
        res[flagged] = 1
        self.age[flagged] = self.tick
        self.stats["victims_kept"] += int(flagged.sum())
        while True:
            try:
                key = self._done.get_nowait()
            except queue.Empty:
                break
            res[key] = 1
            self.age[key] = self.tick
            self.inflight[key] = False

        # misses logged since the previous snapshot
        cnt = int(ring[0])
        new = cnt - self.ring_seen
        if new > self.cap:
            self.stats["ring_overflow"] += new - self.cap
            new = self.cap
        want = np.zeros(0, dtype=np.int64)
        if new > 0:
            keys = ring[1 + np.arange(cnt - new, cnt) % self.cap].astype(np.int64)
            keys = keys[(keys >= 0) & (keys < self.n)]
            u, c = np.unique(keys, return_counts=True)
            ok = (res[u] == 0) & ~self.inflight[u]
            u, c = u[ok], c[ok]
            want = u[np.argsort(-c, kind="stable")]
        self.ring_seen = cnt
        self.stats["masked"] += max(0, new)

        # budget
        inflight_n = int(self.inflight.sum())
        over = int(res.sum()) + inflight_n + len(want) - self.budget
        dropped = np.zeros(0, dtype=np.int64)
        if over > 0:
            c1 = np.nonzero((res == 1) & vram & ~self.pinned)[0]
            t1 = c1[np.argsort(self.age[c1], kind="stable")[:over]]
            t2 = np.zeros(0, dtype=np.int64)
            if over > len(t1):
                m = (res == 1) & ~self.pinned & (self.age <= self.tick - self.min_age)
                m[t1] = False
                c2 = np.nonzero(m)[0]
                t2 = c2[np.argsort(self.age[c2], kind="stable")[: over - len(t1)]]
            dropped = np.concatenate([t1, t2]).astype(np.int64)
            res[dropped] = 0
            self.stats["dropped"] += len(dropped)

        # admission
        free = self.budget - int(res.sum()) - inflight_n
        if self.max_inflight is not None:
            free = min(free, self.max_inflight - inflight_n)
        admit = want[: max(0, free)]
        self.stats["admit_deferred"] += len(want) - len(admit)
        for key in admit.tolist():
            self.inflight[key] = True
            self.stats["fetches"] += 1
            self.fetch(key)

        # upload the changed flags; the dropped keys' release waits for their clear
        diff = np.nonzero(res != res_d)[0].astype(np.int64)
        if len(diff):
            self._upload(diff, res[diff])
            self._last_diff = (diff, res[diff].copy())
        else:
            self._last_diff = None
        if len(dropped):
            self._clears.append((self._event(), self.tick, dropped))
        self.res = res
        self.stats["steps"] += 1
        return int(max(0, new))

    def resident(self) -> int:
        return int(self.res.sum())
