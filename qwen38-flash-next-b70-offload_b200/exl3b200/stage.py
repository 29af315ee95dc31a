"""Prefill with the routed experts on NVMe: the reference's NvTier.stage_forward (plugin/exl3xpu/nvtier.py:545-634).

When the RAM tier holds only part of the experts, a prefill-size MoE call cannot read every expert from host rows
(ExpertStore.forward_prefill_staged copies them from there).  StoreStager streams them from the packed store instead:
  * read-ahead: for each MoE layer, in model order, the records of its experts that are not in VRAM are read from the
    store (pack_store.StoreReader, O_DIRECT where the filesystem allows it) into one of `read_ahead + 1` pinned host
    buffers, on reader threads, `read_ahead` layers before the layer computes;
  * copy: when the layer computes, its records go to one of two device buffers on a copy stream (runs of
    consecutive experts as one cudaMemcpyAsync), and the compute stream waits for that copy only;
  * table: built on the device from the snapshot of the slot map: slots for experts in VRAM, the device buffer for
    the rest (no host round trip per layer);
  * buffer reuse is ordered by events: a host buffer is refilled after the copy that read it, a device buffer after
    the MoE call that read it.
At the first layer of a forward the host synchronises the device and snapshots the slot map once (decode may have
moved cache slots since the last forward, as CUDA graph replays run no host code); nothing else moves slots during
the forward.  Host buffers hold [E, rec] bytes each (rec = the record size), device buffers [E, rec] each.

The store's device tensors may be CPU tensors (tests): copies are then synchronous.
"""
from __future__ import annotations

import concurrent.futures
import time

import numpy as np
import torch

from .moe_offload import _current, _model_order, _on, _record, _wait, s64


class StoreStager:
    def __init__(self, store, reader, read_ahead: int = 2, threads: int = 8, record_layer=None):
        """store: the ExpertStore whose layers are staged; reader: a pack_store.StoreReader of the store file;
        record_layer: {store key: layer index in the store file} (default: the key's row in the store)."""
        meta = reader.meta
        if meta.E != store.E or meta.blob != store.blob:
            raise RuntimeError(f"exl3b200 StoreStager: the store file holds E={meta.E}, blob={meta.blob}; the "
                               f"ExpertStore E={store.E}, blob={store.blob}")
        if read_ahead < 1:
            raise ValueError("exl3b200 StoreStager: read_ahead >= 1")
        self.store, self.reader = store, reader
        self.E, self.rec = store.E, meta.rec
        self.record_layer = dict(record_layer) if record_layer is not None else dict(store.layer_index)
        self.dev = store.dev
        self.D = read_ahead
        self.host = [store.X.host_alloc(self.E * self.rec).view(self.E, self.rec) for _ in range(read_ahead + 1)]
        self.devbuf = [torch.empty((self.E, self.rec), dtype=torch.uint8, device=self.dev) for _ in range(2)]
        self.offsets = torch.arange(self.E, dtype=torch.int64, device=self.dev) * self.rec
        self.pool = concurrent.futures.ThreadPoolExecutor(max_workers=threads, thread_name_prefix="exl3b-stage")
        self.copy_stream = torch.cuda.Stream(self.dev) if self.dev.type == "cuda" else None
        self.host_free = [None] * len(self.host)    # per host buffer: event after the copy that last read it
        self.dev_free = [None, None]                # per device buffer: event after the MoE call that last read it
        self.next_host = 0
        self.next_dev = 0
        self.pending: dict = {}                     # key -> (host buffer, missing experts, read futures)
        self.order: list = []
        self.n_keys = -1
        self.snap_dev = None                        # device copy of the slot map, int64 [L * E]
        self.snap = None                            # its host copy
        self.stats = {"layers": 0, "records": 0}

    def close(self) -> None:
        for _, _, futs in self.pending.values():
            for f in futs:
                f.result()
        self.pending.clear()
        self.pool.shutdown(wait=True)

    def _rows(self, key) -> slice:
        li = self.store.layer_index[key]
        return slice(li * self.E, (li + 1) * self.E)

    def _kick(self, key) -> None:
        """Start the reads of `key`'s records that are not in VRAM into the next host buffer."""
        hb = self.next_host
        self.next_host = (hb + 1) % len(self.host)
        if self.host_free[hb] is not None:
            self.host_free[hb].synchronize()       # the copy that last read this buffer is done
            self.host_free[hb] = None
        missing = np.flatnonzero(self.snap[self._rows(key)] < 0)
        base = self.record_layer[key] * self.E
        rows = self.host[hb]
        futs = [self.pool.submit(self.reader.read, base + int(e), rows[int(e)]) for e in missing]
        self.pending[key] = (hb, missing, futs)

    def stage_forward(self, key, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor) -> torch.Tensor:
        """Prefill-size MoE of layer `key` with its non-VRAM experts streamed from the store (nvtier.py:574-634)."""
        st = self.store
        if self.n_keys != len(st.layer_index):
            self.order, self.n_keys = _model_order(st.layer_index), len(st.layer_index)
        pos = self.order.index(key)
        if pos == 0 or key not in self.pending:
            if self.dev.type == "cuda":
                torch.cuda.synchronize(self.dev)
            self.snap_dev = st.slot_of_dev[: len(st.layer_index) * self.E].to(torch.int64).clone()
            self.snap = self.snap_dev.cpu().numpy()
            for _, _, futs in self.pending.values():
                for f in futs:
                    f.result()
            self.pending.clear()
            for q in range(pos, min(pos + 1 + self.D, len(self.order))):
                self._kick(self.order[q])
        hb, missing, futs = self.pending.pop(key)
        for f in futs:
            f.result()                              # the records are in the host buffer
        buf = self.next_dev
        self.next_dev ^= 1
        dbase, hbase = s64(self.devbuf[buf].data_ptr()), s64(self.host[hb].data_ptr())
        cs, cur = self.copy_stream, _current(self.dev)
        with _on(cs):
            if self.dev_free[buf] is not None:
                _wait(cs, self.dev_free[buf])       # the MoE call that last read this device buffer is done
            if missing.size:
                for run in np.split(missing, np.flatnonzero(np.diff(missing) != 1) + 1):
                    e0 = int(run[0])
                    st.X.memcpy_async(dbase + e0 * self.rec, hbase + e0 * self.rec, len(run) * self.rec)
            copied = _record(cs)
        self.host_free[hb] = copied
        _wait(cur, copied)
        so = self.snap_dev[self._rows(key)]
        table = torch.where(so >= 0, so.clamp_min(0) * st.blob + st.slot_base, self.offsets + dbase)
        y = st.forward(key, x, topk_ids, topk_w, ptrs=table)
        self.dev_free[buf] = _record(cur)
        self.stats["layers"] += 1
        self.stats["records"] += int(missing.size)
        nq = pos + 1 + self.D
        if nq < len(self.order) and self.order[nq] not in self.pending:
            self._kick(self.order[nq])
        return y


class TierDriver:
    """The tier object the plugin drives (the reference's NvTier as called at plugin/sglang_plugin.tier.py:147, 546-550,
    952-953): step() once per decode step and log_stats (exl3b200.tier.TierHost), stage_forward(store, key, li, x,
    ids, w) for prefill-size MoE calls (StoreStager), ensure_for_prefill(li, ids) for smaller eager prefill calls, and
    warm(keys, max_bytes) at start-up."""

    def __init__(self, host, stager: StoreStager):
        self.host, self.stager = host, stager

    def step(self) -> int:
        return self.host.step()

    def ensure_for_prefill(self, li, topk_ids) -> int:
        """Eager prefill below the staging threshold: the layer's picked experts made RAM-resident now."""
        return self.host.ensure_for_prefill(li, topk_ids, self.stager.store.E)

    def warm(self, keys_file, max_bytes):
        """Fill the RAM tier with keys in the store file's numbering (file layer * E + expert), hottest first, up to
        max_bytes of rows; returns (experts fetched, seconds)."""
        st = self.stager.store
        row_of = {rl: st.layer_index[k] for k, rl in self.stager.record_layer.items()}
        keys = [row_of[int(k) // st.E] * st.E + int(k) % st.E for k in keys_file if int(k) // st.E in row_of]
        t0 = time.perf_counter()
        n = self.host.warm(keys, max_keys=int(max_bytes // st.blob))
        return n, time.perf_counter() - t0

    def log_stats(self, logger, every: int = 200) -> None:
        self.host.log_stats(logger, every)

    def stage_forward(self, store, key, li, x, topk_ids, topk_w):
        if store is not self.stager.store or store.layer_index.get(key) != li:
            raise RuntimeError(f"exl3b200 TierDriver.stage_forward: {key!r} (layer {li}) is not a layer of the staged "
                               "store")
        return self.stager.stage_forward(key, x, topk_ids, topk_w)
