"""Two-tier EXL3 routed-expert store on B200: the drop-in for the reference plugin's ExpertStore
(plugin/exl3xpu/moe_offload.py:92-485; API listed at :14-31).

Tier 1 is one pinned host arena per MoE layer ([E, blob] bytes, the GPU reads it at the host address over PCIe/C2C).
Tier 0 is one device arena of n_slots blobs shared by all layers (the expert cache).  Kernels find an expert only
through the per-(layer, expert) int64 pointer table ptrs_all, so moving an expert between tiers rewrites one table
entry, and either pointer stays readable while a kernel may still hold the old one.

Kept from the reference because callers and the op schemas depend on them: the constructor and method signatures,
the names, shapes and dtypes of the device cache-state tensors (they are the arguments of moe_forward_cached and
moe_prefetch), the blob format, and what each method guarantees.  The bookkeeping is this module's own: the host
keeps a mirror of the device slot map shaped like the device tensors (slot_of[key] is a view into it), table
updates are non-blocking copies from pinned memory, and prefill staging is a small double-buffer object.

Expert blob (blob_bytes(H, I, K), 1,786,368 B at H=2048, I=768, K=3):
  gate|up trellis (u32 [H/16][2I/16][8K], PLANAR4) | down trellis ([I/16][H/16][8K], PLANAR4) |
  suh_g[H] suh_u[H] svh_g[I] svh_u[I] suh_d[I] svh_d[H]   (fp16)
"""
from __future__ import annotations

import contextlib
import ctypes
import re
import threading

import numpy as np
import torch

from . import ops as _ops

_lock = threading.Lock()


def ops():
    """The op namespace (torch.ops.exl3b200_moe plus the plain helpers); loads libexl3b200.so once."""
    with _lock:
        _ops.register()
    return _ops.OPS


def s64(p: int) -> int:
    """An address as the signed 64-bit value an int64 pointer table holds."""
    return ctypes.c_int64(p).value


# ------------------------------------------------------------------------------------------------ blob packing
def planar4(tr: torch.Tensor, K: int) -> torch.Tensor:
    """Checkpoint trellis (int16 [rows, tiles, 16K]) -> its int32 words in PLANAR4 order (moe_offload.py:68-73).

    A tile holds 8 periods of K words, period g's word i at 8K-index K*g + i.  For odd K, every run of 4 tiles along a
    row is stored plane-major: [plane i][tile j][period g].  Even K (one word per plane) is planar already, so its
    words keep checkpoint order."""
    rows, tiles, _ = tr.shape
    words = tr.contiguous().view(torch.int32)
    if K % 2 == 0:
        return words.view(rows, tiles, 8 * K)
    if tiles % 4:
        raise ValueError("planar4: tiles per row must be a multiple of 4")
    by_group = words.unflatten(1, (tiles // 4, 4)).unflatten(3, (8, K))   # [row, group, tile j, period g, plane i]
    return by_group.movedim(4, 2).contiguous()                             # [row, group, plane i, tile j, period g]


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8).reshape(-1)


def pack_expert(gate: dict, up: dict, down: dict, K: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """One expert's checkpoint tensors {trellis, suh, svh} -> its blob (moe_offload.py:76-89): a new uint8 CPU tensor,
    or written into `out` (any device, exactly blob-sized).  Each projection's bit width is read from its trellis
    (16K int16 per tile), so K is only a label; gate and up of different widths are packed per k-row as the gate
    tiles (Kg) followed by the up tiles (Ku)."""
    kg, ku, kd = (p["trellis"].shape[2] // 16 for p in (gate, up, down))
    if kg == ku:
        gate_up = planar4(torch.cat((gate["trellis"], up["trellis"]), dim=1), kg)
    else:
        gate_up = torch.cat((planar4(gate["trellis"], kg).flatten(1), planar4(up["trellis"], ku).flatten(1)), dim=1)
    scales = [p[name].to(torch.float16) for name in ("suh", "svh") for p in (gate, up)]   # suh_g suh_u svh_g svh_u
    sections = [_bytes(gate_up), _bytes(planar4(down["trellis"], kd))] + [_bytes(s) for s in scales] + \
               [_bytes(down["suh"].to(torch.float16)), _bytes(down["svh"].to(torch.float16))]
    if out is None:
        return torch.cat(sections)
    sizes = [s.numel() for s in sections]
    if out.numel() != sum(sizes):
        raise ValueError(f"pack_expert: the blob has {sum(sizes)} bytes, out has {out.numel()}")
    for dst, src in zip(out.view(-1).split(sizes), sections):
        dst.copy_(src)
    return out


# ------------------------------------------------------------------------------------------------ device helpers
class _Done:
    """Event stand-in for a CPU store (tests): CPU work is synchronous, so every event has completed."""

    def query(self) -> bool:
        return True

    def synchronize(self) -> None:
        pass


def _current(dev: torch.device):
    return torch.cuda.current_stream(dev) if dev.type == "cuda" else None


def _on(stream):
    return torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()


def _record(stream):
    if stream is None:
        return _Done()
    ev = torch.cuda.Event()
    ev.record(stream)
    return ev


def _wait(stream, ev) -> None:
    if stream is not None and not isinstance(ev, _Done):
        stream.wait_event(ev)


def _as_route(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The tensor itself when it is already contiguous `dtype` (so in-place rewrites by the cached op reach the
    caller), else a contiguous converted copy."""
    return t.contiguous().to(dtype)


_LAYER_NO = re.compile(r"layers\.(\d+)\.")


def _model_order(keys) -> list:
    """Regular MoE layers in model order (the number after "layers."; keys without one last, in add order);
    multi-token-prediction layers ("mtp." keys) are left out.  Layers may be added out of order as their checkpoint
    shards load, so add order is not model order."""
    def number(k):
        m = _LAYER_NO.search(str(k))
        return int(m.group(1)) if m else 1 << 30
    return sorted((k for k in keys if not str(k).startswith("mtp.")), key=number)


class _Staging:
    """Double-buffered layer streaming for prefill (moe_offload.py:348-456): two device buffers of E blobs, a copy
    stream, and per staged layer (buffer, pointer table, copy-done event)."""

    def __init__(self, dev: torch.device):
        self.stream = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        self.staged: dict = {}            # key -> (buffer, table, ready event), staged and not yet computed
        self.busy = [None, None]          # per buffer: event after which its last reader has finished
        self.order: list = []             # regular layers in model order
        self.n_keys = -1
        self.tick = None                  # cache tick when the tables were last validated

    def in_buffer(self, buf: int) -> list:
        return [k for k, (b, _, _) in self.staged.items() if b == buf]


# ------------------------------------------------------------------------------------------------ the store
class ExpertStore:
    """Routed experts of up to max_layers MoE layers (n_experts each, H x I, K bits), n_slots of them in VRAM."""

    def __init__(self, H: int, I: int, K: int, n_experts: int, n_slots: int, device=None, max_layers: int = 64):
        self.H, self.I, self.K, self.E = H, I, K, n_experts
        self.n_slots, self.max_layers = n_slots, max_layers
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.X = ops()
        self.blob = int(self.X.blob_bytes(H, I, K))
        self.slots = torch.empty((n_slots, self.blob), dtype=torch.uint8, device=self.dev) if n_slots else None
        self.slot_base = s64(self.slots.data_ptr()) if n_slots else 0
        self.layer_index: dict = {}       # key -> row of the device tables (add order)
        self.host: dict = {}              # key -> pinned uint8 [E, blob], tier 1
        self._host_ptr: dict = {}         # key -> CPU int64 [E], host address of each expert's blob
        self.slot_of: dict = {}           # key -> CPU int32 [E] view of _mirror_slot: slot of each expert, -1 = host
        # host mirror of the device placement, valid for static placement (make_resident / evict); the device-managed
        # cache (forward_cached, prefetch) moves experts on the device, and the mirror is re-read before the next
        # static operation
        LE = max_layers * n_experts
        self._mirror_slot = torch.full((LE,), -1, dtype=torch.int32)       # mirrors slot_of_dev
        self._mirror_key = np.full(n_slots, -1, dtype=np.int64)             # mirrors slot_key
        self._slot_ready_ev: dict = {}    # slot -> event after which readers of its previous expert are done
        self._cache_used = False          # forward_cached / prefetch ran since the mirror was read
        self._stage = [None, None]        # prefill staging buffers [E, blob], allocated on first use
        self._staging: _Staging | None = None
        self._cepf_stream = None          # the copy stream while copy-engine prefetch runs
        # device cache state, the arguments of moe_forward_cached / moe_prefetch: name -> (entries, dtype, initial)
        i32, i64 = torch.int32, torch.int64
        state = {"ptrs_all": (LE, i64, 0),           # blob address of every (layer, expert): host copy or slot
                 "slot_of_dev": (LE, i32, -1),       # slot of every (layer, expert), -1 = not in VRAM
                 "slot_key": (n_slots, i32, -1),     # (layer * E + expert) held by each slot, -1 = free
                 "slot_last": (n_slots, i32, -1),    # tick of each slot's last use (the LRU order)
                 "tick": (1, i32, 0),                # cached MoE calls so far
                 "host_base": (max_layers, i64, 0),  # each layer's host arena
                 "fill_all": (LE, i64, 0),           # per (layer, expert) fill state of the cache step
                 "fill_list": (1 + n_experts, i32, 0),
                 "pf_list": (1 + n_experts, i32, 0),
                 "pf_slot": (n_experts, i32, 0),
                 "pend": (max_layers * 35, i32, 0),  # copy-engine prefetch state (schema argument)
                 "done_seq": (0, i32, 0)}            # empty: no copy-engine prefetch commits
        for name, (n, dtype, init) in state.items():
            setattr(self, name, torch.full((n,), init, dtype=dtype, device=self.dev))

    # ---- layers
    def _rows(self, key) -> slice:
        li = self.layer_index[key]
        return slice(li * self.E, (li + 1) * self.E)

    def add_layer(self, key, blobs: torch.Tensor | None = None) -> torch.Tensor:
        """Allocate layer `key`'s host arena (filled from `blobs` [E, blob] when given) and point its table there."""
        li = len(self.layer_index)
        if li >= self.max_layers:
            raise RuntimeError(f"ExpertStore: more than max_layers={self.max_layers} MoE layers")
        arena = self.X.host_alloc(self.E * self.blob).view(self.E, self.blob)
        if blobs is not None:
            arena.copy_(blobs)
        base = s64(arena.data_ptr())
        self.layer_index[key] = li
        self.host[key] = arena
        self._host_ptr[key] = torch.arange(self.E, dtype=torch.int64).mul_(self.blob).add_(base)
        self.slot_of[key] = self._mirror_slot[li * self.E:(li + 1) * self.E]
        self.ptrs_all[self._rows(key)].copy_(self._host_ptr[key])
        self.host_base[li] = base
        return arena

    def host_view(self, key) -> torch.Tensor:
        return self.host[key]

    def ptrs(self, key) -> torch.Tensor:
        """Layer `key`'s int64 [E] pointer table (a view of ptrs_all: fixed address)."""
        return self.ptrs_all[self._rows(key)]

    def slot_ptr(self, s: int) -> int:
        return self.slot_base + s * self.blob

    @property
    def free_slots(self) -> list:
        """Free slots by the host mirror, in the order make_resident takes them (lowest first)."""
        return np.flatnonzero(self._mirror_key < 0).tolist()

    @property
    def slot_owner(self) -> list:
        """Per slot (key, expert) by the host mirror, None when free."""
        by_row = {li: k for k, li in self.layer_index.items()}
        return [None if c < 0 else (by_row[int(c) // self.E], int(c) % self.E) for c in self._mirror_key]

    def _to_dev(self, values, dtype: torch.dtype) -> torch.Tensor:
        """A small index/value list (or CPU tensor) on the device, copied from pinned memory without a host sync; the
        copy is ordered on the current stream (the pinned buffer is kept until it has run)."""
        t = values.to(dtype) if isinstance(values, torch.Tensor) else torch.tensor(values, dtype=dtype)
        if self.dev.type != "cuda":
            return t
        return t.pin_memory().to(self.dev, non_blocking=True)

    # ---- static residency
    def make_resident(self, key, experts, stream=None) -> int:
        """Copy `experts` of `key` that are not in VRAM into free slots, then point the table and the device slot map
        at them, all ordered on `stream` (default: the current stream).  Returns the number copied
        (moe_offload.py:154-185)."""
        self._no_copy_prefetch("make_resident")
        self._resync()
        li = self.layer_index[key]
        mine = self.slot_of[key]
        todo = [e for e in dict.fromkeys(int(e) for e in experts) if mine[e] < 0]
        if not todo:
            return 0
        free = self.free_slots[:len(todo)]
        if len(free) < len(todo):
            raise RuntimeError(f"ExpertStore: {len(todo)} experts for {len(free)} free slots "
                               "(evict first or raise n_slots)")
        self.prefill_reset()
        cs = stream if stream is not None else _current(self.dev)
        codes = [li * self.E + e for e in todo]
        with _on(cs):
            for e, s in zip(todo, free):
                ev = self._slot_ready_ev.pop(s, None)
                if ev is not None:
                    _wait(cs, ev)
                self.X.memcpy_async(self.slot_ptr(s), int(self._host_ptr[key][e]), self.blob)
            at = self._to_dev(codes, torch.int64)
            sl = self._to_dev(free, torch.int64)
            self.ptrs_all.index_copy_(0, at, sl * self.blob + self.slot_base)
            self.slot_of_dev.index_copy_(0, at, sl.to(torch.int32))
            self.slot_key.index_copy_(0, sl, at.to(torch.int32))
            self.slot_last.index_fill_(0, sl, 0)
        mine[todo] = torch.tensor(free, dtype=torch.int32)
        self._mirror_key[free] = codes
        return len(todo)

    def evict(self, key, experts) -> None:
        """Point `experts` of `key` back at their host copies; a freed slot is refilled only after the work queued on
        the current stream so far (moe_offload.py:187-216)."""
        self._no_copy_prefetch("evict")
        self._resync()
        li = self.layer_index[key]
        mine = self.slot_of[key]
        gone = [e for e in dict.fromkeys(int(e) for e in experts) if mine[e] >= 0]
        if not gone:
            return
        self.prefill_reset()
        freed = mine[gone].tolist()
        at = self._to_dev([li * self.E + e for e in gone], torch.int64)
        sl = self._to_dev(freed, torch.int64)
        self.ptrs_all.index_copy_(0, at, self._to_dev(self._host_ptr[key][gone], torch.int64))
        self.slot_of_dev.index_fill_(0, at, -1)
        self.slot_key.index_fill_(0, sl, -1)
        self.slot_last.index_fill_(0, sl, -1)
        mine[gone] = -1
        self._mirror_key[freed] = -1
        done = _record(_current(self.dev))
        for s in freed:
            self._slot_ready_ev[s] = done

    def resident_count(self, key=None) -> int:
        """Experts in VRAM by the host mirror (all layers when key is None)."""
        if key is None:
            return int((self._mirror_slot >= 0).sum())
        return int((self.slot_of[key] >= 0).sum())

    def device_resident_count(self, key) -> int:
        """Experts of `key` in VRAM by the device slot map (reads the device)."""
        return int((self.slot_of_dev[self._rows(key)] >= 0).sum().item())

    # ---- compute
    @staticmethod
    def _rt(topk_ids, topk_w):
        """Routing as the ops take it: contiguous int32 ids and fp32 weights, the caller's own tensors when they
        already are (the cached op may rewrite masked picks in place, and callers read that)."""
        return _as_route(topk_ids, torch.int32), _as_route(topk_w, torch.float32)

    def forward(self, key, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, ptrs=None) -> torch.Tensor:
        """Routed-MoE output of layer `key` through its table (or `ptrs`); weights applied, no shared expert."""
        ids, w = self._rt(topk_ids, topk_w)
        return self.X.moe_forward(x, ids, w, self.ptrs(key) if ptrs is None else ptrs, self.I, self.K, self.E)

    def forward_cached(self, key, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor,
                       max_fill: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Decode through the device-managed LRU cache (moe_offload.py:239-249): hits read their slot, up to max_fill
        misses are copied from host into LRU slots and the table is repointed within the call, with no host sync (the
        call can be captured in a CUDA graph).  With the RAM tier on, picks in neither VRAM nor RAM are rewritten in
        place to (safe expert, weight 0) and logged to the miss ring.  `out` (this build's extension) takes the
        output in a caller buffer: the same computation without the torch op dispatch."""
        ids, w = self._rt(topk_ids, topk_w)
        self._cache_used = True
        args = (x, ids, w, self.ptrs_all, self.layer_index[key], self.slot_of_dev, self.slot_key, self.slot_last,
                self.tick, self.host_base, self.slot_base, self.fill_all, self.fill_list,
                self.E if max_fill is None else max_fill, self.I, self.K, self.E, self.pend, self.done_seq)
        if out is not None:
            return _ops._moe_forward_cached_impl(*args, out=out)
        return self.X.moe_forward_cached(*args)

    def forward_cached_routed(self, key, x: torch.Tensor, wr: torch.Tensor, bias: torch.Tensor | None, topk: int,
                              max_fill: int | None = None, out: torch.Tensor | None = None):
        """The router (logits x Wr^T + bias, softmax top-k) and forward_cached on its picks in one call (this build's
        extension: the reference plugin takes its picks from SGLang's TopK).  Returns (out, topk_ids, topk_w) with the
        values router_topk + forward_cached give, ids / w after the tier mask's rewrite; small batches select the
        picks inside the decode kernels, one grid completion fewer per call."""
        self._cache_used = True
        return _ops._moe_forward_cached_routed_impl(
            x, wr, bias, topk, self.ptrs_all, self.layer_index[key], self.slot_of_dev, self.slot_key, self.slot_last,
            self.tick, self.host_base, self.slot_base, self.fill_all, self.fill_list,
            self.E if max_fill is None else max_fill, self.I, self.K, self.E, self.pend, self.done_seq, out=out)

    def prefetch(self, key, ids: torch.Tensor, max_fill: int = 16) -> None:
        """Claim LRU slots for the predicted experts `ids` of `key` and copy them from host, on the CURRENT stream
        (a side stream that waited for the previous MoE call; the compute stream waits for it before the next).  The
        tick is not advanced, so the slots of the last MoE call stay (moe_offload.py:251-262)."""
        if not self.n_slots:
            return
        ids = _as_route(ids, torch.int32)
        self._cache_used = True
        self.X.moe_prefetch(ids.flatten(), self.ptrs_all, self.layer_index[key], self.slot_of_dev, self.slot_key,
                            self.slot_last, self.tick, self.host_base, self.slot_base, self.pf_list, self.pf_slot,
                            max_fill, self.E, self.blob)

    # ---- copy-engine prefetch
    def _no_copy_prefetch(self, what: str) -> None:
        if self._cepf_stream is not None:
            raise RuntimeError(f"ExpertStore.{what}: stop_copy_prefetch first (planned slots may still be filling)")

    def start_copy_prefetch(self) -> None:
        """Start the host worker that turns device-written prefetch plans into copy-engine copies on a stream of its
        own (moe_offload.py:264-280).  While it runs, plan_prefetch publishes plans and every cached MoE call first
        commits the plans that have landed; static placement and staged prefill wait for stop_copy_prefetch."""
        if self._cepf_stream is not None:
            raise RuntimeError("ExpertStore: copy prefetch is already running")
        L, E = len(self.layer_index), self.E
        if not L or not self.n_slots:
            raise RuntimeError("ExpertStore: copy prefetch needs layers and slots")
        self._plans = self.X.host_alloc(L * (4 + 2 * E) * 4)
        self._plans.zero_()
        self._plan_seq = torch.zeros(L, dtype=torch.int32, device=self.dev)
        self.done_seq = torch.zeros(L, dtype=torch.int32, device=self.dev)
        self.pend.zero_()
        bases = torch.zeros(L, dtype=torch.int64)
        for key, li in self.layer_index.items():
            bases[li] = int(self._host_ptr[key][0])
        torch.cuda.synchronize(self.dev)
        stream = torch.cuda.Stream(self.dev)
        with torch.cuda.stream(stream):
            self.X.moe_prefetch_worker_start(self._plans, bases, self.slot_base, self.blob, self.ptrs_all,
                                             self.slot_last, torch.empty(0, dtype=torch.uint8), self.done_seq, L, E,
                                             keep=self)
        self._cepf_stream = stream

    def plan_prefetch(self, key, ids: torch.Tensor, max_fill: int = 16) -> None:
        """On the COMPUTE stream (e.g. right after one layer's MoE call, for the next layer): claim and pin LRU slots
        for the predicted experts `ids` of `key` (at most 16) and publish the plan; the worker copies them on the copy
        engine and a later cached call commits them.  The compute stream never waits (moe_offload.py:282-289)."""
        if self._cepf_stream is None:
            raise RuntimeError("ExpertStore: start_copy_prefetch first")
        ids = _as_route(ids, torch.int32)
        self._cache_used = True
        self.X.moe_prefetch_plan(ids.flatten(), self.ptrs_all, self.layer_index[key], self.slot_of_dev, self.slot_key,
                                 self.slot_last, self.tick, self.host_base, self.slot_base, self.pf_list, self.pf_slot,
                                 self._plans, self._plan_seq, self.pend, self.done_seq, max_fill, self.E, self.blob)

    def stop_copy_prefetch(self) -> list:
        """Stop the worker once it has copied every plan queued so far and commit them; returns [plans handled,
        experts copied] (moe_offload.py:291-302).  Afterwards cached calls run without prefetch commits."""
        if self._cepf_stream is None:
            return [0, 0]
        cs = torch.cuda.current_stream(self.dev)
        cs.synchronize()                                   # every queued plan has been published
        try:
            counts = self.X.moe_prefetch_worker_stop()     # copies them and waits for the copy stream
        finally:
            _ops.cepf_commit(self.pend, self.done_seq, self.E, self.ptrs_all, self.slot_last, self.slot_base,
                             self.blob)
            cs.synchronize()
            self.done_seq = torch.zeros(0, dtype=torch.int32, device=self.dev)
            self._cepf_stream = None
        return counts

    # ---- prefill staging
    def stage_layer(self, key, buf: int, stream) -> torch.Tensor:
        """Queue on `stream` the copy of every expert of `key` that is not in VRAM into staging buffer `buf` (0 or 1),
        runs of consecutive experts as one copy; returns the layer's pointer table for forward(ptrs=...), valid once
        `stream` has been waited on: slots for resident experts, the staging buffer for the rest
        (moe_offload.py:305-329)."""
        self._no_copy_prefetch("stage_layer")
        if _ops.G.ram_res is not None:
            raise RuntimeError("ExpertStore.stage_layer: the RAM tier is on, so host rows may have been released; "
                               "stage from the pack store (exl3b200.stage.StoreStager) instead")
        if self._stage[buf] is None:
            self._stage[buf] = torch.empty((self.E, self.blob), dtype=torch.uint8, device=self.dev)
        base = s64(self._stage[buf].data_ptr())
        self._resync()
        mine = self.slot_of[key]
        missing = np.flatnonzero(mine.numpy() < 0)
        if missing.size:
            runs = np.split(missing, np.flatnonzero(np.diff(missing) != 1) + 1)
            src = self._host_ptr[key]
            with _on(stream):
                for run in runs:
                    e0 = int(run[0])
                    self.X.memcpy_async(base + e0 * self.blob, int(src[e0]), len(run) * self.blob)
        table = torch.arange(self.E, dtype=torch.int64).mul_(self.blob).add_(base)
        held = mine >= 0
        table[held] = mine[held].to(torch.int64) * self.blob + self.slot_base
        return self._to_dev(table, torch.int64)

    def reset_cache(self) -> None:
        """Empty every slot and point every table at host memory (waits for the current stream's queued work)."""
        self._no_copy_prefetch("reset_cache")
        cs = _current(self.dev)
        if cs is not None:
            cs.synchronize()
        for key in self.layer_index:
            self.ptrs_all[self._rows(key)].copy_(self._host_ptr[key])
        for t in (self.slot_of_dev, self.slot_key, self.slot_last):
            t.fill_(-1)
        self.fill_all.zero_()
        self.pend.zero_()
        self._mirror_slot.fill_(-1)
        self._mirror_key.fill(-1)
        self._slot_ready_ev.clear()
        self._cache_used = False
        self.prefill_reset()

    def forward_prefill_staged(self, key, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor) -> torch.Tensor:
        """Prefill-size MoE of layer `key` from a staging buffer (moe_offload.py:348-437).  The layer's experts that
        are not in VRAM were normally copied on the copy stream while the previous layer computed; after queueing this
        layer's compute, the next layer in model order (wrapping to the first: chunked prefill runs forwards back to
        back) is staged into the other buffer.

        At the first layer of a forward the host synchronises the device: decode (graph replays) may have moved
        cache slots since the tables were staged, so when the cache tick moved (or cached calls ran) the placement
        mirror is re-read and pre-staged tables are dropped."""
        if self._staging is None:
            self._staging = _Staging(self.dev)
        sg = self._staging
        if sg.n_keys != len(self.layer_index):
            sg.order, sg.n_keys = _model_order(self.layer_index), len(self.layer_index)
        if sg.order and key == sg.order[0]:
            if self.dev.type == "cuda":
                torch.cuda.synchronize(self.dev)
            tick = int(self.tick.item())
            if tick != sg.tick or self._cache_used:
                self.sync_mirror()
                sg.staged.clear()
                sg.tick = tick
        if key not in sg.staged:
            self._stage_into(key, 1 if sg.in_buffer(0) else 0)
        buf, table, ready = sg.staged.pop(key)
        cs = _current(self.dev)
        _wait(cs, ready)
        y = self.forward(key, x, topk_ids, topk_w, ptrs=table)
        sg.busy[buf] = _record(cs)
        if key in sg.order:
            nxt = sg.order[(sg.order.index(key) + 1) % len(sg.order)]
            if nxt != key and nxt not in sg.staged:
                self._stage_into(nxt, 1 - buf)
        return y

    def _stage_into(self, key, buf: int) -> None:
        """Stage `key` into buffer `buf` on the copy stream, after that buffer's last reader; a layer staged there
        earlier and not computed yet is dropped (its copy is about to be overwritten)."""
        sg = self._staging
        for k in sg.in_buffer(buf):
            del sg.staged[k]
        if sg.busy[buf] is not None:
            _wait(sg.stream, sg.busy[buf])
            sg.busy[buf] = None
        table = self.stage_layer(key, buf, sg.stream)
        sg.staged[key] = (buf, table, _record(sg.stream))

    def prefill_reset(self) -> None:
        """Drop pre-staged layers: their tables hold slot pointers that are valid only until the placement changes."""
        if self._staging is not None:
            self._staging.staged.clear()

    def sync_mirror(self) -> None:
        """Re-read the host mirror of the placement (slot_of, free slots, owners) from the device slot map: a
        device-to-host read that synchronises the current stream, for static placement, never in the decode loop."""
        self._mirror_slot.copy_(self.slot_of_dev.cpu())
        self._mirror_key[:] = self.slot_key.cpu().numpy()
        self._cache_used = False

    def _resync(self) -> None:
        if self._cache_used:
            self.sync_mirror()
