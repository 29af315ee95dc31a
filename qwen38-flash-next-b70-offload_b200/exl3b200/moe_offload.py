"""Two-tier EXL3 routed-expert store on B200: the drop-in for plugin/exl3xpu/moe_offload.py.

Every expert of every MoE layer lives in pinned host memory (tier 1, readable by the GPU at the same address), a
subset lives in device slots (tier 0, the expert cache, one arena shared by all layers).  Kernels address experts
only through a per-layer int64 POINTER TABLE, so moving an expert between tiers is one 8-byte table write
(moe_offload.py:1-31 in the reference).  The API, the blob format and the cache state tensors are the reference's;
torch.xpu becomes torch.cuda and the ops come from libexl3b200.so (torch.ops.exl3b200_moe).

Expert blob (blob_bytes(H, I, K), 1,786,368 B at H=2048, I=768, K=3):
  gate|up trellis (u32 [H/16][2I/16][8K], PLANAR4) | down trellis ([I/16][H/16][8K], PLANAR4) |
  suh_g[H] suh_u[H] svh_g[I] svh_u[I] suh_d[I] svh_d[H]   (fp16)
"""
from __future__ import annotations

import threading

import torch

from . import ops as _ops

_lock = threading.Lock()


def ops():
    """The op namespace (torch.ops.exl3b200_moe plus the plain helpers); loads libexl3b200.so once."""
    with _lock:
        _ops.register()
    return _ops.OPS


def s64(p: int) -> int:
    return p - (1 << 64) if p >= (1 << 63) else p


def planar4(tr: torch.Tensor, K: int) -> torch.Tensor:
    """int16 trellis [rows, tiles, 16K] -> int32 words in PLANAR4 order (moe_offload.py:68-73).  Odd K: D = K planes of
    8 periods per tile; even K (D = 1) is already planar, so the words are returned in checkpoint order."""
    r, n, _ = tr.shape
    w = tr.contiguous().view(torch.int32)
    if K % 2 == 0:
        return w.view(r, n, 8 * K)
    if n % 4:
        raise ValueError("planar4: tiles per row must be a multiple of 4")
    w = w.view(r, n // 4, 4, 8, K)                 # [row, group, tile, period g, plane i]
    return w.permute(0, 1, 4, 2, 3).contiguous()   # [row, group, plane i, tile, g]


def pack_expert(gate: dict, up: dict, down: dict, K: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Checkpoint tensors {trellis, suh, svh} of one expert -> blob (moe_offload.py:76-89).  K is the bit width of
    gate/up/down; a mixed expert packs each tensor with its own K (trellis.shape[2] // 16)."""
    b = lambda z: z.contiguous().view(torch.uint8).flatten()   # noqa: E731
    kg = gate["trellis"].shape[2] // 16
    ku = up["trellis"].shape[2] // 16
    kd = down["trellis"].shape[2] // 16
    if kg == ku:
        gu = b(planar4(torch.cat([gate["trellis"], up["trellis"]], dim=1), kg))
    else:   # per k-row: gate tiles (Kg) then up tiles (Ku)
        pg = planar4(gate["trellis"], kg).reshape(gate["trellis"].shape[0], -1)
        pu = planar4(up["trellis"], ku).reshape(up["trellis"].shape[0], -1)
        gu = b(torch.cat([pg, pu], dim=1))
    parts = [gu, b(planar4(down["trellis"], kd)), b(gate["suh"].half()), b(up["suh"].half()),
             b(gate["svh"].half()), b(up["svh"].half()), b(down["suh"].half()), b(down["svh"].half())]
    if out is None:
        return torch.cat(parts)
    o = 0
    for p in parts:
        out[o:o + p.numel()].copy_(p)
        o += p.numel()
    assert o == out.numel(), (o, out.numel())
    return out


class ExpertStore:
    def __init__(self, H: int, I: int, K: int, n_experts: int, n_slots: int, device=None, max_layers: int = 64):
        self.H, self.I, self.K, self.E = H, I, K, n_experts
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.X = ops()
        self.blob = int(self.X.blob_bytes(H, I, K))
        self.n_slots = n_slots
        self.max_layers = max_layers
        self.slots = torch.empty((n_slots, self.blob), dtype=torch.uint8, device=self.dev) if n_slots else None
        self.slot_owner: list = [None] * n_slots
        self.free_slots = list(range(n_slots - 1, -1, -1))
        self.host: dict = {}
        self.layer_index: dict = {}
        self.slot_of: dict = {}
        self._host_ptr: dict = {}
        self._stage = [None, None]
        self._slot_ready_ev: dict = {}
        LE = max_layers * n_experts
        d = self.dev
        self.ptrs_all = torch.zeros(LE, dtype=torch.int64, device=d)
        self.slot_of_dev = torch.full((LE,), -1, dtype=torch.int32, device=d)
        self.slot_key = torch.full((n_slots,), -1, dtype=torch.int32, device=d)
        self.slot_last = torch.full((n_slots,), -1, dtype=torch.int32, device=d)
        self.tick = torch.zeros(1, dtype=torch.int32, device=d)
        self.host_base = torch.zeros(max_layers, dtype=torch.int64, device=d)
        self.fill_all = torch.zeros(LE, dtype=torch.int64, device=d)
        self.fill_list = torch.zeros(1 + n_experts, dtype=torch.int32, device=d)
        self.pf_list = torch.zeros(1 + n_experts, dtype=torch.int32, device=d)
        self.pf_slot = torch.zeros(n_experts, dtype=torch.int32, device=d)
        self.pend = torch.zeros(max_layers * 35, dtype=torch.int32, device=d)
        self.done_seq = torch.zeros(0, dtype=torch.int32, device=d)
        self.slot_base = s64(self.slots.data_ptr()) if n_slots else 0
        self._cache_used = False

    # ---- layers
    def add_layer(self, key, blobs: torch.Tensor | None = None) -> torch.Tensor:
        li = len(self.layer_index)
        if li >= self.max_layers:
            raise RuntimeError(f"ExpertStore: more than max_layers={self.max_layers} MoE layers")
        self.layer_index[key] = li
        h = self.X.host_alloc(self.E * self.blob).view(self.E, self.blob)
        if blobs is not None:
            h.copy_(blobs)
        self.host[key] = h
        base = s64(h.data_ptr())
        self._host_ptr[key] = base + torch.arange(self.E, dtype=torch.int64) * self.blob
        self.ptrs_all[li * self.E:(li + 1) * self.E].copy_(self._host_ptr[key])
        self.host_base[li] = base
        self.slot_of[key] = torch.full((self.E,), -1, dtype=torch.int32)
        return h

    def host_view(self, key) -> torch.Tensor:
        return self.host[key]

    def ptrs(self, key) -> torch.Tensor:
        li = self.layer_index[key]
        return self.ptrs_all[li * self.E:(li + 1) * self.E]

    def slot_ptr(self, s: int) -> int:
        return self.slot_base + s * self.blob

    # ---- static residency
    def make_resident(self, key, experts, stream=None) -> int:
        """Copy experts into free device slots, then repoint the table and the device slot map, ordered on `stream`
        (default: current stream).  Returns the number copied (moe_offload.py:154-185)."""
        s_ = stream or torch.cuda.current_stream(self.dev)
        self._resync()
        so = self.slot_of[key]
        li = self.layer_index[key]
        todo = [int(e) for e in experts if so[int(e)] < 0]
        if not todo:
            return 0
        es, sls = [], []
        with torch.cuda.stream(s_):
            for e in todo:
                if not self.free_slots:
                    raise RuntimeError("ExpertStore: no free slot (evict first or raise n_slots)")
                sl = self.free_slots.pop()
                ev = self._slot_ready_ev.pop(sl, None)
                if ev is not None:
                    s_.wait_event(ev)
                self.X.memcpy_async(self.slot_ptr(sl), s64(self.host[key][e].data_ptr()), self.blob)
                self.slot_owner[sl] = (key, e)
                so[e] = sl
                es.append(e)
                sls.append(sl)
            d = self.dev
            keys = torch.tensor([li * self.E + e for e in es], dtype=torch.int64)
            slt = torch.tensor(sls, dtype=torch.int64)
            self.ptrs_all.index_copy_(0, keys.to(d), (self.slot_base + slt * self.blob).to(d))
            self.slot_of_dev.index_copy_(0, keys.to(d), slt.to(torch.int32).to(d))
            self.slot_key.index_copy_(0, slt.to(d), keys.to(torch.int32).to(d))
            self.slot_last.index_fill_(0, slt.to(d), 0)
        return len(todo)

    def evict(self, key, experts) -> None:
        """Repoint to the host copy; the slot is reusable after the current stream's queued work."""
        self._resync()
        so = self.slot_of[key]
        li = self.layer_index[key]
        es, sls = [], []
        for e in experts:
            e = int(e)
            sl = int(so[e])
            if sl < 0:
                continue
            es.append(e)
            sls.append(sl)
            so[e] = -1
            self.slot_owner[sl] = None
        if not es:
            return
        d = self.dev
        et = torch.tensor(es, dtype=torch.int64)
        keys = (li * self.E + et).to(d)
        slt = torch.tensor(sls, dtype=torch.int64).to(d)
        self.ptrs_all.index_copy_(0, keys, self._host_ptr[key][et].to(d))
        self.slot_of_dev.index_fill_(0, keys, -1)
        self.slot_key.index_fill_(0, slt, -1)
        self.slot_last.index_fill_(0, slt, -1)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.dev))
        for sl in sls:
            self._slot_ready_ev[sl] = ev
            self.free_slots.append(sl)

    def resident_count(self, key=None) -> int:
        if key is None:
            return sum(int((v >= 0).sum()) for v in self.slot_of.values())
        return int((self.slot_of[key] >= 0).sum())

    def device_resident_count(self, key) -> int:
        li = self.layer_index[key]
        return int((self.slot_of_dev[li * self.E:(li + 1) * self.E] >= 0).sum().item())

    # ---- compute
    @staticmethod
    def _rt(topk_ids, topk_w):
        ids = topk_ids if topk_ids.dtype == torch.int32 and topk_ids.is_contiguous() else topk_ids.to(torch.int32).contiguous()
        w = topk_w if topk_w.dtype == torch.float32 and topk_w.is_contiguous() else topk_w.to(torch.float32).contiguous()
        return ids, w

    def forward(self, key, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, ptrs=None) -> torch.Tensor:
        ids, w = self._rt(topk_ids, topk_w)
        return self.X.moe_forward(x, ids, w, self.ptrs(key) if ptrs is None else ptrs, self.I, self.K, self.E)

    def forward_cached(self, key, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor,
                       max_fill: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Decode with the device-managed LRU cache: misses are copied from host into their LRU slot and the table is
        repointed within the call (no host sync, graph-safe).  With the tier on, picks in neither VRAM nor RAM are
        rewritten in place to (safe expert, weight 0) and logged to the miss ring."""
        ids, w = self._rt(topk_ids, topk_w)
        self._cache_used = True
        if out is not None:   # extension: write into a caller buffer (same computation, no torch op dispatch)
            return _ops._moe_forward_cached_impl(x, ids, w, self.ptrs_all, self.layer_index[key], self.slot_of_dev,
                                                 self.slot_key, self.slot_last, self.tick, self.host_base, self.slot_base,
                                                 self.fill_all, self.fill_list, self.E if max_fill is None else max_fill,
                                                 self.I, self.K, self.E, self.pend, self.done_seq, out=out)
        return self.X.moe_forward_cached(x, ids, w, self.ptrs_all, self.layer_index[key], self.slot_of_dev,
                                         self.slot_key, self.slot_last, self.tick, self.host_base, self.slot_base,
                                         self.fill_all, self.fill_list, self.E if max_fill is None else max_fill,
                                         self.I, self.K, self.E, self.pend, self.done_seq)

    def prefetch(self, key, ids: torch.Tensor, max_fill: int = 16) -> None:
        """Claim LRU slots for predicted experts of `key` and copy them from host on the CURRENT stream (use a side
        stream that waited for the previous MoE call).  The tick is not advanced, so the last call's slots stay."""
        if not self.n_slots:
            return
        ids = ids if ids.dtype == torch.int32 and ids.is_contiguous() else ids.to(torch.int32).contiguous()
        self._cache_used = True
        self.X.moe_prefetch(ids.flatten(), self.ptrs_all, self.layer_index[key], self.slot_of_dev, self.slot_key,
                            self.slot_last, self.tick, self.host_base, self.slot_base, self.pf_list, self.pf_slot,
                            max_fill, self.E, self.blob)

    # ---- prefill staging
    def stage_layer(self, key, buf: int, stream) -> torch.Tensor:
        """Copy every non-resident expert of `key` into staging buffer `buf` on `stream`; returns the pointer table to
        pass to forward(ptrs=...) once `stream` has been waited on (moe_offload.py:305-329)."""
        if self._stage[buf] is None:
            self._stage[buf] = torch.empty((self.E, self.blob), dtype=torch.uint8, device=self.dev)
        st = self._stage[buf]
        self._resync()
        so = self.slot_of[key]
        miss = (so < 0).nonzero().flatten().tolist()
        with torch.cuda.stream(stream):
            i = 0
            while i < len(miss):
                j = i
                while j + 1 < len(miss) and miss[j + 1] == miss[j] + 1:
                    j += 1
                n = j - i + 1
                self.X.memcpy_async(s64(st[miss[i]].data_ptr()), s64(self.host[key][miss[i]].data_ptr()), n * self.blob)
                i = j + 1
        sp = s64(st.data_ptr()) + torch.arange(self.E, dtype=torch.int64) * self.blob
        if self.n_slots:
            dp = self.slot_base + so.clamp_min(0).to(torch.int64) * self.blob
            sp = torch.where(so >= 0, dp, sp)
        return sp.to(self.dev)

    def reset_cache(self) -> None:
        """Empty every slot and repoint all tables to host memory (waits for queued work)."""
        torch.cuda.current_stream(self.dev).synchronize()
        for key, li in self.layer_index.items():
            self.ptrs_all[li * self.E:(li + 1) * self.E].copy_(self._host_ptr[key])
            self.slot_of[key].fill_(-1)
        self.slot_of_dev.fill_(-1)
        self.slot_key.fill_(-1)
        self.slot_last.fill_(-1)
        self.fill_all.zero_()
        self.pend.zero_()
        self.slot_owner = [None] * self.n_slots
        self.free_slots = list(range(self.n_slots - 1, -1, -1))
        self._slot_ready_ev.clear()
        self._cache_used = False

    def forward_prefill_staged(self, key, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor) -> torch.Tensor:
        """Prefill-size MoE for `key` from a device staging buffer, double-buffered across layers on a side stream
        (moe_offload.py:348-437): the layer's non-resident experts are copied H2D (normally while the previous
        layer computed), then the next layer starts staging into the other buffer."""
        if not hasattr(self, "_pf"):
            self._pf = {"stream": torch.cuda.Stream(self.dev), "buf_of": {}, "ready": {}, "free": [None, None],
                        "order": None}
        pf = self._pf
        if pf["order"] is None or len(pf["order"]) != len(self.layer_index):
            pf["order"] = list(self.layer_index)
            import re as _re

            def _lid(k):
                m = _re.search(r"layers\.(\d+)\.", str(k))
                return int(m.group(1)) if m else 1 << 30
            pf["layers"] = sorted((k for k in pf["order"] if not str(k).startswith("mtp.")), key=_lid)
        cs = torch.cuda.current_stream(self.dev)
        if pf["layers"] and key == pf["layers"][0]:
            torch.cuda.synchronize(self.dev)
            t = int(self.tick.item())
            if pf.get("tick") != t or self._cache_used:
                self.sync_mirror()
                self._cache_used = False
                pf["buf_of"].clear()
                pf["ready"].clear()
                pf["tick"] = t
        if key not in pf["buf_of"]:
            used = {b for b, _ in pf["buf_of"].values()}
            self._stage_into(key, 0 if 0 not in used else 1)
        buf, table = pf["buf_of"].pop(key)
        rdy = pf["ready"].pop(key)
        cs.wait_event(rdy)
        ids, w = self._rt(topk_ids, topk_w)
        y = self.X.moe_forward(x, ids, w, table, self.I, self.K, self.E)
        ev = torch.cuda.Event()
        ev.record(cs)
        pf["free"][buf] = ev
        layers = pf["layers"]
        pos = layers.index(key) if key in layers else -1
        if pos >= 0 and layers:
            nxt = layers[(pos + 1) % len(layers)]
            if nxt not in pf["buf_of"] and nxt != key:
                self._stage_into(nxt, 1 - buf)
        return y

    def _stage_into(self, key, buf: int) -> None:
        pf = self._pf
        st = pf["stream"]
        for k_ in [k_ for k_, (b_, _) in pf["buf_of"].items() if b_ == buf]:
            pf["buf_of"].pop(k_)
            pf["ready"].pop(k_, None)
        if pf["free"][buf] is not None:
            st.wait_event(pf["free"][buf])
            pf["free"][buf] = None
        table = self.stage_layer(key, buf, st)
        ev = torch.cuda.Event()
        ev.record(st)
        pf["buf_of"][key] = (buf, table)
        pf["ready"][key] = ev

    def prefill_reset(self) -> None:
        """Drop pre-staged layers (their tables hold slot pointers valid only until the next cache update)."""
        if hasattr(self, "_pf") and self._pf["buf_of"]:
            self._pf["buf_of"].clear()
            self._pf["ready"].clear()

    def sync_mirror(self) -> None:
        """Rebuild the CPU mirror (slot_of, slot_owner, free list) from the device cache state (syncs)."""
        sk = self.slot_key.cpu()
        sod = self.slot_of_dev.cpu()
        keys = {li: key for key, li in self.layer_index.items()}
        for key, li in self.layer_index.items():
            self.slot_of[key] = sod[li * self.E:(li + 1) * self.E].clone()
        self.slot_owner = [None] * self.n_slots
        free = []
        for sl in range(self.n_slots):
            k = int(sk[sl])
            if k < 0:
                free.append(sl)
            else:
                self.slot_owner[sl] = (keys[k // self.E], k % self.E)
        self.free_slots = free[::-1]

    def _resync(self) -> None:
        if self._cache_used:
            self.sync_mirror()
            self._cache_used = False
