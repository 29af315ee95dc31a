"""torch ops with the reference's schemas (namespace exl3b200_moe), backed by libexl3b200.so.

The schemas are those of TORCH_LIBRARY(exl3xpu_moe) (kernels/moe-a8/exl3_moe.a8.sycl:1555-1592); only the namespace
and the device (CUDA) differ.  Every CUDA implementation calls the C ABI on the current stream; nothing syncs the
host, so the ops can be captured in CUDA graphs.  Process-global settings mirror the reference's moe_set_* setters
(:682-790): they are read at call time (and therefore baked into captured graphs), and are not thread-safe.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream

NS = "exl3b200_moe"


class _Globals:
    prefill_min_m = 256        # moe_set_prefill_min_m (exl3_moe.a8.sycl:787); M >= this: prefill path
    pair_max_m = 4             # moe_set_pair_max_m (:730); accepted for schema compatibility
    gu_p, dn_p = 5, 0          # moe_set_splits (:684); tuning knobs of the B70 kernels, accepted and ignored
    mr = 0                     # moe_set_mr (:733)
    debug = 0                  # moe_set_debug (:731)
    host_stride = 0            # moe_set_host_stride (:772); 0 = blob size
    ram_res = None             # moe_set_tier (:775-780): uint8 [L*E], int32 miss ring [1+R], int32 safe [L]
    ring = None
    safe = None
    vict = None                # moe_set_victims (:767-768): int32 [1 + 2E]
    vring = None               # moe_set_victim_ring (a9.patch): (meta, sel, buf)
    skip_zero = True           # picks with weight 0 contribute 0: skip them (output unchanged)


G = _Globals()


def blob_bytes(H: int, I: int, K: int, Ku: int | None = None, Kd: int | None = None) -> int:
    Ku = K if Ku is None else Ku
    Kd = K if Kd is None else Kd
    return int(_lib.lib().exl3b_blob_bytes(H, I, K, Ku, Kd))


# ------------------------------------------------------------------------------------------------ building blocks
_OUT_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

def _check_x(x: torch.Tensor):
    if x.dim() != 2 or x.stride(1) != 1:
        raise RuntimeError("exl3b200: x must be 2-D with unit column stride")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError("exl3b200: x must be bf16 or fp16")
    if not x.is_cuda:
        raise RuntimeError("exl3b200: x must be a CUDA tensor")


def _check_route(ids: torch.Tensor, w: torch.Tensor):
    if ids.dtype != torch.int32 or not ids.is_contiguous():
        raise RuntimeError("exl3b200: topk_ids must be contiguous int32")
    if w.dtype != torch.float32 or not w.is_contiguous():
        raise RuntimeError("exl3b200: topk_w must be contiguous fp32")


def moe_decode(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, ptrs: torch.Tensor, I: int, K: int, E: int,
               kinfo: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed MoE through the decode kernels (any M; sized for small M)."""
    _check_x(x)
    _check_route(ids, w)
    if ptrs.dtype != torch.int64 or not ptrs.is_contiguous():
        raise RuntimeError("exl3b200: ptrs must be contiguous int64")
    M, H = x.shape
    topk = ids.shape[1] if ids.dim() == 2 else 1
    if out is None:
        out = torch.empty_like(x)
    if M == 0:
        return out
    L = _lib.lib()
    wsb = int(L.exl3b_moe_decode_workspace(M, topk, H, I))
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    flags = 1 if G.skip_zero else 0
    check(L.exl3b_moe_decode(x.data_ptr(), x.stride(0), int(x.dtype == torch.bfloat16), ids.data_ptr(), w.data_ptr(),
                             M, topk, ptrs.data_ptr(), ptr(kinfo), H, I, K, E, out.data_ptr(), out.stride(0),
                             _OUT_CODE[out.dtype], ws.data_ptr(), wsb, flags, stream(x.device)),
          "moe_decode")
    return out


def moe_prefill(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, ptrs: torch.Tensor, I: int, K: int, E: int,
                kinfo: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed MoE through the grouped tensor-core prefill kernels (the reference's moe_prefill): H % 256 == 0,
    I % 128 == 0; sized for many tokens."""
    _check_x(x)
    _check_route(ids, w)
    if ptrs.dtype != torch.int64 or not ptrs.is_contiguous():
        raise RuntimeError("exl3b200: ptrs must be contiguous int64")
    M, H = x.shape
    topk = ids.shape[1] if ids.dim() == 2 else 1
    if out is None:
        out = torch.empty_like(x)
    if M == 0:
        return out
    L = _lib.lib()
    wsb = int(L.exl3b_moe_prefill_workspace(M, topk, H, I, E))
    raw = torch.empty(wsb + 1024, dtype=torch.uint8, device=x.device)
    base = (raw.data_ptr() + 1023) & ~1023
    check(L.exl3b_moe_prefill(x.data_ptr(), x.stride(0), int(x.dtype == torch.bfloat16), ids.data_ptr(), w.data_ptr(),
                              M, topk, ptrs.data_ptr(), ptr(kinfo), H, I, K, E, out.data_ptr(), out.stride(0),
                              _OUT_CODE[out.dtype], base, wsb, 0, stream(x.device)),
          "moe_prefill")
    return out


def router_topk(x: torch.Tensor, wr: torch.Tensor, bias: torch.Tensor | None, topk: int):
    """Router GEMV + softmax top-k: returns (ids int32 [T, topk], w fp32 [T, topk])."""
    if x.dtype != torch.bfloat16 or wr.dtype != torch.bfloat16:
        raise RuntimeError("exl3b200 router: x and Wr must be bf16")
    if x.dim() != 2 or x.stride(1) != 1 or not wr.is_contiguous():
        raise RuntimeError("exl3b200 router: x 2-D unit-stride rows, Wr contiguous")
    T, H = x.shape
    E = wr.shape[0]
    ids = torch.empty((T, topk), dtype=torch.int32, device=x.device)
    w = torch.empty((T, topk), dtype=torch.float32, device=x.device)
    logits = torch.empty((T, E), dtype=torch.float32, device=x.device)
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        raise RuntimeError("exl3b200 router: bias must be contiguous fp32")
    check(_lib.lib().exl3b_router_topk(x.data_ptr(), x.stride(0), wr.data_ptr(), ptr(bias), T, H, E, topk,
                                       ids.data_ptr(), w.data_ptr(), logits.data_ptr(), _router_counter(x.device),
                                       stream(x.device)), "router")
    return ids, w


_ctr = {}


def _router_counter(device) -> int:
    """Per (device, stream) int32 arrival counter of the fused router selection.  Zeroed once; every launch leaves it
    at zero.  Created on first use, so the first router call should come before any graph capture on that stream."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream(device))
    t = _ctr.get(key)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=device)
        _ctr[key] = t
    return t.data_ptr()


def dequant(words: torch.Tensor, rows16: int, row_stride: int, tile0: int, ntiles: int, K: int, planar: bool,
            out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty((rows16 * 16, ntiles * 16), dtype=torch.float16, device=words.device)
    check(_lib.lib().exl3b_dequant(words.data_ptr(), rows16, row_stride, tile0, ntiles, K, int(planar),
                                   out.data_ptr(), out.stride(0), stream(words.device)), "dequant")
    return out


def blob_dequant(blob: torch.Tensor, H: int, I: int, Kg: int, Ku: int, Kd: int, proj: int) -> torch.Tensor:
    shape = (H, I) if proj < 2 else (I, H)
    out = torch.empty(shape, dtype=torch.float16, device=blob.device)
    check(_lib.lib().exl3b_blob_dequant(blob.data_ptr(), H, I, Kg, Ku, Kd, proj, out.data_ptr(), stream(blob.device)),
          "blob_dequant")
    return out


def ensure(ids, w, layer, E, ptrs_all, slot_of, slot_key, slot_last, tick, host_base, slot_base, blob, fill_all,
           fill_list, max_fill, prefetch=False, pf_slot=None, tier=True, vict=None):
    """Device cache step (launch_ensure); tier mask / victims from the process globals when `tier`."""
    S = slot_key.numel()
    rr = G.ram_res if (tier and not prefetch) else None
    check(_lib.lib().exl3b_ensure(ids.data_ptr(), ptr(w), ids.numel(), layer, E, S, ptrs_all.data_ptr(),
                                  slot_of.data_ptr(), ptr(slot_key), ptr(slot_last), tick.data_ptr(),
                                  host_base.data_ptr(), slot_base, blob, G.host_stride or blob, ptr(fill_all),
                                  fill_list.data_ptr(), max_fill, int(prefetch), ptr(pf_slot), ptr(rr),
                                  ptr(G.ring if rr is not None else None),
                                  (G.ring.numel() - 1) if rr is not None else 0,
                                  ptr(G.safe if rr is not None else None), ptr(vict), stream(ids.device)), "ensure")


# ------------------------------------------------------------------------------------------------ reference ops
def _moe_forward_impl(x, topk_ids, topk_w, ptrs, I, K, n_experts):
    """moe_forward (exl3_moe.a8.sycl:1263-1314): M >= prefill_min_m takes the prefill GEMMs, else the decode kernels."""
    if x.shape[0] == 0:
        return torch.empty_like(x)
    if x.shape[0] >= G.prefill_min_m and x.shape[1] % 256 == 0:
        return moe_prefill(x, topk_ids, topk_w, ptrs, I, K, n_experts)
    return moe_decode(x, topk_ids, topk_w, ptrs, I, K, n_experts)


def _moe_forward_mixed_impl(x, topk_ids, topk_w, ptrs, kinfo, I, n_experts):
    """Per-expert K (kinfo: Kg | Ku << 4 | Kd << 8); same decode / prefill split as moe_forward."""
    if x.shape[0] >= G.prefill_min_m and x.shape[1] % 256 == 0:
        return moe_prefill(x, topk_ids, topk_w, ptrs, I, 0, n_experts, kinfo=kinfo)
    return moe_decode(x, topk_ids, topk_w, ptrs, I, 0, n_experts, kinfo=kinfo)


def shared_gate(x: torch.Tensor, gate_w: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, shared_id: int):
    """Config-5 shared-expert gate: returns the extended routing (ids [T, topk + 1], w [T, topk + 1]) with the shared
    expert (id shared_id, weight sigmoid(x . gate_w)) after the routed picks."""
    if x.dtype != torch.bfloat16 or gate_w.dtype != torch.bfloat16 or x.stride(1) != 1 or not gate_w.is_contiguous():
        raise RuntimeError("exl3b200 shared_gate: bf16 x with unit-stride rows and contiguous bf16 gate_w")
    _check_route(ids, w)
    T, H = x.shape
    topk = ids.shape[1]
    ids_out = torch.empty((T, topk + 1), dtype=torch.int32, device=x.device)
    w_out = torch.empty((T, topk + 1), dtype=torch.float32, device=x.device)
    check(_lib.lib().exl3b_shared_gate(x.data_ptr(), x.stride(0), gate_w.data_ptr(), T, H, ids.data_ptr(), w.data_ptr(),
                                       topk, int(shared_id), ids_out.data_ptr(), w_out.data_ptr(), stream(x.device)),
          "shared_gate")
    return ids_out, w_out


def _moe_forward_shared_impl(x, topk_ids, topk_w, ptrs, kinfo, gate_w, I, n_experts):
    """Routed experts plus the always-on shared expert (config 5): ptrs / kinfo hold n_experts + 1 entries, the shared
    expert last; it runs as one more pick per token with weight sigmoid(x . gate_w), combined after the routed picks."""
    if ptrs.numel() != n_experts + 1 or kinfo.numel() != n_experts + 1:
        raise RuntimeError("exl3b200 moe_forward_shared: ptrs and kinfo need n_experts + 1 entries (shared last)")
    ids_x, w_x = shared_gate(x, gate_w, topk_ids, topk_w, n_experts)
    return _moe_forward_mixed_impl(x, ids_x, w_x, ptrs, kinfo, I, n_experts + 1)


def _moe_forward_cached_impl(x, topk_ids, topk_w, ptrs_all, layer, slot_of, slot_key, slot_last, tick, host_base,
                             slot_base, fill_all, fill_list, max_fill, I, K, n_experts, pend, done_seq, out=None):
    if ptrs_all.dtype != torch.int64 or fill_all.dtype != torch.int64 or slot_of.dtype != torch.int32:
        raise RuntimeError("exl3b200 moe_forward_cached: int64 ptrs_all / fill_all, int32 slot_of")
    E = n_experts
    M = x.shape[0]
    ptrs_l = ptrs_all.narrow(0, layer * E, E)
    if pend.numel() and done_seq.numel():   # copy-engine prefetch on: commit the plans that have landed first
        cepf_commit(pend, done_seq, E, ptrs_all, slot_last, slot_base, blob_bytes(x.shape[1], I, K))
    if M == 0 or M >= G.prefill_min_m or slot_key.numel() == 0:
        y = _moe_forward_impl(x, topk_ids, topk_w, ptrs_l, I, K, E)
        if out is not None:
            out.copy_(y)
            return out
        return y
    _check_route(topk_ids, topk_w)
    _check_x(x)
    H = x.shape[1]
    blob = blob_bytes(H, I, K)
    topk = topk_ids.shape[1] if topk_ids.dim() == 2 else 1
    S = slot_key.numel()
    if out is None:
        out = torch.empty_like(x)
    L = _lib.lib()
    wsb = int(L.exl3b_moe_decode_workspace(M, topk, H, I))
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    rr = G.ram_res
    vict = G.vict
    if vict is not None and G.vring is not None and G.vring[1].numel() < min(max_fill, E):
        raise RuntimeError("exl3b200 moe_forward_cached: the victim ring's sel needs one entry per possible victim")
    check(L.exl3b_moe_decode_cached(
        x.data_ptr(), x.stride(0), int(x.dtype == torch.bfloat16), topk_ids.data_ptr(), topk_w.data_ptr(), M, topk, layer,
        ptrs_all.data_ptr(), slot_of.data_ptr(), slot_key.data_ptr(), slot_last.data_ptr(), tick.data_ptr(),
        host_base.data_ptr(), slot_base, blob, G.host_stride or blob, fill_all.data_ptr(), fill_list.data_ptr(),
        min(max_fill, E), S, ptr(rr), ptr(G.ring if rr is not None else None),
        (G.ring.numel() - 1) if rr is not None else 0, ptr(G.safe if rr is not None else None), ptr(vict), ptr(rr),
        H, I, K, E, out.data_ptr(), out.stride(0), _OUT_CODE[out.dtype], ws.data_ptr(), wsb,
        1 if G.skip_zero else 0, stream(x.device)), "moe_forward_cached")
    return out


def _moe_forward_cached_routed_impl(x, wr, bias, topk, ptrs_all, layer, slot_of, slot_key, slot_last, tick, host_base,
                                    slot_base, fill_all, fill_list, max_fill, I, K, n_experts, pend, done_seq, out=None):
    """router_topk(x, wr, bias, topk) followed by the cached decode on its picks, as one call: returns (out, ids, w),
    the same values the two calls give.  Small batches select the picks inside the decode kernels."""
    if x.dtype != torch.bfloat16 or wr.dtype != torch.bfloat16:
        raise RuntimeError("exl3b200 moe_forward_cached_routed: x and Wr must be bf16")
    if x.dim() != 2 or x.stride(1) != 1 or not wr.is_contiguous():
        raise RuntimeError("exl3b200 moe_forward_cached_routed: x 2-D unit-stride rows, Wr contiguous")
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        raise RuntimeError("exl3b200 moe_forward_cached_routed: bias must be contiguous fp32")
    E = n_experts
    M, H = x.shape
    if wr.shape[0] != E:
        raise RuntimeError("exl3b200 moe_forward_cached_routed: Wr must have n_experts rows")
    if M == 0 or M >= G.prefill_min_m or slot_key.numel() == 0 or (pend.numel() and done_seq.numel()):
        ids, w = router_topk(x, wr, bias, topk)
        y = _moe_forward_cached_impl(x, ids, w, ptrs_all, layer, slot_of, slot_key, slot_last, tick, host_base,
                                     slot_base, fill_all, fill_list, max_fill, I, K, E, pend, done_seq, out=out)
        return y, ids, w
    if ptrs_all.dtype != torch.int64 or fill_all.dtype != torch.int64 or slot_of.dtype != torch.int32:
        raise RuntimeError("exl3b200 moe_forward_cached_routed: int64 ptrs_all / fill_all, int32 slot_of")
    blob = blob_bytes(H, I, K)
    S = slot_key.numel()
    if out is None:
        out = torch.empty_like(x)
    ids = torch.empty((M, topk), dtype=torch.int32, device=x.device)
    w = torch.empty((M, topk), dtype=torch.float32, device=x.device)
    logits = torch.empty((M, E), dtype=torch.float32, device=x.device)
    L = _lib.lib()
    wsb = int(L.exl3b_moe_decode_workspace(M, topk, H, I))
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    rr = G.ram_res
    vict = G.vict
    if vict is not None and G.vring is not None and G.vring[1].numel() < min(max_fill, E):
        raise RuntimeError("exl3b200 moe_forward_cached: the victim ring's sel needs one entry per possible victim")
    check(L.exl3b_moe_decode_cached_routed(
        x.data_ptr(), x.stride(0), wr.data_ptr(), ptr(bias), logits.data_ptr(), ids.data_ptr(), w.data_ptr(), M, topk,
        layer, ptrs_all.data_ptr(), slot_of.data_ptr(), slot_key.data_ptr(), slot_last.data_ptr(), tick.data_ptr(),
        host_base.data_ptr(), slot_base, blob, G.host_stride or blob, fill_all.data_ptr(), fill_list.data_ptr(),
        min(max_fill, E), S, ptr(rr), ptr(G.ring if rr is not None else None),
        (G.ring.numel() - 1) if rr is not None else 0, ptr(G.safe if rr is not None else None), ptr(vict), ptr(rr),
        H, I, K, E, out.data_ptr(), out.stride(0), _OUT_CODE[out.dtype], ws.data_ptr(), wsb,
        1 if G.skip_zero else 0, _router_counter(x.device), stream(x.device)), "moe_forward_cached_routed")
    return out, ids, w


def tier_prefetch_ids(ids, layer, n_experts, slot_of, ram_res, safe):
    """With the RAM tier on, a predicted expert that is in neither VRAM nor RAM has no valid host row to copy from (its
    row may have been released): it is replaced by the layer's safe expert, which is always resident.  Device ops
    only, no host sync.  The reference's prefetch mode copies without this test.  Out-of-range ids pass through for the
    cache step to reject."""
    if ram_res is None:
        return ids
    lookup = ids.long().clamp(0, n_experts - 1) + layer * n_experts
    ok = (ram_res[lookup] != 0) | (slot_of[lookup] >= 0) | (ids < 0) | (ids >= n_experts)
    return torch.where(ok, ids, safe[layer].to(ids.dtype)).contiguous()


def _moe_prefetch_impl(ids, ptrs_all, layer, slot_of, slot_key, slot_last, tick, host_base, slot_base, pf_list,
                       pf_slot, max_fill, n_experts, blob):
    """Claim LRU slots for predicted experts (tick not advanced), copy them from host, repoint the table
    (moe_prefetch, exl3_moe.a8.sycl:1194-1219)."""
    if ids.dtype != torch.int32 or not ids.is_contiguous():
        raise RuntimeError("exl3b200 moe_prefetch: contiguous int32 ids")
    E, S = n_experts, slot_key.numel()
    if S == 0 or ids.numel() == 0:
        return
    mf = min(max_fill, pf_slot.numel())
    ids = tier_prefetch_ids(ids, layer, E, slot_of, G.ram_res, G.safe)
    ensure(ids, None, layer, E, ptrs_all, slot_of, slot_key, slot_last, tick, host_base, slot_base, blob, None,
           pf_list, mf, prefetch=True, pf_slot=pf_slot, tier=False)
    L = _lib.lib()
    s = stream(ids.device)
    ptrs_l = ptrs_all.narrow(0, layer * E, E)
    nmax = min(mf, ids.numel())
    if nmax > 0:
        check(L.exl3b_fill_copy(pf_list.data_ptr(), ptrs_l.data_ptr(), None, pf_slot.data_ptr(), slot_base, blob, nmax,
                                s), "prefetch copy")
    check(L.exl3b_commit(pf_list.data_ptr(), ptrs_l.data_ptr(), None, pf_slot.data_ptr(), slot_base, blob, s),
          "prefetch commit")


# ------------------------------------------------------------------------------------------------ copy-engine prefetch
_PEND_STRIDE = 35     # int32 per layer in pend: n, seq, T, (expert, slot) x 16
_PLAN_MAX = 16


def cepf_commit(pend, done_seq, n_experts, ptrs_all, slot_last, slot_base, blob) -> None:
    """Commit every landed copy-engine plan (exl3b_cepf_commit) on the current stream."""
    check(_lib.lib().exl3b_cepf_commit(pend.data_ptr(), done_seq.data_ptr(), done_seq.numel(), n_experts,
                                       slot_last.numel(), ptrs_all.data_ptr(), slot_last.data_ptr(), slot_base, blob,
                                       stream(ptrs_all.device)), "copy prefetch commit")


def _moe_prefetch_plan_impl(ids, ptrs_all, layer, slot_of, slot_key, slot_last, tick, host_base, slot_base, pf_list,
                            pf_slot, plans, plan_seq, pend, done_seq, max_fill, n_experts, blob):
    """moe_prefetch_plan (exl3_moe.a8.sycl:1127-1142): claim and pin LRU slots for the predicted experts of `layer`
    and publish the plan to the pinned host buffer `plans` for the copy worker (exl3b_cepf_plan)."""
    if ids.dtype != torch.int32 or not ids.is_contiguous():
        raise RuntimeError("exl3b200 moe_prefetch_plan: contiguous int32 ids")
    E, S, n_layers = n_experts, slot_key.numel(), done_seq.numel()
    if S == 0 or ids.numel() == 0:
        return
    if plans.device.type != "cpu" or not plans.is_pinned() or plans.numel() * plans.element_size() < \
            n_layers * (4 + 2 * E) * 4:
        raise RuntimeError("exl3b200 moe_prefetch_plan: plans must be pinned host memory of n_layers x (4 + 2E) int32")
    if pend.numel() < n_layers * _PEND_STRIDE or plan_seq.numel() < n_layers:
        raise RuntimeError("exl3b200 moe_prefetch_plan: pend needs 35 int32 and plan_seq one per layer")
    mf = min(max_fill, _PLAN_MAX, pf_slot.numel())
    ids = tier_prefetch_ids(ids, layer, E, slot_of, G.ram_res, G.safe)
    check(_lib.lib().exl3b_cepf_plan(ids.data_ptr(), ids.numel(), layer, E, S, ptrs_all.data_ptr(), slot_of.data_ptr(),
                                     slot_key.data_ptr(), slot_last.data_ptr(), tick.data_ptr(), host_base.data_ptr(),
                                     slot_base, blob, G.host_stride or blob, pf_list.data_ptr(), pf_slot.data_ptr(), mf,
                                     plans.data_ptr(), plan_seq.data_ptr(), pend.data_ptr(), done_seq.data_ptr(),
                                     n_layers, stream(ids.device)), "moe_prefetch_plan")


_worker_atexit = False
_worker_keep = None   # what the running worker reads or writes through raw addresses, alive until it stops


def moe_prefetch_worker_start(plans, host_base_cpu, slot_base, blob, ptrs_all, slot_last, commit_host, done_seq,
                              n_layers, n_experts, keep=None) -> None:
    """moe_prefetch_worker_start (exl3_moe.a8.sycl:1092-1115): start the host thread that turns published plans into
    copy-engine copies on the CURRENT stream (call it inside `with torch.cuda.stream(copy_stream)`).  commit_host is
    accepted for the reference's signature; this worker needs no host commit buffer.  The worker uses the plan
    buffer, done_seq and the slot arena by address, so they are kept alive here until the stop, together with `keep`
    (this build's extension: the owner of the slot arena and host arenas, e.g. the ExpertStore)."""
    global _worker_atexit, _worker_keep
    hb = host_base_cpu.to(torch.int64).contiguous()
    if hb.numel() < n_layers:
        raise RuntimeError("exl3b200 moe_prefetch_worker_start: host_base_cpu needs one address per layer")
    dev = done_seq.device
    check(_lib.lib().exl3b_cepf_worker_start(plans.data_ptr(), n_layers, n_experts, slot_last.numel(), hb.data_ptr(),
                                             slot_base, blob, G.host_stride or blob, done_seq.data_ptr(), dev.index,
                                             stream(dev)), "moe_prefetch_worker_start")
    _worker_keep = (plans, done_seq, ptrs_all, slot_last, keep)
    if not _worker_atexit:   # a worker still running at interpreter exit would read freed host memory
        import atexit
        atexit.register(lambda: _lib.lib().exl3b_cepf_worker_stop(None))
        _worker_atexit = True


def moe_prefetch_worker_stop() -> list:
    """moe_prefetch_worker_stop (:1117-1124): handle the plans already published, wait for the copies, stop; returns
    [plans handled, experts copied]."""
    global _worker_keep
    import ctypes
    counts = (ctypes.c_int64 * 2)()
    try:
        check(_lib.lib().exl3b_cepf_worker_stop(counts), "moe_prefetch_worker_stop")
    finally:
        _worker_keep = None   # the worker has exited (stop joins it, also when it reports an error)
    return [int(counts[0]), int(counts[1])]


def align(topk_ids: torch.Tensor, topk_w: torch.Tensor, n_experts: int, pad: int):
    """Routing tables (launch_align, exl3_moe.a8.sycl:639-680): returns (ib int32, fb fp32) laid out as make_route
    (:744-757): ib = [act_expert A | act_start A | act_cnt A | act_pstart A | n_act 1 | pair_tok P | pair_of P |
    pad 16 | blk_a mxb | n_blk 1], fb = pair_w [P], with A = min(P, E), mxb = ceil(P/pad) + A."""
    _check_route(topk_ids, topk_w)
    P = topk_ids.numel()
    topk = topk_ids.shape[-1] if topk_ids.dim() else 1
    E = n_experts
    A = min(P, E)
    mxb = (P + pad - 1) // pad + A
    dev = topk_ids.device
    ib = torch.empty(4 * A + 1 + 2 * P + 16 + mxb + 1, dtype=torch.int32, device=dev)
    fb = torch.empty(max(P, 1), dtype=torch.float32, device=dev)
    L = _lib.lib()
    scratch = torch.empty(max(int(L.exl3b_align_scratch(P, E)), 256), dtype=torch.uint8, device=dev)
    check(L.exl3b_align(topk_ids.data_ptr(), topk_w.data_ptr(), P, topk, E, pad, ib.data_ptr(), fb.data_ptr(), A, mxb,
                        scratch.data_ptr(), scratch.numel(), stream(dev)), "align")
    return ib, fb


def _moe_align_impl(topk_ids, topk_w, n_experts, pad):
    """Debug op moe_align (exl3_moe.a8.sycl:1317-1325) -> [int32 buf, fp32 buf]."""
    ib, fb = align(topk_ids, topk_w, n_experts, pad)
    return [ib, fb]


def host_alloc(nbytes: int) -> torch.Tensor:
    """Pinned host memory readable by the GPU at the same address (host_alloc, exl3_moe.a8.sycl:1529-1536)."""
    return torch.empty(int(nbytes), dtype=torch.uint8, pin_memory=True)


def usm_kind(p: int) -> int:
    """0 unknown/pageable, 1 pinned host, 2 device, 3 managed (usm_kind, exl3_moe.a8.sycl:1539-1543)."""
    return _usm_kind_cudart(p)


_cudart_handle = None


def _cudart():
    """The CUDA runtime torch already loaded (same soname), with the two entry points used here typed once."""
    global _cudart_handle
    if _cudart_handle is None:
        import ctypes
        try:
            rt = ctypes.CDLL("libcudart.so.12")
        except OSError:
            rt = ctypes.CDLL("libcudart.so")
        rt.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                       ctypes.c_void_p]
        rt.cudaMemcpyAsync.restype = ctypes.c_int
        rt.cudaPointerGetAttributes.restype = ctypes.c_int
        _cudart_handle = rt
    return _cudart_handle


def _usm_kind_cudart(p: int) -> int:
    import ctypes

    class Attr(ctypes.Structure):
        _fields_ = [("type", ctypes.c_int), ("device", ctypes.c_int), ("devicePointer", ctypes.c_void_p),
                    ("hostPointer", ctypes.c_void_p)]

    rt = _cudart()
    a = Attr()
    if rt.cudaPointerGetAttributes(ctypes.byref(a), ctypes.c_void_p(p)) != 0:
        rt.cudaGetLastError()
        return 0
    return {0: 0, 1: 1, 2: 2, 3: 3}.get(a.type, 0)


def memcpy_async(dst: int, src: int, nbytes: int) -> None:
    """Async raw copy on the current stream (memcpy_async, exl3_moe.a8.sycl:1546-1549); cudaMemcpyDefault, so any
    pair of host (pinned) and device addresses."""
    rc = _cudart().cudaMemcpyAsync(dst, src, nbytes, 4, torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"exl3b200 memcpy_async: cudaMemcpyAsync failed ({rc})")


# setters (process globals)
def moe_set_splits(gu_p: int, dn_p: int) -> None: G.gu_p, G.dn_p = int(gu_p), int(dn_p)
def moe_set_mr(mr: int) -> None: G.mr = int(mr)
def moe_set_debug(v: int) -> None: G.debug = int(v)
def moe_set_pair_max_m(v: int) -> None: G.pair_max_m = int(v)
def moe_set_prefill_min_m(v: int) -> None: G.prefill_min_m = int(v)
def moe_set_host_stride(s: int) -> None: G.host_stride = int(s)


def moe_set_victims(v: torch.Tensor) -> None:
    G.vict = v if v.numel() else None


def moe_set_victim_ring(meta: torch.Tensor, sel: torch.Tensor, buf: torch.Tensor) -> None:
    """moe_set_victim_ring (experimental/n111-victim-ring/a9.patch): victims that need a write-back go device to
    device into a ring of K = (meta.numel() - 4) / 2 slots of buf instead of to their host rows, and ram_res is not
    set; the host loop (TierHost with vring) drains the ring and flags the keys.  meta int32 [4 + 2K] (meta[3] = K,
    keys -1), sel int32 (one entry per victim of a call), buf uint8 [K, blob] on the device.  Empty meta: ring off."""
    if meta.numel() == 0:
        check(_lib.lib().exl3b_set_victim_ring(None, None, None, 0, 0), "moe_set_victim_ring")
        G.vring = None
        return
    K = (meta.numel() - 4) // 2
    if meta.dtype != torch.int32 or sel.dtype != torch.int32 or meta.numel() != 4 + 2 * K or K < 1 or \
            buf.dtype != torch.uint8 or buf.dim() != 2 or buf.shape[0] != K:
        raise RuntimeError("exl3b200 moe_set_victim_ring: int32 meta [4 + 2K], int32 sel, uint8 buf [K, blob]")
    check(_lib.lib().exl3b_set_victim_ring(meta.data_ptr(), sel.data_ptr(), buf.data_ptr(), buf.numel(), K),
          "moe_set_victim_ring")
    G.vring = (meta, sel, buf)   # kept referenced while the library holds their addresses


def moe_set_tier(ram_res: torch.Tensor, miss: torch.Tensor, safe: torch.Tensor) -> None:
    if ram_res.numel() == 0:
        G.ram_res = G.ring = G.safe = None
        return
    if ram_res.dtype != torch.uint8 or miss.dtype != torch.int32 or safe.dtype != torch.int32:
        raise RuntimeError("exl3b200 moe_set_tier: uint8 ram_res, int32 miss ring, int32 safe")
    if miss.numel() < 2:
        raise RuntimeError("exl3b200 moe_set_tier: the miss ring needs >= 1 entry")
    G.ram_res, G.ring, G.safe = ram_res, miss, safe


def moe_svm_prefetch(ptrs: torch.Tensor, nbytes: int, like: torch.Tensor) -> None:
    """The reference maps RAM-tier pages for the GPU ahead of first touch (SVM); pinned host memory on CUDA is
    always mapped, so there is nothing to do."""
    return None


# ------------------------------------------------------------------------------------------------ registration
_registered = False


def register() -> None:
    """Define the torch ops (torch.ops.exl3b200_moe.*) once."""
    global _registered
    if _registered:
        return
    _lib.lib()   # fail loudly now if the library is missing
    lib = torch.library.Library(NS, "DEF")
    lib.define("moe_forward(Tensor x, Tensor topk_ids, Tensor topk_w, Tensor ptrs, int I, int K, int n_experts) -> Tensor")
    lib.define("moe_forward_cached(Tensor x, Tensor topk_ids, Tensor topk_w, Tensor(a!) ptrs_all, int layer, "
               "Tensor(b!) slot_of, Tensor(c!) slot_key, Tensor(d!) slot_last, Tensor(e!) tick, Tensor host_base, "
               "int slot_base, Tensor(f!) fill_all, Tensor(g!) fill_list, int max_fill, int I, int K, int n_experts, "
               "Tensor(h!) pend, Tensor done_seq) -> Tensor")
    lib.define("moe_prefetch(Tensor ids, Tensor(a!) ptrs_all, int layer, Tensor(b!) slot_of, Tensor(c!) slot_key, "
               "Tensor(d!) slot_last, Tensor tick, Tensor host_base, int slot_base, Tensor(e!) pf_list, "
               "Tensor(f!) pf_slot, int max_fill, int n_experts, int blob) -> ()")
    lib.define("moe_prefetch_plan(Tensor ids, Tensor(a!) ptrs_all, int layer, Tensor(b!) slot_of, Tensor(c!) slot_key, "
               "Tensor(d!) slot_last, Tensor tick, Tensor host_base, int slot_base, Tensor(e!) pf_list, "
               "Tensor(f!) pf_slot, Tensor(g!) plans, Tensor(h!) plan_seq, Tensor(i!) pend, Tensor done_seq, "
               "int max_fill, int n_experts, int blob) -> ()")
    lib.define("moe_align(Tensor topk_ids, Tensor topk_w, int n_experts, int pad) -> Tensor[]")
    lib.define("router_topk(Tensor x, Tensor wr, Tensor? bias, int topk) -> (Tensor, Tensor)")
    lib.define("moe_forward_mixed(Tensor x, Tensor topk_ids, Tensor topk_w, Tensor ptrs, Tensor kinfo, int I, "
               "int n_experts) -> Tensor")
    lib.impl("moe_forward", _moe_forward_impl, "CUDA")
    lib.impl("moe_forward_cached", _moe_forward_cached_impl, "CUDA")
    lib.impl("moe_prefetch", _moe_prefetch_impl, "CUDA")
    lib.impl("moe_prefetch_plan", _moe_prefetch_plan_impl, "CUDA")
    lib.impl("moe_align", _moe_align_impl, "CUDA")
    lib.impl("router_topk", lambda x, wr, bias, topk: router_topk(x, wr, bias, topk), "CUDA")
    lib.impl("moe_forward_mixed", _moe_forward_mixed_impl, "CUDA")
    lib.define("moe_forward_shared(Tensor x, Tensor topk_ids, Tensor topk_w, Tensor ptrs, Tensor kinfo, Tensor gate_w, "
               "int I, int n_experts) -> Tensor")
    lib.impl("moe_forward_shared", _moe_forward_shared_impl, "CUDA")

    torch.library.register_fake(f"{NS}::moe_forward", lambda x, *a: torch.empty_like(x), lib=lib)
    torch.library.register_fake(f"{NS}::moe_forward_cached", lambda x, *a: torch.empty_like(x), lib=lib)
    torch.library.register_fake(f"{NS}::moe_forward_mixed", lambda x, *a: torch.empty_like(x), lib=lib)
    torch.library.register_fake(f"{NS}::moe_forward_shared", lambda x, *a: torch.empty_like(x), lib=lib)
    globals()["_torch_lib"] = lib
    _registered = True


class _Ops:
    """Namespace object mirroring torch.ops.exl3xpu_moe: tensor ops dispatch through torch, the rest are plain."""

    def __getattr__(self, name):
        register()
        if hasattr(torch.ops.exl3b200_moe, name) and name in ("moe_forward", "moe_forward_cached", "moe_prefetch",
                                                               "moe_prefetch_plan", "moe_align", "router_topk",
                                                               "moe_forward_mixed", "moe_forward_shared"):
            return getattr(torch.ops.exl3b200_moe, name)
        fn = {"host_alloc": host_alloc, "usm_kind": usm_kind, "memcpy_async": memcpy_async,
              "blob_bytes": blob_bytes, "moe_set_splits": moe_set_splits, "moe_set_mr": moe_set_mr,
              "moe_set_debug": moe_set_debug, "moe_set_pair_max_m": moe_set_pair_max_m,
              "moe_set_prefill_min_m": moe_set_prefill_min_m, "moe_set_victims": moe_set_victims,
              "moe_set_tier": moe_set_tier, "moe_set_host_stride": moe_set_host_stride,
              "moe_set_victim_ring": moe_set_victim_ring,
              "moe_svm_prefetch": moe_svm_prefetch, "moe_prefetch_worker_start": moe_prefetch_worker_start,
              "moe_prefetch_worker_stop": moe_prefetch_worker_stop}.get(name)
        if fn is None:
            raise AttributeError(name)
        return fn


OPS = _Ops()
