"""Expert-parallel prefill over the GPUs of one node.

The reference runs its MoE prefill (kernels/moe-a8/exl3_moe.a8.sycl:792-828) on one GPU; this spreads it over G ranks
of a torch.distributed group (NCCL on B200s):

* experts are sharded contiguously: rank d owns ids [d E/G, (d+1) E/G) and holds only their blobs;
* every rank routes its own tokens; a token is sent once to every rank owning at least one of its picks, with the
  picks as that rank's local ids (-1 for picks owned elsewhere) and their weights (all-to-all of counts, rows, ids,
  weights);
* each rank runs the grouped prefill GEMMs (or the decode kernels for few rows) on what it received, returning fp32
  partial sums per received row (all-to-all back);
* the source sums a token's partials over the ranks in ascending rank order (exl3b_ep_combine).

Every rank takes the same collective steps in the same order.  The device steps go through the C ABI
(exl3b_ep_plan / _pack / _combine and the MoE entry points); `kernels` may replace them (the CPU tests use a host
implementation of the same contract to check the exchange protocol on gloo ranks).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, stream


class CudaEPKernels:
    """Device side of the exchange through libexl3b200."""

    def plan(self, ids: torch.Tensor, w: torch.Tensor, n_experts: int, G: int) -> dict:
        T, topk = ids.shape
        dev = ids.device
        n = max(T * G, 1)
        out = {
            "bits": torch.empty(max(T, 1), dtype=torch.int32, device=dev),
            "counts": torch.empty(G, dtype=torch.int64, device=dev),
            "offs": torch.empty(G + 1, dtype=torch.int64, device=dev),
            "pos": torch.empty((max(T, 1), G), dtype=torch.int32, device=dev),
            "send_src": torch.empty(n, dtype=torch.int32, device=dev),
            "send_ids": torch.empty((n, topk), dtype=torch.int32, device=dev),
            "send_w": torch.empty((n, topk), dtype=torch.float32, device=dev),
        }
        check(_lib.lib().exl3b_ep_plan(ids.data_ptr(), w.data_ptr(), T, topk, n_experts, G, out["bits"].data_ptr(),
                                       out["counts"].data_ptr(), out["offs"].data_ptr(), out["pos"].data_ptr(),
                                       out["send_src"].data_ptr(), out["send_ids"].data_ptr(), out["send_w"].data_ptr(),
                                       stream(dev)), "ep_plan")
        return out

    def pack(self, x: torch.Tensor, send_src: torch.Tensor, n_rows: int) -> torch.Tensor:
        send_x = torch.empty((n_rows, x.shape[1]), dtype=x.dtype, device=x.device)
        check(_lib.lib().exl3b_ep_pack(x.data_ptr(), x.stride(0), x.shape[1], send_src.data_ptr(), n_rows,
                                       send_x.data_ptr(), stream(x.device)), "ep_pack")
        return send_x

    def combine(self, part: torch.Tensor, pos: torch.Tensor, T: int, G: int, H: int, dtype: torch.dtype) -> torch.Tensor:
        out = torch.empty((T, H), dtype=dtype, device=pos.device)
        code = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}[dtype]
        check(_lib.lib().exl3b_ep_combine(part.data_ptr() if part.numel() else None, pos.data_ptr(), T, G, H,
                                          out.data_ptr(), out.stride(0), code, stream(pos.device)), "ep_combine")
        return out

    def local(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, ptrs: torch.Tensor, kinfo, I: int, K: int,
              n_local: int) -> torch.Tensor:
        from . import ops
        out = torch.empty((x.shape[0], x.shape[1]), dtype=torch.float32, device=x.device)
        if x.shape[0] == 0:
            return out
        if x.shape[0] >= ops.G.prefill_min_m and x.shape[1] % 256 == 0:
            return ops.moe_prefill(x, ids, w, ptrs, I, K, n_local, kinfo=kinfo, out=out)
        return ops.moe_decode(x, ids, w, ptrs, I, K, n_local, kinfo=kinfo, out=out)


class EPPrefill:
    """One MoE layer's expert-parallel prefill on this rank: ptrs_local holds the int64 blob addresses of the rank's
    n_experts / G experts (kinfo_local their packed K when mixed)."""

    def __init__(self, group, n_experts: int, H: int, I: int, K: int, ptrs_local: torch.Tensor,
                 kinfo_local: torch.Tensor | None = None, kernels=None):
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.G:
            raise RuntimeError("exl3b200 EPPrefill: the number of experts must divide evenly over the ranks")
        self.E, self.H, self.I, self.K = n_experts, H, I, K
        self.n_local = n_experts // self.G
        if ptrs_local.numel() != self.n_local:
            raise RuntimeError("exl3b200 EPPrefill: ptrs_local must hold this rank's n_experts / G blob addresses")
        self.ptrs_local, self.kinfo_local = ptrs_local, kinfo_local
        self.k = kernels or CudaEPKernels()
        self.last = {}

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits):
        # A peer that stopped (exited, or stuck past the group's timeout) fails the collective; the error names the
        # layer step so that the caller can tell a lost rank from a bad argument.
        try:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        except RuntimeError as e:   # torch's distributed backend errors derive from RuntimeError
            raise RuntimeError(f"exl3b200 EPPrefill: all-to-all failed on rank {self.rank} of {self.G} "
                               f"(a peer rank stopped or timed out): {e}") from e

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        G, H = self.G, self.H
        T, topk = ids.shape
        p = self.k.plan(ids, w, self.E, G)
        send_counts = p["counts"]
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        both = torch.stack([send_counts, recv_counts]).cpu()
        sc, rc = [int(v) for v in both[0]], [int(v) for v in both[1]]
        n_send, n_recv = sum(sc), sum(rc)
        send_x = self.k.pack(x, p["send_src"], n_send)
        recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=x.device)
        self._a2a(recv_x, send_x, rc, sc)
        recv_ids = torch.empty((n_recv, topk), dtype=torch.int32, device=x.device)
        self._a2a(recv_ids, p["send_ids"][:n_send].contiguous(), rc, sc)
        recv_w = torch.empty((n_recv, topk), dtype=torch.float32, device=x.device)
        self._a2a(recv_w, p["send_w"][:n_send].contiguous(), rc, sc)
        part_recv = self.k.local(recv_x, recv_ids, recv_w, self.ptrs_local, self.kinfo_local, self.I, self.K,
                                 self.n_local)
        part_send = torch.empty((n_send, H), dtype=torch.float32, device=x.device)
        self._a2a(part_send, part_recv, sc, rc)
        self.last = {"send_rows": n_send, "recv_rows": n_recv, "send_counts": sc, "recv_counts": rc}
        return self.k.combine(part_send, p["pos"], T, G, H, x.dtype)
