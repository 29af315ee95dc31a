"""Expert-parallel prefill over the GPUs of one node.

The reference runs its MoE prefill (kernels/moe-a8/exl3_moe.a8.sycl:792-828) on one GPU; this spreads it over G ranks
of a torch.distributed group (NCCL on B200s):

* experts are sharded contiguously: rank d owns ids [d E/G, (d+1) E/G) and holds only their blobs;
* every rank routes its own tokens and sends each token once to every rank owning at least one of its picks: one
  record per (token, destination) holding the token's row of x, its picks as the destination's local expert ids (-1 for
  picks owned elsewhere) and their weights (exl3b_ep_dispatch);
* the records go in fixed-capacity blocks of `cap` rows per destination (cap >= every rank's token count, the same on
  all ranks), unused rows marked "no pick", so one all-to-all with equal splits moves them and no rank has to read the
  counts on the host: a layer queues without a host synchronisation;
* each rank runs the grouped prefill GEMMs (or the decode kernels for few rows) over all G cap received rows (unused
  rows have no picks and cost nothing) and returns fp16 partial sums per row with a second all-to-all;
* the source sums a token's partials over the ranks in ascending rank order (exl3b_ep_combine_h), in fp32;
* with chunks > 1 the batch is split into that many token ranges, and chunk k + 1's outgoing all-to-all and chunk
  k - 1's returning one run on NCCL's stream while chunk k's experts run on the compute stream.

Every rank takes the same collective steps in the same order.  The device steps go through the C ABI; `kernels` may
replace them (the CPU tests use a host implementation of the same contract to run the exchange on gloo ranks).
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
              n_local: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        from . import ops
        out = torch.empty((x.shape[0], x.shape[1]), dtype=dtype, device=x.device)
        if x.shape[0] == 0:
            return out
        if x.shape[0] >= ops.G.prefill_min_m and x.shape[1] % 256 == 0:
            return ops.moe_prefill(x, ids, w, ptrs, I, K, n_local, kinfo=kinfo, out=out)
        return ops.moe_decode(x, ids, w, ptrs, I, K, n_local, kinfo=kinfo, out=out)

    # ---- the exchange EPPrefill runs
    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, n_experts: int, G: int, cap: int) -> dict:
        """Send records [G cap, record bytes] (uint8), pos [T, G] and counts [G] (int64, on the device)."""
        T, topk = ids.shape
        H = x.shape[1]
        dev = x.device
        rec = int(_lib.lib().exl3b_ep_record_bytes(H, topk))
        send = torch.empty((G * cap, rec), dtype=torch.uint8, device=dev)
        counts = torch.empty(2 * G + 1, dtype=torch.int64, device=dev)
        pos = torch.empty((max(T, 1), G), dtype=torch.int32, device=dev)
        bits = torch.empty(max(T, 1), dtype=torch.int32, device=dev)
        src = torch.empty(G * cap, dtype=torch.int32, device=dev)
        check(_lib.lib().exl3b_ep_dispatch(x.data_ptr() if T else None, x.stride(0) if T else H,
                                           ids.data_ptr() if T else None, w.data_ptr() if T else None, T, topk,
                                           n_experts, G, H, cap, bits.data_ptr(), counts.data_ptr(), pos.data_ptr(),
                                           src.data_ptr(), send.data_ptr(), stream(dev)), "ep_dispatch")
        return {"send": send, "pos": pos, "counts": counts[:G]}

    def combine_h(self, part: torch.Tensor, pos: torch.Tensor, T: int, G: int, H: int, dtype: torch.dtype,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = torch.empty((T, H), dtype=dtype, device=pos.device)
        code = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}[dtype]
        check(_lib.lib().exl3b_ep_combine_h(part.data_ptr() if part.numel() else None, pos.data_ptr(), T, G, H,
                                            out.data_ptr(), out.stride(0), code, stream(pos.device)), "ep_combine_h")
        return out


def unpack_records(recv: torch.Tensor, H: int, topk: int, dtype: torch.dtype):
    """Received records -> (x rows as a strided view [rows, H] of `dtype`, contiguous int32 ids and fp32 weights
    [rows, topk])."""
    x = recv[:, :2 * H].view(dtype)
    ids = recv[:, 2 * H:2 * H + 4 * topk].view(torch.int32).contiguous()
    w = recv[:, 2 * H + 4 * topk:2 * H + 8 * topk].view(torch.float32).contiguous()
    return x, ids, w


class EPPrefill:
    """One MoE layer's expert-parallel prefill on this rank: ptrs_local holds the int64 blob addresses of the rank's
    n_experts / G experts (kinfo_local their packed K when mixed).  max_tokens: the token count no rank exceeds in a
    call, the same on every rank (the record blocks' capacity); without it each call first agrees on the largest token
    count with one small all-reduce, which reads the result on the host.  profile=True records CUDA events around the
    phases of each call (read with phase_ms())."""

    def __init__(self, group, n_experts: int, H: int, I: int, K: int, ptrs_local: torch.Tensor,
                 kinfo_local: torch.Tensor | None = None, kernels=None, max_tokens: int | None = None,
                 profile: bool = False, chunks: int = 1):
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
        self.max_tokens = max_tokens
        self.profile = profile
        if chunks < 1:
            raise RuntimeError("exl3b200 EPPrefill: chunks must be >= 1")
        self.chunks = chunks
        self.last = {}
        self._ev = []

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, async_op: bool = False):
        # A peer that stopped (exited, or stuck past the group's timeout) fails the collective; the error names the
        # layer step so that the caller can tell a lost rank from a bad argument.
        try:
            return dist.all_to_all_single(out, inp, group=self.group, async_op=async_op)
        except RuntimeError as e:   # torch's distributed backend errors derive from RuntimeError
            raise RuntimeError(f"exl3b200 EPPrefill: all-to-all failed on rank {self.rank} of {self.G} "
                               f"(a peer rank stopped or timed out): {e}") from e

    def _wait(self, work):
        try:
            work.wait()
        except RuntimeError as e:
            raise RuntimeError(f"exl3b200 EPPrefill: all-to-all failed on rank {self.rank} of {self.G} "
                               f"(a peer rank stopped or timed out): {e}") from e

    def _cap(self, T: int, device) -> int:
        if self.max_tokens is not None:
            if T > self.max_tokens:
                raise RuntimeError(f"exl3b200 EPPrefill: {T} tokens > max_tokens {self.max_tokens}")
            return max(1, int(self.max_tokens))
        t = torch.tensor([T], dtype=torch.int64, device=device)
        try:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        except RuntimeError as e:
            raise RuntimeError(f"exl3b200 EPPrefill: token-count all-reduce failed on rank {self.rank} of {self.G} "
                               f"(a peer rank stopped or timed out): {e}") from e
        return max(1, int(t.item()))

    def _mark(self, dev):
        if self.profile and dev.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._ev.append(ev)

    def phase_ms(self) -> dict:
        """Device time of the last profiled call's phases (synchronises): dispatch, all-to-all out, local MoE,
        all-to-all back, combine."""
        if len(self._ev) != 6:
            return {}
        self._ev[-1].synchronize()
        names = ["dispatch", "a2a_out", "local_moe", "a2a_back", "combine"]
        return {n: self._ev[i].elapsed_time(self._ev[i + 1]) for i, n in enumerate(names)}

    def stats(self) -> dict:
        """Rows and picks of the last call (reads the device): rows sent to / received from each rank, this rank's
        received picks (its expert load)."""
        sc = [int(v) for v in self.last["send_counts"].cpu()]
        idr, cap = self.last["recv_ids"], self.last["cap"]
        valid = (idr >= 0).any(dim=1).view(-1, self.G, cap)   # [chunk][source rank][record]
        rc = [int(v) for v in valid.sum(dim=(0, 2)).cpu()]
        return {"cap": cap, "send_counts": sc, "recv_counts": rc, "send_rows": sum(sc), "recv_rows": sum(rc),
                "recv_picks": int((idr >= 0).sum().item())}

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        if self.chunks > 1:
            return self._forward_chunked(x, ids, w)
        G, H = self.G, self.H
        T, topk = ids.shape
        dev = x.device
        cap = self._cap(T, dev)
        self._ev = []
        self._mark(dev)
        p = self.k.dispatch(x, ids, w, self.E, G, cap)
        self._mark(dev)
        recv = torch.empty_like(p["send"])
        self._a2a(recv, p["send"])
        self._mark(dev)
        xr, idr, wr = unpack_records(recv, H, topk, x.dtype)
        part = self.k.local(xr, idr, wr, self.ptrs_local, self.kinfo_local, self.I, self.K, self.n_local,
                            dtype=torch.float16)
        self._mark(dev)
        back = torch.empty_like(part)
        self._a2a(back, part)
        self._mark(dev)
        out = self.k.combine_h(back, p["pos"], T, G, H, x.dtype)
        self._mark(dev)
        self.last = {"cap": cap, "send_counts": p["counts"], "recv_ids": idr}
        return out

    def _forward_chunked(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """The same exchange over `chunks` token ranges (each with capacity ceil(cap / chunks)), software-pipelined:
        the outgoing all-to-all of every chunk is queued on NCCL's stream ahead of the experts, so chunk k + 1's
        records move while chunk k's experts run, and chunk k's partial sums return while chunk k + 1's run.  The
        result equals the unchunked forward's (each token's partial sums and their order do not depend on the
        split)."""
        G, H, n = self.G, self.H, self.chunks
        T, topk = ids.shape
        dev = x.device
        cap = -(-self._cap(T, dev) // n)
        bounds = [min(T, k * cap) for k in range(n + 1)]
        self._ev = []
        sends, recvs, outs, works = [], [], [], []
        for k in range(n):
            a, b = bounds[k], bounds[k + 1]
            p = self.k.dispatch(x[a:b], ids[a:b], w[a:b], self.E, G, cap)
            recv = torch.empty_like(p["send"])
            works.append(self._a2a(recv, p["send"], async_op=True))
            sends.append(p)
            recvs.append(recv)
        backs, bworks, idrs = [], [], []
        for k in range(n):
            self._wait(works[k])
            xr, idr, wr = unpack_records(recvs[k], H, topk, x.dtype)
            part = self.k.local(xr, idr, wr, self.ptrs_local, self.kinfo_local, self.I, self.K, self.n_local,
                                dtype=torch.float16)
            back = torch.empty_like(part)
            bworks.append(self._a2a(back, part, async_op=True))
            backs.append(back)
            idrs.append(idr)
        out = torch.empty((T, H), dtype=x.dtype, device=dev)
        for k in range(n):
            a, b = bounds[k], bounds[k + 1]
            self._wait(bworks[k])
            if b > a:
                self.k.combine_h(backs[k], sends[k]["pos"], b - a, G, H, x.dtype, out=out[a:b])
        self.last = {"cap": cap, "send_counts": sum(p_["counts"] for p_ in sends),
                     "recv_ids": torch.cat(idrs), "chunk_caps": [cap] * n}
        return out
