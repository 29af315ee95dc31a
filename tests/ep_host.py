"""Test double of the expert-parallel device steps (exl3b200.ep.CudaEPKernels) on host tensors, with the oracle as the
local expert compute: lets the CPU tests run the EPPrefill exchange protocol on gloo ranks.  Same contract as
exl3b_ep_plan / _pack / _combine and exl3b_ep_dispatch / _combine_h (include/exl3b200.h)."""
from __future__ import annotations

import numpy as np
import torch

import oracle as O


class HostEPKernels:
    def __init__(self, blobs_local: list, H: int, I: int, K: int):
        self.blobs, self.H, self.I, self.K = blobs_local, H, I, K

    def plan(self, ids, w, n_experts, G):
        idn, wn = ids.numpy(), w.numpy()
        T, topk = idn.shape
        per = n_experts // G
        owner = np.where(idn >= 0, idn // per, -1)
        pos = np.full((max(T, 1), G), -1, dtype=np.int32)
        counts = np.zeros(G, dtype=np.int64)
        rows = []
        for d in range(G):
            toks = [t for t in range(T) if (owner[t] == d).any()]
            counts[d] = len(toks)
            rows.append(toks)
        offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
        n = max(T * G, 1)
        send_src = np.zeros(n, dtype=np.int32)
        send_ids = np.full((n, topk), -1, dtype=np.int32)
        send_w = np.zeros((n, topk), dtype=np.float32)
        for d in range(G):
            for j, t in enumerate(rows[d]):
                r = offs[d] + j
                pos[t, d] = r
                send_src[r] = t
                mine = owner[t] == d
                send_ids[r] = np.where(mine, idn[t] - d * per, -1)
                send_w[r] = np.where(mine, wn[t], 0.0)
        return {"counts": torch.from_numpy(counts), "offs": torch.from_numpy(offs), "pos": torch.from_numpy(pos),
                "send_src": torch.from_numpy(send_src), "send_ids": torch.from_numpy(send_ids),
                "send_w": torch.from_numpy(send_w)}

    def pack(self, x, send_src, n_rows):
        return x[send_src[:n_rows].long()].contiguous()

    def local(self, x, ids, w, ptrs, kinfo, I, K, n_local, dtype=torch.float32):
        if x.shape[0] == 0:
            return torch.zeros((0, self.H), dtype=dtype)
        xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
        part = O.moe_layer_fast(xb, ids.numpy(), w.numpy(), self.blobs, self.H, self.I, self.K, out_f32=True,
                                y_half=True, threads=2)
        return torch.from_numpy(part).to(dtype)

    @staticmethod
    def record_bytes(H, topk):
        return (2 * H + 8 * topk + 15) // 16 * 16

    def dispatch(self, x, ids, w, n_experts, G, cap):
        idn, wn = ids.numpy(), w.numpy()
        T, topk = idn.shape
        H = x.shape[1]
        per = n_experts // G
        rec = self.record_bytes(H, topk)
        send = np.zeros((G * cap, rec), dtype=np.uint8)
        send[:, 2 * H:2 * H + 4 * topk] = np.full((G * cap, topk), -1, np.int32).view(np.uint8)
        pos = np.full((max(T, 1), G), -1, dtype=np.int32)
        counts = np.zeros(G, dtype=np.int64)
        xb = x.contiguous().view(torch.int16).numpy().view(np.uint8).reshape(T, 2 * H) if T else None
        owner = np.where(idn >= 0, idn // per, -1)
        for d in range(G):
            j = 0
            for t in range(T):
                mine = owner[t] == d
                if not mine.any():
                    continue
                r = d * cap + j
                pos[t, d] = r
                send[r, :2 * H] = xb[t]
                send[r, 2 * H:2 * H + 4 * topk] = np.where(mine, idn[t] - d * per, -1).astype(np.int32).view(np.uint8)
                send[r, 2 * H + 4 * topk:2 * H + 8 * topk] = np.where(mine, wn[t], 0.0).astype(np.float32).view(np.uint8)
                j += 1
            counts[d] = j
        return {"send": torch.from_numpy(send), "pos": torch.from_numpy(pos), "counts": torch.from_numpy(counts)}

    def combine_h(self, part, pos, T, G, H, dtype, out=None):
        r = self.combine(part.to(torch.float32), pos, T, G, H, dtype)
        if out is None:
            return r
        out.copy_(r)
        return out

    def combine(self, part, pos, T, G, H, dtype):
        out = torch.zeros((T, H), dtype=torch.float32)
        pn = pos.numpy()
        for t in range(T):
            for d in range(G):
                if pn[t, d] >= 0:
                    out[t] += part[int(pn[t, d])]
        return out.to(dtype)
