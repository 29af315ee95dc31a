"""Shared test helpers: synthetic layers on the device, oracle inputs, tolerance checks."""
from __future__ import annotations

import numpy as np
import torch

from exl3b200 import synth

ATOL = 2e-2      # north-star layer tolerance: max-abs 2e-2 ...
RTOL_L2 = 1e-3   # ... and rel-L2 1e-3 on bf16 outputs


def make_layer(E, H, I, K, seed, device="cuda", kinfo=None, layer=0):
    """Blobs [E, blob] uint8 on `device` (contiguous, one arena) and the int64 pointer table."""
    if kinfo is None:
        bb = synth.blob_geometry(H, I, K, K, K)["blob"]
        blobs = torch.empty((E, bb), dtype=torch.uint8, device=device)
        for e in range(E):
            synth.fill_blob(blobs[e], seed, layer * E + e, H, I, K)
        ptrs = blobs.data_ptr() + torch.arange(E, dtype=torch.int64) * bb
        return blobs, ptrs.to(device), [blobs[e] for e in range(E)]
    parts = []
    for e in range(E):
        kg, ku, kd = kinfo[e]
        parts.append(synth.make_blob(seed, layer * E + e, H, I, kg, ku, kd, device=device))
    sizes = [p.numel() for p in parts]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]])
    arena = torch.empty(int(sum(sizes)), dtype=torch.uint8, device=device)
    for p, o in zip(parts, offs):
        arena[int(o):int(o) + p.numel()].copy_(p)
    ptrs = arena.data_ptr() + torch.tensor(offs, dtype=torch.int64)
    return arena, ptrs.to(device), [arena[int(o):int(o) + s] for o, s in zip(offs, sizes)]


def oracle_blobs(views, ids: np.ndarray):
    need = set(int(e) for e in np.asarray(ids).ravel())
    return [views[e].cpu().numpy() if e in need else None for e in range(len(views))]


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# Two independent bf16 roundings of values that agree to ~1e-4 (the fp16 intermediates of the reference arithmetic
# flip by one fp16 ulp in a few % of elements under any change of summation order) differ by one bf16 ulp (2^-8
# relative) in a few % of elements: a rel-L2 floor near 1e-3.  The north-star tolerance (max-abs 2e-2, rel-L2 1e-3)
# is therefore asserted on the fp32 layer output before its final rounding (assert_close_f32), and the rounded bf16
# product output is asserted with max-abs 2e-2 and rel-L2 2e-3 (1e-3 plus that floor).
RTOL_L2_BF16 = 2e-3


def assert_close_f32(got: np.ndarray, ref: np.ndarray, atol=ATOL, rl2=RTOL_L2):
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert np.all(np.isfinite(g)), "non-finite output"
    mad = float(np.abs(g - r).max()) if g.size else 0.0
    rel = float(np.linalg.norm(g - r)) / (float(np.linalg.norm(r)) or 1.0)
    assert mad <= atol and rel <= rl2, f"fp32 max-abs {mad:.3g} (tol {atol}), rel-L2 {rel:.3g} (tol {rl2})"
    return mad, rel


def assert_close_layer(got_bits: np.ndarray, ref_bits: np.ndarray, atol=ATOL, rl2=RTOL_L2_BF16):
    g = bf16_to_f32(got_bits).astype(np.float64)
    r = bf16_to_f32(ref_bits).astype(np.float64)
    assert np.all(np.isfinite(g)), "non-finite output"
    mad = float(np.abs(g - r).max()) if g.size else 0.0
    den = float(np.linalg.norm(r)) or 1.0
    rel = float(np.linalg.norm(g - r)) / den
    assert mad <= atol and rel <= rl2, f"max-abs {mad:.3g} (tol {atol}), rel-L2 {rel:.3g} (tol {rl2})"
    return mad, rel
