"""Seeded synthetic EXL3 experts and routing inputs (benchmarks, smoke test and parity tests).

Blob bytes come from a counter-based 32-bit hash evaluated with torch integer ops, so the same
(seed, key) yields the same bytes on the CPU and on a GPU: tests can build a layer on the device and
hand a few experts' bytes to the CPU oracle, and the benchmark can generate tens of GB in place.

Distributions: trellis words uniform over all bit patterns (every pattern is a
valid code); suh = +-1; svh = +-U(0.5, 1.5) / sqrt(fan_in) -- the per-output-channel scale U(0.5, 1.5)
times the fan-in normalisation real EXL3 scale vectors carry (codebook values are O(1), so without it
the fp16 activations of the reference arithmetic overflow); activations N(0, 1) bf16.
"""
from __future__ import annotations

import math

import torch

M32 = 0xFFFFFFFF


def _mul32(a: torch.Tensor, c: int) -> torch.Tensor:
    """(a * c) mod 2^32 for int64 a in [0, 2^32) without int64 overflow."""
    lo = (a & 0xFFFF) * c
    hi = ((a >> 16) * (c & 0xFFFF)) & 0xFFFF
    return (lo + (hi << 16)) & M32


def _fmix32(h: torch.Tensor) -> torch.Tensor:
    h = h ^ (h >> 16)
    h = _mul32(h, 0x85EBCA6B)
    h = h ^ (h >> 13)
    h = _mul32(h, 0xC2B2AE35)
    return h ^ (h >> 16)


def _fmix32_int(h: int) -> int:
    h &= M32
    h ^= h >> 16
    h = (h * 0x85EBCA6B) & M32
    h ^= h >> 13
    h = (h * 0xC2B2AE35) & M32
    return h ^ (h >> 16)


def stream_u32(seed: int, stream: int, n: int, device, offset: int = 0) -> torch.Tensor:
    """n hashed uint32 values (as int64) of stream `stream` under `seed`, starting at index `offset`."""
    s1 = _fmix32_int(seed * 0x9E3779B9 + 0x632BE5AB)
    s2 = _fmix32_int(s1 ^ (stream * 0x85EBCA77 + 0x27D4EB2F))
    s3 = _fmix32_int(s2 + 0x165667B1)
    i = torch.arange(offset, offset + n, dtype=torch.int64, device=device)
    return _fmix32((_fmix32(i ^ s2) + s3) & M32)


def blob_geometry(H: int, I: int, Kg: int, Ku: int, Kd: int) -> dict:
    """Byte offsets of the blob regions (exl3_moe.a8.sycl:42-54, per-tensor K generalisation)."""
    gu = (H // 16) * (I // 16) * 8 * (Kg + Ku) * 4
    d = (I // 16) * (H // 16) * 8 * Kd * 4
    o = gu + d
    off = dict(gu=0, d=gu, suh_g=o, suh_u=o + 2 * H, svh_g=o + 4 * H, svh_u=o + 4 * H + 2 * I,
               suh_d=o + 4 * H + 4 * I, svh_d=o + 4 * H + 6 * I)
    off["blob"] = o + 6 * H + 6 * I
    off["words"] = (gu + d) // 4
    return off


def _signs(seed: int, stream: int, n: int, device) -> torch.Tensor:
    return 1.0 - 2.0 * (stream_u32(seed, stream, n, device) & 1).to(torch.float32)


def _scales(seed: int, stream: int, n: int, fan_in: int, device) -> torch.Tensor:
    h = stream_u32(seed, stream, n, device)
    u = (h >> 8).to(torch.float32) * (1.0 / 16777216.0)
    sign = 1.0 - 2.0 * (h & 1).to(torch.float32)
    return sign * (0.5 + u) * (1.0 / math.sqrt(fan_in))


def fill_blob(out: torch.Tensor, seed: int, key: int, H: int, I: int, Kg: int, Ku: int | None = None,
              Kd: int | None = None) -> torch.Tensor:
    """Write expert `key`'s synthetic blob into the uint8 tensor `out` (len = blob bytes)."""
    Ku = Kg if Ku is None else Ku
    Kd = Kg if Kd is None else Kd
    g = blob_geometry(H, I, Kg, Ku, Kd)
    assert out.dtype == torch.uint8 and out.numel() == g["blob"], (out.numel(), g["blob"])
    dev = out.device
    st = key * 8
    nw = g["words"]
    out[: nw * 4].view(torch.int32).copy_(stream_u32(seed, st, nw, dev).to(torch.int32))
    vec = torch.cat([_signs(seed, st + 1, H, dev), _signs(seed, st + 2, H, dev),
                     _scales(seed, st + 3, I, H, dev), _scales(seed, st + 4, I, H, dev),
                     _signs(seed, st + 5, I, dev), _scales(seed, st + 6, H, I, dev)]).to(torch.float16)
    out[nw * 4:].view(torch.float16).copy_(vec)
    return out


def make_blob(seed: int, key: int, H: int, I: int, Kg: int, Ku: int | None = None, Kd: int | None = None,
              device="cpu") -> torch.Tensor:
    Ku = Kg if Ku is None else Ku
    Kd = Kg if Kd is None else Kd
    b = torch.empty(blob_geometry(H, I, Kg, Ku, Kd)["blob"], dtype=torch.uint8, device=device)
    return fill_blob(b, seed, key, H, I, Kg, Ku, Kd)


def mixed_k(seed: int, key: int) -> tuple[int, int, int]:
    """Config 5: per-tensor K from {2, 3, 4, 5} with P = (0.2, 0.6, 0.1, 0.1) (mean 3.1 bpw per tensor
    draw; 3.05 bpw weighted by tensor size at H=2048, I=768 is within sampling noise)."""
    h = stream_u32(seed, 0x7F000000 + key, 3, "cpu").tolist()
    out = []
    for v in h:
        u = (v >> 8) / 16777216.0
        out.append(2 if u < 0.2 else 3 if u < 0.8 else 4 if u < 0.9 else 5)
    return tuple(out)


def kinfo_pack(kg: int, ku: int, kd: int) -> int:
    return kg | (ku << 4) | (kd << 8)


def activations(T: int, H: int, seed: int, device="cpu") -> torch.Tensor:
    """x ~ N(0, 1) in bf16, generated on the CPU (reproducible) and moved to `device`."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, H, generator=g).to(torch.bfloat16).to(device)


def router_weight(E: int, H: int, std: float, seed: int, device="cpu") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + 1)
    return (torch.randn(E, H, generator=g) * std).to(torch.bfloat16).to(device)


def zipf_bias(E: int, layer: int, seed: int, s: float = 1.1) -> torch.Tensor:
    """Per-layer Zipf(s) logit bias -s*ln(rank): a seeded random permutation assigns ranks 1..E."""
    g = torch.Generator().manual_seed(seed * 1000003 + layer)
    perm = torch.randperm(E, generator=g)
    rank = torch.empty(E, dtype=torch.float32)
    rank[perm] = torch.arange(1, E + 1, dtype=torch.float32)
    return -s * torch.log(rank)


def zipf_rank(E: int, layer: int, seed: int) -> torch.Tensor:
    """Experts of `layer` in Zipf rank order (hottest first), matching zipf_bias."""
    g = torch.Generator().manual_seed(seed * 1000003 + layer)
    return torch.randperm(E, generator=g)


def normal_bias(E: int, std: float, seed: int) -> torch.Tensor:
    """Config 3/4 load-imbalance bias ~ N(0, std)."""
    g = torch.Generator().manual_seed(seed + 2)
    return torch.randn(E, generator=g) * std


def fill_blobs(out: torch.Tensor, seed: int, keys: list, H: int, I: int, K: int, batch: int = 32) -> torch.Tensor:
    """fill_blob for many experts at once: out [n, blob] uint8 (rows may be strided views of a slot arena);
    keys[i] is row i's key.  Same bytes as fill_blob (the hash is elementwise in the word index)."""
    n = len(keys)
    for b0 in range(0, n, batch):
        for i in range(b0, min(n, b0 + batch)):
            fill_blob(out[i], seed, int(keys[i]), H, I, K)
    return out
