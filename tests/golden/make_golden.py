"""Generate tests/golden/golden.npz: small regression fixtures of the CPU oracle.

    python tests/golden/make_golden.py

The reference (SYCL/ESIMD for an Intel GPU) cannot run here and commits no golden vectors for this path, so the
fixtures are the oracle's own outputs on seeded synthetic inputs (exl3b200.synth, hash-based, identical on CPU and
GPU).  They pin the oracle against accidental change and give the GPU tests a reference that needs no recomputation.
What pins the oracle to the REFERENCE is listed in oracle/exl3b_oracle.c (codebook cross-statements, range bound,
blob sizes, blobs packed by the reference's own packer) and checked by tests/test_oracle_codec.py.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "qwen38-flash-next-b70-offload_b200"))

import oracle as O  # noqa: E402
import torch  # noqa: E402
from exl3b200 import synth  # noqa: E402

# small layer case: H=256, I=256, E=16, top-4, K=3, T=3
GH, GI, GE, GTOP, GT, GK, SEED = 256, 256, 16, 4, 3, 3, 11


def layer_case():
    blobs = [synth.make_blob(SEED, e, GH, GI, GK).numpy() for e in range(GE)]
    x = synth.activations(GT, GH, SEED).view(torch.int16).numpy().view(np.uint16)
    wr = synth.router_weight(GE, GH, 0.05, SEED).view(torch.int16).numpy().view(np.uint16)
    ids, w, lg = O.router(x, wr, None, GTOP)
    out, y, ab = O.moe_layer(x, ids, w, blobs, GH, GI, GK, want_y=True)
    return dict(l_x=x, l_wr=wr, l_ids=ids, l_w=w, l_logits=lg, l_out=out, l_y=y, l_abuf=ab)


def tile_case():
    d = {}
    for K in (2, 3, 4, 5):
        words = synth.stream_u32(SEED, 1000 + K, 8 * K * 4, "cpu").to(torch.int64).numpy().astype(np.uint32)
        d[f"t_words_k{K}"] = words
        d[f"t_plain_k{K}"] = O.dequant(words, 1, 8 * K * 4, 0, 4, K, False)
        d[f"t_planar_k{K}"] = O.dequant(words, 1, 8 * K * 4, 0, 4, K, True)
    return d


def main():
    tab = O.mul1_table()
    d = dict(mul1_sha256=np.frombuffer(hashlib.sha256(tab.tobytes()).digest(), dtype=np.uint8),
             mul1_sample=tab[::257].copy())
    d.update(tile_case())
    d.update(layer_case())
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **d)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
