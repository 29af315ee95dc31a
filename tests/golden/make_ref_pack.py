"""Golden blobs from the reference's own packer: plugin/exl3xpu/moe_offload.py pack_expert / planar4 of the reference
checkout given as the argument (read only).  That module is pure torch at import (its SYCL library loads only when
ops() is called), so its packer runs on any CPU.

    python tests/golden/make_ref_pack.py <reference checkout>

writes tests/golden/ref_pack.npz: for K in (3, 5), one expert (H = I = 128) of seeded checkpoint tensors (trellis
int16 [k/16][n/16][16K], suh fp16 [k], svh fp16 [n] for gate, up, down) and the blob bytes the reference packs from
them.  tests/test_oracle_codec.py checks this build's packer and the oracle's blob reader against them.
"""
import importlib.util
import os
import sys

import numpy as np
import torch

H, I = 128, 128


def main(ref_root: str) -> None:
    path = os.path.join(ref_root, "plugin", "exl3xpu", "moe_offload.py")
    spec = importlib.util.spec_from_file_location("reference_moe_offload", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    out = {}
    for K in (3, 5):
        g = torch.Generator().manual_seed(100 + K)

        def tens(k, n):
            return dict(trellis=torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, generator=g),
                        suh=(torch.randint(0, 2, (k,), generator=g) * 2 - 1).half(),
                        svh=(torch.rand(n, generator=g) + 0.5).half())

        gate, up, down = tens(H, I), tens(H, I), tens(I, H)
        blob = ref.pack_expert(gate, up, down, K)
        for name, t in (("gate", gate), ("up", up), ("down", down)):
            for f in ("trellis", "suh", "svh"):
                out[f"k{K}_{name}_{f}"] = t[f].numpy()
        out[f"k{K}_blob"] = blob.numpy()
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_pack.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, {k: v.shape for k, v in out.items() if k.endswith("blob")})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_ref_pack.py <reference checkout>")
    main(sys.argv[1])
