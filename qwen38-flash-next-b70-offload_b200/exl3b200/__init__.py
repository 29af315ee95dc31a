"""exl3b200 -- B200-native (sm_100a) EXL3 routed-expert MoE: the drop-in for the reference plugin's exl3xpu MoE path.

Host code is Python/PyTorch; all compute runs in libexl3b200.so (hand-written CUDA for sm_100a) through its C ABI.
Modules: moe_offload (ExpertStore, pack_expert, planar4, ops()), ops (torch ops with the reference schemas), nvtier
(tier contract), synth (seeded synthetic inputs).
"""
from .moe_offload import ExpertStore, pack_expert, planar4, s64  # noqa: F401

__all__ = ["ExpertStore", "pack_expert", "planar4", "s64"]
