"""exl3b200 -- B200-native (sm_100a) EXL3 routed-expert MoE: the drop-in for the reference plugin's exl3xpu MoE path.

Host code is Python/PyTorch; all compute runs in libexl3b200.so (hand-written CUDA for sm_100a) through its C ABI.
Modules: moe_offload (ExpertStore, pack_expert, planar4, ops()), ops (torch ops with the reference schemas), ep
(expert-parallel prefill over a torch.distributed group), tier (TierHost: the RAM tier's per-step host loop),
checkpoint (EXL3 safetensors checkpoints into ExpertStore host blobs), pack_store (the packed expert store on NVMe and
the reader pool behind TierHost.fetch), stage (StoreStager: prefill with the experts streamed from the pack store),
synth (seeded synthetic inputs), _lib (the C ABI through ctypes).
"""
from .moe_offload import ExpertStore, pack_expert, planar4, s64  # noqa: F401

__all__ = ["ExpertStore", "pack_expert", "planar4", "s64"]
