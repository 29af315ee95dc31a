"""ctypes binding of libexl3b200.so (the C ABI declared in include/exl3b200.h).

The library is built in-tree by build.py and loaded from this directory.  There is no fallback: if the library is
missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("EXL3B200_LIB") or os.path.join(_HERE, "libexl3b200.so")

_lib = None
_lock = threading.Lock()

vp = ctypes.c_void_p
ci = ctypes.c_int
i64 = ctypes.c_int64

_SIGS = {
    "exl3b_last_error": (ctypes.c_char_p, []),
    "exl3b_abi_version": (ci, []),
    "exl3b_device_status": (ci, [vp, ci, vp]),
    "exl3b_blob_bytes": (i64, [ci, ci, ci, ci, ci]),
    "exl3b_dequant": (ci, [vp, ci, i64, ci, ci, ci, ci, vp, i64, vp]),
    "exl3b_blob_dequant": (ci, [vp, ci, ci, ci, ci, ci, ci, vp, vp]),
    "exl3b_router_topk": (ci, [vp, i64, vp, vp, ci, ci, ci, ci, vp, vp, vp, vp, vp]),
    "exl3b_ensure": (ci, [vp, vp, ci, ci, ci, ci, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp, vp, ci, ci, vp, vp, vp, ci,
                          vp, vp, vp]),
    "exl3b_fill_copy": (ci, [vp, vp, vp, vp, i64, i64, ci, vp]),
    "exl3b_victim_copy": (ci, [vp, vp, i64, i64, ci, i64, vp, ci, vp]),
    "exl3b_commit": (ci, [vp, vp, vp, vp, i64, i64, vp]),
    "exl3b_set_victim_ring": (ci, [vp, vp, vp, i64, ci]),
    "exl3b_cepf_plan": (ci, [vp, ci, ci, ci, ci, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp, vp, ci, vp, vp, vp, vp, ci,
                             vp]),
    "exl3b_cepf_commit": (ci, [vp, vp, ci, ci, ci, vp, vp, i64, i64, vp]),
    "exl3b_cepf_worker_start": (ci, [vp, ci, ci, ci, vp, i64, i64, i64, vp, ci, vp]),
    "exl3b_cepf_worker_stop": (ci, [vp]),
    "exl3b_cepf_worker_running": (ci, []),
    "exl3b_moe_decode_workspace": (i64, [ci, ci, ci, ci]),
    "exl3b_moe_decode": (ci, [vp, i64, ci, vp, vp, ci, ci, vp, vp, ci, ci, ci, ci, vp, i64, ci, vp, i64, ci, vp]),
    "exl3b_set_profile_events": (ci, [vp, vp, vp, vp]),
    "exl3b_moe_decode_cached": (ci, [vp, i64, ci, vp, vp, ci, ci, ci, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp, vp, ci, ci,
                                     vp, vp, ci, vp, vp, vp, ci, ci, ci, ci, vp, i64, ci, vp, i64, ci, vp]),
    "exl3b_moe_decode_cached_routed": (ci, [vp, i64, vp, vp, vp, vp, vp, ci, ci, ci, vp, vp, vp, vp, vp, vp, i64, i64,
                                            i64, vp, vp, ci, ci, vp, vp, ci, vp, vp, vp, ci, ci, ci, ci, vp, i64, ci, vp,
                                            i64, ci, vp, vp]),
    "exl3b_align_scratch": (i64, [ci, ci]),
    "exl3b_align": (ci, [vp, vp, ci, ci, ci, ci, vp, vp, ci, ci, vp, i64, vp]),
    "exl3b_ep_plan": (ci, [vp, vp, ci, ci, ci, ci, vp, vp, vp, vp, vp, vp, vp, vp]),
    "exl3b_ep_pack": (ci, [vp, i64, ci, vp, ci, vp, vp]),
    "exl3b_ep_combine": (ci, [vp, vp, ci, ci, ci, vp, i64, ci, vp]),
    "exl3b_ep_record_bytes": (i64, [ci, ci]),
    "exl3b_ep_dispatch": (ci, [vp, i64, vp, vp, ci, ci, ci, ci, ci, ci, vp, vp, vp, vp, vp, vp]),
    "exl3b_ep_combine_h": (ci, [vp, vp, ci, ci, ci, vp, i64, ci, vp]),
    "exl3b_shared_gate": (ci, [vp, i64, vp, ci, ci, vp, vp, ci, ci, vp, vp, vp]),
    "exl3b_moe_decode_noalloc": (ci, [vp, i64, ci, vp, vp, ci, ci, vp, vp, ci, ci, ci, ci, vp, i64, ci, ci, vp]),
    "exl3b_moe_prefill_workspace": (i64, [ci, ci, ci, ci, ci]),
    "exl3b_moe_prefill": (ci, [vp, i64, ci, vp, vp, ci, ci, vp, vp, ci, ci, ci, ci, vp, i64, ci, vp, i64, ci, vp]),
}

OPTIONAL = set()


def lib() -> ctypes.CDLL:
    """Load the library once (raises if it is missing: there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"exl3b200: {LIB_PATH} is not built (run qwen38-flash-next-b70-offload_b200/build.py)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGS.items():
                if not hasattr(L, name):
                    if name in OPTIONAL:
                        continue
                    raise RuntimeError(f"exl3b200: {LIB_PATH} does not export {name}")
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().exl3b_last_error()
        raise RuntimeError(f"exl3b200{(' ' + what) if what else ''}: {msg.decode() if msg else 'error'} (code {rc})")


def ptr(t) -> int | None:
    """Device/host address of a tensor (None for None / empty tensors)."""
    if t is None:
        return None
    if t.numel() == 0:
        return None
    return t.data_ptr()


def stream(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
