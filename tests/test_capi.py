"""CPU: the C-ABI library loads, exports every symbol include/exl3b200.h declares, and rejects bad arguments before
launching anything (no compute runs here)."""
import ctypes
import os
import re

import pytest

from exl3b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "exl3b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(exl3b_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    assert "exl3b_moe_decode" in names and "exl3b_ensure" in names and len(names) >= 14


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared()) <= set(_lib.exported_symbols())


def test_blob_bytes_and_abi():
    L = _lib.lib()
    assert L.exl3b_abi_version() == 1
    assert L.exl3b_blob_bytes(2048, 768, 3, 3, 3) == 1786368
    assert L.exl3b_blob_bytes(2560, 640, 3, 3, 3) == 1862400
    assert L.exl3b_moe_decode_workspace(1, 10, 2048, 768) > 0


def _routed_args(logits=1 << 20, topk=10, H=2048):
    """exl3b_moe_decode_cached_routed arguments for one token (valid pointers as placeholders; nothing launches
    because each case fails a check first)."""
    p = 1 << 20
    return [p, H, p, None, logits, p, p, 1, topk, 0, p, p, p, p, p, p, 0, 1786368, 0, p, p, 8, 8000, None, None, 0,
            None, None, None, H, 768, 3, 512, p, H, 1, p, 1 << 30, 1, None, None]


@pytest.mark.parametrize("call", [
    lambda L: L.exl3b_moe_decode_workspace(0, 10, 2048, 768) == 0,
])
def test_degenerate_sizes(call):
    assert call(_lib.lib())


@pytest.mark.parametrize("call", [
    lambda L: L.exl3b_dequant(None, 1, 24, 0, 4, 3, 1, None, 64, None),
    lambda L: L.exl3b_dequant(1 << 20, 1, 24, 1, 4, 3, 1, 1 << 21, 64, None),      # planar tile0 % 4
    lambda L: L.exl3b_dequant(1 << 20, 1, 24, 0, 4, 7, 0, 1 << 21, 64, None),      # K out of range
    lambda L: L.exl3b_ensure(1 << 20, 1 << 20, 10, 0, 2000, 8, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20,
                             0, 64, 64, 1 << 20, 1 << 20, 8, 0, None, None, None, 0, None, None, None),  # E > 1024
    lambda L: L.exl3b_moe_decode(1 << 20, 2048, 1, 1 << 20, 1 << 20, 1, 10, 1 << 20, None, 2000, 768, 3, 512,
                                 1 << 20, 2048, 1, 1 << 20, 1 << 30, 1, None),    # H % 128
    lambda L: L.exl3b_moe_decode(1 << 20, 2048, 1, 1 << 20, 1 << 20, 1, 10, 1 << 20, None, 2048, 768, 3, 512,
                                 1 << 20, 2048, 1, 1 << 20, 16, 1, None),          # workspace too small
    lambda L: L.exl3b_router_topk(1 << 20, 2048, 1 << 20, None, 1, 2048, 512, 40, 1 << 20, 1 << 20, 1 << 20, None, None),
    lambda L: L.exl3b_align(1 << 20, 1 << 20, 10, 10, 512, 32, 1 << 20, 1 << 20, 9, 10, 1 << 20, 1 << 20, None),
    lambda L: L.exl3b_cepf_plan(*([1 << 20, 4, 0, 512, 8] + [1 << 20] * 6 + [0, 64, 64, 1 << 20, 1 << 20, 17] +
                                  [1 << 20] * 4 + [1, None])),                      # max_fill > 16
    lambda L: L.exl3b_cepf_plan(*([1 << 20, 4, 3, 512, 8] + [1 << 20] * 6 + [0, 64, 64, 1 << 20, 1 << 20, 8] +
                                  [1 << 20] * 4 + [2, None])),                      # layer outside the plan buffer
    lambda L: L.exl3b_cepf_commit(None, 1 << 20, 2, 512, 8, 1 << 20, 1 << 20, 0, 64, None),
    lambda L: L.exl3b_cepf_worker_start(1 << 20, 0, 512, 8, 1 << 20, 0, 64, 64, 1 << 20, 0, None),   # no layers
    lambda L: L.exl3b_moe_decode_cached_routed(*_routed_args(logits=None)),                          # no logits
    lambda L: L.exl3b_moe_decode_cached_routed(*_routed_args(topk=40)),                              # topk > 32
    lambda L: L.exl3b_moe_decode_cached_routed(*_routed_args(H=2000)),                               # router H
    lambda L: L.exl3b_ep_dispatch(1 << 20, 2048, 1 << 20, 1 << 20, 8, 10, 512, 3, 2048, 8, 1 << 20, 1 << 20,
                                  1 << 20, 1 << 20, 1 << 20, None),                 # E % G
    lambda L: L.exl3b_ep_dispatch(1 << 20, 2048, 1 << 20, 1 << 20, 8, 10, 512, 2, 2048, 4, 1 << 20, 1 << 20,
                                  1 << 20, 1 << 20, 1 << 20, None),                 # cap < T
    lambda L: L.exl3b_ep_combine_h(1 << 20, 1 << 20, 4, 2, 2046, 1 << 20, 2048, 0, None),   # H % 4
])
def test_invalid_arguments_rejected_before_launch(call):
    L = _lib.lib()
    assert call(L) == 1
    assert L.exl3b_last_error()


def test_copy_prefetch_worker_idle():
    """No worker running: stop is a no-op that reports zero plans and copies."""
    import ctypes
    L = _lib.lib()
    counts = (ctypes.c_int64 * 2)(7, 7)
    assert L.exl3b_cepf_worker_running() == 0
    assert L.exl3b_cepf_worker_stop(counts) == 0 and list(counts) == [0, 0]


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="not built"):
        _lib.lib()
