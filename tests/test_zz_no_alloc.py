"""exl3b_moe_decode_noalloc (the decode entry point that allocates nothing; its scratch is a fixed 8 MiB device
array of the library) against exl3b_moe_decode with a caller workspace, through the C ABI.

Collected last so that it runs both after the other GPU tests and, alone, in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from exl3b200 import _lib, synth
from helpers import make_layer

DEV = "cuda"


def _decode_ws(L, x, ids, w, ptrs, I, K, E, out):
    M, H = x.shape
    topk = ids.shape[1]
    wsb = int(L.exl3b_moe_decode_workspace(M, topk, H, I))
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    _lib.check(L.exl3b_moe_decode(x.data_ptr(), x.stride(0), 1, ids.data_ptr(), w.data_ptr(), M, topk, ptrs.data_ptr(),
                                  None, H, I, K, E, out.data_ptr(), out.stride(0), 1 if out.dtype == torch.bfloat16 else 2,
                                  ws.data_ptr(), wsb, 0, torch.cuda.current_stream().cuda_stream), "moe_decode")


def _decode_noalloc(L, x, ids, w, ptrs, I, K, E, out):
    M, H = x.shape
    return L.exl3b_moe_decode_noalloc(x.data_ptr(), x.stride(0), 1, ids.data_ptr(), w.data_ptr(), M, ids.shape[1],
                                      ptrs.data_ptr(), None, H, I, K, E, out.data_ptr(), out.stride(0),
                                      1 if out.dtype == torch.bfloat16 else 2, 0,
                                      torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_oversized_call():
    """100 tokens at top-10, H=2048, I=768 need 9.4 MiB of scratch: rejected before any launch (no GPU needed)."""
    L = _lib.lib()
    rc = L.exl3b_moe_decode_noalloc(1 << 20, 2048, 1, 1 << 20, 1 << 20, 100, 10, 1 << 20, None, 2048, 768, 3, 512,
                                    1 << 20, 2048, 1, 0, None)
    assert rc == 1
    assert b"8 MiB" in ctypes.string_at(L.exl3b_last_error())


def test_noalloc_names_a_bad_shape():
    """A shape the decode cannot take is reported as a bad argument, not as a scratch overflow (no GPU needed)."""
    L = _lib.lib()
    rc = L.exl3b_moe_decode_noalloc(1 << 20, 2048, 1, 1 << 20, 1 << 20, 1, 10, 1 << 20, None, 2048, 0, 3, 512,
                                    1 << 20, 2048, 1, 0, None)
    assert rc == 1
    msg = ctypes.string_at(L.exl3b_last_error())
    assert b"multiples of 128" in msg and b"8 MiB" not in msg


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 4])
def test_noalloc_matches_workspace_decode(T):
    """Full decode shape (H=2048, I=768, 512 experts, top-10, K=3): two calls in a row, each equal to the workspace
    entry point bit for bit (the same deterministic kernels run on both), for the bf16 product output and the fp32
    layer output."""
    H, I, E, topk, K = 2048, 768, 512, 10, 3
    L = _lib.lib()
    _, ptrs, _ = make_layer(E, H, I, K, seed=3)
    for call in range(2):
        x = synth.activations(T, H, 60 + call).to(DEV)
        g = torch.Generator().manual_seed(70 + call)
        ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).to(torch.int32).to(DEV)
        w = torch.softmax(torch.rand(T, topk, generator=g), 1).float().to(DEV)
        for dt in (torch.bfloat16, torch.float32):
            ref = torch.empty(T, H, dtype=dt, device=DEV)
            got = torch.full((T, H), float("nan"), dtype=dt, device=DEV)
            _decode_ws(L, x, ids, w, ptrs, I, K, E, ref)
            rc = _decode_noalloc(L, x, ids, w, ptrs, I, K, E, got)
            assert rc == 0, ctypes.string_at(L.exl3b_last_error())
            torch.cuda.synchronize()
            assert torch.equal(got, ref), (call, dt)
    st = np.zeros(1, np.int32)
    _lib.check(L.exl3b_device_status(st.ctypes.data, 1, None))
    assert st[0] == 0
