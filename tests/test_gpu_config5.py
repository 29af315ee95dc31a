"""GPU parity of configs[4]: mixed-bitrate routed experts (per-tensor K in {2, 3, 4, 5}) plus the always-on shared
expert (K = 4) behind a sigmoid gate, decode and prefill, against the oracle: the shared expert is one more pick per
token with weight sigmoid(x . g), combined after the routed picks."""
import numpy as np
import pytest
import torch

import oracle as O
from exl3b200 import _lib, synth
from exl3b200 import ops as X
from helpers import assert_close_f32, assert_close_layer, bits, make_layer

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status():
    X.register()
    yield
    st = np.zeros(1, np.int32)
    _lib.check(_lib.lib().exl3b_device_status(st.ctypes.data, 1, None))
    assert st[0] == 0, f"device status word {st[0]}"


def layer5(E, H, I, seed):
    """E routed experts with mixed K plus the shared expert (K = 4) as entry E of one arena."""
    kin = [synth.mixed_k(seed, e) for e in range(E)] + [(4, 4, 4)]
    arena, ptrs, views = make_layer(E + 1, H, I, 0, seed=seed, kinfo=kin)
    kinfo = torch.tensor([synth.kinfo_pack(*k) for k in kin], dtype=torch.int32)
    return arena, ptrs, views, kinfo


def run_case(T, H, I, E, topk, seed, prefill_min=None):
    arena, ptrs, views, kinfo = layer5(E, H, I, seed)
    x = synth.activations(T, H, seed + 1)
    g = synth.router_weight(1, H, 1.0 / np.sqrt(H), seed + 2).reshape(H)
    wr = synth.router_weight(E, H, 1.0 / np.sqrt(H), seed + 3)
    xd = x.to(DEV)
    ids, w = X.router_topk(xd, wr.to(DEV), None, topk)
    old = X.G.prefill_min_m
    if prefill_min is not None:
        X.moe_set_prefill_min_m(prefill_min)
    try:
        out = torch.ops.exl3b200_moe.moe_forward_shared(xd, ids, w, ptrs, kinfo.to(DEV), g.to(DEV), I, E)
        ids_x, w_x = X.shared_gate(xd, g.to(DEV), ids, w, E)
        o32 = torch.empty(T, H, dtype=torch.float32, device=DEV)
        if T >= X.G.prefill_min_m:
            X.moe_prefill(xd, ids_x, w_x, ptrs, I, 0, E + 1, kinfo=kinfo.to(DEV), out=o32)
        else:
            X.moe_decode(xd, ids_x, w_x, ptrs, I, 0, E + 1, kinfo=kinfo.to(DEV), out=o32)
    finally:
        X.moe_set_prefill_min_m(old)
    torch.cuda.synchronize()
    # gate weights against the oracle's sigmoid(x . g)
    gw = O.shared_gate(bits(x), bits(g))
    np.testing.assert_allclose(w_x[:, topk].cpu().numpy(), gw, rtol=2e-6, atol=0)
    assert torch.equal(ids_x[:, :topk], ids) and torch.equal(w_x[:, :topk], w)
    assert int(ids_x[:, topk].min()) == E == int(ids_x[:, topk].max())
    ki = kinfo.numpy()
    need = set(int(e) for e in ids_x.cpu().numpy().ravel())
    blobs = [views[e].cpu().numpy() if e in need else None for e in range(E + 1)]
    prefill = T >= (prefill_min if prefill_min is not None else X.G.prefill_min_m)
    idn, wn = ids_x.cpu().numpy(), w_x.cpu().numpy()
    ref32 = O.moe_layer_fast(bits(x), idn, wn, blobs, H, I, 3, kinfo=ki, out_f32=True, y_half=prefill)
    ref = O.moe_layer_fast(bits(x), idn, wn, blobs, H, I, 3, kinfo=ki, y_half=prefill)
    assert_close_f32(o32.cpu().numpy(), ref32)
    assert_close_layer(bits(out), ref)


@pytest.mark.parametrize("T", [1, 4])
def test_config5_decode_small(T):
    run_case(T, 256, 256, 16, 4, seed=7)


@pytest.mark.parametrize("T", [1, 4])
def test_config5_decode_full_shape(T):
    """hidden 2048, 512 routed experts, top-10, intermediate 768, per-tensor K in {2..5}, shared expert K = 4."""
    run_case(T, 2048, 768, 512, 10, seed=7)


def test_config5_prefill():
    run_case(300, 256, 256, 16, 4, seed=8)


def test_config5_prefill_full_shape():
    """configs[4] prefill at T = 256 (the parity case; the bench times T = 2048)."""
    run_case(256, 2048, 768, 512, 10, seed=7)
