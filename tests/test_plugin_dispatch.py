"""CPU: the reference plugin's own MoE dispatch, unchanged, driving this build's ExpertStore and TierDriver.

The reference's SGLang plugin calls the expert store from Exl3XpuMoEMethod.apply (plugin/sglang_plugin.tier.py:531-561):
by row count and mode it takes the tier's stage_forward (NVMe staging, big prefill batches), the tier's
ensure_for_prefill followed by forward (smaller prefill batches in tier mode), forward_prefill_staged (prefill batches of
at least EXL3_MOE_STAGE_MIN_M rows, not the MTP layer), forward_cached (decode through the device cache) or forward,
and wraps the result as StandardCombineInput(hidden_states=y.view_as(x)).  This test loads that module from a reference
checkout (beside the repository, or $EXL3B_REFERENCE) with stand-ins for the few SGLang names it imports, builds the
unchanged method class, and calls apply() with this build's store and tier objects on CPU tensors (skipped without a
checkout).  The op namespace is a fake whose forward reads every pick's blob through the pointer table it is given, so
each check compares bytes the kernels would read.
"""
import ctypes
import importlib.util
import os
import sys
import types

import pytest
import torch

from exl3b200 import moe_offload
from exl3b200.moe_offload import ExpertStore
from exl3b200.stage import TierDriver
from exl3b200.tier import TierHost

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("EXL3B_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
PLUGIN = os.path.join(REF, "plugin", "sglang_plugin.tier.py")
pytestmark = pytest.mark.skipif(not os.path.exists(PLUGIN), reason="no reference checkout to load the plugin from")

BLOB, H, E, L = 96, 16, 8, 3


def _bytes_at(addr: int) -> torch.Tensor:
    return torch.frombuffer(bytearray(ctypes.string_at(addr, BLOB)), dtype=torch.uint8).to(torch.float32)


class FakeOps:
    """What the CUDA ops do to memory, on CPU: copies are memmoves; a forward returns, per token, the weighted sum of
    the first H bytes of each pick's blob read through the table (shape [rows, H], like the real output)."""

    def __init__(self):
        self.calls = []

    def blob_bytes(self, H_, I_, K_):
        return BLOB

    def host_alloc(self, n):
        return torch.zeros(n, dtype=torch.uint8)

    def memcpy_async(self, dst, src, n):
        ctypes.memmove(dst, src, n)

    def moe_forward(self, x, ids, w, ptrs, I_, K_, E_):
        p = ptrs.tolist()
        out = torch.zeros(x.shape[0], x.shape[1])
        for t in range(ids.shape[0]):
            for k in range(ids.shape[1]):
                out[t] += float(w[t, k]) * _bytes_at(p[int(ids[t, k])])[: x.shape[1]]
        return out.to(x.dtype)

    def moe_forward_cached(self, x, ids, w, ptrs_all, layer, *rest):
        return self.moe_forward(x, ids, w, ptrs_all[layer * E:(layer + 1) * E], *rest[-5:-2])   # I, K, E

    def moe_set_prefill_min_m(self, v):
        pass


class RecordingStore(ExpertStore):
    """This build's ExpertStore with every entry point the plugin may call recorded (name, key, rows)."""

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self.log = []

    def _rec(self, name, key, x):
        self.log.append((name, key, int(x.shape[0])))

    def forward(self, key, x, topk_ids, topk_w, ptrs=None):
        self._rec("forward", key, x)
        return super().forward(key, x, topk_ids, topk_w, ptrs)

    def forward_cached(self, key, x, topk_ids, topk_w, max_fill=None, out=None):
        self._rec("forward_cached", key, x)
        return super().forward_cached(key, x, topk_ids, topk_w, max_fill, out)

    def forward_prefill_staged(self, key, x, topk_ids, topk_w):
        self._rec("forward_prefill_staged", key, x)
        return super().forward(key, x, topk_ids, topk_w)   # same bytes as the staged copies; staging runs on GPUs

    def prefill_reset(self):
        self.log.append(("prefill_reset", None, 0))
        return super().prefill_reset()


class FakeStager:
    """StoreStager's call surface: stage_forward(key, x, ids, w) -> output (here: the store's forward)."""

    def __init__(self, store):
        self.store, self.calls = store, []

    def stage_forward(self, key, x, topk_ids, topk_w):
        self.calls.append((key, int(x.shape[0])))
        return ExpertStore.forward(self.store, key, x, topk_ids, topk_w)


@pytest.fixture(scope="module")
def plugin():
    """The reference plugin module, loaded with stand-ins for the SGLang names _build_classes imports."""
    names = ["sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.quantization",
             "sglang.srt.layers.quantization.base_config", "sglang.srt.utils", "sglang.srt.utils.common",
             "sglang.srt.layers.moe", "sglang.srt.layers.moe.token_dispatcher",
             "sglang.srt.layers.moe.token_dispatcher.standard"]
    saved = {n: sys.modules.get(n) for n in names}
    mods = {n: types.ModuleType(n) for n in names}

    class _Base:
        def __init__(self, *a, **k):
            pass

    class StandardCombineInput:
        def __init__(self, hidden_states):
            self.hidden_states = hidden_states

    bc = mods["sglang.srt.layers.quantization.base_config"]
    bc.LinearMethodBase = bc.QuantizationConfig = bc.FusedMoEMethodBase = _Base
    mods["sglang.srt.utils.common"].set_weight_attrs = lambda p, attrs: None
    mods["sglang.srt.layers.moe.token_dispatcher.standard"].StandardCombineInput = StandardCombineInput
    sys.modules.update(mods)
    try:
        spec = importlib.util.spec_from_file_location("reference_sglang_plugin_tier", PLUGIN)
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        m.classes()
        yield m
    finally:
        for n, v in saved.items():
            if v is None:
                sys.modules.pop(n, None)
            else:
                sys.modules[n] = v


@pytest.fixture
def env(plugin, monkeypatch):
    fake = FakeOps()
    monkeypatch.setattr(moe_offload, "ops", lambda: fake)
    monkeypatch.setattr(torch.xpu, "is_current_stream_capturing", lambda: False, raising=False)
    for name, v in (("_NVTIER", None), ("_MOE_CACHE", False), ("_STAGE_MIN_M", 512)):
        monkeypatch.setattr(plugin, name, v)
    for v in ("EXL3_NVTIER_PREFILL_M", "EXL3_NVTIER_STAGE", "EXL3_NVTIER_STAGE_M"):
        monkeypatch.delenv(v, raising=False)
    store = RecordingStore(H, 32, 3, E, 4, device="cpu", max_layers=L)
    method = plugin.Exl3XpuMoEMethod("model.layers.3.mlp.experts", {})
    mtp = plugin.Exl3XpuMoEMethod("mtp.layers.0.mlp.experts", {})
    for n, key in enumerate([method.key, mtp.key]):
        blobs = torch.arange(E * BLOB, dtype=torch.int64).view(E, BLOB).add(31 * n).remainder(251).to(torch.uint8)
        store.add_layer(key, blobs)
    store.make_resident(method.key, [1, 4])
    store.log.clear()
    return plugin, store, method, mtp


def _call(method, store, rows, shape=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*(shape or (rows, H)), generator=g).to(torch.bfloat16)
    n = x.numel() // H
    ids = torch.stack([torch.randperm(E, generator=g)[:2] for _ in range(n)]).to(torch.int32)
    w = torch.rand(n, 2, generator=g)
    layer = types.SimpleNamespace(exl3_moe_store=store)
    topk = types.SimpleNamespace(topk_ids=ids.view(*x.shape[:-1], 2), topk_weights=w.view(*x.shape[:-1], 2))
    res = method.apply(layer, types.SimpleNamespace(hidden_states=x, topk_output=topk))
    ref = ExpertStore.forward(store, method.key, x.reshape(n, H), ids, w, ptrs=torch.tensor(
        store._host_ptr[method.key].tolist(), dtype=torch.int64))
    return res.hidden_states, x, ref.view_as(x)


def test_decode_goes_to_forward_or_the_cache(env):
    plugin, store, method, _ = env
    y, x, ref = _call(method, store, 2)
    assert [c[0] for c in store.log] == ["prefill_reset", "forward"] and y.shape == x.shape and torch.equal(y, ref)
    store.log.clear()
    plugin._MOE_CACHE = True
    y, x, ref = _call(method, store, 3, seed=1)
    assert [c[0] for c in store.log] == ["prefill_reset", "forward_cached"] and torch.equal(y, ref)


def test_prefill_streams_at_the_staging_threshold_except_mtp(env):
    plugin, store, method, mtp = env
    y, x, ref = _call(method, store, 511, seed=2)
    assert store.log[-1][0] == "forward" and torch.equal(y, ref)
    y, x, ref = _call(method, store, 512, seed=3)
    assert store.log[-1] == ("forward_prefill_staged", method.key, 512) and torch.equal(y, ref)
    y, x, _ = _call(method, store, 8, shape=(2, 300, H), seed=4)   # [batch, seq, H]: rows are flattened
    assert store.log[-1] == ("forward_prefill_staged", method.key, 600) and y.shape == x.shape
    store.log.clear()
    mtp_layer = types.SimpleNamespace(exl3_moe_store=store)
    xm = torch.randn(600, H).to(torch.bfloat16)
    ids = torch.zeros(600, 2, dtype=torch.int32)
    out = mtp.apply(mtp_layer, types.SimpleNamespace(hidden_states=xm, topk_output=types.SimpleNamespace(
        topk_ids=ids, topk_weights=torch.ones(600, 2))))
    assert [c[0] for c in store.log] == ["prefill_reset", "forward"] and out.hidden_states.shape == xm.shape


def test_tier_mode_prefill_fills_ram_first_or_stages(env, monkeypatch):
    """Tier on: a batch of >= EXL3_NVTIER_PREFILL_M rows makes its experts RAM-resident first (TierHost through
    TierDriver.ensure_for_prefill, with the plugin's arguments), then forward; with EXL3_NVTIER_STAGE=1 a batch of
    >= EXL3_NVTIER_STAGE_M rows goes to stage_forward; decode batches go to the cache as without the tier."""
    plugin, store, method, _ = env
    li = store.layer_index[method.key]
    ram_res = torch.zeros(L * E, dtype=torch.uint8)
    ring = torch.zeros(1 + 16, dtype=torch.int32)
    fetched = []
    host = TierHost(ram_res, ring, store.slot_of_dev, budget=L * E,
                    fetch=lambda k: (fetched.append(k), host.fill_done(k)))
    stager = FakeStager(store)
    plugin._NVTIER = TierDriver(host, stager)
    y, x, ref = _call(method, store, 5, seed=5)
    assert store.log[-1] == ("forward", method.key, 5) and torch.equal(y, ref)
    picked = sorted(set(fetched))
    assert picked and all(k // E == li for k in picked)                      # this layer's keys only
    assert all(int(ram_res[k]) == 1 for k in picked)                         # flagged RAM-resident before forward
    monkeypatch.setenv("EXL3_NVTIER_STAGE", "1")
    monkeypatch.setenv("EXL3_NVTIER_STAGE_M", "256")
    y, x, ref = _call(method, store, 300, seed=6)
    assert stager.calls[-1] == (method.key, 300) and torch.equal(y, ref)
    store.log.clear()
    plugin._MOE_CACHE = True
    y, x, ref = _call(method, store, 2, seed=7)                              # decode: below the tier prefill rows
    assert [c[0] for c in store.log] == ["prefill_reset", "forward_cached"] and torch.equal(y, ref)
