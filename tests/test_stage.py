"""CPU: exl3b200.stage.StoreStager (prefill with the experts streamed from the packed store, the reference's
NvTier.stage_forward) on CPU tensors with the byte-reading fake ops of test_expert_store.py: records are read by
reader threads from a real store file, copied to the staging buffers, and every pick reads its expert's bytes
through the table the stager builds."""
import numpy as np
import pytest
import torch

from exl3b200 import moe_offload, pack_store as P
from exl3b200.moe_offload import ExpertStore
from exl3b200.stage import StoreStager
from test_expert_store import BLOB, FakeOps

E, L = 8, 4


def _rec(layer, e):
    return np.random.default_rng(50 * layer + e).integers(0, 256, BLOB, dtype=np.uint8)


@pytest.fixture
def setup(tmp_path, monkeypatch):
    fake = FakeOps()
    monkeypatch.setattr(moe_offload, "ops", lambda: fake)
    keys = ["model.layers.2.mlp", "model.layers.0.mlp", "model.layers.3.mlp", "model.layers.1.mlp"]
    st = ExpertStore(64, 32, 3, E, 4, device="cpu", max_layers=L)
    for key in keys:
        st.add_layer(key)                              # host rows left empty: only the store file has the data
    row = {key: i for i, key in enumerate(keys)}
    P.pack(str(tmp_path), P.StoreMeta.for_blob(L, E, 3, BLOB, 64, 32), lambda layer, e: _rec(layer, e).tobytes())
    reader = P.StoreReader(str(tmp_path))
    yield st, keys, row, reader, fake
    reader.close()


def test_stage_forward_reads_every_expert_from_the_store(setup):
    st, keys, row, reader, fake = setup
    for key in keys:                                   # VRAM holds two experts of layer 0 (copied by hand here)
        if key == "model.layers.0.mlp":
            for e in (1, 6):
                st.host[key][e] = torch.from_numpy(_rec(row[key], e))
            st.make_resident(key, [1, 6])
    stager = StoreStager(st, reader, read_ahead=2, threads=3)
    order = ["model.layers.0.mlp", "model.layers.1.mlp", "model.layers.2.mlp", "model.layers.3.mlp"]
    rng = np.random.default_rng(0)
    for rep in range(2):
        for key in order:
            ids = torch.from_numpy(rng.integers(0, E, (5, 3)).astype(np.int32))
            y = stager.stage_forward(key, torch.zeros(5, 64), ids, torch.ones(5, 3))
            want = np.stack([_rec(row[key], e) for e in ids.reshape(-1).tolist()])
            assert np.array_equal(y.numpy(), want), (rep, key)
    assert stager.stats["layers"] == 8 and stager.stats["records"] == 2 * (4 * E - 2)   # VRAM experts not read
    stager.close()


def test_stage_forward_resyncs_when_a_layer_is_skipped(setup):
    st, keys, row, reader, fake = setup
    stager = StoreStager(st, reader, read_ahead=1, threads=2)
    for key in ["model.layers.0.mlp", "model.layers.2.mlp", "model.layers.3.mlp"]:   # layer 1 not called
        ids = torch.tensor([[0, 7], [3, 3]], dtype=torch.int32)
        y = stager.stage_forward(key, torch.zeros(2, 64), ids, torch.ones(2, 2))
        assert np.array_equal(y.numpy(), np.stack([_rec(row[key], e) for e in (0, 7, 3, 3)]))
    stager.close()


def test_stager_checks_the_store_file(setup, tmp_path):
    st, keys, row, reader, fake = setup
    other = tmp_path / "other"
    P.pack(str(other), P.StoreMeta.for_blob(L, E + 1, 3, BLOB, 64, 32), lambda layer, e: _rec(layer, e).tobytes())
    r2 = P.StoreReader(str(other))
    with pytest.raises(RuntimeError, match="holds E=9"):
        StoreStager(st, r2)
    r2.close()


def test_tier_driver_takes_the_plugin_calls(setup):
    """The plugin's calls, tier.stage_forward(store, key, li, x, ids, w) and tier.step(), reach the stager and the
    host loop."""
    from exl3b200.stage import TierDriver
    st, keys, row, reader, fake = setup

    class Host:
        steps = 0
        calls = []

        def step(self):
            Host.steps += 1
            return 0

        def ensure_for_prefill(self, li, ids, n_experts):
            Host.calls.append(("ensure", li, n_experts))
            return 0

        def warm(self, keys, max_keys=None):
            Host.calls.append(("warm", keys, max_keys))
            return len(keys)

        def log_stats(self, logger, every=200):
            Host.calls.append(("log", every))

    drv = TierDriver(Host(), StoreStager(st, reader, read_ahead=1, threads=2))
    ids = torch.tensor([[2, 5]], dtype=torch.int32)
    key = "model.layers.0.mlp"
    y = drv.stage_forward(st, key, st.layer_index[key], torch.zeros(1, 64), ids, torch.ones(1, 2))
    assert np.array_equal(y.numpy(), np.stack([_rec(row[key], 2), _rec(row[key], 5)]))
    assert drv.step() == 0 and Host.steps == 1
    drv.ensure_for_prefill(1, ids)
    n, secs = drv.warm([2 * E + 3, 1 * E + 0, 9 * E], 3 * BLOB)     # file layer = store row by default; 9 is none
    drv.log_stats(None, 50)
    assert Host.calls == [("ensure", 1, E), ("warm", [2 * E + 3, 1 * E + 0], 3), ("log", 50)] and n == 2
    with pytest.raises(RuntimeError, match="not a layer"):
        drv.stage_forward(st, key, st.layer_index[key] + 1, torch.zeros(1, 64), ids, torch.ones(1, 2))
    drv.stager.close()
