"""CPU: EXL3 checkpoints into the store (exl3b200.checkpoint) and the packed expert store on disk
(exl3b200.pack_store), on a small synthetic checkpoint (H = I = 128, 4 experts, 2 layers + an MTP layer, K = 3).

The checkpoint files are written by the safetensors library itself (when installed) and by a minimal writer of the
published format, and read back by this build's own header parser.  The store's host arenas are CPU tensors (fake
ops, as in test_expert_store.py)."""
import json
import mmap
import os
import struct
import time

import numpy as np
import pytest
import torch

from exl3b200 import checkpoint as C
from exl3b200 import moe_offload, pack_store as P, synth
from exl3b200.moe_offload import ExpertStore, pack_expert
from exl3b200.tier import TierHost

H = I = 128
E, L, K = 4, 2, 3


class FakeOps:
    def blob_bytes(self, H, I, K):
        return synth.blob_geometry(H, I, K, K, K)["blob"]

    def host_alloc(self, n):
        return torch.zeros(n, dtype=torch.uint8)


@pytest.fixture
def fake(monkeypatch):
    monkeypatch.setattr(moe_offload, "ops", lambda: FakeOps())


def _proj(g, k, n, K):
    return {"trellis": torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, generator=g),
            "suh": (torch.randint(0, 2, (k,), generator=g) * 2 - 1).half(),
            "svh": (torch.rand(n, generator=g) + 0.5).half()}


def _experts(seed=0, Kd=K):
    """{(mtp, layer, e): {role: {part: tensor}}}"""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for mtp, layer in [(False, 0), (False, 1), (True, 0)]:
        for e in range(E):
            out[(mtp, layer, e)] = {"gate": _proj(g, H, I, K), "up": _proj(g, H, I, K), "down": _proj(g, I, H, Kd)}
    return out


def _tensors(experts, codebook="mul1", prefix="model.language_model."):
    t = {}
    for (mtp, layer, e), roles in experts.items():
        base = f"{'mtp.' if mtp else prefix}layers.{layer}.mlp.experts.{e}"
        for role, parts in roles.items():
            for part, v in parts.items():
                t[f"{base}.{role}_proj.{part}"] = v
            if codebook:
                t[f"{base}.{role}_proj.{codebook}"] = torch.zeros((), dtype=torch.int32)
    g = torch.Generator().manual_seed(99)
    attn = _proj(g, H, 256, 4)
    for part, v in attn.items():
        t[f"{prefix}layers.0.self_attn.q_proj.{part}"] = v
    t[f"{prefix}layers.0.self_attn.q_proj.mcg"] = torch.zeros((), dtype=torch.int32)
    t[f"{prefix}embed_tokens.weight"] = torch.randn(8, H, generator=g).to(torch.bfloat16)
    return t


_CODE = {torch.int16: "I16", torch.float16: "F16", torch.bfloat16: "BF16", torch.int32: "I32", torch.float32: "F32"}


def _write_plain(path, tensors):
    """The published safetensors layout: u64 header length, JSON header, data region."""
    header, blobs, o = {"__metadata__": {"format": "pt"}}, [], 0
    for name, v in tensors.items():
        raw = v.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()
        header[name] = {"dtype": _CODE[v.dtype], "shape": list(v.shape), "data_offsets": [o, o + len(raw)]}
        blobs.append(raw)
        o += len(raw)
    text = json.dumps(header).encode()
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)) + text + b"".join(blobs))


def _write_library(path, tensors):
    st = pytest.importorskip("safetensors.torch")
    st.save_file({k: v.contiguous() for k, v in tensors.items()}, path, metadata={"format": "pt"})


def _checkpoint(dirpath, tensors, writer=_write_plain):
    """Two files plus model.safetensors.index.json."""
    names = sorted(tensors)
    parts = {"model-00001-of-00002.safetensors": names[::2], "model-00002-of-00002.safetensors": names[1::2]}
    weight_map = {}
    for fn, ns in parts.items():
        writer(os.path.join(dirpath, fn), {n: tensors[n] for n in ns})
        weight_map.update({n: fn for n in ns})
    with open(os.path.join(dirpath, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    return str(dirpath)


@pytest.mark.parametrize("writer", [_write_plain, _write_library])
def test_reader_returns_the_written_tensors(tmp_path, writer):
    tensors = _tensors(_experts())
    ck = C.Checkpoint(_checkpoint(tmp_path, tensors, writer))
    assert set(ck.tensors) == set(tensors)
    for name, v in tensors.items():
        got = ck.get(name)
        assert got.dtype == v.dtype and got.shape == v.shape and torch.equal(got, v), name


def test_scan_reads_geometry_and_codebook_from_headers(tmp_path):
    geo = C.scan_checkpoint(_checkpoint(tmp_path, _tensors(_experts())))
    assert geo["layers.1.mlp.experts.3.down_proj"] == (I, H, K, C.CODEBOOK["mul1"])
    assert geo["mtp.layers.0.mlp.experts.0.gate_proj"] == (H, I, K, C.CODEBOOK["mul1"])
    assert geo["layers.0.self_attn.q_proj"] == (H, 256, 4, C.CODEBOOK["mcg"])
    assert len(geo) == 3 * E * 3 + 1
    assert C.module_key("model.layers.3.mlp.experts") == "layers.3.mlp.experts"
    assert C.module_key("model.mtp.layers.0.mlp") == "mtp.layers.0.mlp"
    assert C.module_key("lm_head") == "lm_head"


def test_load_experts_packs_every_expert(tmp_path, fake):
    experts = _experts()
    model = _checkpoint(tmp_path, _tensors(experts))
    st = ExpertStore(H, I, K, E, 0, device="cpu", max_layers=4)
    keys = C.load_experts(model, st)
    assert keys == ["layers.0.mlp.experts", "layers.1.mlp.experts", "mtp.layers.0.mlp.experts"]
    for (mtp, layer, e), roles in experts.items():
        want = pack_expert(roles["gate"], roles["up"], roles["down"], K)
        assert torch.equal(st.host_view(C.layer_key(mtp, layer))[e], want), (mtp, layer, e)
    st2 = ExpertStore(H, I, K, E, 0, device="cpu", max_layers=4)
    assert C.load_experts(model, st2, mtp=False) == keys[:2]


def test_packer_takes_tensors_in_any_order_and_refuses_duplicates(fake):
    experts = _experts(seed=5)
    st = ExpertStore(H, I, K, E, 0, device="cpu", max_layers=1)
    st.add_layer("layers.0.mlp.experts")
    geo = {(r, e): ((H, I) if r != "down" else (I, H)) + (K, C.CODEBOOK["mul1"]) for r in ("gate", "up", "down")
           for e in range(E)}
    pk = C.ExpertPacker(st, "layers.0.mlp.experts", geo)
    items = [(e, r, p, experts[(False, 0, e)][r][p]) for e in range(E) for r in ("gate", "up", "down")
             for p in ("trellis", "suh", "svh")]
    for i in np.random.default_rng(0).permutation(len(items)):
        pk.add(*items[i])
        assert len(pk.pending) <= E
    pk.finish()
    for e in range(E):
        ex = experts[(False, 0, e)]
        assert torch.equal(st.host_view("layers.0.mlp.experts")[e], pack_expert(ex["gate"], ex["up"], ex["down"], K))
    pk2 = C.ExpertPacker(st, "layers.0.mlp.experts", geo)
    pk2.add(*items[0])
    with pytest.raises(ValueError, match="twice"):
        pk2.add(*items[0])
    with pytest.raises(ValueError, match="incomplete"):
        pk2.finish()


def _subdir(tmp_path, name):
    (tmp_path / name).mkdir()
    return tmp_path / name


def test_refusals(tmp_path, fake):
    wrong_cb = _checkpoint(_subdir(tmp_path, "cb"), _tensors(_experts(), codebook="mcg"))
    with pytest.raises(ValueError, match="mul1"):
        C.load_experts(wrong_cb, ExpertStore(H, I, K, E, 0, device="cpu", max_layers=4))
    mixed = _checkpoint(_subdir(tmp_path, "mixed"), _tensors(_experts(Kd=4)))
    with pytest.raises(NotImplementedError, match="K"):
        C.load_experts(mixed, ExpertStore(H, I, K, E, 0, device="cpu", max_layers=4))
    ok = _checkpoint(_subdir(tmp_path, "ok"), _tensors(_experts()))
    with pytest.raises(ValueError, match="needs mul1 and"):
        C.load_experts(ok, ExpertStore(H, 256, K, E, 0, device="cpu", max_layers=4))   # store of another I


# ------------------------------------------------------------------------------------------------ pack store
def _store_dir(tmp_path):
    experts = _experts(seed=11)
    model = _checkpoint(_subdir(tmp_path, "model"), _tensors(experts))
    return model, str(tmp_path / "store"), experts


def test_pack_layout_and_verify(tmp_path):
    model, out, experts = _store_dir(tmp_path)
    meta, blob_of = P.checkpoint_source(model)
    blob = synth.blob_geometry(H, I, K, K, K)["blob"]
    assert meta == P.StoreMeta(L, E, K, blob, -(-blob // 4096) * 4096, H, I)
    assert P.pack(out, meta, blob_of)
    raw = open(os.path.join(out, P.BIN), "rb").read()
    assert len(raw) == L * E * meta.rec and meta.rec % 4096 == 0
    assert json.load(open(os.path.join(out, P.META))) == {"L": L, "E": E, "K": K, "blob": blob, "rec": meta.rec,
                                                           "H": H, "I": I}
    for layer in range(L):
        for e in range(E):
            ex = experts[(False, layer, e)]
            o = (layer * E + e) * meta.rec
            assert raw[o:o + blob] == pack_expert(ex["gate"], ex["up"], ex["down"], K).numpy().tobytes()
            assert raw[o + blob:o + meta.rec] == bytes(meta.rec - blob)
    assert P.verify(out, blob_of, n=32) == 0
    mtime = os.path.getmtime(os.path.join(out, P.BIN))
    assert not P.pack(out, meta, blob_of)                   # complete: kept
    assert os.path.getmtime(os.path.join(out, P.BIN)) == mtime
    os.remove(os.path.join(out, P.BIN + ".done"))            # incomplete: rebuilt as a whole
    assert not P.is_complete(out)
    assert P.pack(out, meta, blob_of) and P.is_complete(out)
    os.truncate(os.path.join(out, P.BIN), meta.size - meta.rec)   # marker present, file short: not a store
    assert not P.is_complete(out)
    with pytest.raises(RuntimeError, match="no complete store"):
        P.StoreReader(out)
    assert P.pack(out, meta, blob_of) and P.verify(out, blob_of, n=16) == 0


def test_verify_finds_a_corrupt_record(tmp_path):
    model, out, _ = _store_dir(tmp_path)
    meta, blob_of = P.checkpoint_source(model)
    P.pack(out, meta, blob_of)
    with open(os.path.join(out, P.BIN), "r+b") as f:
        f.seek(5 * meta.rec + 1000)
        b = f.read(1)
        f.seek(5 * meta.rec + 1000)
        f.write(bytes([b[0] ^ 0x40]))
    assert P.verify(out, blob_of, n=64) >= 1


@pytest.mark.parametrize("direct", [False, None])
def test_reader_paths(tmp_path, direct):
    model, out, _ = _store_dir(tmp_path)
    meta, blob_of = P.checkpoint_source(model)
    P.pack(out, meta, blob_of)
    rd = P.StoreReader(out, direct=direct)
    try:
        assert P.probe(out)["store"].endswith(P.BIN)
        page = mmap.mmap(-1, meta.rec)                            # page-aligned: read in place under O_DIRECT
        aligned = torch.from_numpy(np.frombuffer(page, dtype=np.uint8))
        odd = torch.zeros(meta.blob + 64, dtype=torch.uint8)[3:3 + meta.blob]   # unaligned: bounce buffer
        for key in range(L * E):
            want = np.frombuffer(blob_of(key // E, key % E), dtype=np.uint8)
            for out_t in (aligned, odd):
                out_t.zero_()
                rd.read(key, out_t)
                assert np.array_equal(out_t.numpy()[:meta.blob], want), (key, direct)
        with pytest.raises(IndexError):
            rd.read(L * E, aligned)
        del aligned
    finally:
        rd.close()


def test_fetcher_fills_the_ram_tier(tmp_path):
    """TierHost's fetch() served by the store: masked misses are read into their host slots by the reader threads,
    reported with fill_done, and become resident with the record's bytes."""
    model, out, _ = _store_dir(tmp_path)
    meta, blob_of = P.checkpoint_source(model)
    P.pack(out, meta, blob_of)
    n = L * E
    arena = torch.zeros(n, meta.rec, dtype=torch.uint8)             # the RAM tier's host slots
    ram_res = torch.zeros(n, dtype=torch.uint8)
    ring = torch.zeros(1 + 8, dtype=torch.int32)
    slot_of = torch.full((n,), -1, dtype=torch.int32)
    rd = P.StoreReader(out)
    with P.StoreFetcher(rd, dest=lambda key: arena[key], done=lambda key: tier.fill_done(key), threads=3) as fetcher:
        tier = TierHost(ram_res, ring, slot_of, budget=n, fetch=fetcher.fetch)
        tier.step()
        for i, key in enumerate([6, 2, 7, 2]):                 # what a decode step logs for its masked picks
            ring[1 + i % 8] = key
            ring[0] = i + 1
        deadline = time.time() + 10
        while ram_res[[2, 6, 7]].sum() < 3 and time.time() < deadline:
            tier.step()
            time.sleep(0.01)
    rd.close()
    assert ram_res.nonzero().flatten().tolist() == [2, 6, 7] and tier.stats["fetches"] == 3
    for key in (2, 6, 7):
        assert np.array_equal(arena[key][:meta.blob].numpy(), np.frombuffer(blob_of(key // E, key % E), np.uint8))


def test_cli(tmp_path, capsys):
    model, out, _ = _store_dir(tmp_path)
    assert P.main(["probe", "--out", out]) == 1                    # no store yet
    assert P.main(["pack", "--model", model, "--out", out]) == 0
    assert P.main(["verify", "--model", model, "--out", out]) == 0
    assert P.main(["probe", "--out", out]) == 0
    lines = [json.loads(s) for s in capsys.readouterr().out.splitlines()]
    assert lines[-1]["store"].endswith(P.BIN) and lines[-2]["verify_bad"] == 0
