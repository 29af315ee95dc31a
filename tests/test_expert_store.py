"""CPU: ExpertStore's host bookkeeping (exl3b200.moe_offload) on CPU tensors, against a fake op namespace.

The store's device state is plain CPU tensors here; the fake ops do what the CUDA ops do to memory: memcpy_async is
a real memmove between the host arenas, the slot arena and the staging buffers, and moe_forward reads each pick's
blob through the pointer table it is given.  So every check below reads the bytes a kernel would read.  The CUDA
path (the same code with CUDA tensors and streams) is covered by the GPU parity tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from exl3b200 import moe_offload
from exl3b200.moe_offload import ExpertStore

BLOB = 96


class FakeOps:
    def __init__(self):
        self.copies = []          # (dst, src, nbytes)

    def blob_bytes(self, H, I, K):
        return BLOB

    def host_alloc(self, n):
        return torch.zeros(n, dtype=torch.uint8)

    def memcpy_async(self, dst, src, n):
        ctypes.memmove(dst, src, n)
        self.copies.append((dst, src, n))

    def moe_forward(self, x, ids, w, ptrs, I, K, E):
        """Bytes of every pick's blob, read through the table: [picks, BLOB]."""
        ptrs = ptrs.tolist()
        return torch.stack([torch.frombuffer(bytearray(ctypes.string_at(ptrs[e], BLOB)), dtype=torch.uint8)
                            for e in ids.flatten().tolist()])

    def moe_forward_cached(self, x, ids, w, ptrs_all, layer, slot_of, slot_key, slot_last, tick, host_base,
                           slot_base, fill_all, fill_list, max_fill, I, K, E, pend, done_seq):
        """Stand-in for the device cache step: each missed pick takes the lowest free slot, else the least recently
        used one, whose expert is pointed back at its host copy."""
        for e in ids.flatten().tolist():
            code = layer * E + e
            if slot_of[code] >= 0:
                slot_last[slot_of[code]] = int(tick[0]) + 1
                continue
            free = (slot_key < 0).nonzero().flatten()
            s = int(free[0]) if free.numel() else int(torch.argmin(slot_last))
            old = int(slot_key[s])
            if old >= 0:
                slot_of[old] = -1
                ptrs_all[old] = int(host_base[old // E]) + (old % E) * BLOB
            ctypes.memmove(slot_base + s * BLOB, int(ptrs_all[code]), BLOB)
            ptrs_all[code] = slot_base + s * BLOB
            slot_of[code] = s
            slot_key[s] = code
            slot_last[s] = int(tick[0]) + 1   # this call's tick: its own picks are not evicted
        tick += 1
        return self.moe_forward(x, ids, w, ptrs_all[layer * E:(layer + 1) * E], I, K, E)


@pytest.fixture
def fake(monkeypatch):
    f = FakeOps()
    monkeypatch.setattr(moe_offload, "ops", lambda: f)
    return f


def _store(E=8, S=4, L=3, keys=None):
    st = ExpertStore(64, 32, 3, E, S, device="cpu", max_layers=L)
    keys = keys if keys is not None else [f"model.layers.{i}.mlp" for i in range(L)]
    for n, key in enumerate(keys):
        blobs = torch.arange(E * BLOB, dtype=torch.int64).view(E, BLOB).add(997 * n).remainder(251).to(torch.uint8)
        st.add_layer(key, blobs)
    return st, keys


def _reads(st, ptr):
    return torch.frombuffer(bytearray(ctypes.string_at(int(ptr), BLOB)), dtype=torch.uint8)


def _check_tables(st):
    """Every table entry reads its own expert's bytes; the device slot map, slot keys and the mirror agree."""
    for key, li in st.layer_index.items():
        for e in range(st.E):
            assert torch.equal(_reads(st, st.ptrs(key)[e]), st.host[key][e]), (key, e)
            s = int(st.slot_of_dev[li * st.E + e])
            assert s == int(st.slot_of[key][e])
            if s >= 0:
                assert int(st.ptrs(key)[e]) == st.slot_ptr(s)
                assert int(st.slot_key[s]) == li * st.E + e
            else:
                assert int(st.ptrs(key)[e]) == int(st._host_ptr[key][e])


def test_s64_and_routing_conversion(fake):
    assert moe_offload.s64((1 << 64) - 5) == -5 and moe_offload.s64(7) == 7
    ids = torch.zeros(2, 3, dtype=torch.int32)
    w = torch.zeros(2, 3, dtype=torch.float32)
    a, b = ExpertStore._rt(ids, w)
    assert a is ids and b is w                       # in-place rewrites by the cached op reach the caller
    a, b = ExpertStore._rt(torch.zeros(3, 2, dtype=torch.int64).t(), torch.zeros(3, 2, dtype=torch.float16).t())
    assert a.dtype == torch.int32 and a.is_contiguous() and b.dtype == torch.float32 and b.is_contiguous()
    a, _ = ExpertStore._rt(torch.zeros(3, 2, dtype=torch.int32).t(), w)
    assert a.is_contiguous()


def test_add_layer_points_tables_at_host(fake):
    st, keys = _store()
    assert st.blob == BLOB and st.slots.shape == (4, BLOB)
    for li, key in enumerate(keys):
        assert st.layer_index[key] == li
        assert int(st.host_base[li]) == st.host[key].data_ptr()
        assert torch.equal(st.slot_of[key], torch.full((8,), -1, dtype=torch.int32))
    _check_tables(st)
    with pytest.raises(RuntimeError, match="max_layers"):
        st.add_layer("model.layers.9.mlp")


def test_make_resident_and_evict(fake):
    st, keys = _store()
    assert st.make_resident(keys[1], [5, 2, 5]) == 2      # duplicates count once
    assert st.make_resident(keys[1], [2]) == 0            # already resident
    assert st.resident_count() == 2 and st.resident_count(keys[1]) == 2 and st.device_resident_count(keys[1]) == 2
    assert st.slot_of[keys[1]][5] == 0 and st.slot_of[keys[1]][2] == 1   # lowest free slot first
    assert st.free_slots == [2, 3] and st.slot_owner[:2] == [(keys[1], 5), (keys[1], 2)]
    assert int(st.slot_last[0]) == 0 and int(st.slot_last[2]) == -1
    _check_tables(st)
    with pytest.raises(RuntimeError, match="free slots"):
        st.make_resident(keys[0], [0, 1, 3])               # three for two: nothing changes
    assert st.resident_count(keys[0]) == 0 and st.free_slots == [2, 3]
    st.evict(keys[1], [5, 7])                              # 7 is not resident
    assert st.slot_of[keys[1]][5] == -1 and st.free_slots == [0, 2, 3]
    assert int(st.slot_key[0]) == -1 and int(st.slot_last[0]) == -1
    assert st.make_resident(keys[0], [0, 1, 3]) == 3       # the freed slot is reused
    assert st.slot_of[keys[0]].tolist()[:4] == [0, 2, -1, 3]
    _check_tables(st)


def test_stage_layer_copies_runs_and_points_residents_at_slots(fake):
    st, keys = _store(E=10, S=4)
    st.make_resident(keys[2], [3, 7])
    fake.copies.clear()
    table = st.stage_layer(keys[2], 1, None)
    base = st._stage[1].data_ptr()
    runs = sorted(((d - base) // BLOB, n // BLOB) for d, _, n in fake.copies)
    assert runs == [(0, 3), (4, 3), (8, 2)]                # experts 0-2, 4-6, 8-9: one copy per run
    for e in range(10):
        assert torch.equal(_reads(st, table[e]), st.host[keys[2]][e])
        s = int(st.slot_of[keys[2]][e])
        assert int(table[e]) == (st.slot_ptr(s) if s >= 0 else base + e * BLOB)


def test_prefill_staged_streams_layers_in_model_order(fake):
    keys = ["model.layers.2.mlp", "mtp.layers.0.mlp", "model.layers.0.mlp", "model.layers.1.mlp"]
    st, keys = _store(E=8, S=4, L=4, keys=keys)
    st.make_resident("model.layers.1.mlp", [1, 6])
    order = ["model.layers.0.mlp", "model.layers.1.mlp", "model.layers.2.mlp"]
    x = torch.zeros(5, 64)
    staged_into = []                                       # (layer, buffer) per staging, from the copy log
    for rep in range(2):
        for n, key in enumerate(order):
            ids = torch.randint(0, 8, (5, 3), generator=torch.Generator().manual_seed(10 * rep + n), dtype=torch.int32)
            fake.copies.clear()
            y = st.forward_prefill_staged(key, x, ids, torch.ones(5, 3))
            assert torch.equal(y, st.host[key][ids.flatten().long()]), (rep, key)
            for d, s, _ in fake.copies:
                src = next(k for k in keys if st.host[k].data_ptr() <= s < st.host[k].data_ptr() + 8 * BLOB)
                buf = next(b for b in (0, 1) if st._stage[b] is not None and
                           st._stage[b].data_ptr() <= d < st._stage[b].data_ptr() + 8 * BLOB)
                if (src, buf) not in staged_into[-1:]:
                    staged_into.append((src, buf))
    # layer 0 on demand into buffer 0, then each call stages the next layer (wrapping) into the other buffer; the
    # second pass finds layer 0 already staged by the last layer of the first
    assert staged_into == [(order[0], 0), (order[1], 1), (order[2], 0), (order[0], 1), (order[1], 0), (order[2], 1),
                           (order[0], 0)]


def test_cached_calls_move_slots_and_static_ops_resync(fake):
    st, keys = _store(E=8, S=4)
    x = torch.zeros(1, 64)
    y = st.forward_cached(keys[0], x, torch.tensor([[4, 6]], dtype=torch.int32), torch.ones(1, 2))
    assert torch.equal(y, st.host[keys[0]][[4, 6]])
    assert st.resident_count(keys[0]) == 0                 # the mirror is stale until a static op re-reads it
    st.make_resident(keys[1], [0])                         # re-reads first: slots 0 and 1 are taken on the device
    assert st.slot_of[keys[0]].tolist()[4] == 0 and st.slot_of[keys[0]].tolist()[6] == 1
    assert st.slot_of[keys[1]][0] == 2 and st.free_slots == [3]
    _check_tables(st)
    # a staged prefill after cached calls re-reads the placement at its first layer
    st.forward_cached(keys[2], x, torch.tensor([[5]], dtype=torch.int32), torch.ones(1, 1))
    ids = torch.tensor([[5, 4]], dtype=torch.int32)
    y = st.forward_prefill_staged(keys[0], torch.zeros(1, 64), ids, torch.ones(1, 2))
    assert torch.equal(y, st.host[keys[0]][[5, 4]]) and st.slot_of[keys[2]][5] == 3
    st.reset_cache()
    assert st.resident_count() == 0 and st.free_slots == [0, 1, 2, 3]
    assert (st.slot_key < 0).all() and (st.slot_last < 0).all()
    _check_tables(st)


def test_prefill_drops_prestaged_tables_after_decode_moved_slots(fake):
    """The last layer of a prefill pass pre-stages the first layer, its table pointing at slots for resident experts.
    Decode then gives those slots to other experts; the next pass must re-read the placement and re-stage, not read
    the stale table."""
    st, keys = _store(E=8, S=2)
    st.make_resident(keys[0], [1, 2])
    x = torch.zeros(2, 64)
    ids = torch.tensor([[1, 2], [0, 5]], dtype=torch.int32)
    for key in keys:
        st.forward_prefill_staged(key, x, ids, torch.ones(2, 2))
    assert keys[0] in st._staging.staged                   # pre-staged by the last layer
    # decode as a CUDA graph replay runs it: the op alone, no store method (so only the cache tick shows the change)
    fake.moe_forward_cached(x[:1], torch.tensor([[3, 4]], dtype=torch.int32), torch.ones(1, 2), st.ptrs_all, 1,
                            st.slot_of_dev, st.slot_key, st.slot_last, st.tick, st.host_base, st.slot_base,
                            st.fill_all, st.fill_list, 8, st.I, st.K, st.E, st.pend, st.done_seq)
    assert st.slot_key.tolist() == [8 + 3, 8 + 4]          # layer 0's experts 1, 2 lost their slots
    y = st.forward_prefill_staged(keys[0], x, ids, torch.ones(2, 2))
    assert torch.equal(y, st.host[keys[0]][ids.flatten().long()])
    _check_tables(st)


def test_model_order():
    ks = ["model.layers.10.mlp", "mtp.layers.0.mlp", "other", "model.layers.2.mlp"]
    assert moe_offload._model_order(ks) == ["model.layers.2.mlp", "model.layers.10.mlp", "other"]


def test_pack_expert_into_buffer_checks_size():
    g = torch.Generator().manual_seed(3)

    def proj(k, n):
        return dict(trellis=torch.randint(-32768, 32767, (k // 16, n // 16, 48), dtype=torch.int16, generator=g),
                    suh=torch.ones(k, dtype=torch.float16), svh=torch.ones(n, dtype=torch.float16))
    gate, up, down = proj(64, 64), proj(64, 64), proj(64, 64)
    blob = moe_offload.pack_expert(gate, up, down, 3)
    out = torch.zeros(blob.numel(), dtype=torch.uint8)
    assert moe_offload.pack_expert(gate, up, down, 3, out=out) is out and torch.equal(out, blob)
    with pytest.raises(ValueError):
        moe_offload.pack_expert(gate, up, down, 3, out=torch.zeros(blob.numel() + 1, dtype=torch.uint8))
    assert np.array_equal(blob[-64 * 2:].numpy(), torch.ones(64, dtype=torch.float16).view(torch.uint8).numpy())


def test_copy_prefetch_guards(fake):
    """While the copy-engine prefetch worker runs, static placement and staged prefill are refused (their tables
    could point at a slot whose copy has not landed); planning needs a running worker."""
    st, keys = _store()
    with pytest.raises(RuntimeError, match="start_copy_prefetch first"):
        st.plan_prefetch(keys[0], torch.tensor([1], dtype=torch.int32))
    assert st.stop_copy_prefetch() == [0, 0]              # not running: nothing to stop
    st._cepf_stream = object()                             # as start_copy_prefetch leaves it
    for call in (lambda: st.make_resident(keys[0], [1]), lambda: st.evict(keys[0], [1]), st.reset_cache,
                 lambda: st.stage_layer(keys[0], 0, None),
                 lambda: st.forward_prefill_staged(keys[0], torch.zeros(1, 64), torch.zeros(1, 1, dtype=torch.int32),
                                                   torch.ones(1, 1))):
        with pytest.raises(RuntimeError, match="stop_copy_prefetch first"):
            call()


def test_copy_prefetch_worker_buffers_live_until_stop(monkeypatch):
    """The worker reads the plan buffer and writes the slot arena by address: the op layer keeps them (and the
    owner passed as `keep`) referenced until the stop, also when the stop reports a failed copy."""
    from exl3b200 import ops

    class FakeLib:
        def __init__(self, rc):
            self.rc = rc

        def exl3b_cepf_worker_start(self, *args):
            return 0

        def exl3b_cepf_worker_stop(self, counts):
            counts[0], counts[1] = 2, 5
            return self.rc

        def exl3b_last_error(self):
            return b"a copy failed"

    monkeypatch.setattr(ops, "stream", lambda dev=None: 0)
    for rc in (0, 2):
        monkeypatch.setattr(ops._lib, "lib", lambda rc=rc: FakeLib(rc))
        owner, plans, done = object(), torch.zeros(64, dtype=torch.uint8), torch.zeros(2, dtype=torch.int32)
        ops.moe_prefetch_worker_start(plans, torch.zeros(2, dtype=torch.int64), 0, 4096,
                                      torch.zeros(8, dtype=torch.int64), torch.zeros(4, dtype=torch.int32),
                                      torch.empty(0, dtype=torch.uint8), done, 2, 4, keep=owner)
        assert ops._worker_keep[0] is plans and ops._worker_keep[1] is done and ops._worker_keep[-1] is owner
        if rc == 0:
            assert ops.moe_prefetch_worker_stop() == [2, 5]
        else:
            with pytest.raises(RuntimeError, match="a copy failed"):
                ops.moe_prefetch_worker_stop()
        assert ops._worker_keep is None


def test_host_row_staging_refused_with_the_ram_tier(fake, monkeypatch):
    """With the RAM tier on, host rows may have been released: staging from them is refused (StoreStager reads the
    pack store instead)."""
    from exl3b200 import ops
    st, keys = _store()
    monkeypatch.setattr(ops.G, "ram_res", torch.ones(24, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="StoreStager"):
        st.stage_layer(keys[0], 0, None)
    with pytest.raises(RuntimeError, match="StoreStager"):
        st.forward_prefill_staged(keys[0], torch.zeros(1, 64), torch.zeros(1, 1, dtype=torch.int32), torch.ones(1, 1))
