"""CPU: pin the oracle's codec, layout and layer math to the reference's own statements and known answers.

The reference commits no golden vectors for the MoE path (its only harness, experimental/n111-victim-ring/
n111_test.py, needs the B70 and an external NVMe store).  What it does state, and what these tests check:
  - the mul1 codebook twice: vector form kernels/moe-a8/exl3_esimd.h:45-67 and scalar form
    kernels/moe-a8/exl3_moe.a8.sycl:1365-1377 (both restated below in numpy, independently of the C oracle);
  - the codebook bound kQ8WMax = 3.453125 (experimental/n111-victim-ring/csrc/exl3_ops.sycl:522-525);
  - the blob size 1,862,400 B at (H, I, K) = (2560, 640, 3) (kernels/moe-a8/exl3_moe.a8.sycl:7,
    experimental/n111-victim-ring/n111_test.py:21-23);
  - the word/shift form of tile_states (exl3_esimd.h:120-149) and the PLANAR4 view/permute of
    plugin/exl3xpu/moe_offload.py:68-73;
  - blobs packed by the reference's own pack_expert (plugin/exl3xpu/moe_offload.py:76-89), run on the CPU to make
    tests/golden/ref_pack.npz.
"""
import numpy as np
import pytest
import torch

import oracle as O
from exl3b200 import moe_offload, synth


def test_mul1_matches_both_reference_statements():
    tab = O.mul1_table()
    st = np.arange(65536, dtype=np.uint64)
    x = (st * 0x83DCD12D) & 0xFFFFFFFF
    bs = (x & 255) + ((x >> 8) & 255) + ((x >> 16) & 255) + (x >> 24)
    # vector form: h = fp16(0x6400 + bytesum) exact, w = fp16 fma(h, 0x1eee, 0xc931): one rounding of the exact value
    h = (1024 + bs).astype(np.float64)
    c1 = float(np.uint16(0x1EEE).view(np.float16))
    c2 = float(np.uint16(0xC931).view(np.float16))
    vec = (h * c1 + c2).astype(np.float16).view(np.uint16)
    # scalar form: fp32 hsum * k_inv + k_bias, then (half)
    scal = (h.astype(np.float32) * np.float32(c1) + np.float32(c2)).astype(np.float16).view(np.uint16)
    assert np.array_equal(tab, vec)
    assert np.array_equal(tab, scal)


def test_codebook_range_and_size():
    f = O.f16_bits_to_f32(O.mul1_table())
    assert float(np.abs(f).max()) == 3.453125          # kQ8WMax
    assert float(f.min()) == -3.453125 and float(f.max()) == 3.34765625
    assert len(np.unique(f)) == 913


def test_blob_sizes():
    assert O.blob_bytes(2560, 640, 3) == 1862400          # reference model (n111_test.py:21-23)
    assert O.blob_bytes(2048, 768, 3) == 1786368          # BASELINE shapes
    g = synth.blob_geometry(2048, 768, 3, 3, 3)
    assert g["blob"] == 1786368 and g["gu"] == 0 and g["d"] == 1179648


def test_tile_position_map_is_a_permutation():
    pos = {(O.lib().ora_tile_row(t), O.lib().ora_tile_col(t)) for t in range(256)}
    assert len(pos) == 256 and all(0 <= r < 16 and 0 <= c < 16 for r, c in pos)


def _tile_states_wordform(tw: np.ndarray, K: int) -> list:
    """exl3_esimd.h:120-149 restated per value: period g, value u; prev of period 0 = the tile's last word."""
    g_ = np.gcd(K, 32)
    D, V = K // g_, 32 // g_
    W = 8 * K
    out = []
    for t in range(256):
        grp, u = divmod(t, V)
        e = (u + 1) * K
        i1 = (e - 1) // 32
        b0 = e - 16
        i0 = b0 // 32 if b0 >= 0 else -1
        s = (i1 + 1) * 32 - e
        B = int(tw[D * grp + i1])
        if i0 == i1:
            st = B >> s
        else:
            A = int(tw[D * grp + i0]) if i0 >= 0 else int(tw[(D * grp - 1) % W])
            st = B if s == 0 else ((A << (32 - s)) | (B >> s))
        out.append(st & 0xFFFF)
    return out


@pytest.mark.parametrize("K", [2, 3, 4, 5])
def test_tile_state_bitform_equals_wordform(K):
    rng = np.random.default_rng(K)
    for _ in range(4):
        tw = rng.integers(0, 2 ** 32, size=8 * K, dtype=np.uint64).astype(np.uint32)
        wf = _tile_states_wordform(tw, K)
        bf = [O.lib().ora_tile_state(tw, K, t) for t in range(256)]
        assert wf == bf


@pytest.mark.parametrize("K", [3, 5])
def test_planar4_matches_reference_permute(K):
    # reference: w.view(r, n//4, 4, 8, K).permute(0, 1, 4, 2, 3) -> [row][group][plane][tile][period]
    r, n = 2, 8
    tr = torch.randint(-32768, 32767, (r, n, 16 * K), dtype=torch.int16)
    ref = tr.view(torch.int32).view(r, n // 4, 4, 8, K).permute(0, 1, 4, 2, 3).contiguous().view(r, -1)
    got = moe_offload.planar4(tr, K).view(r, -1)
    assert torch.equal(ref, got)
    words = tr.view(torch.int32).view(r, n, 8 * K)
    for j in range(4):
        for w in range(8 * K):
            assert int(got[0, O.lib().ora_planar_offset(K, j, w)]) == int(words[0, j, w])


@pytest.mark.parametrize("K", [2, 3, 4, 5])
def test_pack_round_trip_dequant(K):
    """checkpoint tensors -> pack_expert (blob) -> oracle dequant == oracle dequant of the checkpoint words."""
    H, I = 128, 128
    g = torch.Generator().manual_seed(K)
    def tens(k, n):
        return dict(trellis=torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, generator=g),
                    suh=torch.ones(k, dtype=torch.float16), svh=torch.ones(n, dtype=torch.float16))
    gate, up, down = tens(H, I), tens(H, I), tens(I, H)
    blob = moe_offload.pack_expert(gate, up, down, K).numpy()
    assert blob.size == O.blob_bytes(H, I, K)
    for proj, t, (k, n) in ((0, gate, (H, I)), (1, up, (H, I)), (2, down, (I, H))):
        words = t["trellis"].view(torch.int32).numpy().view(np.uint32).reshape(k // 16, -1)
        ref = O.dequant(words, k // 16, words.shape[1], 0, n // 16, K, False)
        got = O.blob_dequant(blob, H, I, K, K, K, proj)
        assert np.array_equal(ref, got)


def test_mixed_k_pack_round_trip():
    H, I = 128, 128
    ks = (2, 5, 4)
    g = torch.Generator().manual_seed(7)
    def tens(k, n, K):
        return dict(trellis=torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, generator=g),
                    suh=torch.ones(k, dtype=torch.float16), svh=torch.ones(n, dtype=torch.float16))
    gate, up, down = tens(H, I, ks[0]), tens(H, I, ks[1]), tens(I, H, ks[2])
    blob = moe_offload.pack_expert(gate, up, down, 0).numpy()
    assert blob.size == O.blob_bytes(H, I, *ks)
    for proj, t, (k, n), K in ((0, gate, (H, I), ks[0]), (1, up, (H, I), ks[1]), (2, down, (I, H), ks[2])):
        words = t["trellis"].view(torch.int32).numpy().view(np.uint32).reshape(k // 16, -1)
        ref = O.dequant(words, k // 16, words.shape[1], 0, n // 16, K, False)
        assert np.array_equal(ref, O.blob_dequant(blob, H, I, *ks, proj))


def test_fwht_matches_hadamard_matrix():
    Hm = np.array([[1.0]])
    while Hm.shape[0] < 128:
        Hm = np.block([[Hm, Hm], [Hm, -Hm]])
    v = np.random.default_rng(0).standard_normal(128).astype(np.float32)
    got = O.fwht128(v).astype(np.float64)
    ref = Hm @ v.astype(np.float64)
    assert np.allclose(got, ref, rtol=0, atol=1e-4)


def test_synth_blob_identical_cpu_paths():
    a = synth.make_blob(3, 17, 256, 128, 3)
    b = synth.make_blob(3, 17, 256, 128, 3)
    assert torch.equal(a, b)
    assert not torch.equal(a, synth.make_blob(3, 18, 256, 128, 3))
    v = a[synth.blob_geometry(256, 128, 3, 3, 3)["suh_g"]:].view(torch.float16).float()
    assert torch.all(v[:256].abs() == 1.0)


@pytest.mark.parametrize("K", [3, 5])
def test_pack_matches_reference_packer(K):
    """Blobs packed by the reference's own pack_expert / planar4 (tests/golden/ref_pack.npz, written by
    tests/golden/make_ref_pack.py from the reference checkout): this build's pack_expert gives the same bytes, and the
    oracle's blob reader decodes the reference's blob to the checkpoint trellis words' weights."""
    import os
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_pack.npz"))

    def tens(name):
        return {f: torch.from_numpy(d[f"k{K}_{name}_{f}"]) for f in ("trellis", "suh", "svh")}

    gate, up, down = tens("gate"), tens("up"), tens("down")
    blob_ref = d[f"k{K}_blob"]
    assert np.array_equal(moe_offload.pack_expert(gate, up, down, K).numpy(), blob_ref)
    H, I = gate["trellis"].shape[0] * 16, gate["trellis"].shape[1] * 16
    assert blob_ref.size == O.blob_bytes(H, I, K)
    for proj, t, (k, n) in ((0, gate, (H, I)), (1, up, (H, I)), (2, down, (I, H))):
        words = t["trellis"].view(torch.int32).numpy().view(np.uint32).reshape(k // 16, -1)
        assert np.array_equal(O.blob_dequant(blob_ref, H, I, K, K, K, proj),
                              O.dequant(words, k // 16, words.shape[1], 0, n // 16, K, False))


def test_golden_fixtures_reproduce():
    import os
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    import hashlib
    tab = O.mul1_table()
    assert hashlib.sha256(tab.tobytes()).digest() == bytes(d["mul1_sha256"])
    for K in (2, 3, 4, 5):
        w = d[f"t_words_k{K}"]
        assert np.array_equal(O.dequant(w, 1, 8 * K * 4, 0, 4, K, False), d[f"t_plain_k{K}"])
        assert np.array_equal(O.dequant(w, 1, 8 * K * 4, 0, 4, K, True), d[f"t_planar_k{K}"])
    from golden.make_golden import layer_case
    lc = layer_case()
    for k in ("l_ids", "l_out", "l_abuf"):
        assert np.array_equal(lc[k], d[k]), k
    assert np.allclose(lc["l_w"], d["l_w"], rtol=1e-6, atol=0)


def test_oracle_router_ties_and_order():
    H, E = 256, 32
    x = np.zeros((1, H), dtype=np.uint16)
    x[0, 0] = 0x3F80                                       # 1.0 bf16
    wr = np.zeros((E, H), dtype=np.uint16)
    ids, w, lg = O.router(x, wr, np.array([0.0] * 16 + [1.0] * 16, np.float32), 4)
    assert list(ids[0]) == [16, 17, 18, 19]                 # ties -> lower id
    assert np.allclose(w[0], 0.25)


def test_oracle_ensure_lru_rule():
    """Deterministic LRU: misses ascending id, victims = smallest (last+1, slot), paired in slot order."""
    L, E, S = 1, 8, 4
    cs = O.CacheState(L, E, S, np.array([1 << 40], np.int64), 1 << 30, 64)
    cs.slot_last[:] = [5, 3, 3, 9]
    cs.slot_key[:] = [4, 5, 6, 7]
    cs.slot_of[4:8] = [0, 1, 2, 3]
    cs.tick[0] = 9
    ids = np.array([[2, 1, 0]], np.int32)
    w = np.ones((1, 3), np.float32)
    n = cs.ensure(ids, w, 0, max_fill=8)
    assert n == 3
    # victims: (u=4,s=1), (4,2), (6,0); slot order 0,1,2 <- misses 0,1,2
    assert list(cs.fill_list[:4]) == [3, 0, 1, 2]
    assert list(cs.slot_key) == [0, 1, 2, 7]
    assert list(cs.slot_of[:8]) == [0, 1, 2, -1, -1, -1, -1, 3]
    assert list(cs.slot_last) == [10, 10, 10, 9]
