"""numpy front end of the CPU oracle (exl3b_oracle.c).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
reference legs as the checker.  The product path (qwen38-flash-next-b70-offload_b200/exl3b200) never
imports this module.

Parity status: partially pinned (see the header of exl3b_oracle.c for what pins it).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "libexl3b_oracle.so")
_lib = None

u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
vp = ctypes.c_void_p
ci = ctypes.c_int
i64 = ctypes.c_int64
sz = ctypes.c_size_t


def build() -> str:
    """Compile the oracle (make) if the library is missing or older than its source."""
    src = os.path.join(_HERE, "exl3b_oracle.c")
    if not os.path.exists(_LIB) or os.path.getmtime(_LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB)
        sig = {
            "ora_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "ora_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "ora_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
            "ora_mul1": (ctypes.c_uint16, [ctypes.c_uint32]),
            "ora_tile_row": (ci, [ci]),
            "ora_tile_col": (ci, [ci]),
            "ora_tile_state": (ctypes.c_uint32, [u32p, ci, ci]),
            "ora_geo_D": (ci, [ci]),
            "ora_geo_G": (ci, [ci]),
            "ora_planar_offset": (ci, [ci, ci, ci]),
            "ora_decode_tile": (None, [u32p, ci, u16p]),
            "ora_dequant": (None, [u32p, ci, sz, ci, ci, ci, ci, u16p, sz]),
            "ora_blob_bytes": (i64, [ci, ci, ci, ci, ci]),
            "ora_blob_dequant": (None, [vp, ci, ci, ci, ci, ci, ci, u16p]),
            "ora_fwht128": (None, [f32p]),
            "ora_had_in": (None, [u16p, ci, u16p, ci, u16p]),
            "ora_moe_layer": (None, [u16p, ci, i32p, f32p, ci, ci, vp, vp, ci, ci, ci, ci, vp, vp, vp]),
            "ora_dense_glu": (None, [u16p, ci, vp, ci, ci, ci, ci, ci, f32p]),
            "ora_expert_picks": (None, [u16p, ctypes.c_int64, ci, i32p, f32p, ci, vp, ci, ci, ci, ci, ci, ci, f32p]),
            "ora_router_dot": (ctypes.c_float, [u16p, u16p, ci]),
            "ora_shared_gate": (ctypes.c_float, [u16p, u16p, ci]),
            "ora_router": (None, [u16p, u16p, vp, ci, ci, ci, ci, i32p, f32p, vp]),
            "ora_align": (None, [i32p, f32p, ci, ci, ci, ci, i32p, i32p, i32p, i32p, i32p, i32p, f32p, i32p, vp, vp]),
            "ora_ensure": (ci, [i32p, f32p, ci, ci, ci, ci, i64p, i32p, i32p, i32p, i32p, i64p, i64, i64, i64, i64p,
                                i32p, ci, ci, vp, vp, vp, ci, vp, vp]),
            "ora_commit": (None, [i64p, i64p, i32p]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- codec
def mul1_table() -> np.ndarray:
    """fp16 bit patterns of all 65,536 mul1 states."""
    L = lib()
    return np.array([L.ora_mul1(s) for s in range(65536)], dtype=np.uint16)


def f16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    b = f.view(np.uint32).astype(np.uint64)
    lsb = (b >> 16) & 1
    return ((b + 0x7FFF + lsb) >> 16).astype(np.uint16)


def blob_bytes(H: int, I: int, Kg: int, Ku: int | None = None, Kd: int | None = None) -> int:
    Ku = Kg if Ku is None else Ku
    Kd = Kg if Kd is None else Kd
    return int(lib().ora_blob_bytes(H, I, Kg, Ku, Kd))


def blob_dequant(blob: np.ndarray, H: int, I: int, Kg: int, Ku: int, Kd: int, proj: int) -> np.ndarray:
    """fp16 bits W_inner: proj 0/1 -> [H, I] (gate/up), 2 -> [I, H] (down)."""
    blob = np.ascontiguousarray(blob, dtype=np.uint8)
    shape = (H, I) if proj < 2 else (I, H)
    out = np.empty(shape, dtype=np.uint16)
    lib().ora_blob_dequant(_ptr(blob), H, I, Kg, Ku, Kd, proj, out)
    return out


def dequant(words: np.ndarray, rows16: int, row_stride: int, tile0: int, ntiles: int, K: int, planar: bool) -> np.ndarray:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    out = np.empty((rows16 * 16, ntiles * 16), dtype=np.uint16)
    lib().ora_dequant(words, rows16, row_stride, tile0, ntiles, K, int(planar), out, ntiles * 16)
    return out


def fwht128(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32).copy()
    lib().ora_fwht128(v)
    return v


def had_in(x_bits: np.ndarray, suh_bits: np.ndarray, x_is_bf16: bool = True) -> np.ndarray:
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    out = np.empty_like(x_bits)
    lib().ora_had_in(x_bits, int(x_is_bf16), np.ascontiguousarray(suh_bits, dtype=np.uint16), x_bits.size, out)
    return out


# ---------------------------------------------------------------- layer
def moe_layer(x_bits: np.ndarray, ids: np.ndarray, w: np.ndarray, blobs: list, H: int, I: int, K: int = 3,
              kinfo: np.ndarray | None = None, x_is_bf16: bool = True, want_y: bool = False, out_f32: bool = False):
    """Routed MoE layer.  x_bits: uint16 [M, H] (bf16 bits); blobs: list of uint8 arrays indexed by
    expert id (None for unused ids); returns out bf16 bits [M, H] (fp32 [M, H] before the final rounding when
    out_f32), and y fp32 [M*topk, H], abuf fp16 bits [M*topk, I] when want_y."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, topk = ids.shape
    keep = [np.ascontiguousarray(b, dtype=np.uint8) if b is not None else None for b in blobs]
    arr = (ctypes.c_void_p * len(keep))(*[(b.ctypes.data if b is not None else 0) for b in keep])
    out = np.empty((M, H), dtype=np.float32 if out_f32 else np.uint16)
    y = np.empty((M * topk, H), dtype=np.float32) if want_y else None
    ab = np.empty((M * topk, I), dtype=np.uint16) if want_y else None
    ki = np.ascontiguousarray(kinfo, dtype=np.int32) if kinfo is not None else None
    lib().ora_moe_layer(x_bits, int(x_is_bf16), ids, w, M, topk, ctypes.cast(arr, ctypes.c_void_p), _ptr(ki),
                        H, I, K, 2 if out_f32 else 1, _ptr(out), _ptr(y), _ptr(ab))
    return (out, y, ab) if want_y else out


def moe_layer_fast(x_bits: np.ndarray, ids: np.ndarray, w: np.ndarray, blobs: list, H: int, I: int, K: int = 3,
                   kinfo: np.ndarray | None = None, x_is_bf16: bool = True, out_f32: bool = False,
                   threads: int | None = None, y_half: bool = False, rows: np.ndarray | None = None):
    """moe_layer grouped by expert: each expert's weights are dequantised once and all of its picks run on one thread
    (experts on parallel threads; the C code releases the GIL).  Same per-pick arithmetic and the same outputs as
    moe_layer (the combine adds the picks in k order in fp32).  y_half=True gives the prefill semantics: every pick's
    weighted output is rounded to fp16 before the combine (the reference's moe_prefill stores y as fp16).  rows: only
    these token rows are computed (returned in that order)."""
    import concurrent.futures as cf
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows = np.arange(ids.shape[0]) if rows is None else np.asarray(rows)
    sid, sw = ids[rows], w[rows]
    M, topk = sid.shape
    flat_e = sid.ravel()
    flat_t = np.repeat(rows.astype(np.int32), topk)
    flat_w = sw.ravel()
    y = np.zeros((M * topk, H), dtype=np.float32)
    L = lib()
    experts = np.unique(flat_e[flat_e >= 0])   # id -1: no pick (its output row stays zero)

    def run(e):
        sel = np.nonzero(flat_e == e)[0]
        tok = np.ascontiguousarray(flat_t[sel])
        we = np.ascontiguousarray(flat_w[sel])
        ye = np.empty((len(sel), H), dtype=np.float32)
        kg = ku = kd = K
        if kinfo is not None:
            v = int(kinfo[e]); kg, ku, kd = v & 15, (v >> 4) & 15, (v >> 8) & 15
        b = np.ascontiguousarray(blobs[e], dtype=np.uint8)
        L.ora_expert_picks(x_bits, H if x_bits.ndim == 1 else x_bits.shape[1], int(x_is_bf16), tok, we, len(sel),
                           b.ctypes.data, kg, ku, kd, H, I, int(y_half), ye)
        y[sel] = ye

    with cf.ThreadPoolExecutor(threads or (os.cpu_count() or 1)) as ex:
        list(ex.map(run, experts))
    y = y.reshape(M, topk, H)
    acc = np.zeros((M, H), dtype=np.float32)
    for k in range(topk):
        acc += y[:, k]
    if out_f32:
        return acc
    u = acc.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16) if x_is_bf16 else acc.astype(np.float16).view(np.uint16)


def shared_gate(x_bits: np.ndarray, g_bits: np.ndarray) -> np.ndarray:
    """Shared-expert gate weights sigmoid(x . g) fp32 [M] (router dot-product arithmetic) for x bf16 bits [M, H]."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    g_bits = np.ascontiguousarray(g_bits, dtype=np.uint16)
    M, H = x_bits.shape
    return np.array([lib().ora_shared_gate(np.ascontiguousarray(x_bits[m]), g_bits, H) for m in range(M)], dtype=np.float32)


def dense_glu(x_bits: np.ndarray, blob: np.ndarray, H: int, I: int, Kg: int, Ku: int, Kd: int) -> np.ndarray:
    """Un-gated shared-expert output y fp32 [M, H] for x bf16 bits [M, H]."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    blob = np.ascontiguousarray(blob, dtype=np.uint8)
    M = x_bits.shape[0]
    y = np.empty((M, H), dtype=np.float32)
    for m in range(M):
        row = np.empty(H, dtype=np.float32)
        lib().ora_dense_glu(np.ascontiguousarray(x_bits[m]), 1, _ptr(blob), H, I, Kg, Ku, Kd, row)
        y[m] = row
    return y


# ---------------------------------------------------------------- router / align / cache
def router(x_bits: np.ndarray, wr_bits: np.ndarray, bias: np.ndarray | None, topk: int):
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    wr_bits = np.ascontiguousarray(wr_bits, dtype=np.uint16)
    T, H = x_bits.shape
    E = wr_bits.shape[0]
    ids = np.empty((T, topk), dtype=np.int32)
    w = np.empty((T, topk), dtype=np.float32)
    lg = np.empty((T, E), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().ora_router(x_bits, wr_bits, _ptr(b), T, H, E, topk, ids, w, _ptr(lg))
    return ids, w, lg


def align(ids: np.ndarray, w: np.ndarray, E: int, pad: int):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, topk = ids.shape
    n = M * topk
    A = min(n, E)
    r = dict(act_expert=np.zeros(A, np.int32), act_start=np.zeros(A, np.int32), act_cnt=np.zeros(A, np.int32),
             act_pstart=np.zeros(A, np.int32), n_act=np.zeros(1, np.int32), pair_tok=np.zeros(n, np.int32),
             pair_w=np.zeros(n, np.float32), pair_of=np.zeros(n, np.int32))
    mxb = (n + pad - 1) // pad + A
    blk_a = np.zeros(max(mxb, 1), np.int32)
    n_blk = np.zeros(1, np.int32)
    lib().ora_align(ids.ravel(), w.ravel(), n, topk, E, pad, r["act_expert"], r["act_start"], r["act_cnt"],
                    r["act_pstart"], r["n_act"], r["pair_tok"], r["pair_w"], r["pair_of"], _ptr(blk_a), _ptr(n_blk))
    na = int(r["n_act"][0])
    for k in ("act_expert", "act_start", "act_cnt", "act_pstart"):
        r[k] = r[k][:na]
    r["blk_a"] = blk_a[: int(n_blk[0])]
    r["n_blk"] = int(n_blk[0])
    return r


class CacheState:
    """Host copy of the device cache state tensors (moe_offload.py:109-124) for the oracle."""

    def __init__(self, L: int, E: int, S: int, host_base: np.ndarray, slot_base: int, blob: int, hstride: int = 0):
        self.L, self.E, self.S = L, E, S
        self.ptrs_all = np.zeros(L * E, np.int64)
        self.slot_of = np.full(L * E, -1, np.int32)
        self.slot_key = np.full(S, -1, np.int32)
        self.slot_last = np.full(S, -1, np.int32)
        self.tick = np.zeros(1, np.int32)
        self.host_base = np.ascontiguousarray(host_base, dtype=np.int64)
        self.slot_base, self.blob = int(slot_base), int(blob)
        self.hstride = int(hstride or blob)
        self.fill_all = np.zeros(L * E, np.int64)
        self.fill_list = np.zeros(1 + E, np.int32)
        self.pf_slot = np.zeros(E, np.int32)
        for li in range(L):
            self.ptrs_all[li * E:(li + 1) * E] = self.host_base[li] + np.arange(E, dtype=np.int64) * self.hstride

    def copy(self):
        c = CacheState.__new__(CacheState)
        c.__dict__.update({k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in self.__dict__.items()})
        return c

    def ensure(self, ids: np.ndarray, w: np.ndarray, layer: int, max_fill: int, prefetch: bool = False,
               ram_res: np.ndarray | None = None, ring: np.ndarray | None = None, safe: np.ndarray | None = None,
               vict: np.ndarray | None = None) -> int:
        """In-place on ids/w (tier mask) and the state arrays; returns the number of fills."""
        assert ids.dtype == np.int32 and ids.flags.c_contiguous and w.dtype == np.float32 and w.flags.c_contiguous
        cap = 0 if ring is None else ring.size - 1
        return lib().ora_ensure(ids.reshape(-1), w.reshape(-1), ids.size, layer, self.E, self.S, self.ptrs_all,
                                self.slot_of, self.slot_key, self.slot_last, self.tick, self.host_base,
                                self.slot_base, self.blob, self.hstride, self.fill_all, self.fill_list,
                                max_fill, int(prefetch), _ptr(self.pf_slot), _ptr(ram_res), _ptr(ring), cap, _ptr(safe),
                                _ptr(vict))

    def commit(self, layer: int):
        E = self.E
        p = self.ptrs_all[layer * E:(layer + 1) * E].copy()
        f = self.fill_all[layer * E:(layer + 1) * E].copy()
        lib().ora_commit(p, f, self.fill_list)
        self.ptrs_all[layer * E:(layer + 1) * E] = p
        self.fill_all[layer * E:(layer + 1) * E] = f

    # ---- copy-engine prefetch: the plan and commit modes of launch_ensure (exl3_moe.a8.sycl:874-905, 898-1036)
    PINNED = 0x7FFFFFFF

    def cepf_reset(self) -> None:
        self.pend = {}                                   # layer -> (seq, T, [(expert, slot), ...]) in flight
        self.plan_seq = np.zeros(self.L, np.int32)

    def cepf_commit(self, done_seq) -> None:
        """Every layer whose done_seq reached its pending seq: table entries -> slots, slots unpinned (last = T)."""
        for li in sorted(self.pend):
            seq, T, pairs = self.pend[li]
            if int(done_seq[li]) < seq:
                continue
            for e, s in pairs:
                self.ptrs_all[li * self.E + e] = self.slot_base + s * self.blob
                self.slot_last[s] = T
            del self.pend[li]

    def cepf_plan(self, ids: np.ndarray, layer: int, max_fill: int, done_seq):
        """Commit what landed; a layer with a plan in flight plans nothing (returns None); else the prefetch-mode
        cache step claims slots, which are pinned and recorded.  Returns (seq, [(expert, slot), ...])."""
        self.cepf_commit(done_seq)
        if layer in self.pend:
            self.fill_list[0] = 0
            return None
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        n = self.ensure(ids, np.ones(ids.size, np.float32), layer, min(max_fill, 16, self.E), prefetch=True)
        pairs = [(int(self.fill_list[1 + i]), int(self.pf_slot[i])) for i in range(n)]
        for _, s in pairs:
            self.slot_last[s] = self.PINNED
        self.plan_seq[layer] += 1
        seq = int(self.plan_seq[layer])
        if pairs:
            self.pend[layer] = (seq, int(self.tick[0]), pairs)
        return seq, pairs


def vring_claim(vict: np.ndarray, meta: np.ndarray, sel: np.ndarray) -> None:
    """Victim ring claims (the a9 variant of launch_ensure, experimental/n111-victim-ring/a9.patch): in victim-list
    order, every entry that needs a write-back (old key >= 0) takes the first free slot (key < 0) scanning from the
    next search position meta[0]; it records key and claim number meta[1] + 1 there and moves the search position
    past it.  A full ring drops the victim (meta[2] += 1).  sel[i] = the slot of entry i, -1 = no copy.
    meta = [next position, claim sequence, drops, K, key[K], seq[K]]."""
    K = int(meta[3])
    key, seq = meta[4:4 + K], meta[4 + K:4 + 2 * K]
    p = int(meta[0])
    for i in range(int(vict[0])):
        old, r = int(vict[1 + 2 * i]), -1
        if old >= 0:
            r = next(((p + j) % K for j in range(K) if key[(p + j) % K] < 0), -1)
            if r >= 0:
                meta[1] += 1
                key[r], seq[r] = old, meta[1]
                p = (r + 1) % K
            else:
                meta[2] += 1
        sel[i] = r
    meta[0] = p
