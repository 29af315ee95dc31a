"""The packed expert store on local NVMe: the record file the RAM tier is filled from (serve/pack_store.py:1-90).

Layout, the reference's, so a store packed by either side reads on the other:
  * <out>/qwen_experts.bin: one record per (layer, expert) key r = layer * E + e at byte offset r * rec, with
    rec = blob rounded up to 4 KiB (O_DIRECT needs 4 KiB-aligned offsets, sizes and buffers); a record holds the
    expert's blob (pack_expert) followed by zeros;
  * <out>/qwen_experts.json: {"L", "E", "K", "blob", "rec", "H", "I"};
  * <out>/qwen_experts.bin.done: written last; a store without it is incomplete and is rebuilt as a whole.

Records are read with O_DIRECT (page cache bypassed: the RAM tier is the cache) where the filesystem supports it,
else with plain reads.  StoreFetcher runs the reads on a thread pool behind exl3b200.tier.TierHost's fetch().

    python -m exl3b200.pack_store pack   --model DIR --out DIR   build from an EXL3 checkpoint, then verify
    python -m exl3b200.pack_store verify --model DIR --out DIR   size, marker, and 64 random records vs fresh packs
    python -m exl3b200.pack_store probe  --out DIR               the store is complete; whether O_DIRECT reads work
"""
from __future__ import annotations

import argparse
import json
import mmap
import os
import queue
import random
import sys
import threading
from dataclasses import asdict, dataclass

import numpy as np
import torch

PAGE = 4096
BIN, META = "qwen_experts.bin", "qwen_experts.json"


@dataclass(frozen=True)
class StoreMeta:
    L: int
    E: int
    K: int
    blob: int
    rec: int
    H: int
    I: int   # noqa: E741

    @staticmethod
    def for_blob(L: int, E: int, K: int, blob: int, H: int, I: int) -> "StoreMeta":   # noqa: E741
        return StoreMeta(L, E, K, blob, -(-blob // PAGE) * PAGE, H, I)

    def offset(self, key: int) -> int:
        return key * self.rec

    @property
    def size(self) -> int:
        return self.L * self.E * self.rec


def _paths(out_dir: str) -> tuple[str, str, str]:
    b = os.path.join(out_dir, BIN)
    return b, os.path.join(out_dir, META), b + ".done"


def load_meta(out_dir: str) -> StoreMeta:
    with open(_paths(out_dir)[1]) as f:
        m = json.load(f)
    return StoreMeta(*(int(m[k]) for k in ("L", "E", "K", "blob", "rec", "H", "I")))


def is_complete(out_dir: str) -> bool:
    b, m, d = _paths(out_dir)
    if not (os.path.isfile(b) and os.path.isfile(m) and os.path.isfile(d)):
        return False
    return os.path.getsize(b) == load_meta(out_dir).size


def pack(out_dir: str, meta: StoreMeta, blob_of, progress=None) -> bool:
    """Write the store from blob_of(layer, expert) -> bytes (meta.blob of them).  A complete store with the same
    layout is kept (returns False); anything else is rebuilt from scratch (returns True)."""
    os.makedirs(out_dir, exist_ok=True)
    b, m, d = _paths(out_dir)
    if is_complete(out_dir) and load_meta(out_dir) == meta:
        return False
    if os.path.exists(d):
        os.remove(d)
    pad = bytes(meta.rec - meta.blob)
    fd = os.open(b, os.O_RDWR | os.O_CREAT | os.O_TRUNC, 0o644)
    try:
        os.ftruncate(fd, meta.size)
        for layer in range(meta.L):
            for e in range(meta.E):
                data = bytes(blob_of(layer, e))
                if len(data) != meta.blob:
                    raise ValueError(f"exl3b200 pack_store: expert ({layer}, {e}) packs to {len(data)} bytes, "
                                     f"not {meta.blob}")
                os.pwrite(fd, data + pad, meta.offset(layer * meta.E + e))
            if progress is not None:
                progress(layer)
        os.fsync(fd)
    finally:
        os.close(fd)
    with open(m, "w") as f:
        json.dump(asdict(meta), f)
    open(d, "w").close()
    return True


def _aligned(nbytes: int) -> memoryview:
    """A page-aligned, writable host buffer (anonymous mapping)."""
    return memoryview(mmap.mmap(-1, nbytes))


def _direct_fd(path: str):
    """An O_DIRECT descriptor of path when one 4 KiB aligned read through it works, else None."""
    flag = getattr(os, "O_DIRECT", 0)
    if not flag:
        return None
    try:
        fd = os.open(path, os.O_RDONLY | flag)
    except OSError:
        return None
    try:
        os.preadv(fd, [_aligned(PAGE)], 0)
    except OSError:
        os.close(fd)
        return None
    return fd


class StoreReader:
    """Reads records of a complete store into host memory (thread-safe: positioned reads, per-thread buffers)."""

    def __init__(self, out_dir: str, direct: bool | None = None):
        if not is_complete(out_dir):
            raise RuntimeError(f"exl3b200 pack_store: no complete store in {out_dir} ({BIN} + .done + {META})")
        self.meta = load_meta(out_dir)
        path = _paths(out_dir)[0]
        fd = _direct_fd(path) if direct in (None, True) else None
        if direct and fd is None:
            raise RuntimeError(f"exl3b200 pack_store: O_DIRECT reads do not work on {path}")
        self.direct = fd is not None
        self.fd = fd if fd is not None else os.open(path, os.O_RDONLY)
        self._local = threading.local()

    def close(self) -> None:
        if self.fd is not None:
            os.close(self.fd)
            self.fd = None

    def _bounce(self) -> memoryview:
        buf = getattr(self._local, "buf", None)
        if buf is None:
            buf = self._local.buf = _aligned(self.meta.rec)
        return buf

    def read(self, key: int, out: torch.Tensor) -> None:
        """Record `key`'s blob into `out` (uint8 CPU tensor of >= blob bytes, e.g. a pinned host slot).  With O_DIRECT
        the read lands in `out` itself when it is page-aligned and holds a whole record (>= rec bytes): then its
        bytes from blob to rec receive the record's zero padding, so pass a slot of its own, not a view that runs into
        the next one.  Otherwise the read goes through a bounce buffer and only the blob's bytes are written."""
        meta = self.meta
        if not 0 <= key < meta.L * meta.E:
            raise IndexError(f"exl3b200 pack_store: key {key} outside {meta.L} x {meta.E}")
        if out.dtype != torch.uint8 or out.device.type != "cpu" or not out.is_contiguous() or out.numel() < meta.blob:
            raise ValueError("exl3b200 pack_store: out must be a contiguous uint8 CPU tensor of >= blob bytes")
        view = memoryview(out.numpy())
        bounce = self.direct and not (out.data_ptr() % PAGE == 0 and out.numel() >= meta.rec)
        if bounce:
            dst = self._bounce()
        else:
            dst = view[:meta.rec] if self.direct else view[:meta.blob]
        n = os.preadv(self.fd, [dst], meta.offset(key))
        if n != len(dst):
            raise OSError(f"exl3b200 pack_store: short read of record {key} ({n} of {len(dst)} bytes)")
        if bounce:
            view[:meta.blob] = dst[:meta.blob]

    def record(self, key: int) -> np.ndarray:
        out = torch.empty(self.meta.blob, dtype=torch.uint8)
        self.read(key, out)
        return out.numpy()


def verify(out_dir: str, blob_of, n: int = 64, seed: int = 0) -> int:
    """Re-read n random records and compare them with fresh packs; returns the number that differ."""
    reader = StoreReader(out_dir)
    try:
        meta = reader.meta
        rng = random.Random(seed)
        bad = 0
        for _ in range(n):
            layer, e = rng.randrange(meta.L), rng.randrange(meta.E)
            bad += not np.array_equal(reader.record(layer * meta.E + e),
                                      np.frombuffer(bytes(blob_of(layer, e)), dtype=np.uint8))
        return bad
    finally:
        reader.close()


def probe(out_dir: str) -> dict:
    """{"store": path, "o_direct": bool} for a complete store; RuntimeError when it is missing or incomplete."""
    reader = StoreReader(out_dir)
    try:
        return {"store": _paths(out_dir)[0], "o_direct": reader.direct}
    finally:
        reader.close()


class StoreFetcher:
    """The storage behind TierHost.fetch: fetch(key) queues a read of record `key` into dest(key) (the key's host
    slot) on one of `threads` reader threads, which then calls done(key) (TierHost.fill_done).  A failed read is kept
    and raised by the next fetch() or close()."""

    def __init__(self, reader: StoreReader, dest, done, threads: int = 4):
        self.reader, self.dest, self.done = reader, dest, done
        self._q: queue.SimpleQueue = queue.SimpleQueue()
        self._error: BaseException | None = None
        self._closed = False
        self._threads = [threading.Thread(target=self._run, daemon=True, name=f"exl3b-store-{i}")
                         for i in range(threads)]
        for t in self._threads:
            t.start()

    def _run(self) -> None:
        while True:
            key = self._q.get()
            if key is None:
                return
            try:
                self.reader.read(key, self.dest(key))
                self.done(key)
            except BaseException as exc:   # noqa: BLE001 -- handed to the caller's thread
                self._error = exc

    def _raise(self) -> None:
        if self._error is not None:
            exc, self._error = self._error, None
            raise RuntimeError("exl3b200 pack_store: a record read failed") from exc

    def fetch(self, key: int) -> None:
        self._raise()
        if self._closed:
            raise RuntimeError("exl3b200 pack_store: fetch after the fetcher was closed")
        self._q.put(int(key))

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        for _ in self._threads:
            self._q.put(None)
        for t in self._threads:
            t.join()
        self._raise()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ------------------------------------------------------------------------------------------------ checkpoint side
def checkpoint_source(model_dir: str):
    """(StoreMeta, blob_of) for the routed experts of an EXL3 checkpoint's regular layers (layer index = position in
    layer order; the MTP layer is not stored)."""
    from .checkpoint import Checkpoint, expert_layers, scan, module_key
    from .moe_offload import pack_expert
    ck = Checkpoint(model_dir)
    layers = [names for (mtp, _), names in expert_layers(ck).items() if not mtp]
    if not layers:
        raise ValueError(f"exl3b200 pack_store: no routed experts in {model_dir}")
    geo = scan(ck)
    E = 1 + max(e for e, _, _ in layers[0])
    k_gate, n_gate, K, _ = geo[module_key(layers[0][(0, "gate", "trellis")][: -len(".trellis")])]

    def blob_of(layer: int, e: int) -> bytes:
        names = layers[layer]
        parts = {r: {p: ck.get(names[(e, r, p)]) for p in ("trellis", "suh", "svh")} for r in ("gate", "up", "down")}
        return pack_expert(parts["gate"], parts["up"], parts["down"], K).numpy().tobytes()

    blob = len(blob_of(0, 0))
    return StoreMeta.for_blob(len(layers), E, K, blob, k_gate, n_gate), blob_of


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m exl3b200.pack_store")
    ap.add_argument("cmd", choices=["pack", "verify", "probe"])
    ap.add_argument("--model", default=os.environ.get("EXL3_MODEL_PATH"))
    ap.add_argument("--out", default=os.path.dirname(os.environ.get("EXL3_NVTIER_STORE", "")) or None)
    a = ap.parse_args(argv)
    if a.out is None:
        ap.error("--out (or EXL3_NVTIER_STORE) is required")
    if a.cmd == "probe":
        try:
            print(json.dumps(probe(a.out)))
        except RuntimeError as exc:
            print(str(exc), file=sys.stderr)
            return 1
        return 0
    if a.model is None:
        ap.error("--model (or EXL3_MODEL_PATH) is required")
    meta, blob_of = checkpoint_source(a.model)
    if a.cmd == "pack":
        pack(a.out, meta, blob_of, progress=lambda layer: print(json.dumps({"layer": layer}), flush=True))
    bad = verify(a.out, blob_of)
    print(json.dumps({"store": _paths(a.out)[0], "verify_bad": bad, "verify_n": 64}), flush=True)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
