"""EXL3 checkpoints (safetensors) into ExpertStore host blobs.

Follows the reference plugin's checkpoint side: module geometry and codebook read from the safetensors headers only
(plugin/sglang_plugin.tier.py:81-104, scan_checkpoint), and each routed expert packed into its host blob as soon as
its nine tensors are present (:465-495, _maybe_pack), with the same refusals (a codebook other than mul1, a shape
that disagrees with the header, mixed bit widths inside an expert).

safetensors: a little-endian u64 header length n, n bytes of JSON {name: {dtype, shape, data_offsets [begin, end)},
"__metadata__": {...}}, then the data region (offsets are relative to its start).  This module reads headers and
data regions itself (no safetensors dependency at run time).

EXL3 tensors of one linear module (exllamav3): trellis int16 [k/16][n/16][16K] for K bits per weight, suh fp16 [k],
svh fp16 [n], and a marker naming the codebook: "<module>.mul1" (the one these kernels decode), "<module>.mcg", or
neither (3inst).  Routed experts are "<prefix>layers.<l>.mlp.experts.<e>.<gate|up|down>_proj.<suffix>", the prefix
being "model." or "model.language_model."; a multi-token-prediction layer sits under "mtp.".
"""
from __future__ import annotations

import json
import math
import os
import re
from dataclasses import dataclass

import torch

from .moe_offload import pack_expert

CODEBOOK = {"3inst": 0, "mcg": 1, "mul1": 2}          # ids as the reference plugin numbers them
_DTYPE = {"F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64,
          "I8": torch.int8, "U8": torch.uint8, "I16": torch.int16, "I32": torch.int32, "I64": torch.int64,
          "BOOL": torch.bool}
_EXPERT = re.compile(r"^(.*?)layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate|up|down)_proj\.(trellis|suh|svh)$")
_MODULE = re.compile(r"(?:^|\.)(mtp\..+|layers\.\d+\..+)$")


def module_key(name: str) -> str:
    """Canonical module name shared by checkpoint names and engine prefixes: the part from "layers.<n>." on
    ("model.language_model.layers.3.mlp" -> "layers.3.mlp"), from "mtp." on for the MTP layer, else the name."""
    m = _MODULE.search(name)
    return m.group(1) if m else name


def read_header(path: str) -> tuple[dict, int]:
    """(header JSON, byte offset of the data region) of one safetensors file."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"exl3b200 checkpoint: {path}: not a safetensors file")
        n = int.from_bytes(head, "little")
        text = f.read(n)
    if len(text) != n:
        raise ValueError(f"exl3b200 checkpoint: {path}: truncated header")
    return json.loads(text), 8 + n


@dataclass(frozen=True)
class _Tensor:
    path: str
    offset: int          # absolute byte offset in the file
    nbytes: int
    dtype: str
    shape: tuple


class Checkpoint:
    """The tensors of a checkpoint directory: the files named by model.safetensors.index.json when present, else every
    *.safetensors file.  Tensors are read on demand."""

    def __init__(self, model_dir: str):
        self.dir = model_dir
        index = os.path.join(model_dir, "model.safetensors.index.json")
        if os.path.isfile(index):
            with open(index) as f:
                files = sorted(set(json.load(f)["weight_map"].values()))
        else:
            files = sorted(f for f in os.listdir(model_dir) if f.endswith(".safetensors"))
        self.tensors: dict[str, _Tensor] = {}
        for fn in files:
            path = os.path.join(model_dir, fn)
            header, data = read_header(path)
            for name, t in header.items():
                if name == "__metadata__":
                    continue
                begin, end = t["data_offsets"]
                self.tensors[name] = _Tensor(path, data + begin, end - begin, t["dtype"], tuple(t["shape"]))

    def get(self, name: str) -> torch.Tensor:
        t = self.tensors[name]
        dtype = _DTYPE.get(t.dtype)
        if dtype is None:
            raise ValueError(f"exl3b200 checkpoint: {name}: dtype {t.dtype} not supported")
        if math.prod(t.shape) * dtype.itemsize != t.nbytes:
            raise ValueError(f"exl3b200 checkpoint: {name}: {t.nbytes} bytes for shape {t.shape} {t.dtype}")
        with open(t.path, "rb") as f:
            f.seek(t.offset)
            raw = f.read(t.nbytes)
        if len(raw) != t.nbytes:
            raise ValueError(f"exl3b200 checkpoint: {name}: file ends inside the tensor")
        return torch.frombuffer(bytearray(raw), dtype=dtype).reshape(t.shape) if t.nbytes else \
            torch.empty(t.shape, dtype=dtype)


def scan(ck: Checkpoint) -> dict[str, tuple[int, int, int, int]]:
    """{module key: (k, n, K bits, codebook id)} of every EXL3 module, from the headers alone."""
    out = {}
    for name, t in ck.tensors.items():
        if not name.endswith(".trellis"):
            continue
        base = name[: -len(".trellis")]
        cb = next((c for c in ("mcg", "mul1") if f"{base}.{c}" in ck.tensors), "3inst")
        rows, tiles, words = t.shape
        out[module_key(base)] = (rows * 16, tiles * 16, words // 16, CODEBOOK[cb])
    return out


def scan_checkpoint(model_dir: str) -> dict[str, tuple[int, int, int, int]]:
    return scan(Checkpoint(model_dir))


class ExpertPacker:
    """One MoE layer's expert tensors as they arrive, in any order; each expert is packed into
    store.host_view(key)[e] as soon as its nine tensors are present and then dropped, so at most the experts still
    incomplete are held."""

    ROLES = ("gate", "up", "down")
    PARTS = ("trellis", "suh", "svh")

    def __init__(self, store, key, geometry: dict):
        """geometry: {(role, expert): (k, n, K, codebook)} from the headers."""
        self.store, self.key, self.geometry = store, key, geometry
        self.pending: dict[int, dict] = {}
        self.packed = 0

    def add(self, expert: int, role: str, part: str, tensor: torch.Tensor) -> None:
        if role not in self.ROLES or part not in self.PARTS or not 0 <= expert < self.store.E:
            raise ValueError(f"exl3b200 checkpoint: {self.key}: unexpected tensor {role}.{part} of expert {expert}")
        got = self.pending.setdefault(expert, {}).setdefault(role, {})
        if part in got:
            raise ValueError(f"exl3b200 checkpoint: {self.key}: {role} {part} of expert {expert} loaded twice")
        got[part] = tensor.detach().to("cpu")
        if all(len(self.pending[expert].get(r, ())) == 3 for r in self.ROLES):
            self._pack(expert)

    def _pack(self, e: int) -> None:
        parts = self.pending.pop(e)
        st = self.store
        want_kn = {"gate": (st.H, st.I), "up": (st.H, st.I), "down": (st.I, st.H)}
        for role in self.ROLES:
            tr = parts[role]["trellis"]
            shape = (tr.shape[0] * 16, tr.shape[1] * 16, tr.shape[2] // 16)
            k, n, K, cb = self.geometry[(role, e)]
            if shape != (k, n, K) or cb != CODEBOOK["mul1"] or (k, n) != want_kn[role]:
                raise ValueError(f"exl3b200 checkpoint: {self.key}: {role}_proj expert {e}: trellis {tuple(tr.shape)}, "
                                 f"codebook {cb}, header {(k, n, K)} (needs mul1 and {want_kn[role]})")
        widths = {parts[r]["trellis"].shape[2] // 16 for r in self.ROLES}
        if widths != {st.K}:
            raise NotImplementedError(f"exl3b200 checkpoint: {self.key}: expert {e} has K {sorted(widths)}, the store "
                                      f"holds K={st.K} blobs")
        pack_expert(parts["gate"], parts["up"], parts["down"], st.K, out=st.host_view(self.key)[e])
        self.packed += 1

    def finish(self) -> None:
        if self.pending or self.packed != self.store.E:
            raise ValueError(f"exl3b200 checkpoint: {self.key}: {self.packed} of {self.store.E} experts packed, "
                             f"{len(self.pending)} incomplete")


def expert_layers(ck: Checkpoint) -> dict[tuple[bool, int], dict]:
    """{(is_mtp, layer): {(expert, role, part): tensor name}} of the routed experts in a checkpoint."""
    layers: dict[tuple[bool, int], dict] = {}
    for name in ck.tensors:
        m = _EXPERT.match(name)
        if m:
            prefix, layer, e, role, part = m.groups()
            mtp = "mtp" in prefix.split(".")
            layers.setdefault((mtp, int(layer)), {})[(int(e), role, part)] = name
    return dict(sorted(layers.items()))


def layer_key(mtp: bool, layer: int) -> str:
    """The store key of a routed-expert layer: the canonical name of its experts module."""
    return f"{'mtp.' if mtp else ''}layers.{layer}.mlp.experts"


def load_experts(model_dir: str, store, mtp: bool = True) -> list:
    """Pack every routed expert of the checkpoint into `store` (one add_layer per MoE layer, regular layers in order,
    then the MTP layer when `mtp`).  Returns the store keys added."""
    ck = Checkpoint(model_dir)
    geo = scan(ck)
    keys = []
    for (is_mtp, layer), names in expert_layers(ck).items():
        if is_mtp and not mtp:
            continue
        key = layer_key(is_mtp, layer)
        if key not in store.layer_index:
            store.add_layer(key)
        g = {(role, e): geo[module_key(n[: -len(".trellis")])] for (e, role, part), n in names.items()
             if part == "trellis"}
        packer = ExpertPacker(store, key, g)
        for (e, role, part), name in sorted(names.items()):
            packer.add(e, role, part, ck.get(name))
        packer.finish()
        keys.append(key)
    return keys
