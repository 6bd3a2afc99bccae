"""Weight store over a DeepSeek-R1 safetensors checkpoint, for the MoE path.

Replaces the reference's ``WeightStore`` (``inference/weight_store.py:80-255``)
for the calls the MoE path makes: ``get_expert`` (:185), ``get_gate_weight``
(:252), ``get_shared_expert_weights`` (:244), ``get_layer_norm_weights``
(:228), ``get_dense_mlp_weights`` (:236), plus ``get_gate_bias`` (the
``e_score_correction_bias`` the bias-corrected router uses).

Differences in how, not what:

  * The shard index (``model.safetensors.index.json``) and every shard's
    header are parsed once; a tensor is then a byte range of a shard file.
  * An expert is read straight into ONE packed pinned buffer (gate weight,
    gate scale, up weight, up scale, down weight, down scale, 44,050,944 B for
    R1) by ``dsmoe_read_ranges`` (pread on a thread pool): one copy from the
    page cache or the disk, where the reference makes a CPU tensor per key and
    then copies it into a freshly pinned one (:151-180). The returned tensors
    are views into the buffer, in the reference's ``{proj: (weight, scale)}``
    form.
  * Buffers come from torch's pinned-memory caching allocator, which hands a
    freed (evicted) buffer out again only after the asynchronous copies that
    read it have finished, so pinning costs are paid once.
  * Non-expert tensors are loaded on first use (the reference loads all ~40 GB
    of them at start-up).

The LRU policy and byte capacity are the reference's (``ExpertCache``).
"""
from __future__ import annotations

import ctypes
import json
import os
import re
import struct
from pathlib import Path

import torch

from ._lib import check, lib
from .weight_store import ExpertCache

PROJS = ("gate_proj", "up_proj", "down_proj")
EXPERT_PATTERN = re.compile(
    r"model\.layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\.(weight|weight_scale_inv)")

_DTYPES = {
    "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2, "BF16": torch.bfloat16, "F16": torch.float16,
    "F32": torch.float32, "F64": torch.float64, "I64": torch.int64, "I32": torch.int32, "I16": torch.int16,
    "I8": torch.int8, "U8": torch.uint8, "BOOL": torch.bool,
}


def read_header(path: str) -> tuple[int, dict]:
    """(offset of the data section, {key: {"dtype", "shape", "data_offsets"}})
    of one safetensors file: an 8-byte little-endian header length, then the
    JSON header, then the data; offsets are relative to the data section."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return 8 + n, header


class TensorLocation:
    __slots__ = ("path", "offset", "nbytes", "dtype", "shape")

    def __init__(self, path, offset, nbytes, dtype, shape):
        self.path, self.offset, self.nbytes, self.dtype, self.shape = path, offset, nbytes, dtype, shape


class SafetensorsIndex:
    """key -> (shard path, absolute byte offset, size, dtype, shape)."""

    def __init__(self, model_path: str | Path):
        self.root = Path(model_path)
        index_path = self.root / "model.safetensors.index.json"
        if index_path.exists():
            with open(index_path) as f:
                weight_map = json.load(f)["weight_map"]
            shards = sorted(set(weight_map.values()))
        else:  # a single-file checkpoint
            shards = [p.name for p in sorted(self.root.glob("*.safetensors"))]
        self.loc: dict[str, TensorLocation] = {}
        for shard in shards:
            path = str(self.root / shard)
            base, header = read_header(path)
            for key, meta in header.items():
                b, e = meta["data_offsets"]
                dtype = _DTYPES.get(meta["dtype"])
                if dtype is None:
                    raise ValueError(f"{key}: unsupported safetensors dtype {meta['dtype']}")
                self.loc[key] = TensorLocation(path, base + b, e - b, dtype, tuple(meta["shape"]))

    def __contains__(self, key: str) -> bool:
        return key in self.loc

    def __getitem__(self, key: str) -> TensorLocation:
        return self.loc[key]


def read_into(locs: list[TensorLocation], dsts: list[torch.Tensor], threads: int) -> None:
    """Read each location's bytes into the matching contiguous host tensor."""
    n = len(locs)
    paths = (ctypes.c_char_p * n)(*[os.fsencode(l.path) for l in locs])
    offs = (ctypes.c_uint64 * n)(*[l.offset for l in locs])
    sizes = (ctypes.c_uint64 * n)(*[l.nbytes for l in locs])
    ptrs = (ctypes.c_void_p * n)(*[d.data_ptr() for d in dsts])
    for l, d in zip(locs, dsts):
        if d.device.type != "cpu" or not d.is_contiguous() or d.nbytes != l.nbytes:
            raise ValueError("read_into: destinations must be contiguous host tensors of the tensor's size")
    check(lib().dsmoe_read_ranges(n, paths, offs, sizes, ptrs, int(threads)), "dsmoe_read_ranges")


class SafetensorsWeightStore:
    def __init__(self, model_path: str | Path, config, device, expert_cache_bytes: int = 16 * 1024 ** 3,
                 threads: int = 8, pin_memory: bool | None = None, verbose: bool = False):
        self.config = config
        self.device = torch.device(device)
        self.threads = threads
        self.pin_memory = torch.cuda.is_available() if pin_memory is None else pin_memory
        self.verbose = verbose
        self.index = SafetensorsIndex(model_path)
        self.expert_cache = ExpertCache(expert_cache_bytes)
        self._dev: dict[str, torch.Tensor] = {}
        self.bytes_read = 0

    # ------------------------------------------------------------- experts
    @staticmethod
    def expert_keys(layer: int, expert_idx: int) -> list[str]:
        prefix = f"model.layers.{layer}.mlp.experts.{expert_idx}"
        return [f"{prefix}.{proj}.{suffix}" for proj in PROJS for suffix in ("weight", "weight_scale_inv")]

    def _load_expert(self, layer: int, expert_idx: int) -> dict:
        """One expert into one packed pinned buffer; returns the reference's
        cache entry form ``{proj: {"weight", "weight_scale_inv"}}`` (views)."""
        locs = [self.index[k] for k in self.expert_keys(layer, expert_idx)]
        offs, total = [], 0
        for l in locs:
            offs.append(total)
            total += (l.nbytes + 255) // 256 * 256  # every tensor 256-byte aligned in the buffer
        buf = torch.empty(total, dtype=torch.uint8, pin_memory=self.pin_memory)
        views = [buf[o:o + l.nbytes] for o, l in zip(offs, locs)]
        read_into(locs, views, self.threads)
        self.bytes_read += sum(l.nbytes for l in locs)
        entry = {"_buffer": buf}
        for i, proj in enumerate(PROJS):
            w, s = locs[2 * i], locs[2 * i + 1]
            entry[proj] = {"weight": views[2 * i].view(w.dtype).view(w.shape),
                           "weight_scale_inv": views[2 * i + 1].view(s.dtype).view(s.shape)}
        return entry

    def get_expert(self, layer: int, expert_idx: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        """``{proj: (weight, scale)}`` of one routed expert, pinned host memory
        (``inference/weight_store.py:185-206``)."""
        cached = self.expert_cache.get(layer, expert_idx)
        if cached is None:
            if self.verbose:
                print(f"        [expert_cache] MISS  L{layer:02d}/E{expert_idx:03d}")
            cached = self._load_expert(layer, expert_idx)
            self.expert_cache.put(layer, expert_idx, cached)
        return {proj: (cached[proj]["weight"], cached[proj]["weight_scale_inv"]) for proj in PROJS}

    # --------------------------------------------------------- non-experts
    def get(self, key: str) -> torch.Tensor:
        """A non-expert tensor on the store's device, read on first use."""
        t = self._dev.get(key)
        if t is None:
            loc = self.index[key]
            host = torch.empty(loc.nbytes, dtype=torch.uint8, pin_memory=self.pin_memory)
            read_into([loc], [host], self.threads)
            t = host.view(loc.dtype).view(loc.shape).to(self.device)
            self._dev[key] = t
        return t

    def _pairs(self, prefix: str) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        return {p: (self.get(f"{prefix}{p}.weight"), self.get(f"{prefix}{p}.weight_scale_inv")) for p in PROJS}

    def get_gate_weight(self, layer: int) -> torch.Tensor:
        return self.get(f"model.layers.{layer}.mlp.gate.weight")

    def get_gate_bias(self, layer: int) -> torch.Tensor:
        return self.get(f"model.layers.{layer}.mlp.gate.e_score_correction_bias")

    def get_shared_expert_weights(self, layer: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        return self._pairs(f"model.layers.{layer}.mlp.shared_experts.")

    def get_dense_mlp_weights(self, layer: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        return self._pairs(f"model.layers.{layer}.mlp.")

    def get_layer_norm_weights(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        prefix = f"model.layers.{layer}"
        return (self.get(f"{prefix}.input_layernorm.weight"), self.get(f"{prefix}.post_attention_layernorm.weight"))
