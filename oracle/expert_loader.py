"""Restatement of the reference's expert disk read — TEST AND BASELINE
INFRASTRUCTURE ONLY (tests/ and the baseline leg of bench.py use it; the
product never does).

``load_expert`` follows ``WeightStore._load_expert_from_disk``
(``inference/weight_store.py:151-180``) step by step: group the expert's six
keys (``expert_tensor_keys``, :33-40) by shard, open each shard with
safetensors' ``safe_open`` (third-party: the ``safetensors`` package, 0.7.0
in this image; the reference's requirements.txt does not pin it),
``get_tensor`` every key, copy each tensor into a freshly pinned one, and
return ``{proj: {"weight", "weight_scale_inv"}}``.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors import safe_open

PROJS = ("gate_proj", "up_proj", "down_proj")


def expert_tensor_keys(layer: int, expert_idx: int) -> list[str]:
    prefix = f"model.layers.{layer}.mlp.experts.{expert_idx}"
    return [f"{prefix}.{proj}.{suffix}" for proj in PROJS for suffix in ("weight", "weight_scale_inv")]


def shard_map(model_path: str | Path) -> dict[str, str]:
    root = Path(model_path)
    index = root / "model.safetensors.index.json"
    if index.exists():
        with open(index) as f:
            return json.load(f)["weight_map"]
    single = sorted(p.name for p in root.glob("*.safetensors"))[0]
    with safe_open(str(root / single), framework="pt", device="cpu") as f:
        return {k: single for k in f.keys()}


def load_expert(model_path: str | Path, key_to_shard: dict[str, str], layer: int, expert_idx: int,
                pin: bool = True) -> dict:
    root = Path(model_path)
    keys_by_shard: dict[str, list[str]] = {}
    for key in expert_tensor_keys(layer, expert_idx):
        keys_by_shard.setdefault(key_to_shard[key], []).append(key)
    tensors = {}
    for shard, keys in keys_by_shard.items():
        with safe_open(str(root / shard), framework="pt", device="cpu") as f:
            for key in keys:
                t = f.get_tensor(key)
                dst = torch.empty_like(t).pin_memory() if pin else torch.empty_like(t)
                dst.copy_(t)
                tensors[key] = dst
    prefix = f"model.layers.{layer}.mlp.experts.{expert_idx}"
    return {proj: {"weight": tensors[f"{prefix}.{proj}.weight"],
                   "weight_scale_inv": tensors[f"{prefix}.{proj}.weight_scale_inv"]} for proj in PROJS}
