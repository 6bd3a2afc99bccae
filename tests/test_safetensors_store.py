"""The safetensors-backed weight store (dsmoe.safetensors_store) on CPU: a
small checkpoint in the DeepSeek-R1 key layout (inference/weight_store.py:15-17,
:228-255) is written with the safetensors package, then every tensor the store
returns is compared byte for byte with safetensors' own reader."""
import json

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import save_file

from dsmoe.safetensors_store import SafetensorsIndex, SafetensorsWeightStore, read_into
from dsmoe.synthetic import block_quantize

H, F, E, LAYERS = 256, 128, 6, (3, 4)


def fp8(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return block_quantize(torch.randn(shape, generator=g) * 0.02)


def write_checkpoint(root, single_file=False):
    tensors = {}
    seed = 0
    for layer in LAYERS:
        for e in range(E):
            for proj in ("gate_proj", "up_proj", "down_proj"):
                shape = (F, H) if proj != "down_proj" else (H, F)
                w, s = fp8(shape, seed)
                seed += 1
                tensors[f"model.layers.{layer}.mlp.experts.{e}.{proj}.weight"] = w
                tensors[f"model.layers.{layer}.mlp.experts.{e}.{proj}.weight_scale_inv"] = s
        for proj in ("gate_proj", "up_proj", "down_proj"):
            shape = (F, H) if proj != "down_proj" else (H, F)
            w, s = fp8(shape, seed)
            seed += 1
            tensors[f"model.layers.{layer}.mlp.shared_experts.{proj}.weight"] = w
            tensors[f"model.layers.{layer}.mlp.shared_experts.{proj}.weight_scale_inv"] = s
        tensors[f"model.layers.{layer}.mlp.gate.weight"] = (torch.randn(E, H) * 0.006).to(torch.bfloat16)
        tensors[f"model.layers.{layer}.mlp.gate.e_score_correction_bias"] = torch.randn(E) * 0.01
        tensors[f"model.layers.{layer}.input_layernorm.weight"] = torch.rand(H).to(torch.bfloat16)
        tensors[f"model.layers.{layer}.post_attention_layernorm.weight"] = torch.rand(H).to(torch.bfloat16)
    for proj in ("gate_proj", "up_proj", "down_proj"):  # a dense layer
        shape = (2 * F, H) if proj != "down_proj" else (H, 2 * F)
        w, s = fp8(shape, seed)
        seed += 1
        tensors[f"model.layers.0.mlp.{proj}.weight"] = w
        tensors[f"model.layers.0.mlp.{proj}.weight_scale_inv"] = s
    if single_file:
        save_file(tensors, str(root / "model.safetensors"))
        return tensors
    keys = sorted(tensors)
    shards = {"model-00001-of-00002.safetensors": keys[::2], "model-00002-of-00002.safetensors": keys[1::2]}
    weight_map = {}
    for name, ks in shards.items():
        save_file({k: tensors[k] for k in ks}, str(root / name))
        weight_map.update({k: name for k in ks})
    with open(root / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    return tensors


def same_bytes(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.contiguous().view(torch.uint8),
                                                                     b.contiguous().view(torch.uint8))


def reference_read(root, key):
    index = json.load(open(root / "model.safetensors.index.json"))["weight_map"] \
        if (root / "model.safetensors.index.json").exists() else None
    path = root / (index[key] if index else "model.safetensors")
    with safe_open(str(path), framework="pt", device="cpu") as f:
        return f.get_tensor(key)


@pytest.mark.parametrize("single_file", [False, True])
def test_every_tensor_matches_safetensors_reader(tmp_path, single_file):
    write_checkpoint(tmp_path, single_file)
    store = SafetensorsWeightStore(tmp_path, None, "cpu", pin_memory=False, threads=3)
    for layer in LAYERS:
        for e in range(E):
            got = store.get_expert(layer, e)
            for proj, (w, s) in got.items():
                pre = f"model.layers.{layer}.mlp.experts.{e}.{proj}"
                assert same_bytes(w, reference_read(tmp_path, pre + ".weight"))
                assert same_bytes(s, reference_read(tmp_path, pre + ".weight_scale_inv"))
        for proj, (w, s) in store.get_shared_expert_weights(layer).items():
            pre = f"model.layers.{layer}.mlp.shared_experts.{proj}"
            assert same_bytes(w, reference_read(tmp_path, pre + ".weight"))
            assert same_bytes(s, reference_read(tmp_path, pre + ".weight_scale_inv"))
        assert same_bytes(store.get_gate_weight(layer), reference_read(tmp_path, f"model.layers.{layer}.mlp.gate.weight"))
        assert same_bytes(store.get_gate_bias(layer),
                          reference_read(tmp_path, f"model.layers.{layer}.mlp.gate.e_score_correction_bias"))
        ln_in, ln_post = store.get_layer_norm_weights(layer)
        assert same_bytes(ln_post, reference_read(tmp_path, f"model.layers.{layer}.post_attention_layernorm.weight"))
    for proj, (w, s) in store.get_dense_mlp_weights(0).items():
        assert same_bytes(w, reference_read(tmp_path, f"model.layers.0.mlp.{proj}.weight"))


def test_lru_capacity(tmp_path):
    write_checkpoint(tmp_path)
    one = 3 * F * H + 3 * (F // 128) * (H // 128) * 4  # bytes of one expert's tensors
    store = SafetensorsWeightStore(tmp_path, None, "cpu", expert_cache_bytes=2 * one, pin_memory=False)
    for layer, e in [(3, 0), (3, 1), (3, 0), (3, 2), (3, 1), (4, 5), (3, 2)]:
        store.get_expert(layer, e)
    c = store.expert_cache
    assert (c.hits, c.misses) == (1, 6)
    assert list(c.entries) == [(4, 5), (3, 2)]
    assert c.used <= 2 * one
    w, _ = store.get_expert(3, 2)["up_proj"]
    assert same_bytes(w, reference_read(tmp_path, "model.layers.3.mlp.experts.2.up_proj.weight"))


def test_read_errors_are_reported(tmp_path):
    write_checkpoint(tmp_path)
    idx = SafetensorsIndex(tmp_path)
    loc = idx["model.layers.3.mlp.gate.weight"]
    dst = torch.empty(loc.nbytes, dtype=torch.uint8)
    read_into([loc], [dst], 2)
    loc.offset += 1 << 30  # past the end of the shard
    with pytest.raises(RuntimeError, match="past the end"):
        read_into([loc], [dst], 2)
    loc.path = str(tmp_path / "missing.safetensors")
    with pytest.raises(RuntimeError, match="cannot open"):
        read_into([loc], [dst], 2)
    with pytest.raises(ValueError):
        read_into([idx["model.layers.3.mlp.gate.weight"]], [dst[:-1]], 2)


def test_store_matches_the_reference_loader_restatement(tmp_path):
    """The store's packed buffers hold the bytes the reference's
    _load_expert_from_disk (restated in oracle/expert_loader.py) returns."""
    from oracle.expert_loader import load_expert, shard_map

    write_checkpoint(tmp_path)
    store = SafetensorsWeightStore(tmp_path, None, "cpu", pin_memory=False)
    k2s = shard_map(tmp_path)
    for layer, e in [(3, 0), (4, 5)]:
        ref = load_expert(tmp_path, k2s, layer, e, pin=False)
        got = store.get_expert(layer, e)
        for proj in ("gate_proj", "up_proj", "down_proj"):
            assert same_bytes(got[proj][0], ref[proj]["weight"])
            assert same_bytes(got[proj][1], ref[proj]["weight_scale_inv"])
