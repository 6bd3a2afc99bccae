"""Host-side logic that needs no GPU: the pinned-RAM LRU, the expert slot
table of a layer bank, the synthetic generators and the config mirror."""
import os
import sys

import pytest
import torch

from dsmoe import DeepSeekConfig, ExpertCache
from dsmoe.config import load_config
from dsmoe.gpu_transfer import LayerBank
from dsmoe.synthetic import FP8_MAX, SyntheticLayer, activations, block_quantize, expert_weights, score_bias

# the reference source tree: $DSMOE_REFERENCE_ROOT, else a "reference" folder beside this repository
REF_ROOT = os.environ.get("DSMOE_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")


def entry(nbytes):
    return {"gate_proj": {"weight": torch.zeros(nbytes, dtype=torch.uint8)}}


def test_expert_cache_lru_policy():
    c = ExpertCache(300)
    c.put(0, 1, entry(100))
    c.put(0, 2, entry(100))
    c.put(0, 3, entry(100))
    assert c.used == 300
    assert c.get(0, 1) is not None          # 1 becomes most recent
    c.put(0, 4, entry(100))                 # evicts 2 (least recent)
    assert c.get(0, 2) is None
    assert [k[1] for k in c.entries] == [3, 1, 4]
    c.put(0, 5, entry(250))                 # evicts until it fits
    assert [k[1] for k in c.entries] == [5] and c.used == 250
    assert c.hits == 1 and c.misses == 1


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_ROOT, "inference")), reason="reference tree not present")
def test_expert_cache_matches_reference_trace():
    sys.path.insert(0, REF_ROOT)
    from inference.weight_store import ExpertCache as RefCache
    g = torch.Generator().manual_seed(0)
    a, b = ExpertCache(1000), RefCache(1000)
    for _ in range(400):
        key = int(torch.randint(0, 12, (1,), generator=g))
        size = int(torch.randint(50, 300, (1,), generator=g))
        if a.get(0, key) is None:
            assert b.get(0, key) is None
            a.put(0, key, entry(size))
            b.put(0, key, entry(size))
        else:
            assert b.get(0, key) is not None
        assert list(a.entries) == list(b.entries) and a.used == b.used


def test_bank_slot_lru_and_pinning():
    cfg = DeepSeekConfig(hidden_size=128, moe_intermediate_size=128)
    b = LayerBank(cfg, n_slots=4, device=torch.device("cpu"))
    assert b.assign(0) == 0                 # shared expert
    s1, s2, s3 = b.assign(1), b.assign(2), b.assign(3)
    assert (s1, s2, s3) == (1, 2, 3) and not b.fully_resident
    b.assign(1)                             # refresh 1
    s4 = b.assign(4, pinned={1, 4})         # evicts 2 (LRU, not pinned)
    assert s4 == 2 and b.slot_of_host[2] == -1 and b.slot_of_host[4] == 2
    with pytest.raises(RuntimeError):
        b.assign(5, pinned={1, 3, 4, 5})
    b.sync_table(non_blocking=False)
    assert b.slot_of[4].item() == 2 and b.slot_of[0].item() == 0


def test_bank_write_slot_roundtrip():
    cfg = DeepSeekConfig(hidden_size=256, moe_intermediate_size=128)
    b = LayerBank(cfg, n_slots=2, device=torch.device("cpu"))
    ew = expert_weights(1, 3, 5, 256, 128)
    b.write_slot(b.assign(6), ew)
    v = b.views(6)
    for p in ew:
        assert torch.equal(v[p][0].view(torch.uint8), ew[p][0].view(torch.uint8))
        assert torch.equal(v[p][1], ew[p][1])


def test_block_quantize_bounds_and_dequant():
    w = torch.randn(256, 384) * 0.02
    q, s = block_quantize(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (2, 3)
    assert q.float().abs().max() <= FP8_MAX
    deq = (q.float().view(2, 128, 3, 128) * s[:, None, :, None]).view(256, 384)
    assert (deq - w).abs().max() <= 0.07 * w.abs().max()


def test_generators_deterministic():
    a = expert_weights(3, 1, 7, 256, 128)
    b = expert_weights(3, 1, 7, 256, 128)
    c = expert_weights(3, 1, 8, 256, 128)
    assert torch.equal(a["gate_proj"][0].view(torch.uint8), b["gate_proj"][0].view(torch.uint8))
    assert not torch.equal(a["gate_proj"][0].view(torch.uint8), c["gate_proj"][0].view(torch.uint8))
    assert torch.equal(activations(1, 4, 256), activations(1, 4, 256))
    L = SyntheticLayer(0, 3, 256, 128, 256)
    assert L.gate.dtype == torch.bfloat16 and L.gate.shape == (256, 256)


def test_zipf_bias_is_skewed():
    b = score_bias(3, 3, 256, zipf_s=1.1)
    assert b.max() - b.min() > 2.0          # 0.5*log(Zipf) spans several units
    assert len(set(b.tolist())) == 256


def test_config_mirror_and_loader(tmp_path):
    cfg = DeepSeekConfig()
    assert (cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts) == (7168, 2048, 256)
    assert (cfg.n_group, cfg.topk_group, cfg.num_experts_per_tok, cfg.routed_scaling_factor) == (8, 4, 8, 2.5)
    (tmp_path / "config.json").write_text('{"hidden_size": 1024, "n_routed_experts": 64, "n_group": 2,'
                                          ' "quantization_config": {"weight_block_size": [128, 128]}}')
    c2 = load_config(tmp_path, router_mode="v3")
    assert (c2.hidden_size, c2.n_routed_experts, c2.n_group, c2.router_mode) == (1024, 64, 2, "v3")


@pytest.mark.parametrize("check_every", [1, 3, 7, 64])
def test_generate_tokens_loop_rules(check_every):
    """The decode loop's host rules (engine.py:116-151) with a stand-in
    sampler (argmax on the CPU): the first token is kept even if it is the
    end-of-sequence token, a later one ends the output unkept, at most
    max_tokens tokens, whatever the host-check interval."""
    from dsmoe.sampling import generate_tokens

    V = 10
    script = [3, 5, 9, 2, 9, 4, 1, 7, 8, 6, 0, 2]  # token produced by decode step i

    def one_hot(t):
        x = torch.full((1, V), -1.0)
        x[0, t] = 1.0
        return x

    def step(token, i):  # steps past the script (run ahead of the host check) repeat it
        return one_hot(script[i % len(script)])

    def argmax_sampler(logits, temperature, top_p, u, out):
        out.copy_(logits.argmax(dim=-1))
        return out

    def run(first, max_tokens, eos):
        return generate_tokens(step, one_hot(first), max_tokens, eos, temperature=0.0,
                               check_every=check_every, sampler=argmax_sampler)

    assert run(4, 8, None) == [4] + script[:7]
    assert run(4, 1, None) == [4]
    assert run(4, 0, None) == []
    assert run(4, 20, 9) == [4, 3, 5]            # stops at the first 9, unkept
    assert run(9, 20, 9) == [9, 3, 5]            # the first token is kept even when it is the eos
    assert run(4, 3, 9) == [4, 3, 5]             # max_tokens reached before the eos
    assert run(4, 12, 0) == [4] + script[:10]    # eos at decode step 10
