"""The CPU oracle is pinned to the reference: golden vectors in tests/golden
are outputs of the reference's own route(), rms_norm() and moe_block() (made
by tests/golden/make_golden.py)."""
import os

import pytest
import torch

from conftest import GOLDEN
from dsmoe.synthetic import SyntheticLayer, activations, norm_weight
from oracle import moe_oracle as O

BLOCK_CASES = ["small_t16", "mid_t33", "tiny_t1", "c1_t8_full"]
ROUTE_CASES = BLOCK_CASES + ["route_t512_full"]


def load(name):
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"))


def inputs(g):
    layer = SyntheticLayer(g["seed"], g["layer"], g["H"], g["F"], g["E"])
    return layer, activations(g["seed"], g["T"], g["H"])


@pytest.mark.parametrize("name", ROUTE_CASES)
def test_route_matches_reference_exactly(name):
    g = load(name)
    layer, x = inputs(g)
    idx, w = O.route_ref(x, layer.gate, g["n_group"], g["topk_group"], g["top_k"])
    assert torch.equal(idx, g["idx"])
    assert torch.equal(w, g["w"])


@pytest.mark.parametrize("name", ["small_t16", "tiny_t1", "c1_t8_full"])
def test_literal_block_bit_exact(name):
    g = load(name)
    layer, x = inputs(g)
    out, idx, _ = O.moe_block_literal(x.view(1, g["T"], g["H"]), layer.gate, layer.expert, layer.shared())
    assert torch.equal(out.view(g["T"], -1), g["out"])


@pytest.mark.parametrize("name", ["small_t16", "mid_t33", "tiny_t1"])
def test_grouped_block_close(name):
    g = load(name)
    layer, x = inputs(g)
    out = O.moe_block_grouped(x, g["idx"], g["w"], layer.expert, layer.shared())
    # only the fp32 summation order of the matmul differs from the reference
    assert O.rel_rms(out, g["out"]) < 1e-3


def test_golden_metadata():
    for name in ROUTE_CASES:
        g = load(name)
        assert g["idx"].shape == (g["T"], g["top_k"])
        assert g["idx"].dtype == torch.int64 and g["w"].dtype == torch.float32
        if g["kind"] == "block":
            assert g["out"].dtype == torch.bfloat16 and g["out"].shape == (g["T"], g["H"])


def test_route_v3_properties():
    layer = SyntheticLayer(7, 3, 256, 128, 256, bias_zipf=1.1)
    x = activations(7, 64, 256)
    idx, w = O.route_v3(x, layer.gate, layer.bias)
    assert torch.allclose(w.sum(-1), torch.full((64,), 2.5), atol=1e-5)
    s = torch.sigmoid(O.router_logits(x, layer.gate)) + layer.bias
    groups = (idx // 32)
    for t in range(64):
        assert len(set(groups[t].tolist())) <= 4
        # chosen experts are the 8 best by biased score inside the kept groups
        kept = set(groups[t].tolist())
        cand = [e for e in range(256) if e // 32 in kept]
        best = sorted(cand, key=lambda e: -float(s[t, e]))[:8]
        assert sorted(best) == sorted(idx[t].tolist())


def test_index_parity_tie_rule():
    scores = torch.tensor([[0.9, 0.5, 0.5 + 5e-7, 0.1]])
    a = torch.tensor([[0, 1]])
    b = torch.tensor([[0, 2]])
    bad, ties = O.index_parity(a, b, scores)
    assert (bad, ties) == (0, 1)
    c = torch.tensor([[0, 3]])
    bad, ties = O.index_parity(a, c, scores)
    assert (bad, ties) == (1, 0)


NORM_CASES = ["norm_t16_full", "ffn_t16", "ffn_c1_t8_full"]


@pytest.mark.parametrize("name", NORM_CASES)
def test_rms_norm_matches_reference_exactly(name):
    g = load(name)
    x = activations(g["seed"], g["T"], g["H"])
    normed = O.rms_norm(x, norm_weight(g["seed"], g["layer"], 1, g["H"]), g["eps"])
    assert torch.equal(normed, g["normed"])


@pytest.mark.parametrize("name", ["ffn_t16", "ffn_c1_t8_full"])
def test_layer_ffn_close(name):
    """hidden + moe_block(rms_norm(hidden)): the routing on the normalised
    input equals the reference's; the output matches up to the fp32 GEMM
    summation order of the grouped restatement."""
    g = load(name)
    layer, x = inputs(g)
    normed = O.rms_norm(x, norm_weight(g["seed"], g["layer"], 1, g["H"]), g["eps"])
    idx, w = O.route_ref(normed, layer.gate)
    assert torch.equal(idx, g["idx"]) and torch.equal(w, g["w"])
    out = O.moe_layer_ffn(x, norm_weight(g["seed"], g["layer"], 1, g["H"]), g["eps"], layer.gate, layer.expert,
                          layer.shared())
    assert O.rel_rms(out, g["out"]) < 1e-3


SAMPLE_CASES = ["sample_v1000", "sample_v129280", "sample_topp_small", "sample_greedy", "sample_topp1", "sample_hot"]


@pytest.mark.parametrize("name", SAMPLE_CASES)
def test_sampler_matches_reference_exactly(name):
    """oracle/sampler.py against the reference's own sample() (run with the
    same explicit draw): same tokens, same nucleus sizes."""
    from dsmoe.synthetic import logits
    from oracle import sampler as S
    g = load(name)
    x = logits(g["seed"], g["rows"], g["vocab"], g["scale"])
    tokens, nucleus = S.sample_top_p(x, g["temperature"], g["top_p"], g["u"])
    assert torch.equal(tokens, g["tokens"])
    if g["temperature"] != 0:
        assert torch.equal(nucleus, g["nucleus"])


def test_sampler_oracle_properties():
    """Small cases worked by hand: the nucleus rule and the explicit draw."""
    from oracle import sampler as S
    # probabilities 0.5, 0.3, 0.2 (logits = log p, T = 1)
    x = torch.log(torch.tensor([[0.2, 0.5, 0.3]]))
    for top_p, kept in ((0.0, 1), (0.49, 1), (0.5, 2), (0.79, 2), (0.81, 3), (1.0, 3)):
        _, n = S.sample_top_p(x, 1.0, top_p, torch.tensor([0.0]))
        assert int(n) == kept, (top_p, int(n))
    # all kept: u below 0.5 -> index 1, [0.5, 0.8) -> index 2, above -> index 0
    for u, tok in ((0.0, 1), (0.49, 1), (0.51, 2), (0.79, 2), (0.81, 0), (0.999, 0)):
        t, _ = S.sample_top_p(x, 1.0, 1.0, torch.tensor([u]))
        assert int(t) == tok, (u, int(t))
    # top 2 kept (mass 0.8): renormalised 0.625 / 0.375
    for u, tok in ((0.6, 1), (0.63, 2)):
        t, _ = S.sample_top_p(x, 1.0, 0.5, torch.tensor([u]))
        assert int(t) == tok, (u, int(t))
    # temperature 0: argmax, first of equal maxima
    t, _ = S.sample_top_p(torch.tensor([[1.0, 3.0, 3.0, 2.0]]), 0.0, 0.9, None)
    assert int(t) == 1
