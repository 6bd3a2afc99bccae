"""RMSNorm (inference/ops.py:10-13), the MoE layer's FFN half
(inference/forward.py:97-109: hidden + moe_block(rms_norm(hidden))), the dense
FFN of layers 0-2 (inference/ops.py:195-199, intermediate size 18432) and
fp8_linear at attention-projection shapes (inference/ops.py:129-183) on the
GPU, against the reference's golden vectors and the CPU oracle.

Tolerances:
  * rms_norm: the row mean is summed in another order than torch's CPU
    reduction, so 1/sqrt(mean + eps) may differ in its last bit; an output
    element may then differ by one bf16 ulp. At most 1 % of the elements may
    differ, none by more than one ulp.
  * layer FFN: indices identical up to fp32 ties (1e-6); the block's output
    (before the residual add) within rel-RMS 1e-2 of the reference's / the
    oracle's; the fused entry point is bit-identical to the same ops called one
    by one (norm, block, bf16 add), so the residual add itself is exact.
"""
import os

import pytest
import torch

from conftest import GOLDEN
from dsmoe import (DeepSeekConfig, GPUTransfer, SyntheticWeightStore, dense_ffn, fp8_linear, moe_block,
                   moe_layer_ffn, rms_norm)
from dsmoe.synthetic import activations, block_quantize, expert_weights, norm_weight
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REL_RMS_TOL = 1e-2


def golden(name):
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"))


def assert_within_one_ulp(got: torch.Tensor, ref: torch.Tensor, max_frac: float = 0.01):
    got, ref = got.float().cpu(), ref.float().cpu()
    diff = (got - ref).abs()
    # one bf16 ulp of the reference value: 2^(exponent - 7)
    ulp = torch.ldexp(torch.ones_like(ref), torch.frexp(ref).exponent - 8)
    assert bool((diff <= ulp + 0).all()), float((diff / ulp).max())
    frac = float((diff > 0).float().mean())
    assert frac <= max_frac, frac


@pytest.mark.parametrize("name", ["norm_t16_full", "ffn_t16", "ffn_c1_t8_full"])
def test_rms_norm_matches_reference_golden(name):
    g = golden(name)
    x = activations(g["seed"], g["T"], g["H"]).to(DEV)
    w = norm_weight(g["seed"], g["layer"], 1, g["H"]).to(DEV)
    assert_within_one_ulp(rms_norm(x, w, g["eps"]), g["normed"])


@pytest.mark.parametrize("T,H", [(1, 8), (5, 1024), (300, 7168), (3, 8192), (7, 9216), (2, 16384)])
def test_rms_norm_shapes_vs_oracle(T, H):
    """Rows held in registers (H <= 8192) and the two-pass path beyond."""
    gen = torch.Generator().manual_seed(T * 131 + H)
    x = (torch.randn(T, H, generator=gen) * 3.0).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(H, generator=gen)).to(torch.bfloat16)
    got = rms_norm(x.to(DEV), w.to(DEV), 1e-6)
    assert_within_one_ulp(got, O.rms_norm(x, w, 1e-6))


def test_rms_norm_zero_row_and_eps():
    x = torch.zeros(2, 512, dtype=torch.bfloat16)
    x[1, 3] = 1.0
    w = torch.ones(512, dtype=torch.bfloat16)
    got = rms_norm(x.to(DEV), w.to(DEV), 1e-6).cpu()
    assert torch.equal(got[0], torch.zeros(512, dtype=torch.bfloat16))
    assert_within_one_ulp(got, O.rms_norm(x, w, 1e-6), max_frac=1.0)


def layer_setup(g):
    cfg = DeepSeekConfig(hidden_size=g["H"], moe_intermediate_size=g["F"], n_routed_experts=g["E"])
    store = SyntheticWeightStore(cfg, seed=g["seed"], device=DEV, pin_memory=False, gen_device="cpu")
    return cfg, store, GPUTransfer(cfg, store, DEV)


@pytest.mark.parametrize("name", ["ffn_t16", "ffn_c1_t8_full"])
def test_layer_ffn_matches_reference_golden(name):
    g = golden(name)
    cfg, store, gt = layer_setup(g)
    L = store.layer(g["layer"])
    x = activations(g["seed"], g["T"], g["H"]).to(DEV)
    out = moe_layer_ffn(x.view(1, g["T"], -1), g["layer"], store, gt, cfg).view(g["T"], -1)
    # the same ops one by one: norm, block, bf16 residual add
    normed = rms_norm(x, store.get_layer_norm_weights(g["layer"])[1], cfg.rms_norm_eps)
    block, idx, w = moe_block(normed, g["layer"], store, gt, cfg, return_routing=True)
    assert torch.equal(out, x + block)
    # routing on the normalised input and the MoE part against the reference
    scores = torch.sigmoid(O.router_logits(g["normed"], L.gate))
    bad, _ = O.index_parity(idx.cpu(), g["idx"], scores)
    assert bad == 0
    err = O.rel_rms(block.float().cpu(), g["moe"].float())
    assert err < REL_RMS_TOL, err


@pytest.mark.parametrize("T", [1, 200, 1500])
def test_layer_ffn_vs_oracle_sizes(T):
    H, F = 512, 256
    cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F)
    store = SyntheticWeightStore(cfg, seed=90 + T, device=DEV, pin_memory=False, gen_device="cpu")
    gt = GPUTransfer(cfg, store, DEV)
    x = (activations(91 + T, T, H) * 2.0).to(torch.bfloat16)
    out = moe_layer_ffn(x.to(DEV), 4, store, gt, cfg)
    ln = norm_weight(90 + T, 4, 1, H)
    normed = rms_norm(x.to(DEV), ln.to(DEV), cfg.rms_norm_eps)
    block = moe_block(normed, 4, store, gt, cfg)
    assert torch.equal(out, x.to(DEV) + block)
    L = store.layer(4)
    xn = normed.cpu()  # the oracle block on the same normalised input
    idx, w = O.route_ref(xn, L.gate)
    ref = O.moe_block_grouped(xn, idx, w, L.expert, L.shared())
    assert O.rel_rms(block.float().cpu(), ref.float()) < REL_RMS_TOL


def test_layer_ffn_streaming_bank_equals_resident():
    """With a partial slot bank the layer FFN runs norm, block and add as
    separate calls; the result equals the resident fused call."""
    H, F = 256, 128
    cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F)
    store = SyntheticWeightStore(cfg, seed=93, device=DEV, pin_memory=False, gen_device="cpu")
    x = activations(94, 40, H).to(DEV)
    fused = moe_layer_ffn(x, 2, store, GPUTransfer(cfg, store, DEV), cfg)
    streamed = moe_layer_ffn(x, 2, store, GPUTransfer(cfg, store, DEV, slots_per_layer=200), cfg)
    assert torch.equal(fused, streamed)


@pytest.mark.parametrize("T,H,F", [(1, 2048, 18432), (37, 2048, 18432), (3, 7168, 18432)])
def test_dense_ffn_vs_oracle(T, H, F):
    """Dense FFN: 144 K blocks in the down projection (the weight-scale window
    slides past 64 blocks)."""
    w = expert_weights(7, 0, 0, H, F)
    x = activations(8 + T, T, H)
    got = dense_ffn(x.to(DEV), {p: (a.to(DEV), s.to(DEV)) for p, (a, s) in w.items()}).cpu()
    ref = O.expert_ffn(x, w)
    assert O.rel_rms(got.float(), ref.float()) < REL_RMS_TOL


@pytest.mark.parametrize("T,I,O_", [(5, 7168, 576), (33, 512, 200), (2, 1536, 24576), (9, 16384, 7168),
                                    (4, 512, 32768)])
def test_fp8_linear_projection_shapes(T, I, O_):
    """fp8_linear at MLA projection shapes: kv_a_proj_with_mqa (576 outputs, a
    ragged last 128-row block), q_b_proj, o_proj, kv_b_proj."""
    gen = torch.Generator().manual_seed(T + I + O_)
    wq, sc = block_quantize(torch.randn(O_, I, generator=gen) * 0.02)
    x = activations(T + 3, T, I)
    got = fp8_linear(x.to(DEV), wq.to(DEV), sc.to(DEV)).cpu()
    assert got.shape == (T, O_)
    ref = O.fp8_linear(x, wq, sc)
    assert O.rel_rms(got.float(), ref.float()) < REL_RMS_TOL


def test_moe_block_streams_experts_from_safetensors(tmp_path):
    """A checkpoint written in the R1 key layout, read by
    SafetensorsWeightStore (packed pinned buffers, native range reads), streamed
    into a 200-slot bank by GPUTransfer and run through moe_block, matches the
    oracle on the same tensors."""
    from safetensors.torch import save_file

    from dsmoe.safetensors_store import SafetensorsWeightStore

    H, F, E, layer = 512, 256, 256, 5
    cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F)
    tensors = {}
    for e in list(range(E)) + ["shared"]:
        w = expert_weights(11, layer, 300 if e == "shared" else e, H, F)
        pre = f"model.layers.{layer}.mlp." + ("shared_experts." if e == "shared" else f"experts.{e}.")
        for proj, (q, s) in w.items():
            tensors[pre + proj + ".weight"] = q
            tensors[pre + proj + ".weight_scale_inv"] = s
    gate = (torch.randn(E, H, generator=torch.Generator().manual_seed(12)) * 0.006).to(torch.bfloat16)
    tensors[f"model.layers.{layer}.mlp.gate.weight"] = gate
    save_file(tensors, str(tmp_path / "model.safetensors"))
    store = SafetensorsWeightStore(tmp_path, cfg, DEV, expert_cache_bytes=1 << 30)
    gt = GPUTransfer(cfg, store, DEV, slots_per_layer=200)  # 24 tokens use at most 192 experts
    x = activations(13, 24, H)
    out = moe_block(x.to(DEV), layer, store, gt, cfg).cpu()
    assert gt.slot_misses > 0 and store.bytes_read > 0
    idx, w = O.route_ref(x, gate)

    def expert(e):
        pre = f"model.layers.{layer}.mlp.experts.{e}."
        return {p: (tensors[pre + p + ".weight"], tensors[pre + p + ".weight_scale_inv"])
                for p in ("gate_proj", "up_proj", "down_proj")}

    shared = {p: (tensors[f"model.layers.{layer}.mlp.shared_experts.{p}.weight"],
                  tensors[f"model.layers.{layer}.mlp.shared_experts.{p}.weight_scale_inv"])
              for p in ("gate_proj", "up_proj", "down_proj")}
    ref = O.moe_block_grouped(x, idx, w, expert, shared)
    assert O.rel_rms(out.float(), ref.float()) < REL_RMS_TOL
