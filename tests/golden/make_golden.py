"""Generate the golden vectors in this folder from the REFERENCE itself.

Run (needs the reference source tree; not needed to run the tests):

    python tests/golden/make_golden.py /path/to/deepseek-on-one-gpu

It imports the reference's own ``inference.ops.route``, ``inference.ops.rms_norm``
and ``inference.forward.moe_block`` (``inference/ops.py:209-257``,
``inference/ops.py:10-13``, ``inference/forward.py:112-153``) unchanged and runs
them on CPU. The "layer_ffn" cases compose them exactly as the MoE layer's
FFN half does (``inference/forward.py:97-109``): ``hidden +
moe_block(rms_norm(hidden, post_attention_layernorm))``. The three
objects ``moe_block`` touches (``weight_store.get_gate_weight``,
``weight_store.get_shared_expert_weights``, ``gpu_transfer.transfer_experts``,
``inference/forward.py:121,133,147``) are served by in-memory stubs that hand
out seeded synthetic FP8 experts from ``dsmoe.synthetic``.

Only the seeds, shapes and the reference's outputs are stored; the tests
regenerate the inputs from the seeds with the same generator.
"""
from __future__ import annotations

import os
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "deepseek-on-one-gpu_b200"))

from dsmoe.synthetic import SyntheticLayer, activations, logits, norm_weight, uniforms  # noqa: E402

# name: (seed, T, H, F, E, kind)
CASES = {
    "small_t16": (100, 16, 256, 256, 256, "block"),
    "mid_t33": (101, 33, 1024, 512, 256, "block"),
    "tiny_t1": (102, 1, 512, 256, 256, "block"),
    "c1_t8_full": (0, 8, 7168, 2048, 256, "block"),
    "route_t512_full": (1, 512, 7168, 2048, 256, "route"),
    "ffn_t16": (103, 16, 512, 256, 256, "layer_ffn"),
    "ffn_c1_t8_full": (0, 8, 7168, 2048, 256, "layer_ffn"),
    "norm_t16_full": (104, 16, 7168, 2048, 256, "norm"),
}
# Next-token sampling (inference/engine.py:166-190):
# name: (seed, rows, vocab, logit scale, temperature, top_p)
SAMPLE_CASES = {
    "sample_v1000": (200, 8, 1000, 2.0, 0.6, 0.9),
    "sample_v129280": (201, 2, 129280, 3.0, 0.6, 0.9),
    "sample_topp_small": (202, 8, 4096, 1.0, 1.0, 0.05),
    "sample_greedy": (203, 4, 129280, 3.0, 0.0, 0.9),
    "sample_topp1": (204, 4, 2000, 1.5, 0.8, 1.0),
    "sample_hot": (205, 4, 32000, 8.0, 0.3, 0.95),
}
EPS = 1e-6
LAYER = 3


class StubWeightStore:
    """Duck-typed stand-in for ``inference/weight_store.py:WeightStore``."""

    def __init__(self, layer: SyntheticLayer):
        self.layer = layer

    def get_gate_weight(self, layer_idx):
        return self.layer.gate

    def get_shared_expert_weights(self, layer_idx):
        return self.layer.shared()


class StubTransfer:
    """Duck-typed stand-in for ``inference/gpu_transfer.py:GPUTransfer``."""

    def __init__(self, layer: SyntheticLayer):
        self.layer = layer

    def transfer_experts(self, layer_idx, expert_indices, verbose=False):
        return [self.layer.expert(int(e)) for e in expert_indices.tolist()]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from inference import forward as ref_forward  # noqa: E402
    from inference import ops as ref_ops  # noqa: E402
    from inference.config import DeepSeekConfig as RefConfig  # noqa: E402

    torch.set_num_threads(os.cpu_count() or 1)
    only = sys.argv[2:] or list(CASES) + list(SAMPLE_CASES)
    for name in only:
        if name in SAMPLE_CASES:
            make_sample_case(name)
            continue
        seed, T, H, F, E, kind = CASES[name]
        t0 = time.time()
        cfg = RefConfig(hidden_size=H, moe_intermediate_size=F, n_routed_experts=E)
        layer = SyntheticLayer(seed, LAYER, H, F, E)
        x = activations(seed, T, H).view(1, T, H)
        hidden = x
        if kind in ("layer_ffn", "norm"):
            ln = norm_weight(seed, LAYER, 1, H)
            x = ref_ops.rms_norm(hidden, ln, EPS)  # the MoE block's input
        idx, w = ref_ops.route(x, layer.gate, cfg)
        rec = dict(seed=seed, T=T, H=H, F=F, E=E, layer=LAYER, kind=kind,
                   n_group=cfg.n_group, topk_group=cfg.topk_group,
                   top_k=cfg.num_experts_per_tok,
                   routed_scaling_factor=cfg.routed_scaling_factor,
                   idx=idx.reshape(T, -1).clone(), w=w.reshape(T, -1).clone(),
                   torch_version=str(torch.__version__))
        if kind in ("layer_ffn", "norm"):
            rec["eps"] = EPS
            rec["normed"] = x.reshape(T, H).clone()
        if kind in ("block", "layer_ffn"):
            out = ref_forward.moe_block(x, LAYER, StubWeightStore(layer), StubTransfer(layer), cfg)
            if kind == "layer_ffn":
                rec["moe"] = out.reshape(T, H).clone()  # the block's output before the residual add
                out = hidden + out
            rec["out"] = out.reshape(T, H).clone()
        torch.save(rec, HERE / f"{name}.pt")
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)


def make_sample_case(name: str) -> None:
    sys.path.insert(0, str(REPO))
    from inference import engine as ref_engine  # noqa: E402
    from oracle.sampler import inverse_cdf  # noqa: E402

    seed, B, V, scale, temperature, top_p = SAMPLE_CASES[name]
    x = logits(seed, B, V, scale)
    u = uniforms(seed, B)
    seen = {}

    def draw(probs, num_samples, *args, **kwargs):
        seen["kept"] = (probs > 0).sum(dim=-1)
        return inverse_cdf(probs, u)[:, None]

    real = torch.multinomial
    torch.multinomial = draw
    try:
        tokens = ref_engine.sample(x.clone(), temperature, top_p)
    finally:
        torch.multinomial = real
    kept = seen.get("kept", torch.ones(B, dtype=torch.int64))
    rec = dict(seed=seed, rows=B, vocab=V, scale=scale, temperature=temperature, top_p=top_p, u=u.clone(),
               tokens=tokens.reshape(B).clone(), nucleus=kept.reshape(B).clone(), torch_version=str(torch.__version__))
    torch.save(rec, HERE / f"{name}.pt")
    print(f"{name}: tokens {rec['tokens'].tolist()} nucleus {rec['nucleus'].tolist()}", flush=True)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DSMOE_REFERENCE_ROOT", ""))
