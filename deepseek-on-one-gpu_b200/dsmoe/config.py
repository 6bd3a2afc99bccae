"""MoE-block configuration.

Mirrors the reference's frozen ``DeepSeekConfig`` dataclass
(``inference/config.py:6-52``): same field names, same defaults, so a config
object built by the reference's ``load_config`` (``inference/config.py:55-94``)
can be passed to this package unchanged (only attribute access is used).

One field is added: ``router_mode``.
  * ``"ref"`` — the reference router (``inference/ops.py:209-257``): no score
    bias, group score = max of the group, non-selected groups masked to 0.0,
    weights normalised with ``+1e-9`` and ``routed_scaling_factor`` applied
    after the combine (``inference/forward.py:153``).
  * ``"v3"`` — the bias-corrected DeepSeek-V3 router: selection on
    ``sigmoid(logit) + e_score_correction_bias``, group score = sum of the two
    largest biased scores, masked groups at -inf, weights are the unbiased
    scores renormalised and multiplied by ``routed_scaling_factor`` inside the
    router (the combine then does not scale again).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, replace
from pathlib import Path


@dataclass(frozen=True)
class DeepSeekConfig:
    hidden_size: int = 7168
    num_layers: int = 61
    num_attention_heads: int = 128
    num_key_value_heads: int = 128
    vocab_size: int = 129280

    q_lora_rank: int = 1536
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    qk_head_dim: int = 192

    rope_theta: float = 10000.0
    max_position_embeddings: int = 163840
    rope_scaling_factor: float = 40.0
    rope_scaling_beta_fast: int = 32
    rope_scaling_beta_slow: int = 1
    rope_scaling_mscale: float = 1.0
    rope_scaling_mscale_all_dim: float = 1.0
    original_max_position_embeddings: int = 4096

    # MoE (inference/config.py:32-39)
    n_routed_experts: int = 256
    num_experts_per_tok: int = 8
    n_group: int = 8
    topk_group: int = 4
    moe_intermediate_size: int = 2048
    routed_scaling_factor: float = 2.5
    norm_topk_prob: bool = True

    intermediate_size: int = 18432
    first_k_dense_replace: int = 3
    n_shared_experts: int = 1
    rms_norm_eps: float = 1e-6
    fp8_block_size: int = 128

    # Added: router semantics, "ref" (reference) or "v3" (bias-corrected).
    router_mode: str = "ref"

    def with_(self, **kw) -> "DeepSeekConfig":
        return replace(self, **kw)


def load_config(model_path: str | Path, router_mode: str = "ref") -> DeepSeekConfig:
    """Read ``config.json`` the way ``inference/config.py:55-94`` does (MoE
    fields and the block size; the attention fields keep their defaults)."""
    raw = json.loads((Path(model_path) / "config.json").read_text())
    return DeepSeekConfig(
        hidden_size=raw.get("hidden_size", 7168),
        num_layers=raw.get("num_hidden_layers", 61),
        n_routed_experts=raw.get("n_routed_experts", 256),
        num_experts_per_tok=raw.get("num_experts_per_tok", 8),
        n_group=raw.get("n_group", 8),
        topk_group=raw.get("topk_group", 4),
        moe_intermediate_size=raw.get("moe_intermediate_size", 2048),
        routed_scaling_factor=raw.get("routed_scaling_factor", 2.5),
        norm_topk_prob=raw.get("norm_topk_prob", True),
        n_shared_experts=raw.get("n_shared_experts", 1),
        fp8_block_size=raw.get("quantization_config", {}).get("weight_block_size", [128, 128])[0],
        router_mode=router_mode,
    )


def cfg_get(config, name: str, default):
    """Attribute access that tolerates the reference's config (no router_mode)."""
    return getattr(config, name, default)
