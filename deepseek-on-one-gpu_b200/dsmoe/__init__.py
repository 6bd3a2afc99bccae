"""dsmoe — B200-native (sm_100a) DeepSeek-R1 MoE block.

Drop-in for the MoE hot path of sushruta/deepseek-on-one-gpu: ``route``,
``fp8_linear``, ``expert_ffn``, ``rms_norm`` (``inference/ops.py``),
``moe_block`` and the MoE layer's FFN half ``moe_layer_ffn``
(``inference/forward.py``), ``GPUTransfer`` (``inference/gpu_transfer.py``) and
``ExpertCache`` (``inference/weight_store.py``) and the decode step's
``sample`` (``inference/engine.py``), all backed by ``libdsmoe.so``.
"""
from .config import DeepSeekConfig, load_config
from .forward import moe_block, moe_layer_ffn
from .gpu_transfer import GPUTransfer, LayerBank
from .ops import dense_ffn, expert_ffn, fp8_linear, rms_norm, route, swiglu
from .sampling import generate_tokens, sample, sample_with_uniforms
from .weight_store import ExpertCache, SyntheticWeightStore

__all__ = [
    "DeepSeekConfig", "load_config", "moe_block", "moe_layer_ffn", "GPUTransfer", "LayerBank", "dense_ffn",
    "expert_ffn", "fp8_linear", "rms_norm", "route", "swiglu", "ExpertCache", "SyntheticWeightStore", "sample",
    "sample_with_uniforms", "generate_tokens",
]
