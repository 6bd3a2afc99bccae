"""Drop-in replacements for the MoE ops of ``inference/ops.py``.

Same names, argument order and return types as the reference:
  * ``rms_norm(x, weight, eps)``                   — ``inference/ops.py:10-13``
  * ``route(hidden, gate_weight, config)``         — ``inference/ops.py:209-257``
  * ``fp8_linear(x, weight, scale_inv, out_dtype)``— ``inference/ops.py:15-44``
  * ``swiglu(...)`` / ``expert_ffn(hidden, w)``    — ``inference/ops.py:186-206``
  * ``dense_ffn(hidden, mlp_weights)``             — ``inference/ops.py:195-199``
    (the dense FFN of layers 0-2, intermediate size 18432)
Each call goes through ``libdsmoe.so`` on the current CUDA stream; CPU tensors
are rejected (there is no CPU path).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_handle


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight)`` over the last dim
    (bf16 x and weight, last dim a multiple of 8)."""
    H = x.shape[-1]
    x2 = x.reshape(-1, H).contiguous()
    require_cuda(x2, weight)
    if x2.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("rms_norm expects bf16 x and weight")
    out = torch.empty_like(x2)
    check(lib().dsmoe_rms_norm(ptr(x2), ptr(weight.contiguous()), float(eps), x2.shape[0], H, ptr(out),
                               stream_handle(x2.device)), "dsmoe_rms_norm")
    return out.view(x.shape)


def route(hidden: torch.Tensor, gate_weight: torch.Tensor, config, score_bias: torch.Tensor | None = None):
    """Router. ``config.router_mode`` "ref" reproduces the reference; "v3"
    needs ``score_bias`` (e_score_correction_bias). Returns (int64 indices,
    fp32 weights) shaped ``hidden.shape[:-1] + (top_k,)``."""
    H = hidden.shape[-1]
    x = hidden.reshape(-1, H)
    require_cuda(x, gate_weight, score_bias)
    if x.dtype != torch.bfloat16 or gate_weight.dtype != torch.bfloat16:
        raise TypeError("route expects bf16 hidden states and gate weight")
    T = x.shape[0]
    cfg = _lib.moe_config(config)
    K = cfg.top_k
    idx = torch.empty(T, K, dtype=torch.int64, device=x.device)
    w = torch.empty(T, K, dtype=torch.float32, device=x.device)
    ws = _lib.Workspace.get(x.device).ensure(lib().dsmoe_workspace_size(cfg, T))
    check(lib().dsmoe_route(cfg, ptr(x), ptr(gate_weight), ptr(score_bias), T, ptr(idx), ptr(w), ptr(ws),
                            ws.numel(), stream_handle(x.device)), "dsmoe_route")
    shape = tuple(hidden.shape[:-1]) + (K,)
    return idx.view(shape), w.view(shape)


def fp8_linear(x: torch.Tensor, weight: torch.Tensor, scale_inv: torch.Tensor,
               out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``out = x @ dequant(weight, scale_inv).T`` in bf16. In features are a
    multiple of 128; out features a multiple of 8 (the last 128-row scale
    block may be partial, e.g. the 576 outputs of ``kv_a_proj_with_mqa``)."""
    if out_dtype != torch.bfloat16:
        raise TypeError("fp8_linear produces bf16 output")
    O, I = weight.shape
    x2 = x.reshape(-1, I)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    x2 = x2.contiguous()
    require_cuda(x2, weight, scale_inv)
    T = x2.shape[0]
    out = torch.empty(T, O, dtype=torch.bfloat16, device=x2.device)
    ws = _lib.Workspace.get(x2.device).ensure(lib().dsmoe_fp8_linear_workspace_size(T, I, O))
    check(lib().dsmoe_fp8_linear(ptr(x2), T, I, O, ptr(weight), ptr(scale_inv), ptr(out), ptr(ws), ws.numel(),
                                 stream_handle(x2.device)), "dsmoe_fp8_linear")
    return out.view(*x.shape[:-1], O)


def swiglu(x, gate_proj, gate_scale, up_proj, up_scale, down_proj, down_scale) -> torch.Tensor:
    """``down(silu(gate(x)) * up(x))`` as one fused pair of grouped GEMMs."""
    F, H = gate_proj.shape
    x2 = x.reshape(-1, H)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    x2 = x2.contiguous()
    require_cuda(x2, gate_proj, gate_scale, up_proj, up_scale, down_proj, down_scale)
    T = x2.shape[0]
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x2.device)
    ws = _lib.Workspace.get(x2.device).ensure(lib().dsmoe_expert_ffn_workspace_size(T, H, F))
    check(lib().dsmoe_expert_ffn(ptr(x2), T, H, F, ptr(gate_proj), ptr(gate_scale), ptr(up_proj), ptr(up_scale),
                                 ptr(down_proj), ptr(down_scale), ptr(out), ptr(ws), ws.numel(),
                                 stream_handle(x2.device)), "dsmoe_expert_ffn")
    return out.view(*x.shape[:-1], H)


def expert_ffn(hidden: torch.Tensor, expert_weights: dict[str, tuple[torch.Tensor, torch.Tensor]]) -> torch.Tensor:
    return swiglu(hidden, *expert_weights["gate_proj"], *expert_weights["up_proj"], *expert_weights["down_proj"])


def dense_ffn(hidden: torch.Tensor, mlp_weights: dict) -> torch.Tensor:
    """The dense FFN of the first ``first_k_dense_replace`` layers
    (``inference/ops.py:195-199``): the same FP8 SwiGLU as an expert, with
    the dense intermediate size."""
    return swiglu(hidden, *mlp_weights["gate_proj"], *mlp_weights["up_proj"], *mlp_weights["down_proj"])
