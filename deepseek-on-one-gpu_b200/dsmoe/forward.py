"""Drop-in ``moe_block`` (``inference/forward.py:112-153``).

Same signature and result as the reference: ``hidden`` [B, S, H] bf16 ->
``shared_expert(hidden) + routed_scaling_factor * sum_k w_k expert_k(hidden)``
in bf16. The reference routes, then loops over tokens copying each token's 8
experts to the GPU and running 8 single-token FFNs; here the whole block is
one sequence of CUDA kernels on the current stream:

  router -> permute + FP8 hi/lo split -> grouped gate/up GEMM (+SiLU*mul)
  -> grouped down GEMM -> weighted combine with the shared expert.

``gpu_transfer`` must be this package's ``GPUTransfer``: it owns the layer's
device weight bank. In streaming mode (fewer slots than experts) with a
device-managed slot table (``device_slots``) the missing experts are placed
and copied by ``dsmoe_slotcache_step`` on the device; otherwise the routing is
read back once per block (the reference reads it back once per token, via
``.tolist()``) to bring missing experts in before the expert GEMMs.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_handle


def _layer_weights(bank, gate_weight, bias) -> _lib.LayerWeights:
    return _lib.LayerWeights(
        gate_weight=ptr(gate_weight), score_bias=ptr(bias), n_slots=bank.n_slots,
        w_gate=ptr(bank.w["gate_proj"]), s_gate=ptr(bank.s["gate_proj"]),
        w_up=ptr(bank.w["up_proj"]), s_up=ptr(bank.s["up_proj"]),
        w_down=ptr(bank.w["down_proj"]), s_down=ptr(bank.s["down_proj"]),
        slot_of_expert=ptr(bank.slot_of),
    )


def moe_block(hidden: torch.Tensor, layer_idx: int, weight_store, gpu_transfer, config,
              verbose: bool = False, return_routing: bool = False):
    if not hasattr(gpu_transfer, "ensure_resident"):
        raise TypeError("moe_block needs dsmoe.GPUTransfer (it owns the device expert bank)")
    H = hidden.shape[-1]
    x = hidden.reshape(-1, H)
    if x.dtype != torch.bfloat16:
        raise TypeError("moe_block expects bf16 hidden states")
    x = x.contiguous()
    T = x.shape[0]
    gate_weight = weight_store.get_gate_weight(layer_idx)
    bias = None
    if getattr(config, "router_mode", "ref") == "v3":
        bias = weight_store.get_gate_bias(layer_idx)
    require_cuda(x, gate_weight, bias)
    cfg = _lib.moe_config(config)
    K = cfg.top_k
    out = torch.empty_like(x)
    idx = torch.empty(T, K, dtype=torch.int64, device=x.device)
    w = torch.empty(T, K, dtype=torch.float32, device=x.device)
    ws = _lib.Workspace.get(x.device).ensure(lib().dsmoe_workspace_size(cfg, T))
    stream = stream_handle(x.device)
    bank = gpu_transfer.bank(layer_idx)
    if bank.fully_resident:
        lw = _layer_weights(bank, gate_weight, bias)
        check(lib().dsmoe_moe_forward(cfg, lw, ptr(x), T, ptr(out), ptr(idx), ptr(w), ptr(ws), ws.numel(), stream),
              "dsmoe_moe_forward")
    else:
        check(lib().dsmoe_route(cfg, ptr(x), ptr(gate_weight), ptr(bias), T, ptr(idx), ptr(w), ptr(ws), ws.numel(),
                                stream), "dsmoe_route")
        dc = gpu_transfer.device_cache(layer_idx)
        if dc is not None:
            dc.step(idx)  # slot table and copies on the device: no host read
        else:
            experts = torch.unique(idx).tolist()  # one device->host read per block
            if verbose:
                print(f"      [moe L{layer_idx:02d}] {T} tokens -> {len(experts)} distinct experts")
            bank = gpu_transfer.ensure_resident(layer_idx, experts)
        lw = _layer_weights(bank, gate_weight, bias)
        check(lib().dsmoe_moe_experts(cfg, lw, ptr(x), T, ptr(out), ptr(ws), ws.numel(), stream),
              "dsmoe_moe_experts")
    gpu_transfer.mark_used(layer_idx)
    out = out.view(hidden.shape)
    if return_routing:
        shape = tuple(hidden.shape[:-1]) + (K,)
        return out, idx.view(shape), w.view(shape)
    return out


def moe_layer_ffn(hidden: torch.Tensor, layer_idx: int, weight_store, gpu_transfer, config,
                  verbose: bool = False) -> torch.Tensor:
    """The FFN half of a MoE transformer layer (``inference/forward.py:97-109``
    for ``layer_idx >= first_k_dense_replace``):
    ``hidden + moe_block(rms_norm(hidden, post_attention_layernorm))``, bf16.
    With every expert of the layer resident this is one library call
    (``dsmoe_moe_layer_ffn``: the norm kernel, the MoE kernels, and the
    residual add inside the combine)."""
    H = hidden.shape[-1]
    x = hidden.reshape(-1, H).contiguous()
    if x.dtype != torch.bfloat16:
        raise TypeError("moe_layer_ffn expects bf16 hidden states")
    _, post_ln = weight_store.get_layer_norm_weights(layer_idx)
    eps = float(getattr(config, "rms_norm_eps", 1e-6))
    bank = gpu_transfer.bank(layer_idx)
    if not bank.fully_resident:
        from .ops import rms_norm
        normed = rms_norm(x, post_ln, eps)
        return (x + moe_block(normed, layer_idx, weight_store, gpu_transfer, config, verbose=verbose)).view(
            hidden.shape)
    gate_weight = weight_store.get_gate_weight(layer_idx)
    bias = weight_store.get_gate_bias(layer_idx) if getattr(config, "router_mode", "ref") == "v3" else None
    require_cuda(x, gate_weight, bias, post_ln)
    cfg = _lib.moe_config(config)
    T, K = x.shape[0], cfg.top_k
    out = torch.empty_like(x)
    idx = torch.empty(T, K, dtype=torch.int64, device=x.device)
    w = torch.empty(T, K, dtype=torch.float32, device=x.device)
    ws = _lib.Workspace.get(x.device).ensure(lib().dsmoe_moe_layer_ffn_workspace_size(cfg, T))
    lw = _layer_weights(bank, gate_weight, bias)
    check(lib().dsmoe_moe_layer_ffn(cfg, lw, ptr(x), ptr(post_ln), eps, T, ptr(out), ptr(idx), ptr(w), ptr(ws),
                                    ws.numel(), stream_handle(x.device)), "dsmoe_moe_layer_ffn")
    gpu_transfer.mark_used(layer_idx)
    return out.view(hidden.shape)
