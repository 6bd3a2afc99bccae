"""CPU oracle for the DeepSeek-R1 MoE block — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it. The CUDA path in ``dsmoe`` never calls it and fails loudly when its
extension is missing.

It restates, in plain torch-on-CPU fp32/bf16 arithmetic, the reference
algorithm of ``sushruta/deepseek-on-one-gpu``:

  * ``rms_norm``       — ``inference/ops.py:10-13``
  * ``route_ref``      — ``inference/ops.py:209-257``
  * ``fp8_linear``     — ``inference/ops.py:15-44``
  * ``expert_ffn``     — ``inference/ops.py:186-192, 202-206``
  * ``moe_block_literal`` — ``inference/forward.py:112-153`` (per-token loop)
  * ``moe_layer_ffn``  — ``inference/forward.py:97-109`` (the MoE layer's FFN
    half: ``hidden + moe_block(rms_norm(hidden, post_attention_layernorm))``)
  * ``moe_block_grouped`` — the same arithmetic grouped by expert, for sizes the
    literal loop cannot finish in seconds. Per element it performs the same
    fp32 dequant, fp32 dot products, bf16 roundings and bf16 combine order;
    only the summation order inside the fp32 GEMM may differ (batched rows
    against a single row).

The functions are device-agnostic torch code. The golden and small-shape
checks run them on CPU tensors; the full-shape checks of the benchmark
configurations (thousands of rows through all 257 experts) run the same code
on CUDA tensors as a plain fp32 torch reference (TF32 off, so every matmul is
an fp32 matmul; only its summation order differs from the CPU's).

Parity is pinned: ``tests/golden/`` holds outputs of the reference's own
``moe_block`` and ``route`` (imported from the reference tree by
``tests/golden/make_golden.py``) and ``tests/test_oracle_golden.py`` checks this
module against them.

``route_v3`` restates the bias-corrected DeepSeek-V3 router, which the
reference does not implement: it is *parity unpinned* by the reference.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

BLOCK = 128


# --------------------------------------------------------------------------
# Router
# --------------------------------------------------------------------------
def router_logits(hidden: torch.Tensor, gate_weight: torch.Tensor) -> torch.Tensor:
    """fp32 logits, ``inference/ops.py:224``."""
    return hidden.float() @ gate_weight.float().T


def route_ref(hidden: torch.Tensor, gate_weight: torch.Tensor, n_group: int = 8,
              topk_group: int = 4, top_k: int = 8, norm_topk_prob: bool = True):
    """Reference router, ``inference/ops.py:209-257``.

    sigmoid scores (:225); group score is the group's max (:239); the
    ``topk_group`` best groups survive (:240); other experts are set to 0.0
    (:243-248); top-``top_k`` of the masked scores (:251); weights normalised
    by ``sum + 1e-9`` (:254-255). Returns (int64 indices, fp32 weights) in
    descending score order.
    """
    scores = torch.sigmoid(router_logits(hidden, gate_weight))
    E = scores.shape[-1]
    grouped = scores.view(*scores.shape[:-1], n_group, E // n_group)
    gscore = grouped.amax(dim=-1)
    keep_groups = gscore.topk(topk_group, dim=-1).indices
    gmask = torch.zeros_like(gscore, dtype=torch.bool).scatter_(-1, keep_groups, True)
    masked = torch.where(gmask.unsqueeze(-1), grouped, torch.zeros((), dtype=scores.dtype))
    masked = masked.view(*scores.shape[:-1], E)
    w, idx = masked.topk(top_k, dim=-1)
    if norm_topk_prob:
        w = w / (w.sum(dim=-1, keepdim=True) + 1e-9)
    return idx, w


def route_v3(hidden: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor,
             n_group: int = 8, topk_group: int = 4, top_k: int = 8,
             routed_scaling_factor: float = 2.5):
    """Bias-corrected (DeepSeek-V3) router, restated from the published
    description; not implemented by the reference, so parity is unpinned.

    Selection uses ``s + bias``; a group's score is the sum of its two largest
    biased scores; the ``topk_group`` best groups survive, others are -inf;
    top-``top_k`` by biased score; the returned weights are the *unbiased*
    scores at those experts, renormalised, times ``routed_scaling_factor``.
    """
    s = torch.sigmoid(router_logits(hidden, gate_weight))
    sb = s + bias.float()
    E = s.shape[-1]
    g = sb.view(*sb.shape[:-1], n_group, E // n_group)
    gscore = g.topk(2, dim=-1).values.sum(dim=-1)
    keep_groups = gscore.topk(topk_group, dim=-1).indices
    gmask = torch.zeros_like(gscore, dtype=torch.bool).scatter_(-1, keep_groups, True)
    masked = torch.where(gmask.unsqueeze(-1), g, torch.full((), float("-inf")))
    idx = masked.view(*sb.shape[:-1], E).topk(top_k, dim=-1).indices
    w = s.gather(-1, idx)
    w = w / w.sum(dim=-1, keepdim=True)
    return idx, w * routed_scaling_factor


# --------------------------------------------------------------------------
# RMSNorm
# --------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``inference/ops.py:10-13``: fp32 mean of squares, rsqrt, the product
    rounded to x's dtype, then the bf16 product with the weight."""
    r = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps)
    return (x.float() * r).to(x.dtype) * weight


# --------------------------------------------------------------------------
# Expert FFN
# --------------------------------------------------------------------------
def dequant(weight: torch.Tensor, scale_inv: torch.Tensor) -> torch.Tensor:
    """Block dequant to fp32, ``inference/ops.py:37-43``: every element of a
    128x128 block multiplied by that block's ``weight_scale_inv``."""
    O, I = weight.shape
    bo, bi = math.ceil(O / BLOCK), math.ceil(I / BLOCK)
    w = torch.zeros(bo * BLOCK, bi * BLOCK, dtype=torch.float32, device=weight.device)
    w[:O, :I] = weight.float()
    w = (w.view(bo, BLOCK, bi, BLOCK) * scale_inv.float()[:, None, :, None]).view(bo * BLOCK, bi * BLOCK)
    return w[:O, :I]


def fp8_linear(x: torch.Tensor, weight: torch.Tensor, scale_inv: torch.Tensor,
               out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``inference/ops.py:15-44``: fp32 matmul against the fp32-dequantised
    weight, rounded to ``out_dtype``."""
    return (x.float() @ dequant(weight, scale_inv).T).to(out_dtype)


def expert_ffn(x: torch.Tensor, ew: dict) -> torch.Tensor:
    """``inference/ops.py:186-192``: ``down(silu(gate(x)) * up(x))`` with every
    intermediate rounded to bf16 as the reference's dtypes dictate."""
    g = F.silu(fp8_linear(x, *ew["gate_proj"]))
    u = fp8_linear(x, *ew["up_proj"])
    return fp8_linear(g * u, *ew["down_proj"])


# --------------------------------------------------------------------------
# MoE block
# --------------------------------------------------------------------------
def combine_token(routed_rows: list[torch.Tensor], weights: torch.Tensor) -> torch.Tensor:
    """``inference/forward.py:151``: ``routed += w_k * e_out`` in bf16, in top-k
    order. The fp32 0-dim weight is rounded to bf16 by type promotion, the
    product is rounded to bf16, then the running sum is rounded to bf16."""
    acc = torch.zeros_like(routed_rows[0])
    for k, row in enumerate(routed_rows):
        acc += weights[k] * row
    return acc


def moe_block_literal(hidden: torch.Tensor, gate_weight: torch.Tensor, get_expert, shared: dict,
                      n_group=8, topk_group=4, top_k=8, norm_topk_prob=True,
                      routed_scaling_factor=2.5, route_fn=None):
    """Per-token restatement of ``inference/forward.py:112-153``."""
    if route_fn is None:
        idx, w = route_ref(hidden, gate_weight, n_group, topk_group, top_k, norm_topk_prob)
    else:
        idx, w = route_fn(hidden)
    shared_out = expert_ffn(hidden, shared)
    routed = torch.zeros_like(hidden)
    B, S, K = idx.shape
    for b in range(B):
        for s in range(S):
            tok = hidden[b, s].unsqueeze(0).unsqueeze(0)
            for k in range(K):
                e_out = expert_ffn(tok, get_expert(int(idx[b, s, k])))
                routed[b, s] += w[b, s, k] * e_out.squeeze(0).squeeze(0)
    return shared_out + routed * routed_scaling_factor, idx, w


def moe_block_grouped(hidden: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, get_expert,
                      shared: dict, routed_scaling_factor=2.5, final_scale: float | None = None):
    """Grouped-by-expert restatement of ``inference/forward.py:131-153`` for a
    given routing. ``final_scale`` overrides the post-combine scale (1.0 for the
    bias-corrected router, whose weights already carry the factor)."""
    H = hidden.shape[-1]
    x = hidden.reshape(-1, H)
    T = x.shape[0]
    K = idx.shape[-1]
    idx2 = idx.reshape(T, K)
    w2 = w.reshape(T, K)
    shared_out = expert_ffn(x, shared)
    y = torch.empty(T, K, H, dtype=torch.bfloat16, device=x.device)
    for e in torch.unique(idx2).tolist():
        t_sel, k_sel = (idx2 == e).nonzero(as_tuple=True)
        y[t_sel, k_sel] = expert_ffn(x[t_sel], get_expert(e))
    routed = torch.zeros(T, H, dtype=torch.bfloat16, device=x.device)
    for k in range(K):
        routed += (w2[:, k:k + 1].to(torch.bfloat16) * y[:, k]).to(torch.bfloat16)
    scale = routed_scaling_factor if final_scale is None else final_scale
    out = shared_out + routed * scale
    return out.reshape(hidden.shape)


def moe_layer_ffn(hidden: torch.Tensor, ln_weight: torch.Tensor, eps: float, gate_weight: torch.Tensor,
                  get_expert, shared: dict, **kw) -> torch.Tensor:
    """``inference/forward.py:97-109`` for a MoE layer: the block on the
    RMS-normalised hidden state, plus the residual (a bf16 add)."""
    normed = rms_norm(hidden, ln_weight, eps)
    idx, w = route_ref(normed, gate_weight)
    return hidden + moe_block_grouped(normed, idx, w, get_expert, shared, **kw)


def rel_rms(a: torch.Tensor, b: torch.Tensor) -> float:
    """sqrt(mean((a-b)^2)) / sqrt(mean(b^2)), in fp64."""
    a = a.double()
    b = b.double()
    return float(((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt().clamp_min(1e-30)))


def index_parity(idx_a: torch.Tensor, idx_b: torch.Tensor, scores: torch.Tensor,
                 tie_eps: float = 1e-6) -> tuple[int, int]:
    """Compare two top-k index sets row by row.

    A row passes if the index lists are equal, or if every position where they
    differ is explained by an fp32 score tie: the two experts' scores (taken
    from ``scores``, the oracle's selection scores) lie within ``tie_eps``.
    Returns (rows_mismatched_unexplained, rows_differing_at_ties)."""
    a = idx_a.reshape(-1, idx_a.shape[-1]).long()
    b = idx_b.reshape(-1, idx_b.shape[-1]).long()
    sc = scores.reshape(a.shape[0], -1).double()
    bad = ties = 0
    for r in range(a.shape[0]):
        if torch.equal(a[r], b[r]):
            continue
        sa = sc[r, a[r]]
        sb = sc[r, b[r]]
        if torch.all((sa - sb).abs() <= tie_eps) and \
                torch.allclose(sa.sort().values, sb.sort().values, atol=tie_eps, rtol=0):
            ties += 1
        else:
            bad += 1
    return bad, ties
