"""CPU oracle for next-token sampling — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product. Only ``tests/`` may import it;
``dsmoe.sample`` never calls it.

It restates ``sample`` of the reference (``inference/engine.py:166-190``)
step by step in torch-on-CPU fp32, with the one random step made explicit:
the reference draws the token with ``torch.multinomial(sorted_probs, 1)``
(``engine.py:185``); here the caller passes a uniform ``u`` in [0, 1) per row
and the draw is the inverse CDF of ``sorted_probs`` in its (descending)
order: the first position whose running sum exceeds ``u * sum``.

Parity is pinned: ``tests/golden/sample_*.pt`` hold the results of the
reference's own ``sample`` (imported from the reference tree by
``tests/golden/make_golden.py``) run with ``torch.multinomial`` replaced by
``inverse_cdf`` below, and ``tests/test_oracle_golden.py`` checks this module
against them.

``margins`` gives, per row, how close the two decisions were: the distance of
the nucleus boundary's preceding mass from ``top_p`` and of the draw target
from the nearest running-sum boundary. A device implementation that sums the
same probabilities in another order or precision can only disagree with the
oracle where one of them is tiny.
"""
from __future__ import annotations

import torch


def inverse_cdf(probs: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """Position (per row) of the first running sum of ``probs`` (along the
    last dim, in order) that exceeds ``u * total``: what
    ``torch.multinomial(probs, 1)`` returns for the uniform ``u``."""
    c = probs.double().cumsum(dim=-1)
    target = u.double().reshape(-1, 1) * c[:, -1:]
    pos = (c > target).to(torch.int64).argmax(dim=-1)
    last = (probs > 0).to(torch.int64).cumsum(dim=-1).argmax(dim=-1)  # last position with mass
    return torch.minimum(pos, last)


def _filtered(logits: torch.Tensor, temperature: float, top_p: float):
    # engine.py:175-182
    probs = torch.softmax(logits / temperature, dim=-1)
    sorted_probs, sorted_indices = probs.sort(dim=-1, descending=True, stable=True)
    cumulative = sorted_probs.cumsum(dim=-1)
    mask = cumulative - sorted_probs > top_p
    sorted_probs[mask] = 0.0
    sorted_probs /= sorted_probs.sum(dim=-1, keepdim=True)
    return sorted_probs, sorted_indices, cumulative, mask


def sample_top_p(logits: torch.Tensor, temperature: float, top_p: float, u: torch.Tensor | None):
    """(tokens int64 [B], nucleus sizes int64 [B]) for fp32 logits [B, V]."""
    logits = logits.float()
    if temperature == 0:  # engine.py:172-173
        return logits.argmax(dim=-1), torch.ones(logits.shape[0], dtype=torch.int64)
    sorted_probs, sorted_indices, _, mask = _filtered(logits, temperature, top_p)
    pos = inverse_cdf(sorted_probs, u)  # engine.py:185, the draw made explicit
    tokens = sorted_indices.gather(-1, pos[:, None]).squeeze(-1)  # engine.py:186
    return tokens, (~mask).sum(dim=-1)


def margins(logits: torch.Tensor, temperature: float, top_p: float, u: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(nucleus margin, draw margin) per row, as fractions of the total mass."""
    logits = logits.float()
    probs = torch.softmax(logits / temperature, dim=-1).double()
    sp, _ = probs.sort(dim=-1, descending=True, stable=True)
    c = sp.cumsum(dim=-1)
    before = c - sp  # mass preceding each position
    nuc = (before - top_p).abs().min(dim=-1).values
    kept = before <= top_p
    kp = torch.where(kept, sp, torch.zeros_like(sp))
    ck = kp.cumsum(dim=-1)
    target = u.double().reshape(-1, 1) * ck[:, -1:]
    draw = ((ck - target).abs() / ck[:, -1:]).min(dim=-1).values
    return nuc, draw
