"""Seeded synthetic inputs for the MoE block.

No checkpoint is available, so every weight and activation is generated from a
seed with the distributions the benchmark configurations name:

  * activations ``x`` ~ N(0, 1), bf16 ``[T, H]``;
  * router weight ~ N(0, 0.006), bf16 ``[E, H]`` (the reference keeps the gate
    in bf16, ``inference/weight_store.py:252-254``);
  * ``e_score_correction_bias`` ~ N(0, 0.01), fp32 ``[E]`` (or the Zipf skew);
  * expert weights ~ N(0, 0.02), quantised per 128x128 block to FP8-e4m3 with an
    fp32 ``weight_scale_inv = block_amax / 448`` that *multiplies* on dequant
    (``inference/ops.py:37-43``).

Each expert projection has its own generator seeded from
``(seed, layer, expert, proj)``, so an expert can be produced on its own, in any
order, on CPU or GPU. The CPU and CUDA generators give different streams: a
parity test always hands the *same bytes* to both sides.
"""
from __future__ import annotations

import math

import torch

PROJS = ("gate_proj", "up_proj", "down_proj")
FP8_MAX = 448.0
SHARED = -1  # expert id used for the shared expert


def _mix(*parts: int) -> int:
    h = 0x9E3779B97F4A7C15
    for p in parts:
        h ^= (int(p) + 0x632BE59BD9B4E019 + ((h << 6) & 0xFFFFFFFFFFFFFFFF) + (h >> 2))
        h &= 0xFFFFFFFFFFFFFFFF
    return h & 0x7FFFFFFFFFFFFFFF


def _gen(device, *parts: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(_mix(*parts))
    return g


def block_quantize(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``[O, I]`` -> (e4m3 ``[O, I]``, fp32 scale ``[ceil(O/b), ceil(I/b)]``).

    scale = block_amax / 448, q = e4m3(w / scale). Dequantisation is
    ``q * scale`` exactly as ``inference/ops.py:40-43`` expands it.
    """
    O, I = w.shape
    bo, bi = math.ceil(O / block), math.ceil(I / block)
    pad = torch.zeros(bo * block, bi * block, dtype=torch.float32, device=w.device)
    pad[:O, :I] = w
    blocks = pad.view(bo, block, bi, block)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (blocks / scale[:, None, :, None]).clamp_(-FP8_MAX, FP8_MAX)
    q = q.view(bo * block, bi * block)[:O, :I].to(torch.float8_e4m3fn)
    return q.contiguous(), scale.contiguous()


def expert_weights(seed: int, layer: int, expert: int, hidden: int, inter: int,
                   device="cpu", std: float = 0.02) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """One expert in the reference's ``{proj: (weight_fp8, weight_scale_inv)}``
    form (``inference/weight_store.py:203-206``). ``expert == SHARED`` is the
    shared expert (same shapes, shared intermediate = ``inter``)."""
    out = {}
    for pi, proj in enumerate(PROJS):
        shape = (inter, hidden) if proj != "down_proj" else (hidden, inter)
        g = _gen(device, seed, layer, expert + 1000, pi)
        w = torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(std)
        out[proj] = block_quantize(w)
        del w
    return out


def activations(seed: int, T: int, hidden: int, device="cpu") -> torch.Tensor:
    g = _gen(device, seed, 1, 7)
    return torch.randn(T, hidden, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


def gate_weight(seed: int, layer: int, n_experts: int, hidden: int, device="cpu",
                std: float = 0.006) -> torch.Tensor:
    g = _gen(device, seed, layer, 2, 9)
    return torch.randn(n_experts, hidden, generator=g, device=device,
                       dtype=torch.float32).mul_(std).to(torch.bfloat16)


def score_bias(seed: int, layer: int, n_experts: int, device="cpu", std: float = 0.01,
               zipf_s: float | None = None) -> torch.Tensor:
    """``e_score_correction_bias``. With ``zipf_s`` set: 0.5 * log of Zipf(s)
    rank weights, assigned to experts through a seeded random permutation (the
    load-skew configuration)."""
    g = _gen("cpu", seed, layer, 3, 11)
    if zipf_s is None:
        b = torch.randn(n_experts, generator=g, dtype=torch.float32).mul_(std)
    else:
        ranks = torch.arange(1, n_experts + 1, dtype=torch.float64)
        w = ranks.pow(-zipf_s)
        w = w / w.sum()
        perm = torch.randperm(n_experts, generator=g)
        b = torch.empty(n_experts, dtype=torch.float64)
        b[perm] = 0.5 * torch.log(w)
        b = b.float()
    return b.to(device)


def norm_weight(seed: int, layer: int, which: int, hidden: int, device="cpu", std: float = 0.1) -> torch.Tensor:
    """A layer-norm weight (``which`` 0 = input_layernorm, 1 =
    post_attention_layernorm): 1 + N(0, std) in bf16."""
    g = _gen("cpu", seed, layer, 4, 13 + which)
    return (1.0 + torch.randn(hidden, generator=g, dtype=torch.float32) * std).to(torch.bfloat16).to(device)


def logits(seed: int, rows: int, vocab: int, scale: float, device="cpu") -> torch.Tensor:
    """Next-token logits ``[rows, vocab]`` fp32 ~ N(0, scale^2): larger
    ``scale`` gives a more peaked softmax (smaller nucleus)."""
    g = _gen("cpu", seed, 5, 17)
    return torch.randn(rows, vocab, generator=g, dtype=torch.float32).mul_(scale).to(device)


def uniforms(seed: int, rows: int, device="cpu") -> torch.Tensor:
    """One uniform in [0, 1) per row (the sampler's draw)."""
    g = _gen("cpu", seed, 5, 19)
    return torch.rand(rows, generator=g, dtype=torch.float32).to(device)


class SyntheticLayer:
    """Lazily generated weights of one MoE layer (per-expert cache optional)."""

    def __init__(self, seed: int, layer: int, hidden: int, inter: int, n_experts: int,
                 device="cpu", bias_zipf: float | None = None, cache: bool = True):
        self.seed, self.layer, self.hidden, self.inter = seed, layer, hidden, inter
        self.n_experts, self.device = n_experts, device
        self.gate = gate_weight(seed, layer, n_experts, hidden, device)
        self.bias = score_bias(seed, layer, n_experts, device, zipf_s=bias_zipf)
        self._cache: dict[int, dict] | None = {} if cache else None

    def expert(self, e: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        if self._cache is not None and e in self._cache:
            return self._cache[e]
        w = expert_weights(self.seed, self.layer, e, self.hidden, self.inter, self.device)
        if self._cache is not None:
            self._cache[e] = w
        return w

    def shared(self) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        return self.expert(SHARED)
