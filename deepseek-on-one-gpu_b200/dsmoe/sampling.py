"""Next-token sampling on the device: the drop-in for ``sample``
(``inference/engine.py:166-190``) and a decode loop without a per-token host
round trip (the loop of ``InferenceEngine.generate``, ``engine.py:135-157``).

``sample(logits, temperature, top_p)`` has the reference's signature and
result: int64 token ids ``[B]`` on the logits' device. The selection is done
by ``dsmoe_sample_top_p`` (csrc/sampler.cu): softmax(logits / T), the
nucleus (keep a descending position iff the probability mass before it is
<= top_p), and an inverse-CDF draw in descending order. The reference draws
inside ``torch.multinomial``; here the uniform is drawn with ``torch.rand``
on the device (from ``generator`` when given) and handed to the kernel, so a
run is reproducible from the generator's seed, and the same uniform gives the
same token as the reference's steps (``oracle/sampler.py`` restates them with
the draw made explicit).

``generate_tokens`` runs the decode loop with the sampled ids written
straight into a device buffer; the host reads them back only every
``check_every`` steps to look for the end-of-sequence token, instead of
``.item()`` after every step.
"""
from __future__ import annotations

import torch

from ._lib import check, lib, ptr, require_cuda, stream_handle


def _rows(logits: torch.Tensor) -> torch.Tensor:
    if logits.dim() != 2:
        raise ValueError("logits must be (B, vocab_size)")
    x = logits if logits.dtype == torch.float32 else logits.float()
    if x.stride(-1) != 1 or x.stride(0) < x.shape[1]:
        x = x.contiguous()
    return x


def sample_with_uniforms(logits: torch.Tensor, temperature: float, top_p: float, uniforms: torch.Tensor | None,
                         out: torch.Tensor | None = None, return_nucleus: bool = False):
    """Sample with caller-provided uniforms ``[B]`` (fp32, in [0, 1), on the
    device; ignored when ``temperature == 0``). ``out`` (int64 ``[B]``, may
    be a view into a larger buffer) receives the token ids. With
    ``return_nucleus`` also returns the nucleus size of each row (int32)."""
    x = _rows(logits)  # rows may be strided (e.g. logits[:, -1, :] of (B, S, vocab))
    if not x.is_cuda:
        raise RuntimeError("dsmoe runs on CUDA tensors only (no CPU fallback)")
    require_cuda(uniforms, out)
    B, V = x.shape
    tokens = out if out is not None else torch.empty(B, dtype=torch.int64, device=x.device)
    if tokens.dtype != torch.int64 or tokens.numel() != B or not tokens.is_contiguous():
        raise ValueError("out must be a contiguous int64 tensor of B elements")
    u = None
    if temperature != 0:
        if uniforms is None:
            raise ValueError("uniforms are required when temperature > 0")
        u = uniforms.reshape(-1).float().contiguous()
        if u.numel() != B:
            raise ValueError("one uniform per row")
    nucleus = torch.empty(B, dtype=torch.int32, device=x.device) if return_nucleus else None
    check(lib().dsmoe_sample_top_p(ptr(x), B, V, x.stride(0), float(temperature), float(top_p), ptr(u), ptr(tokens),
                                   ptr(nucleus), stream_handle(x.device)), "dsmoe_sample_top_p")
    return (tokens, nucleus) if return_nucleus else tokens


def sample(logits: torch.Tensor, temperature: float, top_p: float,
           generator: torch.Generator | None = None) -> torch.Tensor:
    """``inference/engine.py:166``: (B, vocab) logits -> (B,) int64 token ids,
    on the device, without synchronising the host."""
    x = _rows(logits)
    u = None
    if temperature != 0:
        u = torch.rand(x.shape[0], device=x.device, dtype=torch.float32, generator=generator)
    return sample_with_uniforms(x, temperature, top_p, u)


def generate_tokens(step, first_logits: torch.Tensor, max_tokens: int, eos_token_id: int | None,
                    temperature: float = 0.6, top_p: float = 0.9, generator: torch.Generator | None = None,
                    check_every: int = 16, sampler=None) -> list[int]:
    """The decode loop of ``InferenceEngine.generate`` (``engine.py:116-151``)
    for one sequence, with the tokens kept on the device.

    ``first_logits`` are the prefill's last-position logits ``(1, vocab)``;
    ``step(token, i)`` runs decode step ``i`` (0-based) on the device tensor
    ``token`` (int64 ``[1]``) and returns its logits ``(1, vocab)``. Like the
    reference: the first sampled token is always kept; each later token ends
    the sequence, unkept, if it is ``eos_token_id``; at most ``max_tokens``
    tokens. The host looks at the tokens every ``check_every`` steps, so up to
    ``check_every - 1`` steps may run past the end-of-sequence token; their
    tokens are dropped. ``sampler`` (default ``sample_with_uniforms``) is the
    per-step sampling call, with that function's arguments.
    """
    if max_tokens <= 0:
        return []
    draw_token = sampler or sample_with_uniforms
    dev = first_logits.device
    buf = torch.empty(max_tokens, dtype=torch.int64, device=dev)
    draw_token(first_logits, temperature, top_p, _draw(dev, temperature, generator), out=buf[0:1])
    done = 1
    out: list[int] = []
    checked = 0
    while True:
        stop = min(max_tokens, done + max(1, check_every))
        for i in range(done, stop):
            logits = step(buf[i - 1:i], i - 1)
            draw_token(logits[:, -1, :] if logits.dim() == 3 else logits, temperature, top_p,
                       _draw(dev, temperature, generator), out=buf[i:i + 1])
        done = stop
        host = buf[checked:done].tolist()  # the only host read, once per chunk
        for k, t in enumerate(host):
            if checked + k > 0 and eos_token_id is not None and t == eos_token_id:
                return out
            out.append(t)
        checked = done
        if done >= max_tokens:
            return out


def _draw(dev, temperature: float, generator) -> torch.Tensor | None:
    if temperature == 0:
        return None
    return torch.rand(1, device=dev, dtype=torch.float32, generator=generator)
