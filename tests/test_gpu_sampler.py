"""Device sampler (csrc/sampler.cu through dsmoe_sample_top_p) against the
oracle's restatement of the reference's sample() (oracle/sampler.py), which is
pinned to the reference by tests/golden/sample_*.pt.

Tokens and nucleus sizes must be equal. The one allowed difference: the
kernel sums exact integer masses while the reference sums fp32
probabilities, so a row may disagree where the oracle's nucleus boundary
lies within MARGIN of top_p, or its draw target within MARGIN (as a fraction
of the kept mass) of a running-sum boundary; such rows are counted and must
stay rare.
"""
import os

import pytest
import torch

from conftest import GOLDEN
from dsmoe import sample, sample_with_uniforms, generate_tokens
from dsmoe.synthetic import logits as make_logits, uniforms as make_uniforms
from oracle import sampler as S

pytestmark = pytest.mark.gpu
MARGIN = 1e-5
DEV = "cuda"


def check_rows(x, temperature, top_p, u, max_exempt_frac=0.02):
    tok, nuc = sample_with_uniforms(x.to(DEV), temperature, top_p, None if u is None else u.to(DEV),
                                    return_nucleus=True)
    tok, nuc = tok.cpu(), nuc.cpu().to(torch.int64)
    rt, rn = S.sample_top_p(x.cpu(), temperature, top_p, u)
    if temperature == 0:
        assert torch.equal(tok, rt)
        return
    bad = (tok != rt) | (nuc != rn)
    if bad.any():
        nm, dm = S.margins(x.cpu(), temperature, top_p, u)
        close = (nm < MARGIN) | (dm < MARGIN)
        assert not (bad & ~close).any(), (
            f"rows {torch.nonzero(bad & ~close).flatten().tolist()}: kernel {tok[bad].tolist()} / {nuc[bad].tolist()} "
            f"oracle {rt[bad].tolist()} / {rn[bad].tolist()}")
        assert int(bad.sum()) <= max(1, int(max_exempt_frac * len(bad)))
    return tok, nuc


@pytest.mark.parametrize("name", ["sample_v1000", "sample_v129280", "sample_topp_small", "sample_greedy",
                                  "sample_topp1", "sample_hot"])
def test_sampler_reference_golden(name):
    g = torch.load(os.path.join(GOLDEN, f"{name}.pt"))
    x = make_logits(g["seed"], g["rows"], g["vocab"], g["scale"])
    tok, nuc = sample_with_uniforms(x.to(DEV), g["temperature"], g["top_p"], g["u"].to(DEV), return_nucleus=True)
    assert torch.equal(tok.cpu(), g["tokens"])
    if g["temperature"] != 0:
        assert torch.equal(nuc.cpu().to(torch.int64), g["nucleus"])


@pytest.mark.parametrize("V", [1, 2, 3, 1001, 4096, 16384, 16385, 50000, 129280, 131072])
@pytest.mark.parametrize("scale,temperature,top_p", [(1.0, 1.0, 0.9), (3.0, 0.6, 0.9), (0.3, 0.7, 0.5)])
def test_sampler_vs_oracle(V, scale, temperature, top_p):
    B = 16
    seed = 300 + V % 97
    x = make_logits(seed, B, V, scale)
    u = make_uniforms(seed, B)
    check_rows(x, temperature, top_p, u)


def test_sampler_many_rows_and_uniform_sweep():
    """One row repeated with uniforms across [0, 1): every draw equals the
    oracle's; u = 0 gives the top element, u just below 1 the last kept."""
    V = 3000
    x = make_logits(7, 1, V, 2.0).repeat(400, 1)
    u = torch.linspace(0, 1, 400, dtype=torch.float64).clamp(max=1 - 2 ** -24).float()
    tok, nuc = check_rows(x, 0.8, 0.9, u, max_exempt_frac=0.01)
    rt, _ = S.sample_top_p(x, 0.8, 0.9, u)
    assert int(tok[0]) == int(x[0].argmax())
    assert torch.equal(tok[[0, -1]], rt[[0, -1]])
    assert len(set(nuc.tolist())) == 1


def test_sampler_edge_cases():
    # temperature 0: argmax, first of equal maxima
    x = torch.zeros(3, 40000)
    x[0, 12345] = 5.0
    x[1, [100, 39000]] = 7.0
    x[2, :] = -1.0
    tok = sample(x.to(DEV), 0.0, 0.9).cpu()
    assert tok.tolist() == [12345, 100, 0]
    # top_p = 0 keeps only the top element; top_p >= 1 keeps everything
    y = make_logits(11, 8, 5000, 1.0)
    u = make_uniforms(11, 8)
    t0, n0 = sample_with_uniforms(y.to(DEV), 1.0, 0.0, u.to(DEV), return_nucleus=True)
    assert torch.equal(t0.cpu(), y.argmax(dim=-1)) and (n0 == 1).all()
    _, n1 = sample_with_uniforms(y.to(DEV), 1.0, 1.5, u.to(DEV), return_nucleus=True)
    assert (n1 == 5000).all()
    # -inf logits are never drawn and do not count
    z = make_logits(12, 8, 3000, 1.0)
    z[:, ::2] = float("-inf")
    tz, nz = sample_with_uniforms(z.to(DEV), 0.7, 0.95, u.to(DEV), return_nucleus=True)
    assert (tz.cpu() % 2 == 1).all()
    check_rows(z, 0.7, 0.95, u)
    # a row without a finite maximum gets -1 (the reference's softmax is NaN)
    w = make_logits(13, 3, 1000, 1.0)
    w[0, 5] = float("nan")
    w[1, :] = float("-inf")
    w[2, 7] = float("inf")
    assert sample_with_uniforms(w.to(DEV), 1.0, 0.9, u[:3].to(DEV)).cpu().tolist() == [-1, -1, -1]
    # temperature 0 follows torch.argmax: a NaN counts as the maximum
    assert sample(w.to(DEV), 0.0, 0.9).cpu().tolist() == w.argmax(dim=-1).tolist()


def test_sampler_equal_logits_stable_order():
    """All logits equal: the nucleus is the first floor(top_p * V) + 1
    positions of a stable sort, i.e. the smallest indices, and the draw picks
    by index."""
    V = 5003
    x = torch.full((6, V), 0.25)
    u = torch.tensor([0.0, 0.1, 0.5, 0.9, 0.99, 0.999999])
    tok, nuc = sample_with_uniforms(x.to(DEV), 1.0, 0.9, u.to(DEV), return_nucleus=True)
    kept = int(0.9 * V) + 1
    assert (nuc.cpu() == kept).all()
    rt, rn = S.sample_top_p(x, 1.0, 0.9, u)
    assert torch.equal(tok.cpu(), rt) and (rn == kept).all()
    assert tok.cpu().tolist() == [int(v * kept) for v in u.tolist()]


def test_sampler_strided_rows_and_determinism():
    B, S_, V = 4, 3, 129280
    full = make_logits(21, B * S_, V, 3.0).view(B, S_, V).to(DEV)
    u = make_uniforms(21, B).to(DEV)
    a = sample_with_uniforms(full[:, -1, :], 0.6, 0.9, u)        # strided rows, no copy
    b = sample_with_uniforms(full[:, -1, :].contiguous(), 0.6, 0.9, u)
    c = sample_with_uniforms(full[:, -1, :], 0.6, 0.9, u)
    assert torch.equal(a, b) and torch.equal(a, c)
    check_rows(full[:, -1, :].cpu(), 0.6, 0.9, u.cpu())


def test_sample_distribution():
    """sample() draws its own uniforms: over many rows of one distribution the
    token frequencies follow the renormalised nucleus probabilities."""
    x = torch.tensor([[2.0, 1.0, 0.5, 0.0, -1.0, -3.0]]).repeat(40000, 1)
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    tok = sample(x.to(DEV), 1.0, 0.9, generator=g).cpu()
    p = torch.softmax(x[0], dim=-1).double()
    sp, si = p.sort(descending=True)
    keep = (sp.cumsum(0) - sp) <= 0.9
    q = torch.zeros_like(p)
    q[si[keep]] = sp[keep] / sp[keep].sum()
    freq = torch.bincount(tok, minlength=6).double() / tok.numel()
    sd = (q * (1 - q) / tok.numel()).sqrt()
    assert ((freq - q).abs() <= 5 * sd + 1e-12).all(), (freq, q)


def test_generate_tokens_matches_per_token_loop():
    """The device-resident decode loop gives the per-token loop's tokens
    (engine.py:116-151 with the oracle's sampler), including the stop at the
    end-of-sequence token and the max_tokens limit."""
    V = 2000
    table = make_logits(31, V, V, 3.0)  # logits of the next step = row of the previous token
    first = make_logits(32, 1, V, 3.0)
    table_dev = table.to(DEV)

    def step(tok, i):
        return table_dev[tok]

    def per_token(temperature, top_p, max_tokens, eos, seed):
        g = torch.Generator(device=DEV)
        g.manual_seed(seed)
        draw = (lambda: torch.rand(1, device=DEV, generator=g).cpu()) if temperature else (lambda: None)
        tok, _ = S.sample_top_p(first, temperature, top_p, draw())
        out = [int(tok)]
        for _ in range(max_tokens - 1):
            tok, _ = S.sample_top_p(table[int(tok)].view(1, V), temperature, top_p, draw())
            if eos is not None and int(tok) == eos:
                break
            out.append(int(tok))
        return out

    for temperature in (0.0, 0.8):
        ref = per_token(temperature, 0.9, 40, None, 9)
        g = torch.Generator(device=DEV)
        g.manual_seed(9)
        got = generate_tokens(step, first.to(DEV), 40, None, temperature, 0.9, generator=g, check_every=7)
        assert got == ref
        eos = ref[12]
        stop = ref.index(eos, 1) if eos in ref[1:] else None
        g.manual_seed(9)
        got = generate_tokens(step, first.to(DEV), 40, eos, temperature, 0.9, generator=g, check_every=5)
        assert got == ref[:stop]
