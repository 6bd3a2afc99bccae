"""Output parity at the shapes ``bench.py`` times, at the DeepSeek-R1
dimensions (H=7168, F=2048, 256 routed experts + the shared one).

Each case builds exactly the bench's inputs (same seeds, same layer) and
checks

  * routing indices of EVERY row against the oracle's router run on CPU
    (identical except rows that differ only at fp32 score ties within 1e-6),
    and routing weights to 1e-5 where the indices agree;
  * the block output of a row subset (32 rows spread over the batch plus
    every row routed to the hottest expert, whose group runs the most token
    tiles) within 1e-2 relative RMS of the reference arithmetic
    (``inference/forward.py:112-153``): the oracle's grouped restatement run as
    a plain fp32 torch reference on the GPU (TF32 off), over every expert
    those rows touch.

Cases: config 2 (T=4096, reference router, seed 1), config 4 (T=16384,
bias-corrected router with a Zipf(1.1) bias, seed 3) and config 3's
expert-parallel step with 8 ranks emulated on one GPU (T=8192 per rank,
seed 2).
"""
import pytest
import torch

from dsmoe import DeepSeekConfig, GPUTransfer, SyntheticWeightStore, _lib, moe_block
from dsmoe.ep import EPLayer, emulate_step
from dsmoe.synthetic import activations
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

REL_RMS_TOL = 1e-2
W_TOL = 1e-5
DEV = torch.device("cuda", 0)
H, F, E, K = 7168, 2048, 256, 8
LAYER = 3  # the layer bench.py builds


@pytest.fixture(autouse=True)
def fp32_matmuls():
    """The GPU-side reference must multiply in fp32, not TF32."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    assert torch.get_float32_matmul_precision() == "highest"
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def check_routing(idx, w, idx_r, w_r, keys):
    idx = idx.reshape(idx_r.shape).cpu()
    w = w.reshape(w_r.shape).cpu()
    bad, ties = O.index_parity(idx, idx_r, keys)
    assert bad == 0, f"{bad} rows with unexplained index differences ({ties} tie rows)"
    same = (idx == idx_r).all(-1)
    assert (w[same] - w_r[same]).abs().max().item() <= W_TOL
    return ties


def check_rows(idx_r: torch.Tensor):
    """32 rows spread over the batch + every row routed to the hottest expert."""
    T = idx_r.shape[0]
    counts = torch.bincount(idx_r.reshape(-1), minlength=E)
    hot = int(counts.argmax())
    rows = torch.cat([torch.linspace(0, T - 1, 32).long(), (idx_r == hot).any(-1).nonzero().view(-1)])
    return torch.unique(rows), hot, int(counts[hot]), float(counts.max() / counts.float().mean())


def bank_expert(bank, group):
    return {p: (w, s) for p, (w, s) in bank.views(group).items()}


def single_gpu_case(seed, T, router_mode, zipf):
    cfg = DeepSeekConfig(router_mode=router_mode)
    store = SyntheticWeightStore(cfg, seed=seed, device=DEV, pin_memory=False, gen_device="cuda", bias_zipf=zipf)
    gt = GPUTransfer(cfg, store, DEV)
    x = activations(seed, T, H, device=DEV)
    out, idx, w = moe_block(x, LAYER, store, gt, cfg, return_routing=True)
    torch.cuda.synchronize()
    xc, gate = x.cpu(), store.get_gate_weight(LAYER).cpu()
    if router_mode == "v3":
        bias = store.get_gate_bias(LAYER).cpu()
        idx_r, w_r = O.route_v3(xc, gate, bias)
        keys = torch.sigmoid(O.router_logits(xc, gate)) + bias
        final_scale = 1.0
    else:
        idx_r, w_r = O.route_ref(xc, gate)
        keys = torch.sigmoid(O.router_logits(xc, gate))
        final_scale = None
    check_routing(idx, w, idx_r, w_r, keys)
    rows, hot, n_hot, skew = check_rows(idx_r)
    bank = gt.bank(LAYER)
    r = rows.to(DEV)
    ref = O.moe_block_grouped(x[r], idx_r[rows].to(DEV), w_r[rows].to(DEV), lambda e: bank_expert(bank, e + 1),
                              bank_expert(bank, 0), final_scale=final_scale)
    err = O.rel_rms(out[r].float(), ref.float())
    return err, rows.numel(), n_hot, skew


def test_config2_t4096_output_parity():
    err, n_rows, n_hot, _ = single_gpu_case(seed=1, T=4096, router_mode="ref", zipf=None)
    assert n_rows >= n_hot > 128
    assert err <= REL_RMS_TOL, (err, n_rows)


def test_config4_t16384_zipf_output_parity():
    err, n_rows, n_hot, skew = single_gpu_case(seed=3, T=16384, router_mode="v3", zipf=1.1)
    assert skew >= 10.0, skew  # the configuration's premise: the hottest expert >= 10x the mean
    assert n_hot >= 10 * 16384 * K // E
    assert err <= REL_RMS_TOL, (err, n_rows)


def test_config3_ep8_emulated_t8192_output_parity():
    """8 expert-parallel ranks on one GPU (32 experts each), 8192 tokens per
    rank: every rank's output rows against the oracle over all 256 experts."""
    W, T, seed = 8, 8192, 2
    cfg = DeepSeekConfig()
    store = SyntheticWeightStore(cfg, seed=seed, device=DEV, pin_memory=False, gen_device="cuda")
    layers = [EPLayer(cfg, store, DEV, LAYER, W, r, expert_source=store.device_expert) for r in range(W)]
    xs = [activations(1000 * seed + r, T, H, device=DEV) for r in range(W)]  # bench.py's per-rank inputs
    # The emulated ranks run one after the other on one GPU, so one workspace
    # sized for the most rows a rank can receive (every token once) serves all.
    need = _lib.lib().dsmoe_moe_local_workspace_size(_lib.moe_config(layers[0].lcfg), W * T)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    for r in range(W):
        layers[r]._ws = ws
    outs = emulate_step(layers, xs)
    torch.cuda.synchronize()
    gate = store.get_gate_weight(LAYER).cpu()

    def expert(e):
        return bank_expert(layers[e // 32].bank, e % 32 + 1)

    shared = bank_expert(layers[0].bank, 0)
    x_all = torch.cat(xs)
    x_cpu = x_all.cpu()
    idx_r, w_r = O.route_ref(x_cpu, gate)
    scores = torch.sigmoid(O.router_logits(x_cpu, gate))
    for r in range(W):  # each rank routes its own tokens with the replicated gate
        idx, w = layers[r].route(xs[r])
        sl = slice(r * T, (r + 1) * T)
        check_routing(idx, w, idx_r[sl], w_r[sl], scores[sl])
    rows, hot, n_hot, _ = check_rows(idx_r)
    rows = torch.unique(torch.cat([rows, torch.arange(W) * T + 5]))  # at least one row of every rank
    out_all = torch.cat(outs)
    r = rows.to(DEV)
    ref = O.moe_block_grouped(x_all[r], idx_r[rows].to(DEV), w_r[rows].to(DEV), expert, shared)
    err = O.rel_rms(out_all[r].float(), ref.float())
    assert err <= REL_RMS_TOL, (err, rows.numel(), n_hot)
