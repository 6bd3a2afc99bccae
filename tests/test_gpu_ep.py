"""Expert-parallel step (dsmoe.ep) on one GPU: W ranks emulated in one process
(the all-to-alls become slicing), each rank's output compared with the
single-GPU moe_block on the same tokens and with the CPU oracle."""
import pytest
import torch

from dsmoe import DeepSeekConfig, GPUTransfer, SyntheticWeightStore, moe_block
from dsmoe.ep import EPLayer, emulate_step
from dsmoe.synthetic import activations
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REL_RMS_TOL = 1e-2


@pytest.mark.parametrize("W,T,mode", [(2, 64, "ref"), (4, 96, "ref"), (8, 40, "ref"), (8, 300, "v3"), (1, 33, "ref")])
def test_ep_emulated_matches_single_gpu(W, T, mode):
    H, F = 512, 256
    cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F, router_mode=mode)
    store = SyntheticWeightStore(cfg, seed=31, device=DEV, pin_memory=False, gen_device="cpu",
                                 bias_zipf=1.1 if mode == "v3" else None)
    layers = [EPLayer(cfg, store, DEV, 3, W, r, expert_source=store.device_expert) for r in range(W)]
    xs = [activations(40 + r, T, H).to(DEV) for r in range(W)]
    outs = emulate_step(layers, xs)
    gt = GPUTransfer(cfg, store, DEV)
    L = store.layer(3)
    for r in range(W):
        single = moe_block(xs[r], 3, store, gt, cfg)
        assert O.rel_rms(outs[r].float().cpu(), single.float().cpu()) < 5e-3
        x = xs[r].cpu()
        if mode == "v3":
            idx, w = O.route_v3(x, L.gate, L.bias)
            ref = O.moe_block_grouped(x, idx, w, L.expert, L.shared(), final_scale=1.0)
        else:
            idx, w = O.route_ref(x, L.gate)
            ref = O.moe_block_grouped(x, idx, w, L.expert, L.shared())
        assert O.rel_rms(outs[r].float().cpu(), ref.float()) < REL_RMS_TOL


def test_ep_emulated_balanced_placement_matches_single_gpu():
    """Skewed routing (bias-corrected router, Zipf expert bias) with the experts
    placed by load (dsmoe.ep.balanced_placement): each rank holds the experts
    the placement gives it, the router's ids are relabelled on the device, and
    every rank's output matches the single-GPU block."""
    from dsmoe.ep import balanced_placement

    H, F = 512, 256
    cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F, router_mode="v3")
    store = SyntheticWeightStore(cfg, seed=31, device=DEV, pin_memory=False, gen_device="cpu", bias_zipf=1.1)
    W, T = 8, 300
    xs = [activations(40 + r, T, H).to(DEV) for r in range(W)]
    probe = EPLayer(cfg, store, DEV, 3, W, 0, expert_source=store.device_expert)
    loads = sum(torch.bincount(probe.route(x)[0].reshape(-1), minlength=256) for x in xs).double().cpu()
    placement = balanced_placement(loads.tolist(), W)
    El = 256 // W
    contiguous = loads.view(W, El).sum(1)
    spread = torch.zeros(W, dtype=torch.float64)
    for e, pos in enumerate(placement):
        spread[pos // El] += loads[e]
    assert spread.max() <= contiguous.max()
    layers = [EPLayer(cfg, store, DEV, 3, W, r, expert_source=store.device_expert, placement=placement)
              for r in range(W)]
    for r in (0, 5):
        lay = layers[r]
        for el in (0, El - 1):
            e = lay.owned[el]
            assert placement[e] == r * El + el
            slot = lay.bank.slot_of_host[el + 1]
            want = store.device_expert(3, e)["gate_proj"][0]
            assert torch.equal(lay.bank.w["gate_proj"][slot].view(torch.uint8), want.view(torch.uint8))
    outs = emulate_step(layers, xs)
    gt = GPUTransfer(cfg, store, DEV)
    for r in range(W):
        single = moe_block(xs[r], 3, store, gt, cfg)
        assert O.rel_rms(outs[r].float().cpu(), single.float().cpu()) < 5e-3


def test_ep_full_dims_w8():
    cfg = DeepSeekConfig()
    store = SyntheticWeightStore(cfg, seed=41, device=DEV, pin_memory=False, gen_device="cuda")
    W, T = 8, 128
    layers = [EPLayer(cfg, store, DEV, 3, W, r, expert_source=store.device_expert) for r in range(W)]
    xs = [activations(50 + r, T, 7168).to(DEV) for r in range(W)]
    outs = emulate_step(layers, xs)
    gt = GPUTransfer(cfg, store, DEV)
    for r in (0, 5):
        single = moe_block(xs[r], 3, store, gt, cfg)
        assert O.rel_rms(outs[r].float().cpu(), single.float().cpu()) < 5e-3
    assert all(torch.isfinite(o.float()).all() for o in outs)


def test_ep_rank_with_no_tokens_for_it():
    """A rank that receives nothing (all tokens routed elsewhere) still returns."""
    H, F = 256, 128
    cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F)
    store = SyntheticWeightStore(cfg, seed=5, device=DEV, pin_memory=False, gen_device="cpu")
    gate = torch.zeros(256, H)
    gate[[0, 1, 2, 3, 4, 5, 6, 7]] = 0.05  # experts 0-7 live on rank 0 of 8
    store._gate[3] = gate.to(torch.bfloat16).to(DEV)
    W = 8
    layers = [EPLayer(cfg, store, DEV, 3, W, r, expert_source=store.device_expert) for r in range(W)]
    xs = [activations(60 + r, 16, H).abs().to(DEV) for r in range(W)]
    outs = emulate_step(layers, xs)
    gt = GPUTransfer(cfg, store, DEV)
    for r in range(W):
        single = moe_block(xs[r], 3, store, gt, cfg)
        assert O.rel_rms(outs[r].float().cpu(), single.float().cpu()) < 5e-3


@pytest.mark.parametrize("chunks,reserve", [(1, 0), (1, 16), (2, 0), (3, 16), (5, 0)])
def test_ep_overlapped_two_stream_step(chunks, reserve):
    """The overlapped step (exchange on a side stream, shared expert while the
    rows travel, optional chunking and SM reserve) on a one-rank group gives
    the plain step's output and the single-GPU block's."""
    from dsmoe.ep import LocalExchange

    H, F = 512, 256
    cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F)
    store = SyntheticWeightStore(cfg, seed=71, device=DEV, pin_memory=False, gen_device="cpu")
    layer = EPLayer(cfg, store, DEV, 2, 1, 0, exchange=LocalExchange(), expert_source=store.device_expert)
    x = activations(72, 203, H).to(DEV)
    layer.overlap = False
    plain = layer.forward(x)
    layer.overlap = True
    layer.sm_reserve = reserve
    ov = layer.forward(x, chunks=chunks)
    again = layer.forward(x, chunks=chunks)
    torch.cuda.synchronize()
    assert torch.equal(ov, again)
    assert O.rel_rms(ov.float().cpu(), plain.float().cpu()) < 1e-3
    if chunks == 1:
        assert torch.equal(ov, plain)
    gt = GPUTransfer(cfg, store, DEV)
    single = moe_block(x, 2, store, gt, cfg)
    assert O.rel_rms(ov.float().cpu(), single.float().cpu()) < 5e-3
    L = store.layer(2)
    idx, w = O.route_ref(x.cpu(), L.gate)
    ref = O.moe_block_grouped(x.cpu(), idx, w, L.expert, L.shared())
    assert O.rel_rms(ov.float().cpu(), ref.float()) < REL_RMS_TOL


def test_ep_peer_memory_one_rank_group():
    """The peer-memory exchange (rows pushed into mapped receive buffers,
    partials written back into the origin's return buffer, tiny NCCL
    barriers, received rows counted on the device) on a one-rank NCCL group
    gives the all-to-all step's output bit for bit, with the pushes
    overlapping the shared expert or not."""
    import socket

    import torch.distributed as dist

    from dsmoe.ep import DistExchange

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1, device_id=DEV)
    try:
        H, F = 512, 256
        cfg = DeepSeekConfig(hidden_size=H, moe_intermediate_size=F)
        store = SyntheticWeightStore(cfg, seed=81, device=DEV, pin_memory=False, gen_device="cpu")
        layer = EPLayer(cfg, store, DEV, 2, 1, 0, exchange=DistExchange(), expert_source=store.device_expert)
        xs = [activations(82 + i, T, H).to(DEV) for i, T in enumerate((100, 1, 37))]
        plain = [layer.forward(x) for x in xs]
        layer.use_peer_memory(cap=128)
        try:
            for push_sms in (16, 0):  # pushes beside the shared expert on a side stream, then in order
                layer.push_sms = push_sms
                peer = [layer.forward(x) for x in xs]
                torch.cuda.synchronize()
                for a, b in zip(plain, peer):
                    assert torch.equal(a, b)
                assert layer.push_status() == 0
            with pytest.raises(ValueError):
                layer.forward(activations(90, 129, H).to(DEV))
        finally:
            layer.close()
    finally:
        dist.destroy_process_group()
