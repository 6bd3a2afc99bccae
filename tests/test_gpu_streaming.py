"""Streaming decode (dsmoe.streaming): experts in pinned host memory, small
GPU slot caches, next-layer prefetch. The hidden state after every step must
equal the same chain computed with every expert resident."""
import pytest
import torch

from dsmoe import DeepSeekConfig, GPUTransfer, SyntheticWeightStore, moe_block
from dsmoe.streaming import StreamingDecoder
from dsmoe.synthetic import activations

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("prefetch", [True, False])
def test_streaming_matches_resident_chain(prefetch):
    cfg = DeepSeekConfig(hidden_size=512, moe_intermediate_size=256)
    layers = [0, 1, 2]
    store = SyntheticWeightStore(cfg, seed=9, device=DEV, pin_memory=True, gen_device="cpu",
                                 layer_seeds={0: 10, 1: 11, 2: 12})
    store.preload_host(layers)
    dec = StreamingDecoder(cfg, store, DEV, layers, slots_per_layer=17, prefetch=prefetch)
    resident = GPUTransfer(cfg, store, DEV)
    h_s = h_r = activations(3, 2, 512).to(DEV)
    for step in range(12):
        h_s = dec.step(h_s)
        for layer in layers:
            h_r = h_r + moe_block(h_r, layer, store, resident, cfg)
        assert torch.equal(h_s, h_r), step
    assert dec.gt.slot_misses > 0 and dec.gt.bytes_h2d > 0
    if prefetch:
        assert dec.gt.prefetched > 0


def test_device_slots_match_resident_chain():
    """Device-managed slot tables (dsmoe_slotcache_step: placement and copies
    on the GPU, no host read per layer) give the resident chain's hidden
    state bit for bit, through steps of 1 and 3 tokens that keep evicting."""
    cfg = DeepSeekConfig(hidden_size=512, moe_intermediate_size=256)
    layers = [0, 1, 2]
    store = SyntheticWeightStore(cfg, seed=9, device=DEV, pin_memory=True, gen_device="cpu",
                                 layer_seeds={0: 10, 1: 11, 2: 12})
    store.preload_host(layers)
    dec = StreamingDecoder(cfg, store, DEV, layers, slots_per_layer=25, device_slots=True)
    assert dec.device_slots
    resident = GPUTransfer(cfg, store, DEV)
    for T in (1, 3):
        h_s = h_r = activations(30 + T, T, 512).to(DEV)
        for step in range(10):
            h_s = dec.step(h_s)
            for layer in layers:
                h_r = h_r + moe_block(h_r, layer, store, resident, cfg)
            assert torch.equal(h_s, h_r), (T, step)
    hits, misses, moved = dec.device_counters()
    assert misses > 0 and hits > 0 and moved > 0
    assert all(dec.gt.device_cache(l).device_status() == 0 for l in layers)


def _lru_model(n_slots, E, steps):
    """The slot policy of dsmoe_slotcache_step restated in Python: hits
    refresh their slot's step; each missing expert (ascending id) takes the
    slot with the smallest last step among those the step does not use
    (empty slots first, then the lowest slot), never the shared expert's."""
    slot_of = [-1] * (E + 1)
    group_in_slot = [-1] * n_slots
    last = [-1] * n_slots
    slot_of[0], group_in_slot[0], last[0] = 0, 0, None  # shared expert pinned in slot 0
    history = []
    for clock, experts in enumerate(steps, start=1):
        need = sorted({e + 1 for e in experts})
        for g in need:
            if slot_of[g] >= 0:
                last[slot_of[g]] = clock
        for g in [g for g in need if slot_of[g] < 0]:
            v = min((last[s] + 1, s) for s in range(n_slots) if last[s] is not None and last[s] != clock)[1]
            if group_in_slot[v] > 0:
                slot_of[group_in_slot[v]] = -1
            slot_of[g], group_in_slot[v], last[v] = v, g, clock
        history.append(list(slot_of))
    return history


def test_device_slot_policy_and_contents():
    """The device slot table follows the policy step by step, and every
    resident expert's slot holds that expert's bytes."""
    from dsmoe.synthetic import PROJS

    cfg = DeepSeekConfig(hidden_size=512, moe_intermediate_size=256)
    store = SyntheticWeightStore(cfg, seed=4, device=DEV, pin_memory=True, gen_device="cpu")
    store.preload_host([5])
    gt = GPUTransfer(cfg, store, DEV, slots_per_layer=20, device_slots=True)
    dc = gt.device_cache(5)
    g = torch.Generator().manual_seed(7)
    steps = [torch.randint(0, 256, (int(torch.randint(1, 12, (1,), generator=g)),), generator=g).tolist()
             for _ in range(25)]
    steps += [steps[-1], steps[-2] + steps[-1][:2]]  # repeats: hits
    want = _lru_model(20, 256, steps)
    for i, experts in enumerate(steps):
        dc.step(torch.tensor(experts, dtype=torch.int64, device=DEV))
        assert gt.bank(5).slot_of.tolist() == want[i], i
    assert dc.device_status() == 0
    dc.refresh_host_mirror()
    bank = gt.bank(5)
    for grp, s in enumerate(bank.slot_of_host):
        if grp == 0 or s < 0:
            continue
        ref = store.get_expert(5, grp - 1)
        for p in PROJS:
            assert torch.equal(bank.w[p][s].cpu().view(torch.uint8), ref[p][0].view(torch.uint8)), (grp, p)
            assert torch.equal(bank.s[p][s].cpu(), ref[p][1]), (grp, p)
    hits, misses = dc.counters()
    assert misses == sum(len(set(e)) for e in steps) - hits
