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
