"""Device error reporting: a weight-slot table entry outside the expert bank
(a corrupted table) is caught by the grouped GEMM's own bounds check before
anything is read through it. The kernel records DSMOE device error 4 (bad
slot) in the workspace status word, stops every role, lets its copies and
MMAs in flight finish, and returns; the call itself returns normally, the
status read reports the error once, and the next call with a sound table is
bit-identical to the one before. No GPU fault is involved."""
import pytest
import torch

from dsmoe import DeepSeekConfig, GPUTransfer, SyntheticWeightStore, moe_block
from dsmoe._lib import Workspace
from dsmoe.synthetic import activations

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
BAD_SLOT = 4  # kDevBadSlot


@pytest.mark.parametrize("T", [24, 300])
def test_bad_slot_is_reported_and_the_next_call_is_clean(T):
    cfg = DeepSeekConfig(hidden_size=512, moe_intermediate_size=256)
    store = SyntheticWeightStore(cfg, seed=13, device=DEV, pin_memory=False, gen_device="cpu")
    gt = GPUTransfer(cfg, store, DEV)
    x = activations(14, T, 512).to(DEV)
    good = moe_block(x, 3, store, gt, cfg)
    torch.cuda.synchronize()
    assert Workspace.get(DEV).status() == 0
    bank = gt.bank(3)
    saved = bank.slot_of.clone()
    bank.slot_of[1:] = bank.n_slots + 7  # every routed expert points past the bank; the shared one stays
    moe_block(x, 3, store, gt, cfg)
    torch.cuda.synchronize()
    assert Workspace.get(DEV).status() == BAD_SLOT
    assert Workspace.get(DEV).status() == 0  # read and cleared
    bank.slot_of.copy_(saved)
    again = moe_block(x, 3, store, gt, cfg)
    torch.cuda.synchronize()
    assert Workspace.get(DEV).status() == 0
    assert torch.equal(again, good)
