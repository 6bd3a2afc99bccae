"""The allocation-free expert FFN entry point (dsmoe_expert_ffn_noalloc).

It exists for callers that cannot allocate device memory when they call in:
a runtime that owns all device memory through its own fixed pool, code that
runs while an allocator lock is held, latency-critical paths that must not
block, synchronize or fail on an allocation. Its scratch is a fixed array
inside libdsmoe instead of a caller workspace.

This file is named so that pytest collects it last: if it fails, a run that
stops at the first failure has already run every other test. It must pass
both alone in a fresh process and after the other tests (the scratch array
keeps whatever the previous call left in it).
"""
import ctypes

import pytest
import torch

from dsmoe import _lib, ops
from dsmoe.synthetic import activations, expert_weights
from oracle.moe_oracle import rel_rms

pytestmark = pytest.mark.gpu

REL_RMS_TOL = 1e-2  # the output tolerance used by the other GPU parity tests
DEV = torch.device("cuda", 0)


def call_noalloc(x, ew, out):
    L = _lib.lib()
    T, H = x.shape
    F = ew["gate_proj"][0].shape[0]
    p = _lib.ptr
    return L.dsmoe_expert_ffn_noalloc(
        p(x), T, H, F, p(ew["gate_proj"][0]), p(ew["gate_proj"][1]), p(ew["up_proj"][0]), p(ew["up_proj"][1]),
        p(ew["down_proj"][0]), p(ew["down_proj"][1]), p(out), _lib.stream_handle(DEV))


@pytest.mark.parametrize("T,H,F,seed", [(48, 7168, 2048, 1), (200, 1024, 512, 2)])
def test_noalloc_matches_workspace_entry_point_twice(T, H, F, seed):
    ew = {p: (w.to(DEV), s.to(DEV)) for p, (w, s) in expert_weights(seed, 3, 7, H, F).items()}
    for call in range(2):  # two calls in a row share (and reuse) the static scratch
        x = activations(seed * 10 + call, T, H).to(DEV)
        ref = ops.expert_ffn(x, ew)  # the existing entry point, caller-provided workspace
        out = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc = call_noalloc(x, ew, out)
        assert rc == 0, _lib.lib().dsmoe_last_error()
        torch.cuda.synchronize()
        err = rel_rms(out.float().cpu(), ref.float().cpu())
        assert err <= REL_RMS_TOL, (call, err)


def test_noalloc_rejects_oversized_calls():
    L = _lib.lib()
    T, H, F = 4096, 7168, 2048  # needs ~110 MB of scratch, above the fixed 8 MiB
    assert L.dsmoe_expert_ffn_workspace_size(T, H, F) > 8 * 1024 * 1024
    dummy = ctypes.c_void_p(256)  # never dereferenced: the size check runs first
    rc = L.dsmoe_expert_ffn_noalloc(dummy, T, H, F, dummy, dummy, dummy, dummy, dummy, dummy, dummy,
                                    _lib.stream_handle(DEV))
    assert rc == -3
    assert b"scratch" in L.dsmoe_last_error()
