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
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

REL_RMS_TOL = 1e-2  # the output tolerance used by the other GPU parity tests
DEV = torch.device("cuda", 0)
SCRATCH = 8 * 1024 * 1024  # DSMOE_NOALLOC_SCRATCH_BYTES


def call_noalloc(x, ew, out):
    L = _lib.lib()
    T, H = x.shape
    F = ew["gate_proj"][0].shape[0]
    p = _lib.ptr
    return L.dsmoe_expert_ffn_noalloc(
        p(x), T, H, F, p(ew["gate_proj"][0]), p(ew["gate_proj"][1]), p(ew["up_proj"][0]), p(ew["up_proj"][1]),
        p(ew["down_proj"][0]), p(ew["down_proj"][1]), p(out), _lib.stream_handle(DEV))


def noalloc_status():
    """The scratch's device error word (read and cleared)."""
    st = ctypes.c_int32(-1)
    rc = _lib.lib().dsmoe_read_status(None, ctypes.byref(st), _lib.stream_handle(DEV))
    return rc, st.value


def max_tokens(H, F):
    L = _lib.lib()
    T = 1
    while L.dsmoe_expert_ffn_workspace_size(T + 1, H, F) <= SCRATCH:
        T += 1
    return T


def run(x, ew):
    out = torch.full(x.shape, float("nan"), dtype=torch.bfloat16, device=DEV)
    rc = call_noalloc(x, ew, out)
    assert rc == 0, _lib.lib().dsmoe_last_error()
    return out


@pytest.mark.parametrize("T,H,F,seed", [(48, 7168, 2048, 1), (200, 1024, 512, 2)])
def test_noalloc_matches_oracle_and_workspace_entry_point_twice(T, H, F, seed):
    ew_cpu = expert_weights(seed, 3, 7, H, F)
    ew = {p: (w.to(DEV), s.to(DEV)) for p, (w, s) in ew_cpu.items()}
    for call in range(2):  # two calls in a row share (and reuse) the static scratch
        x = activations(seed * 10 + call, T, H)
        out = run(x.to(DEV), ew)
        torch.cuda.synchronize()
        ref = O.expert_ffn(x, ew_cpu)  # the reference arithmetic (CPU oracle)
        err = O.rel_rms(out.float().cpu(), ref.float())
        assert err <= REL_RMS_TOL, (call, err)
        # the same kernels as the workspace entry point: bit-identical
        assert torch.equal(out, ops.expert_ffn(x.to(DEV), ew)), call
    assert noalloc_status() == (0, 0)


def test_noalloc_largest_then_small_call():
    """The largest call the scratch takes, then a small one: the small call
    must not pick up anything the large one left in the shared array."""
    H, F = 7168, 2048
    ew = {p: (w.to(DEV), s.to(DEV)) for p, (w, s) in expert_weights(4, 3, 11, H, F).items()}
    T_max = max_tokens(H, F)
    assert T_max >= 256
    for T, seed in ((T_max, 40), (5, 41), (T_max - 31, 42)):
        x = activations(seed, T, H).to(DEV)
        out = run(x, ew)
        assert torch.equal(out, ops.expert_ffn(x, ew)), T
    assert noalloc_status() == (0, 0)


def test_noalloc_allocates_no_device_memory():
    """After a first call (module loading, the one-time set-up), further calls
    leave the device's free memory unchanged."""
    H, F = 1024, 512
    ew = {p: (w.to(DEV), s.to(DEV)) for p, (w, s) in expert_weights(5, 3, 2, H, F).items()}
    xs = [activations(50 + i, 64, H).to(DEV) for i in range(4)]
    outs = [torch.empty(64, H, dtype=torch.bfloat16, device=DEV) for _ in range(4)]
    assert call_noalloc(xs[0], ew, outs[0]) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(DEV)[0]
    for i in range(1, 4):
        assert call_noalloc(xs[i], ew, outs[i]) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(DEV)[0] >= free0


def test_noalloc_rejects_oversized_calls():
    L = _lib.lib()
    T, H, F = 4096, 7168, 2048  # needs ~110 MB of scratch, above the fixed 8 MiB
    assert L.dsmoe_expert_ffn_workspace_size(T, H, F) > SCRATCH
    dummy = ctypes.c_void_p(256)  # never dereferenced: the size check runs first
    rc = L.dsmoe_expert_ffn_noalloc(dummy, T, H, F, dummy, dummy, dummy, dummy, dummy, dummy, dummy,
                                    _lib.stream_handle(DEV))
    assert rc == -3
    assert b"scratch" in L.dsmoe_last_error()
