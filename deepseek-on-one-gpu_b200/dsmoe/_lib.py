"""ctypes binding of ``libdsmoe.so`` (the C ABI in ``include/dsmoe.h``).

There is no fallback: if the library is missing or a call fails, a
``RuntimeError`` is raised. Workspaces are cached per device and grown on
demand; the library itself never allocates.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdsmoe.so")

ROUTER_MODES = {"ref": 0, "v3": 1}
ERRORS = {-1: "invalid argument", -2: "CUDA error", -3: "workspace too small", -4: "unsupported", -5: "device error"}

EXPORTED = (
    "dsmoe_last_error", "dsmoe_version", "dsmoe_workspace_size", "dsmoe_route", "dsmoe_moe_forward",
    "dsmoe_moe_experts", "dsmoe_expert_ffn_workspace_size", "dsmoe_fp8_linear_workspace_size",
    "dsmoe_expert_ffn", "dsmoe_fp8_linear", "dsmoe_read_status", "dsmoe_set_profile_events",
    "dsmoe_expert_ffn_noalloc", "dsmoe_ep_dispatch", "dsmoe_moe_local_workspace_size", "dsmoe_moe_local",
    "dsmoe_ep_combine", "dsmoe_set_gemm_sm_limit", "dsmoe_rms_norm", "dsmoe_moe_layer_ffn_workspace_size",
    "dsmoe_moe_layer_ffn", "dsmoe_read_ranges", "dsmoe_ep_plan", "dsmoe_ep_push", "dsmoe_moe_local_peer",
    "dsmoe_ep_meta_bytes", "dsmoe_ipc_alloc", "dsmoe_ipc_open", "dsmoe_ipc_close", "dsmoe_ipc_free",
    "dsmoe_sample_top_p", "dsmoe_slotcache_state_bytes", "dsmoe_slotcache_step", "dsmoe_map_host_pointers",
    "dsmoe_clock_probe",
)


class MoeConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("n_routed", ctypes.c_int32),
        ("n_group", ctypes.c_int32), ("topk_group", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("router_mode", ctypes.c_int32), ("norm_topk_prob", ctypes.c_int32),
        ("routed_scaling_factor", ctypes.c_float),
    ]


class LayerWeights(ctypes.Structure):
    _fields_ = [
        ("gate_weight", ctypes.c_void_p), ("score_bias", ctypes.c_void_p), ("n_slots", ctypes.c_int32),
        ("w_gate", ctypes.c_void_p), ("s_gate", ctypes.c_void_p),
        ("w_up", ctypes.c_void_p), ("s_up", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p), ("s_down", ctypes.c_void_p),
        ("slot_of_expert", ctypes.c_void_p),
    ]


class SlotCacheDesc(ctypes.Structure):
    """``dsmoe_slotcache_t`` (include/dsmoe.h)."""
    _fields_ = [
        ("n_experts", ctypes.c_int32), ("n_slots", ctypes.c_int32), ("hidden", ctypes.c_int32),
        ("inter", ctypes.c_int32),
        ("w_gate", ctypes.c_void_p), ("s_gate", ctypes.c_void_p), ("w_up", ctypes.c_void_p),
        ("s_up", ctypes.c_void_p), ("w_down", ctypes.c_void_p), ("s_down", ctypes.c_void_p),
        ("slot_of", ctypes.c_void_p), ("state", ctypes.c_void_p), ("host_src", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"libdsmoe.so is not built ({LIB_PATH}); run __graft_entry__.build()")
                L = ctypes.CDLL(LIB_PATH)
                vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
                cfgp = ctypes.POINTER(MoeConfig)
                wp = ctypes.POINTER(LayerWeights)
                L.dsmoe_last_error.restype = ctypes.c_char_p
                L.dsmoe_version.restype = ctypes.c_int
                L.dsmoe_workspace_size.argtypes = [cfgp, i32]
                L.dsmoe_workspace_size.restype = sz
                L.dsmoe_route.argtypes = [cfgp, vp, vp, vp, i32, vp, vp, vp, sz, vp]
                L.dsmoe_moe_forward.argtypes = [cfgp, wp, vp, i32, vp, vp, vp, vp, sz, vp]
                L.dsmoe_moe_experts.argtypes = [cfgp, wp, vp, i32, vp, vp, sz, vp]
                L.dsmoe_expert_ffn_workspace_size.argtypes = [i32, i32, i32]
                L.dsmoe_expert_ffn_workspace_size.restype = sz
                L.dsmoe_fp8_linear_workspace_size.argtypes = [i32, i32, i32]
                L.dsmoe_fp8_linear_workspace_size.restype = sz
                L.dsmoe_expert_ffn.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
                L.dsmoe_fp8_linear.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp, sz, vp]
                L.dsmoe_read_status.argtypes = [vp, ctypes.POINTER(ctypes.c_int32), vp]
                L.dsmoe_set_profile_events.argtypes = [ctypes.POINTER(vp), i32]
                L.dsmoe_clock_probe.argtypes = [vp, i32, vp]
                L.dsmoe_expert_ffn_noalloc.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]
                L.dsmoe_ep_dispatch.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]
                L.dsmoe_moe_local_workspace_size.argtypes = [cfgp, i32]
                L.dsmoe_moe_local_workspace_size.restype = sz
                L.dsmoe_moe_local.argtypes = [cfgp, wp, vp, i32, vp, vp, vp, vp, sz, vp]
                L.dsmoe_ep_combine.argtypes = [vp, vp, i32, i32, i32, vp, ctypes.c_float, vp, vp]
                L.dsmoe_set_gemm_sm_limit.argtypes = [i32]
                L.dsmoe_rms_norm.argtypes = [vp, vp, ctypes.c_float, i32, i32, vp, vp]
                L.dsmoe_moe_layer_ffn_workspace_size.argtypes = [cfgp, i32]
                L.dsmoe_moe_layer_ffn_workspace_size.restype = sz
                L.dsmoe_moe_layer_ffn.argtypes = [cfgp, wp, vp, vp, ctypes.c_float, i32, vp, vp, vp, vp, sz, vp]
                L.dsmoe_ep_plan.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]
                L.dsmoe_ep_push.argtypes = [vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, i32, vp]
                L.dsmoe_moe_local_peer.argtypes = [cfgp, wp, vp, i32, vp, i32, i32, i32, vp, vp, vp, sz, vp]
                L.dsmoe_ep_meta_bytes.argtypes = [i32, i32, i32]
                L.dsmoe_ep_meta_bytes.restype = sz
                L.dsmoe_ipc_alloc.argtypes = [sz, ctypes.POINTER(vp), vp]
                L.dsmoe_ipc_open.argtypes = [vp, ctypes.POINTER(vp)]
                L.dsmoe_ipc_close.argtypes = [vp]
                L.dsmoe_ipc_free.argtypes = [vp]
                L.dsmoe_sample_top_p.argtypes = [vp, i32, i32, ctypes.c_int64, ctypes.c_float, ctypes.c_float, vp, vp,
                                                 vp, vp]
                u64p = ctypes.POINTER(ctypes.c_uint64)
                L.dsmoe_slotcache_state_bytes.argtypes = [i32]
                L.dsmoe_slotcache_state_bytes.restype = sz
                L.dsmoe_slotcache_step.argtypes = [ctypes.POINTER(SlotCacheDesc), vp, i32, vp]
                L.dsmoe_map_host_pointers.argtypes = [u64p, i32, u64p]
                L.dsmoe_read_ranges.argtypes = [i32, ctypes.POINTER(ctypes.c_char_p), u64p, u64p,
                                                ctypes.POINTER(vp), i32]
                for name in EXPORTED:
                    getattr(L, name).restype = getattr(L, name).restype or ctypes.c_int
                _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().dsmoe_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({ERRORS.get(rc, rc)}): {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("dsmoe runs on CUDA tensors only (no CPU fallback)")
        if not t.is_contiguous():
            raise RuntimeError("dsmoe expects contiguous tensors")


class Workspace:
    """Per-device scratch buffer, zero-initialised once (the first bytes hold
    the device error word) and grown on demand."""

    _by_device: dict[int, "Workspace"] = {}

    def __init__(self, device: torch.device):
        self.device = device
        self.buf = torch.zeros(0, dtype=torch.uint8, device=device)

    @classmethod
    def get(cls, device: torch.device) -> "Workspace":
        idx = device.index if device.index is not None else torch.cuda.current_device()
        ws = cls._by_device.get(idx)
        if ws is None:
            ws = cls._by_device[idx] = Workspace(torch.device("cuda", idx))
        return ws

    def ensure(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            # Grow by 25 % to avoid re-allocating for every new token count.
            self.buf = torch.zeros(int(nbytes * 1.25) + 4096, dtype=torch.uint8, device=self.device)
        return self.buf

    def status(self) -> int:
        st = ctypes.c_int32(0)
        lib().dsmoe_read_status(ptr(self.buf), ctypes.byref(st), stream_handle(self.device))
        return int(st.value)


def moe_config(config) -> MoeConfig:
    mode = getattr(config, "router_mode", "ref")
    return MoeConfig(
        hidden=config.hidden_size, inter=config.moe_intermediate_size, n_routed=config.n_routed_experts,
        n_group=config.n_group, topk_group=config.topk_group, top_k=config.num_experts_per_tok,
        router_mode=ROUTER_MODES[mode], norm_topk_prob=int(bool(config.norm_topk_prob)),
        routed_scaling_factor=float(config.routed_scaling_factor),
    )


def set_gemm_sm_limit(max_ctas: int) -> None:
    """Cap this thread's later grouped-GEMM launches at ``max_ctas`` CTAs (one
    per SM; 0 = all SMs) so that a collective on another stream finds free
    SMs."""
    check(lib().dsmoe_set_gemm_sm_limit(int(max_ctas)), "dsmoe_set_gemm_sm_limit")


class ClockProbe:
    """Mean SM clock over a region of a stream: ``start()`` and ``stop()``
    enqueue a probe in which every SM records its cycle counter and the
    global ns timer; ``mhz()`` (after the stream is synchronised) is the
    median over SMs of cycles / ns between the two."""

    def __init__(self, device):
        import torch

        self.n = torch.cuda.get_device_properties(device).multi_processor_count
        self.a = torch.zeros(2 * self.n, dtype=torch.int64, device=device)
        self.b = torch.zeros_like(self.a)

    def _probe(self, buf):
        import torch

        check(lib().dsmoe_clock_probe(buf.data_ptr(), self.n, torch.cuda.current_stream(buf.device).cuda_stream),
              "dsmoe_clock_probe")

    def start(self):
        self._probe(self.a)

    def stop(self):
        self._probe(self.b)

    def mhz(self) -> float | None:
        a, b = self.a.view(-1, 2).cpu().double(), self.b.view(-1, 2).cpu().double()
        dt = b[:, 1] - a[:, 1]
        ok = (a[:, 1] > 0) & (b[:, 1] > 0) & (dt > 0)
        if not bool(ok.any()):
            return None
        return float(((b[:, 0] - a[:, 0])[ok] / dt[ok]).median() * 1e3)


def set_profile_events(events: list | None) -> None:
    """Record ``events`` (torch.cuda.Event, up to 8) at the stage boundaries of
    later MoE calls from this thread; ``None`` switches it off."""
    if not events:
        check(lib().dsmoe_set_profile_events(None, 0), "dsmoe_set_profile_events")
        return
    for e in events:
        if e.cuda_event == 0:  # torch creates the CUDA event lazily
            e.record()
    arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
    check(lib().dsmoe_set_profile_events(arr, len(events)), "dsmoe_set_profile_events")
