"""Streaming decode through a stack of MoE layers with experts held in pinned
host memory (the reference's deployment: ``inference/engine.py`` decode loop
over ``moe_block`` with ``GPUTransfer`` / ``WeightStore.get_expert``).

Each layer keeps a GPU slot cache (``LayerBank``, LRU over slots). Per layer
and step:

  1. route the hidden state with this layer's gate, and - when prefetching -
     with the NEXT layer's gate as a prediction of its experts;
  2. one device->host read of both expert lists (the reference reads the
     routing back once per token and layer too, ``gpu_transfer.py:60``);
  3. missing experts of this layer are copied on the side stream (the compute
     stream waits on an event; prefetched copies of this layer are waited for
     the same way);
  4. the expert GEMMs of this layer are enqueued, then the predicted experts
     of the next layer start copying on the side stream, overlapping them -
     but only while the prediction has been right: each layer keeps a running
     precision (predicted experts that were then used); below 50 % the copies
     would spend host-link bandwidth on experts nobody needs, so they stop
     (predictions continue and re-enable them if they improve);
  5. ``h <- h + moe(h)``: the block's residual connection
     (``inference/forward.py:109``) carries the hidden state to the next layer.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_handle
from .forward import _layer_weights
from .gpu_transfer import GPUTransfer


class StreamingDecoder:
    def __init__(self, config, weight_store, device, layers, slots_per_layer: int = 65, prefetch: bool = True,
                 device_slots: bool = False):
        self.config = config
        self.store = weight_store
        self.device = torch.device(device)
        self.layers = list(layers)
        self.prefetch = prefetch
        self.gt = GPUTransfer(config, weight_store, self.device, slots_per_layer=slots_per_layer,
                              device_slots=device_slots)
        self.cfg = _lib.moe_config(config)
        self.K = config.num_experts_per_tok
        self.ws = torch.zeros(0, dtype=torch.uint8, device=self.device)
        self.pred_ws = torch.zeros(0, dtype=torch.uint8, device=self.device)
        self.predicted = 0
        self.predicted_used = 0
        self.precision = {layer: 1.0 for layer in self.layers}  # running prefetch precision per layer
        self.min_precision = 0.5
        for layer in self.layers:
            self.gt.bank(layer)
        # device-managed slot tables: every layer's experts in pinned host memory
        self.device_slots = device_slots and all(self.gt.device_cache(l) is not None for l in self.layers)
        if device_slots and not self.device_slots:
            raise ValueError("device_slots needs every routed expert of the layers in pinned host memory "
                             "(weight_store.preload_host)")

    def _route(self, x, layer, ws, idx, w):
        T = x.shape[0]
        need = lib().dsmoe_workspace_size(self.cfg, T)
        if ws.numel() < need:
            ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        gate = self.store.get_gate_weight(layer)
        bias = self.store.get_gate_bias(layer) if getattr(self.config, "router_mode", "ref") == "v3" else None
        check(lib().dsmoe_route(self.cfg, ptr(x), ptr(gate), ptr(bias), T, ptr(idx), ptr(w), ptr(ws), ws.numel(),
                                stream_handle(self.device)), "dsmoe_route")
        return ws

    def step(self, h: torch.Tensor) -> torch.Tensor:
        """One decode step: h [T, H] bf16 through every layer."""
        if self.device_slots:
            return self._step_device(h)
        T = h.shape[0]
        idx = torch.empty(T, self.K, dtype=torch.int64, device=self.device)
        w = torch.empty(T, self.K, dtype=torch.float32, device=self.device)
        pidx = torch.empty(T, self.K, dtype=torch.int64, device=self.device)
        pw = torch.empty(T, self.K, dtype=torch.float32, device=self.device)
        pending_pred = None
        for i, layer in enumerate(self.layers):
            x = h.contiguous()
            self.ws = self._route(x, layer, self.ws, idx, w)
            nxt = self.layers[i + 1] if self.prefetch and i + 1 < len(self.layers) else None
            if nxt is not None:
                self.pred_ws = self._route(x, nxt, self.pred_ws, pidx, pw)
            both = torch.cat([idx.view(-1), pidx.view(-1)]).cpu().tolist() if nxt is not None else idx.view(-1).cpu().tolist()
            experts = sorted(set(both[: T * self.K]))
            if pending_pred is not None:
                used = len(pending_pred & set(experts))
                self.predicted_used += used
                self.precision[layer] = 0.8 * self.precision[layer] + 0.2 * used / max(1, len(pending_pred))
            bank = self.gt.ensure_resident(layer, experts)
            out = torch.empty_like(x)
            lw = _layer_weights(bank, self.store.get_gate_weight(layer), None)
            check(lib().dsmoe_moe_experts(self.cfg, lw, ptr(x), T, ptr(out), ptr(self.ws), self.ws.numel(),
                                          stream_handle(self.device)), "dsmoe_moe_experts")
            self.gt.mark_used(layer)
            if nxt is not None:
                pending_pred = set(both[T * self.K:])
                self.predicted += len(pending_pred)
                if self.precision[nxt] >= self.min_precision:
                    self.gt.prefetch(nxt, sorted(pending_pred))
            else:
                pending_pred = None
            h = x + out
        return h

    def _step_device(self, h: torch.Tensor) -> torch.Tensor:
        """The decode step with device-managed slot tables: per layer the
        router, ``dsmoe_slotcache_step`` (slot placement and host->device
        copies of the missing experts by the SMs) and the expert GEMMs, all
        enqueued on the current stream; the host reads nothing and waits for
        nothing. No next-layer prefetch on this path."""
        T = h.shape[0]
        idx = torch.empty(T, self.K, dtype=torch.int64, device=self.device)
        w = torch.empty(T, self.K, dtype=torch.float32, device=self.device)
        for layer in self.layers:
            x = h.contiguous()
            self.ws = self._route(x, layer, self.ws, idx, w)
            self.gt.device_cache(layer).step(idx)
            bank = self.gt.bank(layer)
            out = torch.empty_like(x)
            lw = _layer_weights(bank, self.store.get_gate_weight(layer), None)
            check(lib().dsmoe_moe_experts(self.cfg, lw, ptr(x), T, ptr(out), ptr(self.ws), self.ws.numel(),
                                          stream_handle(self.device)), "dsmoe_moe_experts")
            h = x + out
        return h

    def device_counters(self) -> tuple[int, int, int]:
        """(hits, misses, bytes moved) of the device-managed slot tables (a
        host read)."""
        hits = misses = 0
        for layer in self.layers:
            a, b = self.gt.device_cache(layer).counters()
            hits, misses = hits + a, misses + b
        c = self.config
        per_expert = 3 * c.hidden_size * c.moe_intermediate_size + \
            3 * (c.hidden_size // 128) * (c.moe_intermediate_size // 128) * 4
        return hits, misses, misses * per_expert
