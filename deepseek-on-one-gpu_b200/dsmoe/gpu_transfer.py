"""GPU expert residency: per-layer weight banks and the H2D slot cache.

Replaces ``GPUTransfer`` (``inference/gpu_transfer.py:7-89``). The reference
owns 8 GPU slots, copies the 8 experts of ONE token into them on a side stream
and blocks the host on ``synchronize()`` before every token's FFNs
(:68-79). Here each MoE layer owns a ``LayerBank``: ``n_slots`` expert slots
laid out as three stacked e4m3 weight tensors plus their scales, and a
device-side ``slot_of`` table (group -> slot) that the grouped GEMMs read.

  * Resident mode (``slots_per_layer = n_routed + 1``): every expert of the
    layer lives in HBM (11.3 GB FP8 per DeepSeek-R1 layer), nothing moves.
  * Streaming mode (fewer slots): ``ensure_resident`` brings missing experts
    in on a side stream with one ``cudaMemcpyAsync`` per tensor, evicting the
    least recently used slot, and makes the compute stream wait on an event;
    the host never blocks on the copy itself.

``transfer_experts`` keeps the reference signature and return value (a list
of ``{proj: (weight, scale)}`` per requested expert, views into the bank).

Device-managed streaming (``device_slots=True``, when the weight store holds
every routed expert of a layer in pinned host memory): the slot table is kept
on the GPU by ``dsmoe_slotcache_step`` (``DeviceSlotCache``), which places the
step's missing experts in least-recently-used slots and copies them from host
memory with the SMs, all on the compute stream: the routing is never read
back and the host never waits.
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_handle
from .synthetic import PROJS

PINNED_SLOT = 0x7FFFFFFF  # last_use of the shared expert's slot: never taken


class LayerBank:
    def __init__(self, config, n_slots: int, device: torch.device):
        E, H, F = config.n_routed_experts, config.hidden_size, config.moe_intermediate_size
        self.n_slots, self.device, self.n_groups = n_slots, device, E + 1
        e4m3 = torch.float8_e4m3fn
        self.w = {
            "gate_proj": torch.empty(n_slots, F, H, dtype=e4m3, device=device),
            "up_proj": torch.empty(n_slots, F, H, dtype=e4m3, device=device),
            "down_proj": torch.empty(n_slots, H, F, dtype=e4m3, device=device),
        }
        self.s = {
            "gate_proj": torch.empty(n_slots, F // 128, H // 128, dtype=torch.float32, device=device),
            "up_proj": torch.empty(n_slots, F // 128, H // 128, dtype=torch.float32, device=device),
            "down_proj": torch.empty(n_slots, H // 128, F // 128, dtype=torch.float32, device=device),
        }
        self.slot_of = torch.full((E + 1,), -1, dtype=torch.int32, device=device)
        self.slot_of_host = [-1] * (E + 1)
        self.group_in_slot = [-1] * n_slots
        self.lru: OrderedDict[int, int] = OrderedDict()  # group -> slot, routed experts only
        self.free = list(range(n_slots))
        self.last_use: torch.cuda.Event | None = None
        self.pending: torch.cuda.Event | None = None  # prefetch copies in flight
        self.dirty = False

    @property
    def fully_resident(self) -> bool:
        return all(s >= 0 for s in self.slot_of_host)

    def assign(self, group: int, pinned: set[int] | None = None) -> int:
        """Slot for `group` (already resident, a free slot, or the LRU victim)."""
        s = self.slot_of_host[group]
        if s >= 0:
            if group in self.lru:
                self.lru.move_to_end(group)
            return s
        if self.free:
            s = self.free.pop(0)
        else:
            victim = next((g for g in self.lru if not pinned or g not in pinned), None)
            if victim is None:
                raise RuntimeError("expert slot cache too small for the experts one step needs")
            s = self.lru.pop(victim)
            self.slot_of_host[victim] = -1
        self.slot_of_host[group] = s
        self.group_in_slot[s] = group
        if group != 0:
            self.lru[group] = s
        self.dirty = True
        return s

    def write_slot(self, slot: int, expert: dict, non_blocking: bool = False) -> int:
        """Copy one expert ``{proj: (weight, scale)}`` into `slot`; returns bytes."""
        n = 0
        for p in PROJS:
            w, s = expert[p]
            if isinstance(w, dict):  # ExpertCache entry form
                w, s = w["weight"], w["weight_scale_inv"]
            self.w[p][slot].copy_(w, non_blocking=non_blocking)
            self.s[p][slot].copy_(s, non_blocking=non_blocking)
            n += w.nbytes + s.nbytes
        return n

    def sync_table(self, non_blocking: bool = True) -> None:
        if self.dirty:
            host = torch.tensor(self.slot_of_host, dtype=torch.int32)
            if torch.cuda.is_available():
                host = host.pin_memory()
            self.slot_of.copy_(host, non_blocking=non_blocking)
            self.dirty = False

    def views(self, group: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        s = self.slot_of_host[group]
        return {p: (self.w[p][s], self.s[p][s]) for p in PROJS}


class DeviceSlotCache:
    """The slot table of one ``LayerBank`` kept on the device
    (``dsmoe_slotcache_step``): each step marks the experts its routing needs,
    refreshes their recency, gives every missing expert the least recently
    used slot the step does not need and copies it in from pinned host memory.
    After construction the bank's host-side mirrors are no longer maintained;
    ``refresh_host_mirror`` reads the device table back (a host sync, for
    inspection only)."""

    def __init__(self, bank: LayerBank, config, host_ptrs: list[int]):
        E, H, F = config.n_routed_experts, config.hidden_size, config.moe_intermediate_size
        if len(host_ptrs) != 6 * E:
            raise ValueError("need 6 host tensors per routed expert")
        self.bank, self.device = bank, bank.device
        src = (ctypes.c_uint64 * (6 * E))(*host_ptrs)
        dev = (ctypes.c_uint64 * (6 * E))()
        check(lib().dsmoe_map_host_pointers(src, 6 * E, dev), "dsmoe_map_host_pointers")
        self.src = torch.tensor([int(v) for v in dev], dtype=torch.int64).to(self.device)  # uint64 bits
        n = bank.n_slots
        st = torch.zeros(lib().dsmoe_slotcache_state_bytes(n) // 4, dtype=torch.int32)
        st[4:4 + n] = torch.tensor(bank.group_in_slot, dtype=torch.int32)
        last = [-1 if g < 0 else (PINNED_SLOT if g == 0 else 0) for g in bank.group_in_slot]
        st[4 + n:4 + 2 * n] = torch.tensor(last, dtype=torch.int32)
        bank.sync_table(non_blocking=False)
        self.state = st.to(self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.desc = _lib.SlotCacheDesc(
            n_experts=E, n_slots=n, hidden=H, inter=F,
            w_gate=ptr(bank.w["gate_proj"]), s_gate=ptr(bank.s["gate_proj"]), w_up=ptr(bank.w["up_proj"]),
            s_up=ptr(bank.s["up_proj"]), w_down=ptr(bank.w["down_proj"]), s_down=ptr(bank.s["down_proj"]),
            slot_of=ptr(bank.slot_of), state=ptr(self.state), host_src=ptr(self.src), status=ptr(self.status))
        bank.device_managed = True

    def step(self, topk_idx: torch.Tensor) -> None:
        """Make the experts of ``topk_idx`` (int64, any shape) resident, on
        the current stream."""
        idx = topk_idx.contiguous()
        check(lib().dsmoe_slotcache_step(ctypes.byref(self.desc), ptr(idx), idx.numel(),
                                         stream_handle(self.device)), "dsmoe_slotcache_step")

    def counters(self) -> tuple[int, int]:
        """(hits, misses) so far (a host read)."""
        v = self.state[2:4].tolist()
        return int(v[0]), int(v[1])

    def device_status(self) -> int:
        return int(self.status.item())

    def refresh_host_mirror(self) -> None:
        b = self.bank
        b.slot_of_host = b.slot_of.tolist()
        n = b.n_slots
        b.group_in_slot = self.state[4:4 + n].tolist()


class GPUTransfer:
    """Expert residency manager with the reference's constructor and
    ``transfer_experts`` signature (``inference/gpu_transfer.py:15-16,50-52``)."""

    def __init__(self, config, weight_store, device, verbose: bool = False, slots_per_layer: int | None = None,
                 device_slots: bool = False):
        self.config = config
        self.weight_store = weight_store
        self.device = torch.device(device)
        self.verbose = verbose
        self.slots = slots_per_layer or (config.n_routed_experts + 1)
        if self.slots < config.num_experts_per_tok + 1:
            raise ValueError("need at least top_k + 1 slots per layer")
        self.transfer_stream = torch.cuda.Stream(device=self.device)
        self.banks: dict[int, LayerBank] = {}
        self.bytes_h2d = 0
        self.slot_hits = 0
        self.slot_misses = 0
        self.prefetched = 0
        self.device_slots = device_slots
        self.dcache: dict[int, DeviceSlotCache] = {}

    @property
    def resident(self) -> bool:
        return self.slots >= self.config.n_routed_experts + 1

    def bank(self, layer: int) -> LayerBank:
        b = self.banks.get(layer)
        if b is None:
            b = LayerBank(self.config, self.slots, self.device)
            self.banks[layer] = b
            if self.resident and hasattr(self.weight_store, "fill_bank"):
                self.weight_store.fill_bank(layer, b)
            else:
                b.write_slot(b.assign(0), self.weight_store.get_shared_expert_weights(layer))
                if self.resident:
                    for e in range(self.config.n_routed_experts):
                        b.write_slot(b.assign(e + 1), self.weight_store.get_expert(layer, e))
            b.sync_table(non_blocking=False)
            torch.cuda.current_stream(self.device).synchronize()
        return b

    def device_cache(self, layer: int) -> DeviceSlotCache | None:
        """The layer's device-managed slot table (streaming mode with
        ``device_slots`` and every routed expert in pinned host memory)."""
        if self.resident or not self.device_slots:
            return None
        dc = self.dcache.get(layer)
        if dc is None:
            ptrs = getattr(self.weight_store, "host_expert_pointers", lambda _l: None)(layer)
            if ptrs is None:
                return None
            dc = self.dcache[layer] = DeviceSlotCache(self.bank(layer), self.config, ptrs)
        return dc

    def prefetch(self, layer: int, experts) -> int:
        """Start bringing `experts` (routed ids) into the layer's bank on the side
        stream without making the compute stream wait; the next
        ``ensure_resident`` on this layer waits for them. Returns the number of
        experts whose copy was started."""
        b = self.bank(layer)
        missing = [g for g in dict.fromkeys(int(e) + 1 for e in experts) if b.slot_of_host[g] < 0]
        if not missing:
            return 0
        ts = self.transfer_stream
        if b.last_use is not None:
            ts.wait_event(b.last_use)
        with torch.cuda.stream(ts):
            for g in missing:
                slot = b.assign(g, pinned=set(missing))
                self.bytes_h2d += b.write_slot(slot, self.weight_store.get_expert(layer, g - 1), non_blocking=True)
            b.sync_table(non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(ts)
        b.pending = ev
        self.prefetched += len(missing)
        return len(missing)

    def ensure_resident(self, layer: int, experts) -> LayerBank:
        """Make `experts` (routed ids) resident in the layer's bank. Copies run
        on the side stream after the bank's last use; the current stream waits
        for them (and for any prefetch of this layer) with an event."""
        b = self.bank(layer)
        if b.pending is not None:
            torch.cuda.current_stream(self.device).wait_event(b.pending)
            b.pending = None
        need = [int(e) for e in experts]
        groups = {e + 1 for e in need}
        missing = [g for g in dict.fromkeys(e + 1 for e in need) if b.slot_of_host[g] < 0]
        self.slot_hits += len(groups) - len(missing)
        self.slot_misses += len(missing)
        for g in groups - set(missing):
            b.assign(g)  # refresh recency
        if not missing:
            return b
        ts = self.transfer_stream
        if b.last_use is not None:
            ts.wait_event(b.last_use)
        with torch.cuda.stream(ts):
            for g in missing:
                slot = b.assign(g, pinned=groups)
                self.bytes_h2d += b.write_slot(slot, self.weight_store.get_expert(layer, g - 1), non_blocking=True)
            b.sync_table(non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(ts)
        torch.cuda.current_stream(self.device).wait_event(ev)
        return b

    def mark_used(self, layer: int) -> None:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.banks[layer].last_use = ev

    def transfer_experts(self, layer: int, expert_indices: torch.Tensor, verbose: bool = False):
        indices = [int(i) for i in expert_indices.reshape(-1).tolist()]
        b = self.ensure_resident(layer, indices)
        if verbose or self.verbose:
            print(f"      [gpu_transfer] L{layer:02d}: experts {indices} resident")
        return [b.views(e + 1) for e in indices]
