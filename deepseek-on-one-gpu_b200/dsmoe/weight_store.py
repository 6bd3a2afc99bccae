"""Host-side expert storage: the pinned-RAM LRU and a synthetic weight store.

``ExpertCache`` keeps the reference's interface and policy
(``inference/weight_store.py:42-78``): entries keyed ``(layer, expert)`` hold
``{proj: {"weight", "weight_scale_inv"}}`` pinned tensors; ``get`` refreshes
recency, ``put`` evicts least-recently-used entries until the new entry fits
the byte capacity. Hit/miss counters are added.

``SyntheticWeightStore`` answers the calls the MoE path makes on the
reference's ``WeightStore`` (``get_gate_weight`` :252, ``get_shared_expert_weights``
:244, ``get_expert`` :185) with seeded synthetic FP8 weights, so the block can
run without the 689 GB checkpoint. It also adds ``get_gate_bias`` (the
``e_score_correction_bias`` the bias-corrected router needs) and
``fill_bank``, which generates a whole layer directly on the GPU.
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from .synthetic import PROJS, SHARED, SyntheticLayer, expert_weights, norm_weight


class ExpertCache:
    def __init__(self, capacity_bytes: int):
        self.capacity = int(capacity_bytes)
        self.used = 0
        self.entries: OrderedDict[tuple[int, int], dict] = OrderedDict()
        self.hits = 0
        self.misses = 0

    @staticmethod
    def entry_bytes(expert_dict: dict) -> int:
        return sum(t.nbytes for proj in expert_dict.values() if isinstance(proj, dict) for t in proj.values())

    def get(self, layer: int, expert_idx: int) -> dict | None:
        key = (layer, expert_idx)
        entry = self.entries.get(key)
        if entry is None:
            self.misses += 1
            return None
        self.hits += 1
        self.entries.move_to_end(key)
        return entry

    def peek(self, layer: int, expert_idx: int) -> dict | None:
        """The entry without touching the LRU order or the counters."""
        return self.entries.get((layer, expert_idx))

    def put(self, layer: int, expert_idx: int, expert_dict: dict) -> None:
        need = self.entry_bytes(expert_dict)
        self._evict_until(need)
        self.entries[(layer, expert_idx)] = expert_dict
        self.used += need

    def _evict_until(self, needed: int) -> None:
        while self.entries and self.used + needed > self.capacity:
            _, old = self.entries.popitem(last=False)
            self.used -= self.entry_bytes(old)


class SyntheticWeightStore:
    """Seeded stand-in for the reference's ``WeightStore`` on the MoE path."""

    def __init__(self, config, seed: int, device, expert_cache_bytes: int = 16 * 1024 ** 3,
                 pin_memory: bool = True, bias_zipf: float | None = None, layer_seeds: dict | None = None,
                 gen_device: str = "cpu"):
        self.config = config
        self.gen_device = gen_device
        self.seed = seed
        self.device = torch.device(device)
        self.pin_memory = pin_memory and torch.cuda.is_available()
        self.bias_zipf = bias_zipf
        self.layer_seeds = layer_seeds or {}
        self.expert_cache = ExpertCache(expert_cache_bytes)
        self._layers: dict[int, SyntheticLayer] = {}
        self._gate: dict[int, torch.Tensor] = {}
        self._bias: dict[int, torch.Tensor] = {}
        self._shared: dict[int, dict] = {}
        self._norm: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def _seed(self, layer: int) -> int:
        return self.layer_seeds.get(layer, self.seed)

    def layer(self, layer: int) -> SyntheticLayer:
        if layer not in self._layers:
            c = self.config
            self._layers[layer] = SyntheticLayer(self._seed(layer), layer, c.hidden_size, c.moe_intermediate_size,
                                                 c.n_routed_experts, "cpu", bias_zipf=self.bias_zipf, cache=False)
        return self._layers[layer]

    def get_gate_weight(self, layer: int) -> torch.Tensor:
        if layer not in self._gate:
            self._gate[layer] = self.layer(layer).gate.to(self.device)
        return self._gate[layer]

    def get_layer_norm_weights(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(input_layernorm, post_attention_layernorm) weights, as the
        reference's ``WeightStore.get_layer_norm_weights`` (weight_store.py:228-234)."""
        if layer not in self._norm:
            c = self.config
            self._norm[layer] = tuple(norm_weight(self._seed(layer), layer, i, c.hidden_size, self.device)
                                      for i in (0, 1))
        return self._norm[layer]

    def get_gate_bias(self, layer: int) -> torch.Tensor:
        if layer not in self._bias:
            self._bias[layer] = self.layer(layer).bias.to(self.device)
        return self._bias[layer]

    def _generate(self, layer: int, e: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        """Expert ``e`` (``SHARED`` for the shared expert) from the generator
        ``gen_device`` names; every accessor below returns these same bytes."""
        c = self.config
        if self.gen_device == "cpu":
            return self.layer(layer).expert(e)
        return expert_weights(self._seed(layer), layer, e, c.hidden_size, c.moe_intermediate_size,
                              device=self.device)

    def get_shared_expert_weights(self, layer: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        if layer not in self._shared:
            ew = self._generate(layer, SHARED)
            self._shared[layer] = {p: (w.to(self.device), s.to(self.device)) for p, (w, s) in ew.items()}
        return self._shared[layer]

    def get_expert(self, layer: int, expert_idx: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        cached = self.expert_cache.get(layer, expert_idx)
        if cached is None:
            ew = self._generate(layer, expert_idx)
            cached = {}
            for p, (w, s) in ew.items():
                w, s = w.cpu(), s.cpu()
                if self.pin_memory:
                    w, s = w.pin_memory(), s.pin_memory()
                cached[p] = {"weight": w, "weight_scale_inv": s}
            self.expert_cache.put(layer, expert_idx, cached)
        return {p: (cached[p]["weight"], cached[p]["weight_scale_inv"]) for p in PROJS}

    def preload_host(self, layers) -> int:
        """Fill the pinned host LRU with every routed expert of `layers` (the
        host-resident expert store of the streaming configuration): one pinned
        arena per layer, experts generated by ``gen_device`` and copied straight
        into it. Returns the pinned bytes."""
        c = self.config
        E, H, F = c.n_routed_experts, c.hidden_size, c.moe_intermediate_size
        wbytes = {"gate_proj": F * H, "up_proj": F * H, "down_proj": H * F}
        sshape = {"gate_proj": (F // 128, H // 128), "up_proj": (F // 128, H // 128), "down_proj": (H // 128, F // 128)}
        per_w = sum(wbytes.values())
        per_s = sum(a * b for a, b in sshape.values())
        total = 0
        for layer in layers:
            warena = torch.empty(E * per_w, dtype=torch.uint8, pin_memory=self.pin_memory)
            sarena = torch.empty(E * per_s, dtype=torch.float32, pin_memory=self.pin_memory)
            total += warena.nbytes + sarena.nbytes
            for e in range(E):
                ew = self._generate(layer, e)
                wo, so = e * per_w, e * per_s
                entry = {}
                for p in PROJS:
                    w, sc = ew[p]
                    hw = warena[wo: wo + wbytes[p]].view(torch.float8_e4m3fn).view(w.shape)
                    hs = sarena[so: so + sc.numel()].view(sc.shape)
                    hw.copy_(w)
                    hs.copy_(sc)
                    wo += wbytes[p]
                    so += sc.numel()
                    entry[p] = {"weight": hw, "weight_scale_inv": hs}
                self.expert_cache.put(layer, e, entry)
        return total

    def host_expert_pointers(self, layer: int) -> list[int] | None:
        """Host addresses of every routed expert's six tensors (w_gate,
        s_gate, w_up, s_up, w_down, s_down) when all of them sit in pinned
        host memory (after ``preload_host``), else None. The device-side slot
        cache reads experts from there."""
        out = []
        for e in range(self.config.n_routed_experts):
            ent = self.expert_cache.peek(layer, e)
            if ent is None:
                return None
            for p in PROJS:
                w, sc = ent[p]["weight"], ent[p]["weight_scale_inv"]
                if not (w.is_pinned() and sc.is_pinned()):
                    return None
                out += [w.data_ptr(), sc.data_ptr()]
        return out

    def device_expert(self, layer: int, e: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        """Expert ``e`` on the store's device (same bytes as ``get_expert``)."""
        return {p: (w.to(self.device), s.to(self.device)) for p, (w, s) in self._generate(layer, e).items()}

    def fill_bank(self, layer: int, bank, experts=None) -> None:
        """Write the shared expert and `experts` (default: all) into a device
        ``LayerBank``. With ``gen_device="cuda"`` they are generated on the GPU
        by the CUDA generator (fast, but different values from the CPU
        generator that the oracle uses); with ``"cpu"`` they are the same bytes
        ``layer(l).expert(e)`` returns."""
        experts = range(self.config.n_routed_experts) if experts is None else experts
        for e in [SHARED, *experts]:
            bank.write_slot(bank.assign(0 if e == SHARED else e + 1), self.device_expert(layer, e))
