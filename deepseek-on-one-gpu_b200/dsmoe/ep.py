"""Expert parallelism for the MoE block (no counterpart in the single-GPU
reference; the same arithmetic as ``inference/forward.py:112-153``).

W ranks, rank r owns routed experts ``[r*El, (r+1)*El)`` (``El = E / W``), or
the experts an expert placement gives it (``EPLayer.set_placement``,
``balanced_placement`` for skewed routing); the gate and the shared expert are
replicated, tokens stay on their rank. One
layer step (``EPLayer.forward``):

  1. route the rank's tokens (``dsmoe_route``);
  2. ``dsmoe_ep_dispatch``: one send row per (token, owning rank), grouped by
     destination, with the token's local expert ids and weights;
  3. exchange counts, then rows and routing lists (all-to-all);
  4. ``dsmoe_moe_local``: grouped FP8 GEMMs over the rank's experts for the
     received rows, one pre-reduced bf16 row per received row;
  5. exchange the partial rows back (all-to-all, reversed splits);
  6. shared expert on the rank's own tokens (``dsmoe_expert_ffn``) and
     ``dsmoe_ep_combine``: ``out = bf16(shared + bf16(scale * sum_ranks))``.

The exchange is a small interface so the same step runs over
``torch.distributed`` (NCCL between GPUs, Gloo on CPU for the bookkeeping
tests) or over an in-process emulation of W ranks on one GPU.

Overlap (CUDA tensors, ``EPLayer.overlap``, the default): the count and row
exchanges run on a side stream; the shared expert, which needs no exchange,
is queued on the compute stream right after the packing, so it runs while
the counts make their device->host trip and the rows travel. With
``chunks=C`` > 1 the tokens are routed once and packed in C chunks under one
count exchange; the expert GEMMs of a chunk then run while the next chunk's
rows or the previous chunk's partials travel (each chunk re-reads the rank's
expert weights, so this pays only where the exchange is long next to the
GEMMs). While they overlap an exchange the grouped GEMMs leave ``sm_reserve``
SMs free (``dsmoe_set_gemm_sm_limit``) so that the collective's kernels are
not queued behind the persistent GEMM grid. Per token the arithmetic is the
same in every mode.

Peer-memory exchange (``EPLayer.peer`` set, ``PeerBuffers``): no NCCL
all-to-all. Every rank maps the other ranks' receive and return buffers
(CUDA IPC); ``dsmoe_ep_push`` writes each token row straight into its
destination rank's receive buffer, and the combine of ``dsmoe_moe_local_peer``
writes each partial row straight into its origin rank's return buffer. Only
the per-rank counts are gathered (NCCL all-gather of W ints) and two tiny
all-reduces act as stream-ordered barriers between the writes and the reads.
The host never reads a count: the rows a rank receives are summed from the
gathered counts on the device, and the workspace is sized once for
``world * cap`` rows. The pushes run on a side stream on ``2 * push_sms``
CTAs while the shared expert's GEMMs leave ``push_sms`` SMs free.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_handle
from .gpu_transfer import LayerBank
from .ops import expert_ffn, route
from .synthetic import PROJS


class DistExchange:
    """All-to-all over a torch.distributed process group. The per-peer row
    counts cross the device->host boundary once per exchange (NCCL needs the
    split sizes on the host)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)

    def counts(self, send_counts: torch.Tensor) -> tuple[list[int], list[int]]:
        recv = torch.empty_like(send_counts)
        self.dist.all_to_all_single(recv, send_counts, group=self.group)
        both = torch.cat([send_counts, recv]).tolist()
        return both[: self.world], both[self.world:]

    def counts_chunks(self, counts_wc: torch.Tensor) -> tuple[list[list[int]], list[list[int]]]:
        """One exchange for C chunks. ``counts_wc`` [W, C] int32: rows this
        rank sends to rank d in chunk c. Returns per chunk the send splits
        and the receive splits (by source rank)."""
        W, C = counts_wc.shape
        send = counts_wc.contiguous().reshape(-1)
        recv = torch.empty_like(send)
        self.dist.all_to_all_single(recv, send, group=self.group)
        both = torch.cat([send, recv]).tolist()
        s, r = both[: W * C], both[W * C:]
        return ([[s[d * C + c] for d in range(W)] for c in range(C)],
                [[r[q * C + c] for q in range(W)] for c in range(C)])

    def rows(self, send: torch.Tensor, send_splits: list[int], recv_splits: list[int]) -> torch.Tensor:
        out = send.new_empty((sum(recv_splits),) + tuple(send.shape[1:]))
        self.dist.all_to_all_single(out, send[: sum(send_splits)].contiguous(), output_split_sizes=recv_splits,
                                    input_split_sizes=send_splits, group=self.group)
        return out


def _device_view(addr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor over ``nbytes`` of device memory at ``addr`` (memory this
    module owns; the tensor does not free it)."""

    class _Arr:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (addr, False), "version": 3}

    return torch.as_tensor(_Arr(), device=device)


class PeerBuffers:
    """Receive and return buffers of one expert-parallel layer, mapped by every
    rank of the group: receive rows [world * cap][H] bf16, receive routing
    metadata (``dsmoe_ep_meta_bytes``), return rows [world * cap][H] bf16.
    Allocated once (``dsmoe_ipc_alloc``), handles exchanged with an
    all-gather, peers' buffers mapped with ``dsmoe_ipc_open``; ``tables[name]``
    holds the W buffer addresses (in this process) on the device."""

    NAMES = ("x", "meta", "back")

    def __init__(self, world: int, rank: int, cap: int, hidden: int, top_k: int, device, group=None):
        import torch.distributed as dist

        self.world, self.rank, self.cap, self.device = world, rank, cap, torch.device(device)
        self.nbytes = {"x": world * cap * hidden * 2, "meta": lib().dsmoe_ep_meta_bytes(world, cap, top_k),
                       "back": world * cap * hidden * 2}
        self.own, handles = {}, {}
        with torch.cuda.device(self.device):
            for name in self.NAMES:
                ptr_, h = ctypes.c_void_p(), (ctypes.c_char * 64)()
                check(lib().dsmoe_ipc_alloc(self.nbytes[name], ctypes.byref(ptr_), h), "dsmoe_ipc_alloc")
                self.own[name] = ptr_.value
                handles[name] = bytes(h)
            everyone = [None] * world
            dist.all_gather_object(everyone, handles, group=group)
            self.addr = {name: [0] * world for name in self.NAMES}
            self._opened = []
            for r in range(world):
                for name in self.NAMES:
                    if r == rank:
                        a = self.own[name]
                    else:
                        ptr_ = ctypes.c_void_p()
                        h = (ctypes.c_char * 64).from_buffer_copy(everyone[r][name])
                        check(lib().dsmoe_ipc_open(h, ctypes.byref(ptr_)), "dsmoe_ipc_open")
                        a = ptr_.value
                        self._opened.append(a)
                    self.addr[name][r] = a
        self.tables = {n: torch.tensor(self.addr[n], dtype=torch.int64, device=self.device) for n in self.NAMES}
        self.views = {n: _device_view(self.own[n], self.nbytes[n], self.device) for n in self.NAMES}
        self.group = group
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (a collective: every
        rank calls it, after its last step)."""
        import torch.distributed as dist

        if not self.own:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for a in self._opened:
                lib().dsmoe_ipc_close(ctypes.c_void_p(a))
            dist.barrier(group=self.group)
            for a in self.own.values():
                lib().dsmoe_ipc_free(ctypes.c_void_p(a))
        self.own, self._opened, self.views = {}, [], {}


class LocalExchange:
    """The exchange of a one-rank group: every row stays on the rank. Lets the
    chunked, two-stream step run (and be tested) on a single GPU."""

    world = 1

    def counts(self, send_counts: torch.Tensor) -> tuple[list[int], list[int]]:
        c = send_counts.tolist()
        return c, c

    def counts_chunks(self, counts_wc: torch.Tensor) -> tuple[list[list[int]], list[list[int]]]:
        c = counts_wc.t().tolist()
        return c, [list(x) for x in c]

    def rows(self, send: torch.Tensor, send_splits: list[int], recv_splits: list[int]) -> torch.Tensor:
        return send[: sum(send_splits)].clone()


def local_config(config, world: int):
    """Config of one rank's share: El = E / world routed experts."""
    E = config.n_routed_experts
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    El = E // world
    ng = max(1, El // 32)
    if El % 32:
        raise ValueError("experts per rank must be a multiple of 32")
    return config.with_(n_routed_experts=El, n_group=ng, topk_group=ng)


def balanced_placement(loads, world: int) -> list[int]:
    """Expert placement for skewed routing: ``loads[e]`` is expert e's expected
    number of (token, expert) pairs (e.g. counted over a calibration batch).
    Experts are taken in decreasing load and each goes to the rank with the
    smallest load so far among ranks with a free slot (E / world slots each):
    the longest-processing-time rule. Returns ``placement`` with
    ``placement[e] = rank * (E / world) + slot``, a permutation of range(E)."""
    loads = [float(v) for v in loads]
    E = len(loads)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    El = E // world
    rank_load = [0.0] * world
    used = [0] * world
    placement = [0] * E
    for e in sorted(range(E), key=lambda i: (-loads[i], i)):
        r = min((q for q in range(world) if used[q] < El), key=lambda q: (rank_load[q], q))
        placement[e] = r * El + used[r]
        used[r] += 1
        rank_load[r] += loads[e]
    return placement


PEER_PHASES = ("route_plan_count_gather", "push_beside_shared_expert", "barrier_rows_landed",
               "expert_gemms_partials_return", "barrier_partials_back", "combine")


class EPLayer:
    """One MoE layer, expert-parallel. ``expert_source(layer, e)`` returns expert
    ``e``'s ``{proj: (weight, scale)}`` (any device); by default the weight
    store's ``get_expert``. ``placement`` (optional, every rank the same):
    expert e lives on rank ``placement[e] // El`` in its slot
    ``placement[e] % El``; by default rank r owns experts ``[r*El, (r+1)*El)``.
    The router's expert ids are relabelled through it on the device, so the
    exchange kernels see contiguous ranges either way."""

    def __init__(self, config, weight_store, device, layer: int, world: int, rank: int, exchange=None,
                 expert_source=None, placement=None):
        self.config = config
        self.store = weight_store
        self.device = torch.device(device)
        self.layer = layer
        self.world, self.rank = world, rank
        self.exchange = exchange
        self.lcfg = local_config(config, world)
        self.El = self.lcfg.n_routed_experts
        self._src = expert_source or weight_store.get_expert
        self.bank = LayerBank(self.lcfg, self.El + 1, self.device)
        self.bank.write_slot(self.bank.assign(0), weight_store.get_shared_expert_weights(layer))
        self.relabel = None  # device int64 [E]: router expert id -> rank * El + slot
        self.set_placement(placement)
        self.shared = {p: (self.bank.w[p][0], self.bank.s[p][0]) for p in PROJS}
        self._ws = torch.zeros(0, dtype=torch.uint8, device=self.device)
        self._comm = None  # side stream of the overlapped step
        self.peer: PeerBuffers | None = None  # set by use_peer_memory()
        self._flag = None
        self.overlap = True  # CUDA tensors: exchange on a side stream, shared expert while rows travel
        self.sm_reserve = 0  # SMs left to the collectives while GEMMs and all-to-alls overlap
        # peer-memory step: SMs the shared expert leaves to the row pushes (0 =
        # no overlap). The rows a rank sends to other GPUs grow with the world
        # size (at T tokens: ~T rows at 2 ranks, ~2.2 T at 4, ~3.5 T at 8) and
        # SM-issued stores to a peer reach ~9 GB/s per CTA up to ~690 GB/s, so
        # the share grows with it until pushes and shared expert take about
        # equally long.
        self.push_sms = {1: 16, 2: 8, 4: 14}.get(world, min(32, 2 + 5 * world // 2))
        self._push_status = None
        # Optional timing of the peer-memory step (CUDA events recorded on the
        # compute stream): phase_events[0..6] at the PEER_PHASES boundaries,
        # lib_events (7) handed to the library around the rank's expert GEMMs.
        self.phase_events = None
        self.lib_events = None
        self.last_counts_all = None

    def set_placement(self, placement=None) -> None:
        """(Re)load this rank's experts for ``placement`` (see the class
        docstring; None = contiguous ranges). Every rank must use the same."""
        E, El = self.config.n_routed_experts, self.El
        if placement is None:
            owned = [self.rank * El + el for el in range(El)]
            self.relabel = None
        else:
            placement = [int(v) for v in placement]
            if sorted(placement) != list(range(E)):
                raise ValueError("placement must be a permutation of the expert ids")
            inv = [0] * E
            for e, pos in enumerate(placement):
                inv[pos] = e
            owned = [inv[self.rank * El + el] for el in range(El)]
            self.relabel = torch.tensor(placement, dtype=torch.int64, device=self.device)
        for el, e in enumerate(owned):
            # local expert el is group el + 1 of the rank's bank (group 0: shared)
            self.bank.write_slot(self.bank.assign(el + 1), self._src(self.layer, e))
        self.bank.sync_table(non_blocking=False)
        self.owned = owned

    # -------------------------------------------------------------- phases
    def route(self, x: torch.Tensor):
        cfg = self.config
        bias = self.store.get_gate_bias(self.layer) if getattr(cfg, "router_mode", "ref") == "v3" else None
        idx, w = route(x, self.store.get_gate_weight(self.layer), cfg, score_bias=bias)
        if self.relabel is not None:
            idx = self.relabel[idx]  # rank * El + slot: contiguous ranges for the exchange kernels
        return idx, w

    def dispatch(self, x: torch.Tensor):
        """Route and pack. Returns (counts[W] int32 device, tok_rows, send_x, send_meta)."""
        idx, w = self.route(x)
        return self.pack(x, idx, w)

    def pack(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor):
        """Pack routed tokens for the exchange (``dsmoe_ep_dispatch``)."""
        cfg = self.config
        T, H = x.shape
        K = cfg.num_experts_per_tok
        idx, w = idx.contiguous(), w.contiguous()
        cap = max(1, T * min(K, self.world))
        dev = x.device
        counts = torch.empty(self.world, dtype=torch.int32, device=dev)
        tok_rows = torch.empty(T, self.world, dtype=torch.int32, device=dev)
        send_tok = torch.empty(cap, dtype=torch.int32, device=dev)
        meta = torch.empty(cap, 2 * K, dtype=torch.int32, device=dev)  # [local idx x K | weights (fp32 bits) x K]
        send_idx = torch.empty(cap, K, dtype=torch.int32, device=dev)
        send_w = torch.empty(cap, K, dtype=torch.float32, device=dev)
        send_x = torch.empty(cap, H, dtype=torch.bfloat16, device=dev)
        check(lib().dsmoe_ep_dispatch(ptr(idx), ptr(w), ptr(x), T, K, H, self.world, self.El, ptr(counts),
                                      ptr(tok_rows), ptr(send_tok), ptr(send_idx), ptr(send_w), ptr(send_x),
                                      stream_handle(dev)), "dsmoe_ep_dispatch")
        meta[:, :K] = send_idx
        meta[:, K:] = send_w.view(torch.int32)
        return counts, tok_rows, send_x, meta

    def compute(self, recv_x: torch.Tensor, recv_meta: torch.Tensor) -> torch.Tensor:
        """The rank's experts on the received rows -> one partial row each."""
        R, H = recv_x.shape
        K = self.config.num_experts_per_tok
        out = torch.empty(R, H, dtype=torch.bfloat16, device=recv_x.device)
        if R == 0:
            return out
        lidx = recv_meta[:, :K].contiguous()
        lw = recv_meta[:, K:].contiguous().view(torch.float32)
        cfg = _lib.moe_config(self.lcfg)
        need = lib().dsmoe_moe_local_workspace_size(cfg, R)
        if self._ws.numel() < need:
            self._ws = torch.zeros(int(need * 1.25) + 4096, dtype=torch.uint8, device=recv_x.device)
        b = self.bank
        lw_struct = _lib.LayerWeights(
            gate_weight=None, score_bias=None, n_slots=b.n_slots,
            w_gate=ptr(b.w["gate_proj"]), s_gate=ptr(b.s["gate_proj"]), w_up=ptr(b.w["up_proj"]),
            s_up=ptr(b.s["up_proj"]), w_down=ptr(b.w["down_proj"]), s_down=ptr(b.s["down_proj"]),
            slot_of_expert=ptr(b.slot_of))
        if self.lib_events:
            _lib.set_profile_events(self.lib_events)
        try:
            check(lib().dsmoe_moe_local(cfg, lw_struct, ptr(recv_x), R, ptr(lidx), ptr(lw), ptr(out), ptr(self._ws),
                                        self._ws.numel(), stream_handle(recv_x.device)), "dsmoe_moe_local")
        finally:
            if self.lib_events:
                _lib.set_profile_events(None)
        return out

    def shared_ffn(self, x: torch.Tensor) -> torch.Tensor:
        """The shared expert on the rank's own tokens (needs no exchange)."""
        return expert_ffn(x, self.shared)

    def combine(self, shared: torch.Tensor, back: torch.Tensor, tok_rows: torch.Tensor) -> torch.Tensor:
        """``out = bf16(shared + bf16(scale * sum of the returned partials))``."""
        T, H = shared.shape
        out = torch.empty_like(shared)
        scale = 1.0 if getattr(self.config, "router_mode", "ref") == "v3" else float(self.config.routed_scaling_factor)
        check(lib().dsmoe_ep_combine(ptr(back) if back.numel() else None, ptr(tok_rows), T, self.world, H,
                                     ptr(shared), scale, ptr(out), stream_handle(shared.device)), "dsmoe_ep_combine")
        return out

    def finish(self, x: torch.Tensor, back: torch.Tensor, tok_rows: torch.Tensor) -> torch.Tensor:
        """Shared expert on the rank's tokens + sum of the returned partials."""
        return self.combine(self.shared_ffn(x), back, tok_rows)

    def use_peer_memory(self, cap: int, group=None) -> None:
        """Exchange through mapped peer buffers sized for up to ``cap`` tokens
        per rank and step (a collective: every rank calls it)."""
        self.peer = PeerBuffers(self.world, self.rank, cap, self.config.hidden_size, self.config.num_experts_per_tok,
                                self.device, group)

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _barrier(self, dev):
        """Stream-ordered barrier: completes on every rank only after every rank's
        earlier kernels on its stream have completed."""
        if self._flag is None:
            self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self.exchange.dist.all_reduce(self._flag, group=self.exchange.group)

    def _peer_workspace(self, dev):
        """Workspace of the peer-memory step, sized once for the most rows a
        rank can receive (world * cap), so that the step never needs the
        received-row count on the host."""
        pb = self.peer
        need = lib().dsmoe_moe_local_workspace_size(_lib.moe_config(self.lcfg), self.world * pb.cap)
        if self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        if self._push_status is None:
            self._push_status = torch.zeros(1, dtype=torch.int32, device=dev)
        return self._ws

    def push_status(self) -> int:
        """The push kernel's device error word (read and cleared; a host sync:
        diagnostics only). Non-zero: gathered counts that did not fit the
        receive buffers."""
        if self._push_status is None:
            return 0
        v = int(self._push_status.item())
        self._push_status.zero_()
        return v

    def _forward_peer(self, x: torch.Tensor) -> torch.Tensor:
        cfg, pb = self.config, self.peer
        T, H = x.shape
        K, W, dev = cfg.num_experts_per_tok, self.world, x.device
        if T > pb.cap:
            raise ValueError(f"{T} tokens exceed the peer buffers' capacity of {pb.cap}")
        ws = self._peer_workspace(dev)
        ev = self.phase_events
        cs = torch.cuda.current_stream(dev)
        if ev:
            ev[0].record(cs)
        idx, w = self.route(x)
        counts = torch.empty(W, dtype=torch.int32, device=dev)
        tok_rows = torch.empty(T, W, dtype=torch.int32, device=dev)
        n_send = max(1, T * min(K, W))
        send_tok = torch.empty(n_send, dtype=torch.int32, device=dev)
        send_idx = torch.empty(n_send, K, dtype=torch.int32, device=dev)
        send_w = torch.empty(n_send, K, dtype=torch.float32, device=dev)
        check(lib().dsmoe_ep_plan(ptr(idx), ptr(w), T, K, W, self.El, ptr(counts), ptr(tok_rows), ptr(send_tok),
                                  ptr(send_idx), ptr(send_w), stream_handle(dev)), "dsmoe_ep_plan")
        counts_all = torch.empty(W * W, dtype=torch.int32, device=dev)  # row s: what rank s sends to each rank
        self.exchange.dist.all_gather_into_tensor(counts_all, counts, group=self.exchange.group)
        self.last_counts_all = counts_all
        if ev:
            ev[1].record(cs)
        overlap = self.overlap and self.push_sms > 0
        push_stream = cs
        if overlap:
            # The pushes travel over NVLink on a side stream, on a capped grid,
            # while the shared expert (which needs no exchange) computes on the
            # SMs its GEMMs leave free of them.
            if self._comm is None:
                self._comm = torch.cuda.Stream(device=dev)
            push_stream = self._comm
            ready = torch.cuda.Event()
            ready.record(cs)
            push_stream.wait_event(ready)
            for t_ in (x, counts_all, send_tok, send_idx, send_w, tok_rows):
                t_.record_stream(push_stream)
        check(lib().dsmoe_ep_push(ptr(x), T, K, H, W, self.rank, pb.cap, ptr(counts_all), ptr(send_tok),
                                  ptr(send_idx), ptr(send_w), ptr(tok_rows), ptr(pb.tables["x"]),
                                  ptr(pb.tables["meta"]), ptr(self._push_status),
                                  2 * self.push_sms if overlap else 0, push_stream.cuda_stream), "dsmoe_ep_push")
        if overlap:
            n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
            try:
                _lib.set_gemm_sm_limit(max(1, n_sm - self.push_sms))
                shared = self.shared_ffn(x)
            finally:
                _lib.set_gemm_sm_limit(0)
            pushed = torch.cuda.Event()
            pushed.record(push_stream)
            cs.wait_event(pushed)
        else:
            shared = self.shared_ffn(x)
        if ev:
            ev[2].record(cs)
        self._barrier(dev)  # every rank's rows have landed
        if ev:
            ev[3].record(cs)
        lcfg = _lib.moe_config(self.lcfg)
        b = self.bank
        lw = _lib.LayerWeights(
            gate_weight=None, score_bias=None, n_slots=b.n_slots,
            w_gate=ptr(b.w["gate_proj"]), s_gate=ptr(b.s["gate_proj"]), w_up=ptr(b.w["up_proj"]),
            s_up=ptr(b.s["up_proj"]), w_down=ptr(b.w["down_proj"]), s_down=ptr(b.s["down_proj"]),
            slot_of_expert=ptr(b.slot_of))
        # rows received are counted on the device from counts_all; W * cap bounds them
        if self.lib_events:
            _lib.set_profile_events(self.lib_events)
        try:
            check(lib().dsmoe_moe_local_peer(lcfg, lw, pb.own["x"], W * pb.cap, pb.own["meta"], W, self.rank,
                                             pb.cap, ptr(pb.tables["back"]), ptr(counts_all), ptr(ws), ws.numel(),
                                             stream_handle(dev)), "dsmoe_moe_local_peer")
        finally:
            if self.lib_events:
                _lib.set_profile_events(None)
        if ev:
            ev[4].record(cs)
        self._barrier(dev)  # every partial is back at its origin
        if ev:
            ev[5].record(cs)
        back = pb.views["back"].view(torch.bfloat16).view(W * pb.cap, H)
        out = self.combine(shared, back, tok_rows)
        if ev:
            ev[6].record(cs)
        return out

    def received_pairs(self) -> tuple[int, int]:
        """(rows, (row, local expert) pairs) this rank received in the last
        peer-memory step (a host read: diagnostics only)."""
        W, K = self.world, self.config.num_experts_per_tok
        rows = int(self.last_counts_all.view(W, W)[:, self.rank].sum().item())
        meta = self.peer.views["meta"].view(torch.int32)[: W * self.peer.cap * K].view(W * self.peer.cap, K)
        return rows, int((meta[:rows] >= 0).sum().item())

    def forward(self, x: torch.Tensor, chunks: int = 1) -> torch.Tensor:
        """One expert-parallel MoE step for this rank's tokens ``x`` [T, H] bf16.
        With ``overlap`` (default, CUDA tensors) the exchange runs on a side
        stream while the shared expert runs; ``chunks`` > 1 also overlaps the
        all-to-alls of one chunk with the expert GEMMs of another (each chunk
        re-reads the rank's expert weights)."""
        shape = x.shape
        x = x.reshape(-1, shape[-1]).contiguous()
        if self.peer is not None:
            return self._forward_peer(x).view(shape)
        if self.overlap and x.is_cuda and x.shape[0] >= chunks:
            return self._forward_overlapped(x, chunks).view(shape)
        counts, tok_rows, send_x, meta = self.dispatch(x)
        send_splits, recv_splits = self.exchange.counts(counts)
        recv_x = self.exchange.rows(send_x, send_splits, recv_splits)
        recv_meta = self.exchange.rows(meta, send_splits, recv_splits)
        part = self.compute(recv_x, recv_meta)
        back = self.exchange.rows(part, recv_splits, send_splits)
        return self.finish(x, back, tok_rows).view(shape)


    def _forward_overlapped(self, x: torch.Tensor, C: int) -> torch.Tensor:
        T, H = x.shape
        dev = x.device
        cs = torch.cuda.current_stream(dev)
        if self._comm is None:
            self._comm = torch.cuda.Stream(device=dev)
        comm = self._comm
        n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
        limit = max(1, n_sm - self.sm_reserve) if self.sm_reserve > 0 else 0
        bounds = [T * c // C for c in range(C + 1)]
        idx, w = self.route(x)
        packs = [self.pack(x[bounds[c]:bounds[c + 1]], idx[bounds[c]:bounds[c + 1]], w[bounds[c]:bounds[c + 1]])
                 for c in range(C)]
        counts_wc = torch.stack([p[0] for p in packs], dim=1)
        packed = torch.cuda.Event()
        packed.record(cs)
        # The shared expert needs no exchange: it is queued first on the
        # compute stream and runs while the counts and rows travel.
        try:
            _lib.set_gemm_sm_limit(limit)
            shared = self.shared_ffn(x)
        finally:
            _lib.set_gemm_sm_limit(0)
        comm.wait_event(packed)
        arrived = []
        with torch.cuda.stream(comm):
            counts_wc.record_stream(comm)
            send_sp, recv_sp = self.exchange.counts_chunks(counts_wc)  # the host waits for the side stream only
            for c, (_, _, send_x, meta) in enumerate(packs):
                send_x.record_stream(comm)
                meta.record_stream(comm)
                rx = self.exchange.rows(send_x, send_sp[c], recv_sp[c])
                rm = self.exchange.rows(meta, send_sp[c], recv_sp[c])
                rx.record_stream(cs)
                rm.record_stream(cs)
                ev = torch.cuda.Event()
                ev.record(comm)
                arrived.append((rx, rm, ev))
        back = []
        for c, (rx, rm, ev) in enumerate(arrived):
            cs.wait_event(ev)
            try:
                # chunks before the last overlap the next chunk's traffic
                _lib.set_gemm_sm_limit(limit if c < C - 1 else 0)
                part = self.compute(rx, rm)
            finally:
                _lib.set_gemm_sm_limit(0)
            done = torch.cuda.Event()
            done.record(cs)
            comm.wait_event(done)
            with torch.cuda.stream(comm):
                part.record_stream(comm)
                b = self.exchange.rows(part, recv_sp[c], send_sp[c])
                b.record_stream(cs)
                ev_b = torch.cuda.Event()
                ev_b.record(comm)
            back.append((b, ev_b))
        outs = []
        for c, (b, ev_b) in enumerate(back):
            cs.wait_event(ev_b)
            t0, t1 = bounds[c], bounds[c + 1]
            outs.append(self.combine(shared[t0:t1], b, packs[c][1]))
        return outs[0] if C == 1 else torch.cat(outs)


def emulate_step(layers: list[EPLayer], xs: list[torch.Tensor]) -> list[torch.Tensor]:
    """Run one expert-parallel step of W ranks in one process (one device):
    the all-to-alls become slicing and concatenation. For tests and
    single-GPU measurements of the per-rank kernels."""
    W = len(layers)
    plans = [layers[r].dispatch(xs[r]) for r in range(W)]
    counts = [p[0].tolist() for p in plans]  # counts[src][dst]
    # rows src -> dst, in the order an all-to-all delivers them (by source rank)
    starts = [[sum(counts[s][:d]) for d in range(W)] for s in range(W)]
    recv_x, recv_m = [], []
    for d in range(W):
        recv_x.append(torch.cat([plans[s][2][starts[s][d]: starts[s][d] + counts[s][d]] for s in range(W)]))
        recv_m.append(torch.cat([plans[s][3][starts[s][d]: starts[s][d] + counts[s][d]] for s in range(W)]))
    parts = [layers[d].compute(recv_x[d], recv_m[d]) for d in range(W)]
    outs = []
    for s in range(W):
        back = []
        for d in range(W):
            off = sum(counts[q][d] for q in range(s))
            back.append(parts[d][off: off + counts[s][d]])
        outs.append(layers[s].finish(xs[s], torch.cat(back), plans[s][1]))
    return outs
