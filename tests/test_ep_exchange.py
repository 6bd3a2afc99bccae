"""The expert-parallel exchange (dsmoe.ep.DistExchange) on CPU with two Gloo
ranks: count exchange (one chunk and several), variable-split all-to-all
there and back."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "deepseek-on-one-gpu_b200"))
    from dsmoe.ep import DistExchange
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        ex = DistExchange()
        # rank r sends (r + d + 1) rows to rank d, each row = [src, dst, i] * 4
        send_counts = torch.tensor([rank + d + 1 for d in range(world)], dtype=torch.int32)
        rows = [torch.tensor([rank, d, i, 7] * 4, dtype=torch.int32) for d in range(world)
                for i in range(rank + d + 1)]
        send = torch.stack(rows + [torch.full((16,), -9, dtype=torch.int32)])  # one unused capacity row
        sc, rc = ex.counts(send_counts)
        assert sc == [rank + d + 1 for d in range(world)]
        assert rc == [s + rank + 1 for s in range(world)]
        recv = ex.rows(send, sc, rc)
        off = 0
        for s in range(world):
            for i in range(rc[s]):
                assert recv[off].tolist()[:3] == [s, rank, i]
                off += 1
        back = ex.rows(recv * 2, rc, sc)  # the partial rows go back in the senders' order
        assert torch.equal(back, send[: sum(sc)] * 2)
        # one count exchange for 3 chunks: rank r sends (10 r + 3 d + c) rows to d in chunk c
        C = 3
        cwc = torch.tensor([[10 * rank + 3 * d + c for c in range(C)] for d in range(world)], dtype=torch.int32)
        scc, rcc = ex.counts_chunks(cwc)
        assert scc == [[10 * rank + 3 * d + c for d in range(world)] for c in range(C)]
        assert rcc == [[10 * s + 3 * rank + c for s in range(world)] for c in range(C)]
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_dist_exchange_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}


def test_balanced_placement_is_a_permutation_with_equal_slots_and_spreads_load():
    """balanced_placement (longest-processing-time rule): a permutation of the
    expert ids, E / W experts per rank, and under Zipf-skewed loads the busiest
    rank within the rule's bound (mean + the largest single load)."""
    import random

    from dsmoe.ep import balanced_placement

    E = 256
    for W in (2, 4, 8):
        rng = random.Random(W)
        loads = [1.0 / (i + 1) ** 1.1 for i in range(E)]
        rng.shuffle(loads)
        p = balanced_placement(loads, W)
        assert sorted(p) == list(range(E))
        El = E // W
        per_rank = [0] * W
        load = [0.0] * W
        for e, pos in enumerate(p):
            per_rank[pos // El] += 1
            load[pos // El] += loads[e]
        assert per_rank == [El] * W
        mean = sum(loads) / W
        assert max(load) <= mean + max(loads) + 1e-12
        # contiguous ranges over the same (shuffled) loads are worse or equal
        contiguous = [sum(loads[r * El:(r + 1) * El]) for r in range(W)]
        assert max(load) <= max(contiguous) + 1e-12
    # uniform loads keep every rank equal
    p = balanced_placement([1.0] * E, 8)
    assert sorted(p) == list(range(E))
