#!/usr/bin/env python
"""Benchmark: DeepSeek-R1 MoE-layer tokens/s on B200 (libdsmoe).

Default workload (N=1): one MoE layer at the DeepSeek-R1 shape, prefill
T=4096 tokens, all 256 routed experts + the shared expert resident in HBM
(11.3 GB FP8), seeded synthetic weights and activations (no checkpoint, no
dataset). One "step" = one full ``moe_block`` forward.

Printed JSON keys (one line, rank 0):
  value      tokens/s over all ranks, inputs resident in HBM, CUDA-event timed
  e2e        same metric through ``moe_block`` with the input copied from pinned
             host memory and the output read back every step
  roofline   the dominant kernel (grouped gate/up GEMM): algorithmic bytes (or
             FLOPs, whichever bound its arithmetic intensity sets) per launch /
             its event-timed duration, against the measured peak; the compute
             roof is the measured sustained bf16 GEMM rate, because the kernel
             runs two FP8 MMAs (hi and lo terms) per useful multiply-add
  cpu_baseline  the CPU oracle (a restatement of the reference's per-token
             moe_block) timed on a bounded token sample on this host
  widened_rows  RMSNorm, the MoE layer's FFN half, the dense FFN, the expert
             loader and next-token sampling, measured on the same GPU
  decode_rows   the same layer at decode batches T=8 and T=64 (tokens/s and
             the GEMMs' fraction of measured HBM bandwidth)
  streaming_config5  32 steps of config 5 (B=1 decode through 8 layers,
             experts in pinned host memory): tokens/s, host-link GB/s, slot
             hit rate
  stages_ms  per-kernel CUDA-event times, recorded by the library at its
             stage boundaries inside the timed steps
  clocks     nvidia-smi samples inside the timed region, and sm_mhz_device:
             the SMs' own cycle counters over the timed steps (median over
             SMs, dsmoe_clock_probe)
``--impl reference`` times only that CPU path and prints its own line.
With N > 1 (torchrun, one rank per GPU) the step is expert-parallel (config
3: 4096 tokens per rank by default, the N=1 batch, with config 3's 8192
measured in the same run as ``config3_t8192``; each rank owning 256/N experts, token rows and
partial sums exchanged over peer memory; ``--nccl-exchange`` for the NCCL
all-to-all, ``--mode replica`` for independent replicas); weak scaling. When
the step's routing would load the busiest rank more than 1.25x the mean
(config 4's skew), the experts are placed over the ranks by load
(``--ep-placement``); the roofline and stage times are the critical rank's.
"""
from __future__ import annotations

import argparse
from datetime import datetime
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "deepseek-on-one-gpu_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "MoE-layer tokens/s (DeepSeek-R1 FP8 shape) at 1/2/4/8 B200; % of FP8 TC peak"
UNIT = "tokens/s"
H, F, E, TOPK = 7168, 2048, 256, 8
LAYER = 3
FP8_DENSE_NOMINAL_TFLOPS = 4500.0
# DRAM bytes (read + write) per launch of a grouped GEMM, measured by ncu on
# exactly the workload bench.py runs (one-pass capture of
# dram__bytes_read.sum + dram__bytes_write.sum; the profile summaries under
# profiles/ give the command). Keyed (stage, config, tokens per GPU, routed
# experts); a workload without a capture reports traffic null.
MEASURED_DRAM_BYTES: dict[tuple[str, int, int, int], float] = {
    # profiles/grouped_gemm_t4096_dram.md: 8.91 GB read + 0.288 GB written
    ("gate_up", 2, 4096, 256): 8.91e9 + 0.28765e9,
    # same capture: 4.30 GB read + 0.4825 GB written
    ("down", 2, 4096, 256): 4.30e9 + 0.4825e9,
}


def expert_load_rates(cfg, dev, n_experts: int = 16, layer: int = 7) -> dict:
    """Expert disk step (the loader that feeds the pinned expert cache): read n R1-size experts
    from a safetensors file (written just before, so from the page cache)
    into pinned host memory, with the store (packed buffers, native pread
    pool) and with the reference's own steps (safe_open, get_tensor, copy into
    a fresh pinned tensor; oracle/expert_loader.py). Each is timed on its
    second pass, after torch's pinned allocator has warmed up."""
    import tempfile

    from safetensors.torch import save_file

    from dsmoe.safetensors_store import SafetensorsWeightStore
    from dsmoe.synthetic import expert_weights
    from oracle.expert_loader import load_expert, shard_map

    tensors = {}
    for e in range(n_experts):
        for proj, (w, s) in expert_weights(21, layer, e, cfg.hidden_size, cfg.moe_intermediate_size, "cuda").items():
            pre = f"model.layers.{layer}.mlp.experts.{e}.{proj}"
            tensors[pre + ".weight"] = w.cpu()
            tensors[pre + ".weight_scale_inv"] = s.cpu()
    nbytes = sum(t.nbytes for t in tensors.values())
    out = {}
    with tempfile.TemporaryDirectory() as td:
        save_file(tensors, os.path.join(td, "model.safetensors"))
        del tensors
        for rep in range(2):
            store = SafetensorsWeightStore(td, cfg, dev, expert_cache_bytes=1 << 40, threads=16)
            t0 = time.perf_counter()
            got = [store.get_expert(layer, e) for e in range(n_experts)]
            t1 = time.perf_counter()
            del got, store
            k2s = shard_map(td)
            t2 = time.perf_counter()
            ref = [load_expert(td, k2s, layer, e) for e in range(n_experts)]
            t3 = time.perf_counter()
            del ref
        out = {"expert_load_GB_s": nbytes / (t1 - t0) / 1e9, "reference_loader_GB_s": nbytes / (t3 - t2) / 1e9,
               "expert_load_sample": f"{n_experts} R1 experts ({nbytes / 1e9:.2f} GB) from the page cache into "
                                     f"pinned host memory, 16 pread threads"}
    return out


def _torch_sort_sample(logits, temperature: float, top_p: float):
    """The reference's sampling steps (softmax, full sort, cumsum, mask,
    renormalise, multinomial, gather) as plain torch ops on the GPU: the
    comparison point for the device sampler."""
    probs = torch.softmax(logits / temperature, dim=-1)
    sp, si = probs.sort(dim=-1, descending=True)
    cum = sp.cumsum(dim=-1)
    sp[cum - sp > top_p] = 0.0
    sp /= sp.sum(dim=-1, keepdim=True)
    return si.gather(-1, torch.multinomial(sp, num_samples=1)).squeeze(-1)


def sampler_rates(dev, dev_ms) -> dict:
    """Next-token sampling at DeepSeek's vocabulary (129,280 fp32 logits per
    row, T = 0.6, top_p = 0.9): the device sampler (dsmoe.sample) against the
    reference's steps as torch ops, device-timed per call, for 1 and 64 rows."""
    from dsmoe import sample
    from dsmoe.synthetic import logits as make_logits
    out = {}
    for B in (1, 64):
        x = make_logits(40, B, 129280, 3.0, dev)
        out[f"sampler_us_b{B}"] = 1e3 * dev_ms(lambda: sample(x, 0.6, 0.9), n=50)
        out[f"torch_sort_sampler_us_b{B}"] = 1e3 * dev_ms(lambda: _torch_sort_sample(x, 0.6, 0.9), n=50)
    return out


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured")
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self, window: tuple[float, float] | None = None):
        """Median SM clock and the throttle reasons seen; with ``window``
        (host time.time() bounds of the timed region) only samples inside it
        count, if there are any."""
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for row in csv.reader(io.StringIO(out)):
            if len(row) < 10:
                continue
            try:
                ts = datetime.strptime(row[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
                idx = int(row[1])
                rows.append((ts, idx, float(row[2]), float(row[3]),
                             {n for n, v in zip(names, row[6:10]) if v.strip().lower() == "active"}))
            except ValueError:
                continue
        rows = [r for r in rows if r[1] in self.gpus]
        inside = [r for r in rows if window and window[0] <= r[0] <= window[1]]
        use = inside or rows
        if not use:
            return None
        return {"sm_mhz": statistics.median(r[2] for r in use), "sm_max_mhz": max(r[3] for r in use),
                "reasons": sorted(set().union(*(r[4] for r in use))), "samples": len(use),
                "samples_in_timed_region": len(inside)}


def workload_config(args, world: int) -> dict:
    """The ``config`` object of the bench line, shared by both arms so that
    the reference arm reports exactly the workload of this arm."""
    ep = world > 1 and args.mode == "ep"
    T, E_ = args.tokens, args.experts
    if ep:
        workload = (f"1 DeepSeek-R1 MoE layer, expert-parallel over {world} GPUs ({E_ // world} experts per GPU, "
                    f"gate and shared expert replicated), T={T} tokens per GPU, "
                    f"{'NCCL all-to-all' if args.nccl_exchange else 'peer-memory'} dispatch/combine "
                    f"(config {args.config})")
    else:
        workload = (f"1 DeepSeek-R1 MoE layer, prefill T={T} tokens per GPU, {E_}+1 experts resident "
                    f"(config {args.config})" + ("; independent replica per GPU" if world > 1 else ""))
    c = {"workload": workload, "tokens_per_gpu": T, "hidden": H, "moe_intermediate": F, "experts": E_,
         "top_k": TOPK, "router": "v3" if args.config == 4 else "ref", "baseline_config": args.config,
         "l2": "weights 11.3 GB per step > 126 MB L2 (no flush needed)",
         "parallelism": (f"ep{world}" if ep else f"replica x{world}") if world > 1 else "single GPU"}
    if ep:
        c.update({"ep_exchange": "NCCL all-to-all" if args.nccl_exchange else "peer memory (IPC-mapped buffers)",
                  "ep_overlap": not args.no_overlap, "ep_chunks": args.chunks, "ep_sm_reserve": args.sm_reserve})
    return c


def time_cpu_reference(x_sample, gate, get_expert, shared, steps: int, warmup: int, bias=None):
    """The reference's per-token ``moe_block`` (restated step by step by the
    oracle, ``inference/forward.py:112-153``) on the host cores: every step
    runs the same token sample through it. The experts the sample routes to
    are fetched before the timed region (the reference's weight store holds
    them in its pinned host cache). Returns (tokens/s, seconds timed)."""
    from oracle import moe_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    n = x_sample.shape[0]
    if bias is None:
        route_fn, scale = None, 2.5
        idx, _ = O.route_ref(x_sample, gate)
    else:
        def route_fn(h):
            return O.route_v3(h, gate, bias)
        scale = 1.0  # the bias-corrected router's weights carry the factor
        idx, _ = O.route_v3(x_sample, gate, bias)
    experts = {e: get_expert(e) for e in sorted(set(idx.reshape(-1).tolist()))}
    xs = x_sample.view(1, n, -1)
    for _ in range(warmup):
        O.moe_block_literal(xs, gate, experts.__getitem__, shared, route_fn=route_fn, routed_scaling_factor=scale)
    t0 = time.perf_counter()
    for _ in range(steps):
        O.moe_block_literal(xs, gate, experts.__getitem__, shared, route_fn=route_fn, routed_scaling_factor=scale)
    dt = time.perf_counter() - t0
    return n * steps / dt, dt


def run_reference(args, rank, world):
    """``--impl reference``: the reference's CPU path on this host's cores, on
    this arm's workload. Each step is a bounded sample of it: the first
    ``--ref-tokens-per-step`` tokens of rank 0's batch through the per-token
    loop; the loop's cost is linear in the token count, so tokens/s
    extrapolates to the whole batch."""
    if rank != 0:
        return
    from dsmoe.synthetic import SyntheticLayer, activations

    T, n = args.tokens, args.ref_tokens_per_step
    seed = {2: 1, 3: 2, 4: 3}.get(args.config, 1)
    ep = world > 1 and args.mode == "ep"
    L = SyntheticLayer(seed, LAYER, H, F, args.experts, "cpu", bias_zipf=1.1 if args.config == 4 else None,
                       cache=True)
    x = activations(1000 * seed if ep else seed, n, H)  # rank 0's first n tokens (same generator, CPU stream)
    v, dt = time_cpu_reference(x, L.gate, L.expert, L.shared(), args.steps, args.warmup,
                               bias=L.bias if args.config == 4 else None)
    sample = (f"{n} tokens of rank 0's T={T} batch per step through the oracle's step-by-step restatement of the "
              f"reference moe_block (inference/forward.py:112-153; the reference tree does not travel to this "
              f"host), {args.steps} steps in {dt:.1f} s; experts of the same seeds and distributions generated "
              f"on the CPU; tokens/s is linear in T")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def streaming_measure(local: int, steps: int, warmup: int, prefetch: bool = True,
                      modes: tuple[str, ...] = ("device", "host")) -> dict:
    """Config 5: B=1 decode steps through 8 MoE layers (seeds 10..17), all
    routed experts in pinned host memory, a 64-expert GPU slot cache per layer
    (+ the shared expert). Two ways to run the slot caches, on the same pinned
    store: "device" (dsmoe_slotcache_step: placement and copies on the GPU, no
    host read per layer, no prefetch) and "host" (host-side LRU, cudaMemcpyAsync
    on a side stream, adaptive next-layer prefetch, one routing read-back per
    layer). Returns the measured figures per mode (device-timed)."""
    from dsmoe import DeepSeekConfig, SyntheticWeightStore
    from dsmoe.streaming import StreamingDecoder
    from dsmoe.synthetic import activations

    dev = torch.device("cuda", local)
    layers = list(range(8))
    cfg = DeepSeekConfig()
    store = SyntheticWeightStore(cfg, seed=10, device=dev, pin_memory=True, gen_device="cuda",
                                 layer_seeds={l: 10 + l for l in layers}, expert_cache_bytes=1 << 40)
    t0 = time.perf_counter()
    pinned = store.preload_host(layers)
    setup_s = time.perf_counter() - t0
    # host-link reference: one pinned -> device copy of 1 GiB
    src = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty_like(src, device=dev)
    for _ in range(2):
        dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(3):
        dst.copy_(src, non_blocking=True)
    c1.record()
    torch.cuda.synchronize()
    link_gbs = 3 * src.nbytes / (c0.elapsed_time(c1) / 1e3) / 1e9
    del src, dst
    # a new token every step (N(0,1) hidden state), carried through the 8 layers
    h_host = activations(10, warmup + steps, H).pin_memory()
    out_host = torch.empty(1, H, dtype=torch.bfloat16).pin_memory()
    res = {"pinned_copy_GB_s": link_gbs, "pinned_host_gb": pinned / 1e9, "host_setup_s": setup_s,
           "layers": len(layers), "steps": steps, "warmup": warmup}
    for mode in modes:
        device = mode == "device"
        dec = StreamingDecoder(cfg, store, dev, layers, slots_per_layer=65, prefetch=prefetch and not device,
                               device_slots=device)

        def moved_hits_misses():
            if device:
                h, m, b = dec.device_counters()
                return b, h, m
            return dec.gt.bytes_h2d, dec.gt.slot_hits, dec.gt.slot_misses

        for i in range(warmup):
            dec.step(h_host[i:i + 1].to(dev))
        torch.cuda.synchronize()
        b0, hit0, m0 = moved_hits_misses()
        p0, u0 = dec.predicted, dec.predicted_used
        sampler = ClockSampler({local})
        sampler.start()
        time.sleep(0.3)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_begin = time.time()
        e0.record()
        for i in range(steps):
            hd = h_host[warmup + i: warmup + i + 1].to(dev, non_blocking=True)  # the token in
            h = dec.step(hd)
            out_host.copy_(h, non_blocking=True)  # its final hidden state out
        e1.record()
        torch.cuda.synchronize()
        clocks = sampler.stop((t_begin, time.time()))
        ms = e0.elapsed_time(e1) / steps
        b1, hit1, m1 = moved_hits_misses()
        moved, hits, misses = b1 - b0, hit1 - hit0, m1 - m0
        achieved = moved / (steps * ms / 1e3) / 1e9
        res[mode] = {"tokens_per_s": 1e3 / ms, "ms_per_step": ms, "host_link_GB_s": achieved,
                     "host_link_frac": achieved / link_gbs, "h2d_gb_per_step": moved / steps / 1e9,
                     "slot_hit_rate": hits / max(1, hits + misses),
                     "misses_per_layer_step": misses / (steps * len(layers)),
                     "host_reads_per_layer": 0 if device else 1, "clocks": clocks}
        if not device:
            res[mode].update({"prefetch_precision": (dec.predicted_used - u0) / max(1, dec.predicted - p0),
                              "prefetched_experts": dec.gt.prefetched})
        del dec
        torch.cuda.empty_cache()
    del store
    torch.cuda.empty_cache()
    return res


def run_streaming(args, rank, world, local):
    """Config 5 as its own bench line (``--config 5``): the device-managed
    slot caches are the line's value; the host-managed ones are reported
    beside them."""
    if rank != 0:
        return
    torch.cuda.set_device(local)
    r = streaming_measure(local, args.steps, args.warmup, prefetch=not args.no_prefetch)
    d = r["device"]
    line = {
        "metric": METRIC, "value": d["tokens_per_s"], "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": d["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8-e4m3 (hi/lo activations) x e4m3 weights, fp32 accumulate",
        "data": "synthetic (seeded; per-layer seeds 10..17)",
        "config": {"workload": "B=1 decode through 8 DeepSeek-R1 MoE layers, experts in pinned host memory "
                               "(config 5), h <- h + moe(h) per layer, device-managed slot caches",
                   "slots_per_layer": 64, "pinned_host_gb": r["pinned_host_gb"],
                   "host_setup_s": r["host_setup_s"], "baseline_config": 5},
        "e2e": {"value": d["tokens_per_s"], "unit": UNIT, "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 2},
        "roofline": {"kernel": "expert host->device copies (slot-cache fill kernel)", "bound": "host-link",
                     "achieved": d["host_link_GB_s"], "peak": r["pinned_copy_GB_s"], "unit": "GB/s",
                     "frac": d["host_link_frac"], "peak_source": "measured pinned->device copy of 1 GiB in this run",
                     "traffic": None},
        "streaming": r,
        # per layer and step: router 2, slot plan + fill 2, count/plan/scatter 3, GEMMs 2, swiglu 1, combine 1
        "gpu_launches": 11 * r["layers"] * args.steps,
        "clocks": d["clocks"],
        "cpu_baseline": None,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="dsmoe", choices=["dsmoe", "reference"])
    ap.add_argument("--config", type=int, default=None, choices=[2, 3, 4, 5],
                    help="BASELINE config: 2 = prefill T=4096 on 1 GPU (default at N=1), 3 = expert-parallel "
                         "T=8192 per GPU (default at N>1), 4 = load skew: bias-corrected router with Zipf(1.1) "
                         "bias, T=16384 per GPU, 5 = streaming decode through 8 layers with experts in pinned "
                         "host memory (1 GPU)")
    ap.add_argument("--no-prefetch", action="store_true",
                    help="config 5: no next-layer expert prediction (default: adaptive prefetch)")
    ap.add_argument("--tokens", type=int, default=None, help="tokens per GPU (default: the config's)")
    ap.add_argument("--mode", default="ep", choices=["ep", "replica"],
                    help="N > 1: expert-parallel over NCCL (default) or independent replicas")
    ap.add_argument("--chunks", type=int, default=1,
                    help="expert-parallel step: token chunks whose all-to-alls overlap the expert GEMMs (1 = none)")
    ap.add_argument("--sm-reserve", type=int, default=0,
                    help="expert-parallel step: SMs the grouped GEMMs leave to the all-to-alls while they overlap")
    ap.add_argument("--nccl-exchange", action="store_true",
                    help="expert-parallel step: NCCL all-to-all instead of the default peer-memory exchange")
    ap.add_argument("--no-overlap", action="store_true",
                    help="expert-parallel step: exchange and GEMMs in one stream, one after the other")
    ap.add_argument("--ref-tokens-per-step", type=int, default=8)
    ap.add_argument("--ep-placement", default="auto", choices=["auto", "contiguous", "balanced"],
                    help="expert placement over ranks at N>1 (auto: balanced when routing is skewed)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=E, help="routed experts (32 per group); smaller = profiling case")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the T=8 / T=64 decode rows of the N=1 line")
    ap.add_argument("--no-streaming", action="store_true",
                    help="skip the config-5 streaming row of the N=1 line (90 GB of pinned host memory)")
    ap.add_argument("--no-widened", action="store_true", help="skip the widened rows of the N=1 line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    default_run = args.config is None
    if args.config is None:
        args.config = 2 if world == 1 else 3
    if args.tokens is None:
        # The default N > 1 run keeps the N = 1 line's per-GPU batch (4096
        # tokens) so that the 1 -> N curve compares equal per-GPU work (weak
        # scaling); config 3's own 8192 tokens per GPU is measured in the same
        # run (config3_t8192) and is the default of an explicit --config 3.
        args.tokens = {2: 4096, 3: 4096 if default_run else 8192, 4: 16384, 5: 1}[args.config]
    args.extra_config3 = default_run and world > 1 and args.mode == "ep" and args.tokens != 8192
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    if args.config == 5:
        run_streaming(args, rank, world, local)
        return

    import torch.distributed as dist
    from datetime import timedelta

    from dsmoe import DeepSeekConfig, GPUTransfer, SyntheticWeightStore, moe_block
    from dsmoe._lib import ClockProbe, Workspace, set_profile_events
    from dsmoe.ep import PEER_PHASES
    from dsmoe.synthetic import activations

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    T = args.tokens
    n_group = max(1, args.experts // 32)
    skew = args.config == 4
    cfg = DeepSeekConfig(n_routed_experts=32 * n_group, n_group=n_group, topk_group=min(4, n_group),
                         router_mode="v3" if skew else "ref")
    zipf = 1.1 if skew else None
    seed = {2: 1, 3: 2, 4: 3}[args.config]
    ep = world > 1 and args.mode == "ep"
    if ep:
        # one set of layer weights sharded over the ranks, every rank with its
        # own tokens
        from dsmoe.ep import DistExchange, EPLayer

        store = SyntheticWeightStore(cfg, seed=seed, device=dev, pin_memory=False, gen_device="cuda", bias_zipf=zipf)
        ep_layer = EPLayer(cfg, store, dev, LAYER, world, rank, exchange=DistExchange(),
                           expert_source=store.device_expert)
        ep_layer.sm_reserve = args.sm_reserve
        ep_layer.overlap = not args.no_overlap
        if not args.nccl_exchange:
            ep_layer.use_peer_memory(cap=max(T, 8192 if args.extra_config3 else 0))
        bank = None
        x = activations(1000 * seed + rank, T, H, device=dev)
        # Expert placement: contiguous ranges unless the routing of this
        # step's tokens (counted over all ranks) would load the busiest rank
        # more than 1.25x the mean, as skewed routing does; then experts are
        # spread by load (dsmoe.ep.balanced_placement), every rank alike.
        from dsmoe.ep import balanced_placement
        cal_idx, _ = ep_layer.route(x)
        loads = torch.bincount(cal_idx.reshape(-1), minlength=cfg.n_routed_experts).double()
        dist.all_reduce(loads)
        loads = loads.cpu()
        El = cfg.n_routed_experts // world
        rank_loads = loads.view(world, El).sum(1)
        contiguous_imbalance = float(rank_loads.max() / rank_loads.mean())
        placement_info = {"placement": "contiguous", "expected_rank_load_max_over_mean": contiguous_imbalance}
        if args.ep_placement == "balanced" or (args.ep_placement == "auto" and contiguous_imbalance > 1.25):
            placement = balanced_placement(loads.tolist(), world)
            ep_layer.set_placement(placement)
            bal = torch.zeros(world, dtype=torch.float64)
            for e, pos in enumerate(placement):
                bal[pos // El] += loads[e]
            placement_info = {"placement": "balanced by expert load (longest-processing-time rule)",
                              "expected_rank_load_max_over_mean": float(bal.max() / bal.mean()),
                              "contiguous_expected_rank_load_max_over_mean": contiguous_imbalance}

        def step(inp):
            return ep_layer.forward(inp, chunks=args.chunks)
    else:
        store = SyntheticWeightStore(cfg, seed=seed + rank, device=dev, pin_memory=False, gen_device="cuda",
                                     bias_zipf=zipf)
        gt = GPUTransfer(cfg, store, dev)
        bank = gt.bank(LAYER)
        x = activations(seed + rank, T, H, device=dev)

        def step(inp):
            return moe_block(inp, LAYER, store, gt, cfg)

    # ---------------------------------------------------------- device-timed
    # Single-GPU step: the library records one set of stage-boundary events
    # per timed step (dsmoe_set_profile_events; on the launching stream), so
    # the per-kernel times and the roofline come from the timed steps
    # themselves. The expert-parallel step is timed whole; its phases are
    # measured in a separate pass below.
    names = ["router", "permute", "gate_up", "swiglu_quant", "down", "combine"]
    evsets = [[torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)] for _ in range(args.steps)]
    # expert-parallel peer-memory step: its phases on the compute stream
    phsets = ([[torch.cuda.Event(enable_timing=True) for _ in range(len(PEER_PHASES) + 1)]
               for _ in range(args.steps)] if ep and not args.nccl_exchange else None)
    for evs in evsets + (phsets or []):
        for e in evs:
            e.record()  # create the CUDA events before the timed region
    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    sampler = ClockSampler({local} if world == 1 else set(range(world)))
    if rank == 0:
        sampler.start()
        time.sleep(0.5)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    probe = ClockProbe(dev)  # the SMs' own cycle counters across the timed region
    t_begin = time.time()
    probe.start()
    e0.record()
    for i in range(args.steps):
        if ep:  # the library's events around the rank's expert GEMMs only
            ep_layer.lib_events = evsets[i]
            ep_layer.phase_events = phsets[i] if phsets else None
        else:
            set_profile_events(evsets[i])
        step(x)
    e1.record()
    probe.stop()
    torch.cuda.synchronize()
    t_end = time.time()
    if ep:
        ep_layer.lib_events = ep_layer.phase_events = None
    else:
        set_profile_events(None)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop((t_begin, t_end)) if rank == 0 else None
    if rank == 0:
        clocks = clocks or {}
        # mean SM clock over the timed steps from the SMs' cycle counters (median over SMs)
        clocks["sm_mhz_device"] = probe.mhz()
    ms = e0.elapsed_time(e1) / args.steps
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = world * T / (ms_max / 1000.0)

    # ------------------------------------------------- per-stage (roofline)
    stage_ms = [0.0] * len(names)
    first = 2 if ep else 0  # expert-parallel: the library events cover the rank's expert GEMMs (stages 2..5)
    for evs in evsets:
        for i in range(first, len(names)):
            stage_ms[i] += evs[i].elapsed_time(evs[i + 1]) / len(evsets)
    ep_phases = None
    if phsets:
        ep_phases = {nm: sum(ev[i].elapsed_time(ev[i + 1]) for ev in phsets) / len(phsets)
                     for i, nm in enumerate(PEER_PHASES)}
        ep_phases["decomposition"] = ("peer-memory step, phase by phase on the compute stream inside the timed "
                                      "steps (the pushes run on a side stream beside the shared expert)")
    if not ep:
        out, idx, _w = moe_block(x, LAYER, store, gt, cfg, return_routing=True)  # the (deterministic) routing
    else:
        names[0] = names[1] = None  # not timed separately on the expert-parallel path
        # what this rank's GEMMs processed: its local (row, expert) pairs
        if args.nccl_exchange:
            counts_d, tok_rows, send_x, meta = ep_layer.dispatch(x)
            sc, rc = ep_layer.exchange.counts(counts_d)
            lidx = ep_layer.exchange.rows(meta, sc, rc)[:, :TOPK].reshape(-1)
        else:
            step(x)
            rows_recv, _ = ep_layer.received_pairs()
            pbm = ep_layer.peer.views["meta"].view(torch.int32)
            lidx = pbm[: world * ep_layer.peer.cap * TOPK].view(-1, TOPK)[:rows_recv].reshape(-1)
            ep_phases["rows_per_rank_received"] = rows_recv
            # load balance across ranks (skewed routing concentrates rows on the
            # ranks owning the hot experts)
            rr = torch.tensor([rows_recv], dtype=torch.int64, device=dev)
            rr_all = [torch.zeros_like(rr) for _ in range(world)]
            dist.all_gather(rr_all, rr)
            rows_all = [int(t.item()) for t in rr_all]
            ep_phases["rows_received_by_rank"] = rows_all
            ep_phases["rows_received_max_over_mean"] = max(rows_all) / (sum(rows_all) / world)
        lidx = lidx[lidx >= 0].long()
    config3 = None
    if args.extra_config3:
        # config 3's own shape (8192 tokens per GPU), same layer and exchange
        x8 = activations(1000 * seed + rank, 8192, H, device=dev)
        for _ in range(3):
            step(x8)
        torch.cuda.synchronize()
        dist.barrier()
        a8, b8 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a8.record()
        for _ in range(10):
            step(x8)
        b8.record()
        torch.cuda.synchronize()
        ms8 = torch.tensor([a8.elapsed_time(b8) / 10], device=dev)
        dist.all_reduce(ms8, op=dist.ReduceOp.MAX)
        config3 = {"tokens_per_gpu": 8192, "value": world * 8192 / (float(ms8.item()) / 1e3),
                   "ms_per_step": float(ms8.item()), "steps": 10, "unit": UNIT}
        del x8
    from dsmoe.ops import route as _route
    _gidx, _ = _route(x, store.get_gate_weight(LAYER), cfg,
                      score_bias=store.get_gate_bias(LAYER) if skew else None)
    gcounts = torch.bincount(_gidx.reshape(-1), minlength=cfg.n_routed_experts).float()
    hottest_over_mean = float(gcounts.max() / gcounts.mean())
    if ep:
        # the rank's own GEMM work: its experts over the rows it received (no shared expert there)
        counts = torch.bincount(lidx, minlength=ep_layer.El).cpu()
        touched = int((counts > 0).sum())
        rows = int(lidx.numel())
    else:
        counts = torch.bincount(idx.reshape(-1), minlength=cfg.n_routed_experts).cpu()
        touched = int((counts > 0).sum()) + 1  # + shared expert
        rows = T * TOPK + T
    gu_ms, dn_ms = stage_ms[2], stage_ms[4]
    crit_rank, gemm_ms_by_rank = 0, None
    if ep:
        # The roofline is the critical rank's: under skewed routing some ranks
        # get few rows (or none: at 8 ranks a rank owns exactly one expert
        # group, which group-limited routing can skip entirely).
        mine = torch.tensor([float(rows), float(touched)] + list(stage_ms), dtype=torch.float64, device=dev)
        allv = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allv, mine)
        allv = [v.tolist() for v in allv]
        gemm_ms_by_rank = [round(v[2 + 2] + v[2 + 4], 4) for v in allv]
        crit_rank = max(range(world), key=lambda r: gemm_ms_by_rank[r])
        rows, touched = int(allv[crit_rank][0]), int(allv[crit_rank][1])
        stage_ms = allv[crit_rank][2:]
        gu_ms, dn_ms = stage_ms[2], stage_ms[4]
    w13 = 2 * F * H + 2 * (F // 128) * (H // 128) * 4
    w2 = F * H + (F // 128) * (H // 128) * 4
    # algorithmic bytes per launch: weights of every expert used, activations
    # read once per (token, expert) row (hi + lo = 2 B/element + scales), outputs
    gateup_bytes = touched * w13 + rows * (H * 2 + (H // 128) * 4) + rows * 2 * F * 2
    swiglu_bytes = rows * 2 * F * 2 + rows * (F * 2 + (F // 128) * 4)
    down_bytes = touched * w2 + rows * (F * 2 + (F // 128) * 4) + rows * H * 2
    algo_flops = 2.0 * rows * 3 * F * H  # useful FP8-GEMM work (hi/lo doubles what the tensor pipe executes)
    hbm_peak, bf16_peak, bf16_sustained, peak_src = peaks()
    dominant = "gate_up" if gu_ms >= dn_ms else "down"
    dom_bytes, dom_ms = (gateup_bytes, gu_ms) if dominant == "gate_up" else (down_bytes, dn_ms)
    dom_flops = 2.0 * rows * (2 * F if dominant == "gate_up" else F) * H  # algorithmic (one pass over x)
    traffic = None if ep else MEASURED_DRAM_BYTES.get((dominant, args.config, T, cfg.n_routed_experts))
    # The bound is the roof the launch's algorithmic intensity meets first.
    # The kernel executes two FP8 MMAs (hi and lo activation terms) per
    # multiply-add of the reference, so its compute roof in useful FLOP/s is
    # the FP8 rate / 2 = the measured bf16 GEMM rate; sustained, because the
    # kernel is timed inside a long step under the 1000 W cap.
    tensor_roof = bf16_sustained
    dom_ms = max(dom_ms, 1e-6)
    hbm_frac = dom_bytes / (dom_ms / 1000.0) / 1e9 / hbm_peak
    if dom_bytes > 0 and dom_flops / dom_bytes > tensor_roof * 1e12 / (hbm_peak * 1e9):
        achieved = dom_flops / (dom_ms / 1000.0) / 1e12
        roofline = {"kernel": f"grouped_gemm_kernel ({dominant})", "bound": "tensor", "achieved": achieved,
                    "peak": tensor_roof, "unit": "TFLOP/s", "frac": achieved / tensor_roof,
                    "peak_source": f"{peak_src}: bf16 GEMM sustained (= FP8 rate / 2, two FP8 MMAs per useful "
                                   "multiply-add)", "traffic": traffic,
                    "executed_fp8_tflops": 2.0 * achieved, "hbm_frac": hbm_frac,
                    "algorithmic_flops_per_launch": dom_flops, "algorithmic_bytes_per_launch": dom_bytes}
    else:
        achieved = dom_bytes / (dom_ms / 1000.0) / 1e9
        roofline = {"kernel": f"grouped_gemm_kernel ({dominant})", "bound": "hbm", "achieved": achieved,
                    "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak, "peak_source": peak_src,
                    "traffic": traffic, "algorithmic_bytes_per_launch": dom_bytes,
                    "algorithmic_flops_per_launch": dom_flops,
                    "tensor_frac": dom_flops / (dom_ms / 1000.0) / 1e12 / tensor_roof}
    if ep:
        roofline["rank"] = crit_rank  # the rank whose expert GEMMs took longest
        roofline["gemm_ms_by_rank"] = gemm_ms_by_rank
    roofline["traffic_source"] = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch on this "
                                  "workload (profiles/)" if traffic else None)
    roofline["timing"] = ("mean of the launch's CUDA-event duration over the timed steps (events recorded by the "
                          "library at its stage boundaries on the launching stream)")
    layer_bytes = gateup_bytes + swiglu_bytes + down_bytes
    layer_ms = sum(stage_ms)

    # ------------------------------------------------------------------ e2e
    if args.skip_e2e:
        args.steps_e2e = 0
    # A stream of batches through the public call, as a serving loop runs it:
    # every step copies its input from pinned host memory and reads its output
    # back; the copies run on two copy streams (one per direction) with two
    # device input buffers, so step i+1's input and step i-1's output move
    # while step i computes. The timed region runs from the first input copy
    # to the last output copy.
    x_host = x.cpu().pin_memory()
    outs_host = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    x_in = [torch.empty_like(x) for _ in range(2)]
    cs = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n, start=None, end=None):
        if start is not None:
            start.record(h2d)
        with torch.cuda.stream(h2d):
            x_in[0].copy_(x_host, non_blocking=True)
        in_ready[0].record(h2d)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                nb = (i + 1) % 2
                if i >= 1:
                    h2d.wait_event(computed[nb])  # step i-1 is done with that buffer
                with torch.cuda.stream(h2d):
                    x_in[nb].copy_(x_host, non_blocking=True)
                in_ready[nb].record(h2d)
            cs.wait_event(in_ready[b])
            y = step(x_in[b])
            computed[b].record(cs)
            d2h.wait_event(computed[b])
            with torch.cuda.stream(d2h):
                y.record_stream(d2h)
                outs_host[b].copy_(y, non_blocking=True)
        if end is not None:
            end.record(d2h)

    if not args.skip_e2e:
        e2e_run(3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = 1 if args.skip_e2e else args.steps
    e2e_run(n_e2e, e2, e3)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e2.elapsed_time(e3) / n_e2e], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = world * T / (float(e2e_ms.item()) / 1000.0)
    # ------------------------------------ widened rows (1 GPU, same layer)
    # The MoE layer's FFN half (norm + block + residual in one library call),
    # RMSNorm alone, and the dense FFN of layers 0-2 (intermediate 18432)
    # through the same FP8 GEMM, on this batch. Device-timed.
    widened = None
    if world == 1 and not ep and not args.no_widened:
        from dsmoe import dense_ffn, moe_layer_ffn, rms_norm
        from dsmoe.synthetic import expert_weights

        def dev_ms(fn, n=10):
            for _ in range(3):
                fn()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(n):
                fn()
            b.record()
            torch.cuda.synchronize()
            return a.elapsed_time(b) / n

        ln = store.get_layer_norm_weights(LAYER)[1]
        norm_ms = dev_ms(lambda: rms_norm(x, ln, cfg.rms_norm_eps))
        ffn_ms = dev_ms(lambda: moe_layer_ffn(x, LAYER, store, gt, cfg))
        dense_w = {p: (w.to(dev), s.to(dev)) for p, (w, s) in expert_weights(5, 0, 0, H, 18432, "cuda").items()}
        dn_ms = dev_ms(lambda: dense_ffn(x, dense_w))
        dense_bytes = 3 * 18432 * H + T * H * 2 * 2
        loader = expert_load_rates(cfg, dev)
        sampler = sampler_rates(dev, dev_ms)
        widened = {"rms_norm_ms": norm_ms, "rms_norm_GB_s": 2 * T * H * 2 / (norm_ms / 1e3) / 1e9,
                   "moe_layer_ffn_ms": ffn_ms, "moe_layer_ffn_over_block": ffn_ms / ms_max,
                   "dense_ffn_ms": dn_ms, "dense_ffn_tflops": 2.0 * T * 3 * 18432 * H / (dn_ms / 1e3) / 1e12,
                   "dense_ffn_weight_GB": dense_bytes / 1e9, **loader, **sampler}
        del dense_w
    # -------------------------------- decode batches (north star: T=64) --
    # The same layer and bank at decode batch sizes, timed like the main
    # step (CUDA events per stage, inside the timed steps).
    decode = None
    if world == 1 and not ep and args.config == 2 and not args.no_decode:
        decode = {}
        for Td in (8, 64):
            xd = activations(seed + 100 + Td, Td, H, device=dev)
            n_d = 50
            ev_d = [[torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)] for _ in range(n_d)]
            for evs in ev_d:
                for e in evs:
                    e.record()
            for _ in range(5):
                step(xd)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            probe_d = ClockProbe(dev)
            probe_d.start()
            a.record()
            for i in range(n_d):
                set_profile_events(ev_d[i])
                step(xd)
            b.record()
            probe_d.stop()
            torch.cuda.synchronize()
            set_profile_events(None)
            ms_d = a.elapsed_time(b) / n_d
            st = [sum(evs[i].elapsed_time(evs[i + 1]) for evs in ev_d) / n_d for i in range(len(names))]
            _, idx_d, _ = moe_block(xd, LAYER, store, gt, cfg, return_routing=True)
            touched_d = int(torch.unique(idx_d).numel()) + 1  # + the shared expert
            rows_d = Td * TOPK + Td
            gu_b = touched_d * w13 + rows_d * (H * 2 + (H // 128) * 4) + rows_d * 2 * F * 2
            dn_b = touched_d * w2 + rows_d * (F * 2 + (F // 128) * 4) + rows_d * H * 2
            decode[f"t{Td}"] = {
                "tokens_per_s": Td / (ms_d / 1e3), "ms_per_step": ms_d, "steps": n_d,
                "experts_touched": touched_d, "stages_ms": dict(zip(names, st)),
                "gate_up_hbm_frac": gu_b / (st[2] / 1e3) / 1e9 / hbm_peak,
                "down_hbm_frac": dn_b / (st[4] / 1e3) / 1e9 / hbm_peak,
                "step_hbm_frac": (gu_b + dn_b) / (ms_d / 1e3) / 1e9 / hbm_peak,
                "algorithmic_bytes_gemms": gu_b + dn_b, "sm_mhz_device": probe_d.mhz()}
        decode["note"] = ("hbm fractions: algorithmic bytes (weights of the experts touched + activation rows in "
                          "and out) / CUDA-event time, of measured HBM " + f"{hbm_peak:.0f} GB/s")

    # ------------------------------------- config 5 (streaming decode) ----
    streaming = None
    if world == 1 and not ep and args.config == 2 and not args.no_streaming:
        try:
            import psutil
            enough = psutil.virtual_memory().available > 120e9
        except Exception:
            enough = False
        streaming = (streaming_measure(local, 32, 3) if enough else
                     {"skipped": "less than 120 GB of free host memory for the 90 GB pinned expert store"})

    status = Workspace.get(dev).status()

    # ---------------------------------------------------------- CPU oracle
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        def get_expert(e):
            return {p: (w.cpu(), s.cpu()) for p, (w, s) in bank.views(e + 1).items()}

        shared = {p: (w.cpu(), s.cpu()) for p, (w, s) in bank.views(0).items()}
        n_cpu = args.ref_tokens_per_step
        v, dt = time_cpu_reference(x[:n_cpu].cpu(), store.get_gate_weight(LAYER).cpu(), get_expert, shared,
                                   steps=2, warmup=1, bias=store.get_gate_bias(LAYER).cpu() if skew else None)
        cpu = {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"the first {n_cpu} tokens of the T={T} batch, 2 timed passes ({dt:.1f} s) through the "
                         f"oracle's step-by-step restatement of the reference moe_block "
                         f"(inference/forward.py:112-153), experts copied from this run's bank beforehand; "
                         f"tokens/s extrapolates linearly in T (the reference loops per token)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8-e4m3 (hi/lo activations) x e4m3 weights, fp32 accumulate",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) FP8 block-quantised experts)",
            "config": workload_config(args, world),
            "routing": {"hottest_expert_over_mean": hottest_over_mean},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2,
                    "copies": "pinned host buffers; H2D and D2H on their own streams, double-buffered, "
                              "overlapping the neighbouring steps' compute"},
            "roofline": roofline,
            "stages_ms": {nm: v for nm, v in zip(names, stage_ms) if nm},
            "stages_rank": crit_rank if ep else None,
            "stages_sum_over_step": None if ep else sum(stage_ms) / ms_max,
            **({"config3_t8192": config3} if config3 else {}),
            **({"ep_phases_ms": ep_phases} if ep_phases else {}),
            **({"ep_placement": placement_info} if ep else {}),
            "layer": {"algorithmic_bytes": layer_bytes, "GB_s": layer_bytes / (layer_ms / 1e3) / 1e9,
                      "hbm_frac": layer_bytes / (layer_ms / 1e3) / 1e9 / hbm_peak,
                      "fp8_tflops_algorithmic": algo_flops / (ms_max / 1e3) / 1e12,
                      "fp8_frac_of_nominal_dense": algo_flops / (ms_max / 1e3) / 1e12 / FP8_DENSE_NOMINAL_TFLOPS,
                      "experts_touched": touched},
            **({"widened_rows": widened} if widened else {}),
            **({"decode_rows": decode} if decode else {}),
            **({"streaming_config5": streaming} if streaming else {}),
            # library kernels per step: router 2, count/plan/scatter 3, GEMMs 2, swiglu 1, combine 1;
            # expert-parallel over peer memory: router 2, plan 2, push 1, shared-expert FFN 5 (plan,
            # scatter, 2 GEMMs, swiglu), received-row count 1, the rank's experts 7 (count, plan, scatter,
            # 2 GEMMs, swiglu, combine-and-return), final combine 1
            "gpu_launches": (19 if ep else 9) * args.steps,
            "device_status": status,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        if ep:
            ep_layer.close()  # peer buffers (a collective when in use)
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
