#!/usr/bin/env python
"""Benchmark of the B200 MoE expert path (PDScope per-layer expert execution).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl pdx|reference]

Workload (synthetic seeded data, random-init weights):
  * headline ``value``: config 2 -- a 48-layer Qwen3-30B-A3B-shaped MoE stack
    (H=2048, E=128, I=768, top-8; all 6144 experts resident in HBM) decoding a
    batch of 64 tokens; one step = all 48 layers (route, pack, grouped FFN,
    combine) replayed from one CUDA graph.  Expert weights streamed per step
    (~3.6 GB) far exceed the 126 MB L2, so no L2 flush is needed.
  * also reported: decode at batch 1 and 8, and config 3 -- a ragged prefill of
    8 sequences (lengths ~U[256, 4096], seeded) through the same 48 layers with a
    Zipf(1.1) router skew.
  * ``e2e``: the same decode step through the public stack API with the input
    copied host->device from pinned memory and the output copied back every step.
  * ``roofline``: the grouped expert FFN of the decode path (one launch of
    k_decode_ffn: gate/up and down projections, weights streamed by TMA into
    tcgen05 MMAs) timed on its own stream with CUDA events; algorithmic
    bytes = active experts x 9,437,184 B + activation rows.
  * ``cpu_baseline``: the reference's CPU layer path (oracle/cpu_path.py, torch
    CPU ops) on this host's cores, a bounded sample of layers.
Multi-GPU (N>1, torchrun): expert parallel, 128/N experts per GPU, each rank
routing its own decode batch (64 tokens per GPU, weak scaling) and exchanging
rows over NVLink peer memory (``--ep-transport nccl``: NCCL all-to-all);
value = tokens of all ranks / max-over-ranks time.  ``--ep-shape 235b`` runs
config 5 instead (Qwen3-235B shape, 256 decode tokens in all).

``--impl reference`` times the reference's own CPU implementation of the path
(the torch-CPU restatement in oracle/cpu_path.py) on all host cores on the
pdx arm's whole-job workload (at N GPUs the N x 64-token batch, or config 5's
shape) and prints the same metric; under torchrun rank 0 alone runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode & prefill tok/s, Qwen3-30B-A3B-shape MoE, 1–8 B200; % HBM/tensor roofline"
CFG = dict(hidden=2048, experts=128, inter=768, top_k=8, layers=48)
EXPERT_BYTES = 3 * CFG["hidden"] * CFG["inter"] * 2          # 9,437,184
FLOPS_PER_ROW = 6 * CFG["hidden"] * CFG["inter"]              # 9,437,184 (x2 flops, 3 matmuls)
FALLBACK_PEAKS = dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0)


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("pdx", "reference"), default="pdx")
    ap.add_argument("--layers", type=int, default=CFG["layers"])
    ap.add_argument("--decode-batch", type=int, default=64, help="headline decode batch")
    ap.add_argument("--decode-batches", default="1,8", help="other decode batches reported beside the headline")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--prefill-steps", type=int, default=3)
    ap.add_argument("--cpu-layers", type=int, default=2, help="layers in the CPU baseline sample")
    ap.add_argument("--cpu-threads", type=int, default=0, help="0 = all usable cores")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--ep-transport", choices=("p2p", "nccl"), default="p2p",
                    help="N>1 decode exchange: NVLink peer stores + flags (p2p) or NCCL all-to-all")
    ap.add_argument("--ep-shape", choices=("30b", "235b"), default="30b",
                    help="N>1 expert-parallel workload: 30b (config 2 per GPU) or 235b (config 5)")
    ap.add_argument("--offload", action="store_true",
                    help="config 4 instead: experts in pinned host memory, 24 GiB HBM cap, hot 16/layer")
    ap.add_argument("--offload-prefills", default="512,1024,2048,4096")
    ap.add_argument("--offload-decode-steps", type=int, default=64)
    ap.add_argument("--offload-cap-gib", type=float, default=24.0)
    ap.add_argument("--offload-hot", type=int, default=16)
    ap.add_argument("--offload-warm", type=int, default=30,
                    help="static cache tier: the next experts per layer by the hot table's rank")
    ap.add_argument("--offload-python", action="store_true",
                    help="per-layer orchestration in Python instead of the C++ engine (pdx_offload_*)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=float(d["hbm_gbs"]), bf16_tflops=float(d["bf16_tflops"]),
                    bf16_tflops_sustained=float(d["bf16_tflops_sustained"]), source="measured")
    return dict(FALLBACK_PEAKS, source="fallback")


def usable_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------
REASON_FIELDS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(f"/tmp/pdx_clocks_{os.getpid()}.csv")

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"], samples=0)
        sm, smax, power, reasons = [], None, [], set()
        for line in self.path.read_text().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(REASON_FIELDS, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=smax,
                    power_w_max=max(power) if power else None, reasons=sorted(reasons), samples=len(sm))


# ----------------------------------------------------------------------------
# CPU baseline (reference CPU path, oracle/cpu_path.py)
# ----------------------------------------------------------------------------


def cpu_baseline(tokens, layers, threads, steps=1):
    from oracle import cpu_path
    import torch
    cores = threads or usable_cores()
    sample = [cpu_path.make_layer(CFG["hidden"], CFG["experts"], CFG["inter"], seed=100 + i) for i in range(layers)]
    cpu_path.time_layers(sample[:1], tokens, CFG["hidden"], cores, repeats=1)  # warm
    per_layer, active = cpu_path.time_layers(sample, tokens, CFG["hidden"], cores, repeats=steps)
    tok_s = tokens / (per_layer * CFG["layers"])
    try:
        model = next((l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name")), "")
    except OSError:
        model = ""
    return dict(value=tok_s, unit="tok/s", cores=cores, kind="port",
                sample=(f"{layers} random-init Qwen3-30B-A3B layers x {steps} pass(es) at decode batch {tokens}, "
                        f"torch CPU route/compact_expert_groups/expert_forward/index_add_ "
                        f"(oracle/cpu_path.py); {per_layer * 1e3:.1f} ms/layer, scaled to 48 layers; "
                        f"mean active experts {statistics.mean(active):.1f}; cpu '{model}'"),
                ms_per_layer=per_layer * 1e3, torch_threads=torch.get_num_threads())


def ep_layers(args, world, H, I):
    """Layers of the config-5 stack that fit one GPU's share of the experts."""
    fit = int(150e9 // ((CFG["experts"] // world) * 3 * H * I * 2))
    return min(94 if args.layers == CFG["layers"] else args.layers, fit)


def headline_config(args, world):
    """The workload of the headline line, identical for both arms: the pdx arm
    runs it on the GPUs, the reference arm on the host cores."""
    E, k = CFG["experts"], CFG["top_k"]
    if world > 1 and args.ep_shape == "235b":
        H, I = 4096, 1536
        L = ep_layers(args, world, H, I)
        per_gpu = max(1, 256 // world)
        return dict(workload=f"config5 decode batch {per_gpu * world} in all ({per_gpu} per GPU): {L}-layer "
                             f"Qwen3-235B-A22B-shape MoE stack, experts split evenly over {world} GPUs",
                    hidden=H, experts=E, inter=I, top_k=k, layers=L, decode_batch=per_gpu,
                    global_batch=per_gpu * world, parallelism=f"ep{world}",
                    l2="not flushed: every step streams the routed experts' weights (GBs, > 126 MB L2)"), "strong"
    t = args.decode_batch
    if world > 1:
        workload = (f"config2 decode batch {t} per GPU: {args.layers}-layer Qwen3-30B-A3B-shape MoE stack, "
                    f"experts split evenly over {world} GPUs")
    else:
        workload = f"config2 decode batch {t}: {args.layers}-layer Qwen3-30B-A3B-shape MoE stack, all experts resident"
    return dict(workload=workload, hidden=CFG["hidden"], experts=E, inter=CFG["inter"], top_k=k, layers=args.layers,
                decode_batch=t, global_batch=t * world, parallelism=f"ep{world}" if world > 1 else "single",
                l2="not flushed: every step streams the routed experts' weights (GBs, > 126 MB L2)"), "weak"


def run_reference(args, rank):
    """The reference's CPU layer path (oracle/cpu_path.py: route ->
    compact_expert_groups -> per-expert torch CPU expert_forward -> index_add_
    merge) on all host cores, timing the whole headline workload: every step
    runs every layer of the stack on the whole job's token batch (N x the
    per-GPU batch at N GPUs).  The stack's layers cycle through
    ``--cpu-layers`` distinct random-init layers (the weights of all 48 would
    not fit host memory), with x <- layer_norm(MoE(x) + x) between layers as
    on the GPU arm."""
    if rank != 0:
        return 0
    import torch
    from oracle import cpu_path
    steps = max(1, args.steps)
    warm = max(0, args.warmup)
    cores = args.cpu_threads or usable_cores()
    world = max(1, args.gpus)
    config, scaling = headline_config(args, world)
    H, E, I, L = config["hidden"], config["experts"], config["inter"], config["layers"]
    t_count = config["global_batch"]
    torch.set_num_threads(cores)
    sample = [cpu_path.make_layer(H, E, I, seed=100 + i) for i in range(max(1, args.cpu_layers))]
    gen = torch.Generator(device="cpu").manual_seed(5)
    x0 = torch.randn(t_count, H, generator=gen).to(torch.bfloat16)
    for _ in range(warm):
        cpu_path.stack_step(x0, sample, L)
    times, active = [], []
    t0 = time.perf_counter()
    for _ in range(steps):
        s0 = time.perf_counter()
        _, act = cpu_path.stack_step(x0, sample, L)
        times.append(time.perf_counter() - s0)
        active.extend(act)
    elapsed = time.perf_counter() - t0
    ms = elapsed / steps * 1e3
    value = t_count * steps / elapsed
    line = dict(metric=METRIC, value=value, unit="tok/s", impl="reference", n_gpus=args.gpus, steps=steps,
                warmup=warm, ms_per_step=ms, higher_is_better=True, scaling=scaling, vs_baseline=None,
                dtype="bf16", data="synthetic", config=config,
                cpu_baseline=dict(value=value, unit="tok/s", cores=cores, kind="port",
                                  sample=(f"every step runs all {L} layers at batch {t_count} on the reference's "
                                          f"CPU path (torch CPU, oracle/cpu_path.py), cycling {len(sample)} "
                                          f"random-init layers; {steps} steps in {elapsed:.1f} s wall, "
                                          f"median {statistics.median(times) * 1e3:.0f} ms/step, mean active "
                                          f"experts {statistics.mean(active):.1f}")),
                e2e=dict(value=value, unit="tok/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
                timed_layers_per_step=L, extrapolated=False)
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# GPU benchmark
# ----------------------------------------------------------------------------


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import datetime
    import torch
    import torch.distributed as dist
    from pdscope_b200 import _lib
    from pdscope_b200.stack import (ResidentMoEStack, activations, build_stack, prefill_lengths, ZIPF_ALPHA,
                                    ZIPF_S)

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    K, W = max(1, args.steps), max(3, args.warmup)
    pk = peaks()
    L = args.layers
    if world > 1:
        return run_expert_parallel(args, rank, local_rank, world, dev, dist, K, W, pk, L)
    if args.offload:
        return run_offload(args, dev, W, pk, L)
    stack = build_stack(L, CFG["hidden"], CFG["experts"], CFG["inter"], CFG["top_k"], device=dev, seed=rank)
    torch.cuda.synchronize(dev)

    def timed(fn, steps, warm, sampler=None):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            fn()
        e1.record(s)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    def active_per_layer(t_count):
        b = stack.buffers(t_count)
        return [int((st.counts > 0).sum().item()) for st in b["stages"]]

    # ---- decode: batches 1, 8 and the headline batch --------------------------------
    decode = {}
    headline_t = args.decode_batch
    extra = [int(v) for v in args.decode_batches.split(",") if v.strip()]
    for t_count in sorted(set(extra) | {headline_t}):
        stack.input(t_count).copy_(activations(t_count, CFG["hidden"], device=dev, seed=10 + t_count + 1000 * rank))
        launches0 = _lib.lib.pdx_launch_count()
        stack.step(t_count)  # capture (counts the kernels of one step)
        torch.cuda.synchronize(dev)
        launches_per_step = (_lib.lib.pdx_launch_count() - launches0) // 2  # warm call + captured call
        sampler = ClockSampler(local_rank) if t_count == headline_t else None
        if sampler:
            with sampler:
                ms = timed(lambda: stack.step(t_count), K, W)
            clocks = sampler.summary()
        else:
            ms = timed(lambda: stack.step(t_count), K, W)
            clocks = None
        act = active_per_layer(t_count)
        decode[t_count] = dict(ms_per_step=ms / K, tok_s=sum_over_ranks(t_count) * K / (ms / 1e3),
                               active_experts_per_layer=statistics.mean(act),
                               weight_gb_per_step=sum(act) * EXPERT_BYTES / 1e9,
                               launches_per_step=launches_per_step, clocks=clocks)
        decode[t_count]["hbm_gbs_step"] = decode[t_count]["weight_gb_per_step"] / (decode[t_count]["ms_per_step"] / 1e3)
        decode[t_count]["stage_us_per_layer"] = stack.stage_times_us(t_count)

    # ---- roofline of the dominant kernel: grouped FFN GEMV at the headline batch ----
    t_count = headline_t
    stack.stage_once(t_count)
    g = stack.ffn_graph(t_count)
    ffn_ms = timed(g.replay, K, W)
    act = active_per_layer(t_count)
    n_rows = t_count * CFG["top_k"]
    act_bytes = t_count * CFG["hidden"] * 2 + n_rows * CFG["inter"] * 2 * 2 + n_rows * CFG["hidden"] * 2
    bytes_per_launch = statistics.mean(act) * EXPERT_BYTES + act_bytes
    per_launch_s = ffn_ms / 1e3 / (K * L)
    achieved = bytes_per_launch / per_launch_s / 1e9
    traffic = None
    tt = ROOT / "profiles" / "traffic.txt"   # figure from an ncu capture (see the file's header)
    if tt.exists():
        for line in tt.read_text().splitlines():
            f = line.split()
            if len(f) == 2 and f[0] == "decode_ffn_dram_bytes_per_active_expert":
                traffic = float(f[1]) * statistics.mean(act)
    roofline = dict(bound="hbm", kernel="pdx_moe_ffn_grouped decode path (k_decode_ffn: gate/up + down in one launch, TMA weight stream, tcgen05 swap-AB)",
                    achieved=achieved, peak=pk["hbm_gbs"], unit="GB/s", frac=achieved / pk["hbm_gbs"],
                    peak_source=pk["source"], frac_of_8000_nominal=achieved / 8000.0, traffic=traffic,
                    bytes_per_launch=bytes_per_launch, us_per_launch=per_launch_s * 1e6)

    # ---- e2e: public API with host buffers (pinned H2D in, D2H out) --------------------
    # (right after the device-timed headline, at the same clocks)
    t_count = headline_t
    host_in = activations(t_count, CFG["hidden"], device=dev, seed=5).cpu().pin_memory()
    host_out = torch.empty((t_count, CFG["hidden"]), dtype=torch.bfloat16).pin_memory()
    x_dev, y_dev = stack.input(t_count), stack.output(t_count)

    def e2e_step():
        x_dev.copy_(host_in, non_blocking=True)
        stack.step(t_count)
        host_out.copy_(y_dev, non_blocking=True)

    e2e_ms = timed(e2e_step, K, W)
    e2e = dict(value=sum_over_ranks(t_count) * K / (e2e_ms / 1e3), unit="tok/s",
               h2d_bytes_per_step=host_in.numel() * 2, d2h_bytes_per_step=host_out.numel() * 2,
               ms_per_step=e2e_ms / K)

    # ---- config 1: one layer (pdx_moe_layer, one C-ABI call) at T = 1 and 512 ----------
    # (timed before the prefill section: the HBM-bound layer then runs at the clocks
    # the decode sections see, not in the power-capped aftermath of the prefill GEMMs)
    from pdscope_b200.runtime import LayerOutputs, ResidentMoELayer
    layer0 = ResidentMoELayer(stack.gates[0], stack.slabs[0])
    config1 = {}
    for t_count, reps in ((1, 200), (512, 50)):
        x1 = activations(t_count, CFG["hidden"], device=dev, seed=300 + t_count)
        outs = layer0.forward(x1)
        # ten pdx_moe_layer calls per CUDA graph, as a serving loop replays them
        # (the layer's 1.2 GB of expert weights exceed L2, so no call hits in it)
        torch.cuda.synchronize(dev)
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1):
            for _ in range(10):
                layer0.forward(x1, outputs=outs)
        ms1 = timed(g1.replay, reps // 10, W) / (reps // 10 * 10)
        del g1
        u = int((outs.counts > 0).sum().item())
        layer_bytes = u * EXPERT_BYTES + CFG["experts"] * CFG["hidden"] * 2 + 2 * t_count * CFG["hidden"] * 2
        config1[str(t_count)] = dict(us_per_layer=ms1 * 1e3, active_experts=u,
                                     hbm_gbs=layer_bytes / (ms1 / 1e3) / 1e9,
                                     hbm_frac=layer_bytes / (ms1 / 1e3) / 1e9 / pk["hbm_gbs"],
                                     tflops=t_count * CFG["top_k"] * FLOPS_PER_ROW / (ms1 / 1e3) / 1e12)
    if world == 1 and not args.no_cpu:
        from oracle import cpu_path
        cores = args.cpu_threads or usable_cores()
        sample = [cpu_path.make_layer(CFG["hidden"], CFG["experts"], CFG["inter"], seed=100)]
        for t_count in (1, 512):
            per_layer, _ = cpu_path.time_layers(sample, t_count, CFG["hidden"], cores, repeats=1)
            config1[str(t_count)]["cpu_reference_us_per_layer"] = per_layer * 1e6
            config1[str(t_count)]["cpu_cores"] = cores
    del layer0

    # ---- prefill (config 3): ragged 8-sequence batch, Zipf router skew -----------------
    prefill = None
    if not args.no_prefill:
        lengths = prefill_lengths(8, seed=rank)
        tp = sum(lengths)
        zgates = []
        gen = torch.Generator(device=dev).manual_seed(1234 + rank)
        for l in range(L):
            gte = stack.gates[l].clone()
            perm = torch.randperm(CFG["experts"], device=dev, generator=gen)
            ranks = torch.empty(CFG["experts"], device=dev)
            ranks[perm] = torch.arange(1, CFG["experts"] + 1, device=dev, dtype=torch.float32)
            gte[:, 0] = (-ZIPF_ALPHA * ZIPF_S * torch.log(ranks)).to(torch.bfloat16)
            zgates.append(gte)
        pstack = ResidentMoEStack(zgates, stack.slabs, top_k=CFG["top_k"])
        pstack.input(tp).copy_(activations(tp, CFG["hidden"], device=dev, seed=77 + rank, zipf=True))
        stack.release_graphs()
        pstack.step(tp)
        pk_steps = max(1, args.prefill_steps)
        with ClockSampler(local_rank) as psampler:
            ms = timed(lambda: pstack.step(tp), pk_steps, 1)
        prefill_clocks = psampler.summary()
        b = pstack.buffers(tp)
        c0 = b["stages"][0].counts.float()
        top16 = float(torch.topk(c0, 16).values.sum() / c0.sum())
        stages_p = pstack.stage_times_us(tp, layers=4, repeats=1)
        pstack.stage_once(tp)
        gp = pstack.ffn_graph(tp)
        ffn_ms_p = timed(gp.replay, pk_steps, 1)
        flops_launch = tp * CFG["top_k"] * FLOPS_PER_ROW
        per_launch_p = ffn_ms_p / 1e3 / (pk_steps * L)
        tflops = flops_launch / per_launch_p / 1e12
        prefill = dict(tokens=tp, lengths=lengths, ms_per_step=ms / pk_steps,
                       tok_s=sum_over_ranks(tp) * pk_steps / (ms / 1e3), top16_share_layer0=top16,
                       stage_us_per_layer=stages_p, clocks=prefill_clocks,
                       zipf=dict(s=ZIPF_S, alpha=ZIPF_ALPHA),
                       roofline=dict(bound="tensor", kernel="pdx_moe_ffn_grouped tcgen05 (gather + 2x k_grouped_gemm)",
                                     achieved=tflops, unit="TFLOP/s", peak=pk["bf16_tflops_sustained"],
                                     frac=tflops / pk["bf16_tflops_sustained"],
                                     frac_of_burst=tflops / pk["bf16_tflops"], peak_source=pk["source"],
                                     flops_per_launch=flops_launch, us_per_launch=per_launch_p * 1e6))
        pstack.release_graphs()
        del pstack

    # ---- parity of the timed path (after the timed regions) ---------------------------
    # routing ids against the reference's own device route (F.linear/softmax/topk on this
    # GPU) over whole rows, and the graph-replayed step against the eager step
    from pdscope_b200.agreement import route_agreement
    parity = dict(route_vs_device_reference={})
    for t_count, zipf in ((1, False), (64, False), (512, False), (12450, True)):
        gate0 = stack.gates[0]
        if zipf:
            gen = torch.Generator(device=dev).manual_seed(4321)
            ranks_z = torch.randperm(CFG["experts"], device=dev, generator=gen).float() + 1
            gate0 = gate0.clone()
            gate0[:, 0] = (-ZIPF_ALPHA * ZIPF_S * torch.log(ranks_z)).to(torch.bfloat16)
        xa = activations(t_count, CFG["hidden"], device=dev, seed=600 + t_count, zipf=zipf)
        parity["route_vs_device_reference"][str(t_count)] = route_agreement(xa, gate0, CFG["top_k"], True)
    t_count = headline_t
    stack.input(t_count).copy_(activations(t_count, CFG["hidden"], device=dev, seed=606))
    stack.step(t_count, graph=False)
    eager_out = stack.output(t_count).clone()
    stack.step(t_count)
    torch.cuda.synchronize(dev)
    parity["graph_step_equals_eager_step"] = bool(torch.equal(stack.output(t_count), eager_out))

    # ---- CPU baseline (rank 0, N = 1 only) -------------------------------------------
    cpu = None
    if world == 1 and not args.no_cpu:
        cpu = cpu_baseline(headline_t, args.cpu_layers, args.cpu_threads)

    stack.release_graphs()
    if rank == 0:
        d = decode[headline_t]
        line = dict(metric=METRIC, value=d["tok_s"], unit="tok/s", n_gpus=world, steps=K, warmup=W,
                    ms_per_step=d["ms_per_step"], higher_is_better=True, scaling="weak", vs_baseline=None,
                    dtype="bf16", data="synthetic",
                    config=headline_config(args, 1)[0],
                    execution="all experts resident in HBM; one CUDA graph per 48-layer step",
                    roofline=roofline, cpu_baseline=cpu, e2e=e2e, clocks=d["clocks"],
                    gpu_launches=d["launches_per_step"] * K,
                    decode={str(t): {k: v for k, v in r.items() if k != "clocks"} for t, r in decode.items()},
                    prefill=prefill, config1_layer=config1, parity=parity)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_offload(args, dev, W, pk, L):
    """Config 4: the 48-layer stack with the process capped at 24 GiB of HBM,
    16 hot experts per layer (by Zipf rank, written and read back as a
    ``layer,expert`` hot file) resident, all other experts in pinned host memory
    and fetched by the copy engine; the gate-fallback predictor prefetches the
    next layer.  One request per prefill length (prefill, then single-token
    decode steps), as the reference's offload runs.  Host-link roofline: pinned
    H2D GB/s measured in the same process."""
    import tempfile
    import torch
    from pdscope_b200 import _lib
    from pdscope_b200.offload import (NativeOffloadMoEStack, OffloadMoEStack, PinnedHostBuffer, load_hot_file,
                                      measure_h2d_gbs, write_hot_file, zipf_hot_sets)
    from pdscope_b200.stack import activations, ZIPF_ALPHA, ZIPF_S

    H, E, I, k = CFG["hidden"], CFG["experts"], CFG["inter"], CFG["top_k"]
    per = EXPERT_BYTES // 2
    total = torch.cuda.get_device_properties(dev).total_memory
    cap = int(args.offload_cap_gib * 2 ** 30)
    torch.cuda.set_per_process_memory_fraction(min(1.0, cap / total), dev)
    link_gbs = measure_h2d_gbs(dev)
    torch.cuda.empty_cache()

    gen = torch.Generator(device=dev).manual_seed(0)
    host_buf = PinnedHostBuffer(L * E * per * 2)
    host = host_buf.tensor.view(torch.bfloat16).view(L, E, per)
    gates = []
    for l in range(L):
        gate = torch.randn(E, H, device=dev, generator=gen) * 0.02
        perm = torch.randperm(E, device=dev, generator=gen)
        ranks = torch.empty(E, device=dev)
        ranks[perm] = torch.arange(1, E + 1, device=dev, dtype=torch.float32)
        gate[:, 0] = -ZIPF_ALPHA * ZIPF_S * torch.log(ranks)
        gates.append(gate.to(torch.bfloat16))
        for e0 in range(0, E, 16):
            chunk = (torch.randn((16, per), device=dev, generator=gen) * 0.02).to(torch.bfloat16)
            host[l, e0:e0 + 16].copy_(chunk)
    del chunk
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    with tempfile.TemporaryDirectory() as td:
        hot_path = Path(td) / "hot_offload.txt"
        write_hot_file(hot_path, zipf_hot_sets(gates, E))          # full Zipf ranking, hottest first
        ranked = load_hot_file(hot_path, args.offload_hot + args.offload_warm, L)
    hot = [r[:args.offload_hot] for r in ranked]
    warm = [r[args.offload_hot:] for r in ranked]
    hot_bytes = sum(len(h) + len(w) for h, w in zip(hot, warm)) * EXPERT_BYTES
    reserve = int(1.5 * 2 ** 30)   # activations, packing and FFN workspace at the largest prefill
    free = cap - torch.cuda.memory_allocated(dev) - hot_bytes - reserve
    slots = max(E, free // EXPERT_BYTES)
    prefills = [int(v) for v in args.offload_prefills.split(",") if v.strip()]
    if args.offload_python:
        stack = OffloadMoEStack(gates, host, hot, hidden=H, inter=I, cache_slots=slots, top_k=k, warm=warm)
    else:
        stack = NativeOffloadMoEStack(gates, host, hot, hidden=H, inter=I, cache_slots=slots, top_k=k, warm=warm,
                                      max_tokens=max(prefills + [16]))

    n_dec = max(1, args.offload_decode_steps)
    for w in range(W):   # warm: tensor maps, device attributes, allocator
        stack.forward(activations(16 if w == 0 else 1, H, device=dev, seed=900 + w, zipf=True))
    torch.cuda.synchronize(dev)
    s = torch.cuda.current_stream(dev)

    def timed(inputs):
        before = stack.stats.as_dict()
        l0 = _lib.lib.pdx_launch_count()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for x in inputs:
            stack.forward(x)
        e1.record(s)
        torch.cuda.synchronize(dev)
        after = stack.stats.as_dict()
        d = {key: after[key] - before[key] for key in after}
        d["launches"] = _lib.lib.pdx_launch_count() - l0
        return e0.elapsed_time(e1) / 1e3, d

    requests = []
    with ClockSampler(dev.index or 0) as sampler:
        for r, P in enumerate(prefills):
            xp = activations(P, H, device=dev, seed=2000 + r, zipf=True)
            dec = [activations(1, H, device=dev, seed=3000 + 100 * r + i, zipf=True) for i in range(n_dec)]
            tp, dp = timed([xp])
            td_, dd = timed(dec)
            nonhot_uses = dd["expert_uses"] - dd["hot_hits"]
            requests.append(dict(
                prefill_tokens=P, prefill_s=tp, prefill_tok_s=P / tp,
                prefill_h2d_gb=dp["h2d_bytes"] / 1e9, prefill_h2d_gbs=dp["h2d_bytes"] / 1e9 / tp,
                prefill_link_frac=dp["h2d_bytes"] / 1e9 / tp / link_gbs,
                decode_steps=n_dec, decode_s=td_, decode_tok_s=n_dec / td_,
                decode_h2d_gb=dd["h2d_bytes"] / 1e9, decode_h2d_gbs=dd["h2d_bytes"] / 1e9 / td_,
                decode_link_frac=dd["h2d_bytes"] / 1e9 / td_ / link_gbs,
                decode_hot_hit_rate=dd["hot_hits"] / max(1, dd["expert_uses"]),
                decode_warm_hit_rate=dd["warm_hits"] / max(1, dd["expert_uses"]),
                decode_ring_hit_rate=dd["cache_hits"] / max(1, nonhot_uses - dd["warm_hits"]),
                decode_prefetch_used=dd["prefetch_used"], decode_prefetch_copies=dd["prefetch_copies"],
                decode_demand_copies=dd["demand_copies"], launches=dp["launches"] + dd["launches"]))
    clocks = sampler.summary()
    dec_vals = [q["decode_tok_s"] for q in requests]
    line = dict(metric="offload single-request decode tok/s (config 4), Qwen3-30B-A3B-shape MoE, 1 B200, "
                       "24 GiB HBM cap; host-link roofline",
                value=statistics.mean(dec_vals), unit="tok/s", n_gpus=1, steps=len(requests), warmup=W,
                ms_per_step=1e3 / statistics.mean(dec_vals), higher_is_better=True, scaling="weak",
                vs_baseline=None, dtype="bf16", data="synthetic",
                config=dict(workload="config4 offload: 48 layers, hot %d/layer by Zipf rank (+%d/layer static "
                                     "cache tier), rest in pinned host memory, prefills %s then %d decode steps "
                                     "each" % (args.offload_hot, args.offload_warm, prefills, n_dec),
                            orchestration="python" if args.offload_python else "native (pdx_offload_*)",
                            hbm_cap_gib=args.offload_cap_gib, hot_per_layer=args.offload_hot,
                            warm_per_layer=args.offload_warm, hot_and_warm_gib=hot_bytes / 2 ** 30,
                            cache_ring_slots=int(slots), cache_ring_gib=slots * EXPERT_BYTES / 2 ** 30,
                            host_gib=L * E * EXPERT_BYTES / 2 ** 30, zipf=dict(s=ZIPF_S, alpha=ZIPF_ALPHA),
                            value="mean decode tok/s over the requests"),
                roofline=dict(bound="host link", achieved=max(q["prefill_h2d_gbs"] for q in requests),
                              peak=link_gbs, unit="GB/s",
                              frac=max(q["prefill_h2d_gbs"] for q in requests) / link_gbs,
                              peak_source="pinned cudaMemcpyAsync H2D, 1 GiB, measured in this run",
                              traffic=None),
                requests=requests, clocks=clocks,
                gpu_launches=sum(q["launches"] for q in requests),
                reference_a100_for_context=dict(prefill_tok_s={"512": 343.92, "1024": 597.18, "2048": 1086.83,
                                                               "4096": 1671.54},
                                                decode_tok_s={"512": 7.984, "1024": 7.689, "2048": 7.902,
                                                              "4096": 7.765},
                                                note="whole model (attention + MoE) on A100 PCIe with kt CPU "
                                                     "experts; not like for like"))
    print(json.dumps(line), flush=True)
    if hasattr(stack, "close"):
        stack.close()
    del stack
    host_buf.close()
    return 0


def run_expert_parallel(args, rank, local_rank, world, dev, dist, K, W, pk, L):
    """N > 1: experts sharded 128/N per GPU (expert e on rank e // (128/N)),
    NCCL all-to-all dispatch/combine, one CUDA graph per decode step.

    ``--ep-shape 30b`` (default; the driver's scaling runs): the 48-layer
    Qwen3-30B-A3B stack, decode batch per rank fixed (weak scaling).
    ``--ep-shape 235b`` (config 5): Qwen3-235B-A22B shape (H=4096, I=1536,
    94 layers, as many as fit in HBM at 2 GPUs), decode batch 256 tokens in all
    (256/N per rank) and a Zipf(1.1) prefill of 16 sequences ~U[512, 4096]
    split over the ranks."""
    import torch
    from pdscope_b200 import _lib
    from pdscope_b200.expert_parallel import ExpertParallelStack, PeerExchange, TorchDistExchange
    from pdscope_b200.runtime import ExpertSlab
    from pdscope_b200.stack import activations, prefill_lengths, ZIPF_ALPHA, ZIPF_S

    big = args.ep_shape == "235b"
    E, k = CFG["experts"], CFG["top_k"]
    H, I = (4096, 1536) if big else (CFG["hidden"], CFG["inter"])
    expert_bytes = 3 * H * I * 2
    if E % world:
        raise SystemExit(f"{E} experts do not divide over {world} GPUs")
    el = E // world
    if big:
        L = ep_layers(args, world, H, I)             # leave ~30 GB of HBM for activations and workspaces
    g_gate = torch.Generator(device=dev).manual_seed(0)          # routers replicated on every rank
    g_w = torch.Generator(device=dev).manual_seed(1000 + rank)   # this rank's experts
    gates = []
    for _ in range(L):
        g = torch.randn(E, H, device=dev, generator=g_gate) * 0.02
        if big:   # Zipf(1.1) skew through hidden column 0 (used by the prefill; decode inputs keep it random)
            ranks = torch.randperm(E, device=dev, generator=g_gate).float() + 1
            g[:, 0] = -ZIPF_ALPHA * ZIPF_S * torch.log(ranks)
        gates.append(g.to(torch.bfloat16))
    slabs = [ExpertSlab.allocate(el, H, I, dev, generator=g_w) for _ in range(L)]
    if big:
        decode_sizes = [max(1, 256 // world)]
    else:
        decode_sizes = sorted(set(int(v) for v in args.decode_batches.split(",") if v.strip()) | {args.decode_batch})
    peer = None
    if args.ep_transport == "p2p":
        peer = PeerExchange(L, max(decode_sizes), world=world, rank=rank, local_experts=el, hidden=H, top_k=k,
                            device=dev)
    stack = ExpertParallelStack(gates, slabs, rank=rank, world=world, exchange=TorchDistExchange(), top_k=k,
                                peer=peer)
    torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def timed(fn, steps, warm):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            fn()
        e1.record(s)
        torch.cuda.synchronize(dev)
        dist.barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    decode = {}
    headline_t = max(1, 256 // world) if big else args.decode_batch
    batches = decode_sizes
    clocks = None
    for t_count in batches:
        x, _ = stack.io(t_count)
        x.copy_(activations(t_count, H, device=dev, seed=10 + t_count + 1000 * rank))
        n0 = _lib.lib.pdx_launch_count()
        stack.step(t_count)
        torch.cuda.synchronize(dev)
        launches = (_lib.lib.pdx_launch_count() - n0) // 2
        if t_count == headline_t:
            sampler = ClockSampler(local_rank)
            with sampler:
                ms = timed(lambda: stack.step(t_count), K, W)
            clocks = sampler.summary()
        else:
            ms = timed(lambda: stack.step(t_count), K, W)
        act = stack.local_active_experts()   # this rank's experts that received rows, per layer
        local_bytes = sum(act) * expert_bytes
        decode[t_count] = dict(ms_per_step=ms / K, tok_s=world * t_count * K / (ms / 1e3),
                               launches_per_step=launches,
                               local_active_experts_per_layer=statistics.mean(act),
                               local_weight_gb_per_step=local_bytes / 1e9,
                               hbm_gbs_step_per_gpu=local_bytes / 1e9 / (ms / K / 1e3))
        if peer is not None:
            # where a layer's time goes: eager layers (host launch gaps included) with CUDA events between the
            # exchange stages (max over ranks of each stage's mean)
            stages = stack.stage_times_us(t_count, layers=min(8, L), repeats=2)
            decode[t_count]["stage_us_per_layer_eager"] = {name: max_over_ranks(v) for name, v in sorted(stages.items())}
    t_count = headline_t
    x, y = stack.io(t_count)
    host_in = activations(t_count, H, device=dev, seed=5 + rank).cpu().pin_memory()
    host_out = torch.empty((t_count, H), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        x.copy_(host_in, non_blocking=True)
        stack.step(t_count)
        host_out.copy_(y, non_blocking=True)

    e2e_ms = timed(e2e_step, K, W)
    stack.release_graphs()

    prefill = None
    if big and not args.no_prefill:
        lengths = prefill_lengths(16, lo=512, hi=4096, seed=0)
        mine = lengths[rank::world]                    # sequences of this rank
        tp = sum(mine)
        xp = activations(tp, H, device=dev, seed=77 + rank, zipf=True)
        xin, _ = stack.io(tp)
        xin.copy_(xp)
        stack.step(tp, graph=False)                    # warm (exact exchange: one host sync per layer)
        ms = timed(lambda: stack.step(tp, graph=False), max(1, args.prefill_steps), 1)
        total = sum_over_ranks(tp)
        flops = total * k * 6 * H * I * L
        prefill = dict(tokens_total=int(total), lengths=lengths, tokens_this_rank=tp,
                       ms_per_step=ms / max(1, args.prefill_steps),
                       tok_s=total * max(1, args.prefill_steps) / (ms / 1e3),
                       tflops_per_gpu=flops / world / (ms / max(1, args.prefill_steps) / 1e3) / 1e12,
                       zipf=dict(s=ZIPF_S, alpha=ZIPF_ALPHA))
        prefill["frac_of_sustained_bf16"] = prefill["tflops_per_gpu"] / pk["bf16_tflops_sustained"]

    d = decode[headline_t]
    if rank == 0:
        config, scaling = headline_config(args, world)
        line = dict(metric=METRIC, value=d["tok_s"], unit="tok/s", n_gpus=world, steps=K, warmup=W,
                    ms_per_step=d["ms_per_step"], higher_is_better=True, scaling=scaling, vs_baseline=None,
                    dtype="bf16", data="synthetic", config=config,
                    execution=(f"expert parallel, {el} experts per GPU, dispatch/combine exchange over NVLink, "
                               f"one CUDA graph per step"),
                    roofline=dict(bound="hbm", kernel="whole expert-parallel decode step (weights of the local "
                                                      "experts that received rows / step time, per GPU)",
                                  achieved=d["hbm_gbs_step_per_gpu"], peak=pk["hbm_gbs"], unit="GB/s",
                                  frac=d["hbm_gbs_step_per_gpu"] / pk["hbm_gbs"], peak_source=pk["source"],
                                  traffic=None),
                    cpu_baseline=None,
                    e2e=dict(value=world * t_count * K / (e2e_ms / 1e3), unit="tok/s",
                             h2d_bytes_per_step=host_in.numel() * 2, d2h_bytes_per_step=host_out.numel() * 2,
                             ms_per_step=e2e_ms / K),
                    clocks=clocks, gpu_launches=d["launches_per_step"] * K,
                    decode={str(t): r for t, r in decode.items()}, prefill=prefill)
        line["exchange"] = ("NVLink peer stores + flags (pdx_ep_*_p2p)" if peer is not None
                            else "NCCL all-to-all")
        print(json.dumps(line), flush=True)
    stack.release_graphs()
    if peer is not None:
        peer.close()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
