"""B200 per-expert cost table in the reference's ``pdscope_cost_table`` schema.

AdaptSched (expertbench/pdscope_policy.py) plans placement from a table of
per-expert completion times by routed token count, read by ``FileCosts``
(benchmarks/pdscope_compare.py:55-85; shipped table costs/cost_table.json,
measured on an A100 PCIe).  This module measures the same three columns on a
B200 so the policy makes B200-appropriate decisions unchanged:

* ``gpu_ms``  what one more resident expert with n routed rows adds to a
              layer on the B200: one grouped FFN launch (``pdx_moe_ffn_grouped``,
              row gather + the tcgen05 GEMMs) over G experts of n rows each,
              divided by G.  The reference runs one cuBLAS chain per expert, so
              its per-expert time is a whole launch; here experts share one
              launch and each costs its weight stream (about 1.5 us at one
              token) or its tensor-core time.  The time of a lone single-expert
              launch (``pdx_expert_ffn``, the gpu_backend hook) is kept as
              ``gpu_single_launch_ms``;
* ``h2d_ms``  one expert's 9 MiB gate|up|down slot from pinned host memory on
              a dedicated copy stream (the executor's load path, executor.py:333-372);
* ``cpu_ms``  the reference's CPU expert path without kt (``ExpertExecutor.cpu``
              with cpu_backend=None -> torch CPU ``expert_forward``,
              executor.py:513-530), on all host cores.

    python -m pdscope_b200.costs --out pdscope_b200/cost_table_b200.json

``TableCosts`` reads a table as FileCosts does (exact points, linear
interpolation inside the 1..4096 domain) for callers without the
reference's harness module.
"""
from __future__ import annotations

import argparse
import bisect
import ctypes
import json
import os
import statistics
import time
from pathlib import Path

import torch

LOADS = (1, 4, 16, 64, 128, 256, 1024, 4096)   # FileCosts requires the 1..4096 domain
DEFAULT_TABLE = Path(__file__).resolve().parent / "cost_table_b200.json"


class TableCosts:
    """``for_load(n)`` over a pdscope_cost_table file, as FileCosts computes it
    (benchmarks/pdscope_compare.py:55-85): the measured point at n, else the
    linear interpolation between the two measured loads around n; loads
    outside the measured domain raise ValueError."""

    def __init__(self, path=DEFAULT_TABLE):
        payload = json.loads(Path(path).read_text())
        self.loads = validate(payload)
        self.points = {int(n): {k: float(v) for k, v in p.items()} for n, p in payload["points"].items()}
        self.path = str(path)

    def for_load(self, n):
        if not self.loads[0] <= n <= self.loads[-1]:
            raise ValueError("expert load outside the measured domain")
        if n in self.points:
            return dict(tokens=n, **self.points[n])
        hi = bisect.bisect_left(self.loads, n)
        lo, up = self.loads[hi - 1], self.loads[hi]
        r = (n - lo) / (up - lo)
        return dict(tokens=n, **{k: self.points[lo][k] + r * (self.points[up][k] - self.points[lo][k])
                                 for k in self.points[lo]})


def _median_ms(fn, repeats, stream):
    times = []
    for _ in range(repeats):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        stream.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def _grouped_ms_per_expert(n, hidden, inter, experts, repeats, dev, gen, slab):
    """One grouped FFN launch over ``experts`` experts with n rows each (the
    layer's gather + GEMMs), its median time divided by the expert count."""
    from . import _lib
    rows = n * experts
    x = torch.randn((rows, hidden), device=dev, generator=gen).to(torch.bfloat16)
    tokens = torch.arange(rows, dtype=torch.int32, device=dev)
    offsets = (torch.arange(experts + 1, dtype=torch.int32, device=dev) * n).contiguous()
    active = torch.cat([torch.tensor([experts], dtype=torch.int32),
                        torch.arange(experts, dtype=torch.int32)]).to(dev)
    y = torch.empty((rows, hidden), dtype=torch.bfloat16, device=dev)
    ws = torch.empty(_lib.lib.pdx_ffn_workspace_bytes(rows, experts, hidden, inter, _lib.FFN_AUTO),
                     dtype=torch.uint8, device=dev)
    comp = torch.cuda.current_stream(dev)
    s = ctypes.c_void_p(comp.cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())

    def launch():
        _lib.check(_lib.lib.pdx_moe_ffn_grouped(p(x), rows, p(tokens), p(offsets), p(active), experts, rows,
                                                ctypes.byref(slab.struct), hidden, inter, p(y), _lib.FFN_AUTO,
                                                p(ws), ws.numel(), s))
    for _ in range(3):
        launch()
    return _median_ms(launch, repeats, comp) / experts


def calibrate(device="cuda", hidden=2048, inter=768, loads=LOADS, repeats=20, cpu_threads=0, cpu_repeats=2,
              seed=0, experts=128):
    from .runtime import ExpertSlab, expert_forward
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    slab = ExpertSlab.allocate(experts, hidden, inter, dev, generator=gen)
    w = slab.expert_tensors(0)
    w_cpu = {k: v.cpu() for k, v in w.items()}
    slot_bytes = 3 * hidden * inter * 2
    host = torch.empty(slot_bytes, dtype=torch.uint8).pin_memory()
    slot = torch.empty(slot_bytes, dtype=torch.uint8, device=dev)
    copy_stream = torch.cuda.Stream(device=dev)
    comp = torch.cuda.current_stream(dev)
    threads = cpu_threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)

    def h2d():
        with torch.cuda.stream(copy_stream):
            slot.copy_(host, non_blocking=True)

    # device columns first, before any CPU work (host threads left spinning by
    # the CPU matmuls disturb the copy timings)
    h2d()
    dev_ms = {}
    for n in loads:
        x = torch.randn((n, hidden), device=dev, generator=gen).to(torch.bfloat16)
        for _ in range(3):
            expert_forward(x, w)
        single = _median_ms(lambda: expert_forward(x, w), repeats, comp)
        grouped = _grouped_ms_per_expert(n, hidden, inter, experts, max(5, repeats // 2), dev, gen, slab)
        dev_ms[n] = (x, grouped, single, _median_ms(h2d, repeats, copy_stream))
    points = {}
    for n in loads:
        x, grouped, single, h2d_ms = dev_ms[n]
        xc = x.cpu()
        g, u, d = w_cpu["gate_proj"], w_cpu["up_proj"], w_cpu["down_proj"]

        def cpu_expert():   # qwen.py:87-90 on torch CPU tensors
            h = torch.nn.functional.silu(torch.nn.functional.linear(xc, g)) * torch.nn.functional.linear(xc, u)
            return torch.nn.functional.linear(h, d)
        cpu_expert()
        ct = []
        for _ in range(cpu_repeats):
            t0 = time.perf_counter()
            cpu_expert()
            ct.append((time.perf_counter() - t0) * 1e3)
        points[str(n)] = dict(cpu_ms=round(statistics.median(ct), 6), gpu_ms=round(grouped, 6),
                              h2d_ms=round(h2d_ms, 6), gpu_single_launch_ms=round(single, 6))
    props = torch.cuda.get_device_properties(dev)
    try:
        cpu_model = next((l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name")),
                         "")
    except OSError:
        cpu_model = ""
    return {
        "schema_version": 1,
        "kind": "pdscope_cost_table",
        "model": f"Qwen3-30B-A3B-shape expert (H={hidden}, I={inter}) BF16, random-init weights",
        "platform": f"{props.name} ({props.multi_processor_count} SMs) + {cpu_model}",
        "native_operator": "none: cpu_ms is torch CPU expert_forward (the cpu_backend=None path); "
                           f"gpu_ms is one grouped pdx_moe_ffn_grouped launch over {experts} experts divided by "
                           f"{experts} (sm_100a tcgen05 kernels); gpu_single_launch_ms is pdx_expert_ffn alone",
        "workers": threads,
        "loads": list(loads),
        "points": points,
        "scope": "per-expert completion time by routed token count: CPU torch, resident GPU (libpdx_moe, "
                 "marginal per expert in a grouped launch), pinned host->device copy of one 9 MiB expert slot "
                 "on a copy stream",
    }


def validate(table):
    """The checks FileCosts applies (pdscope_compare.py:62-71)."""
    if table.get("kind") != "pdscope_cost_table":
        raise ValueError("cost table file has an unexpected kind")
    loads = sorted(int(n) for n in table["points"])
    if loads[0] != 1 or loads[-1] != 4096:
        raise ValueError("cost table must cover the measured 1..4096 domain")
    for n, p in table["points"].items():
        for key in ("cpu_ms", "gpu_ms", "h2d_ms"):
            if not float(p[key]) > 0:
                raise ValueError(f"load {n}: {key} must be positive")
    return loads


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", required=True)
    ap.add_argument("--repeats", type=int, default=20)
    ap.add_argument("--cpu-threads", type=int, default=0)
    args = ap.parse_args()
    table = calibrate(repeats=args.repeats, cpu_threads=args.cpu_threads)
    validate(table)
    with open(args.out, "w") as f:
        json.dump(table, f, indent=2)
        f.write("\n")
    print(json.dumps(table["points"]))


if __name__ == "__main__":
    main()
