"""A stack of HBM-resident MoE layers driven as one decode/prefill step.

``ResidentMoEStack`` owns every buffer a step needs (no allocation inside a
step) and can capture the whole multi-layer step as one CUDA graph, so the
per-layer host work of the reference (``.tolist()`` syncs in grouping,
pdscope_runtime.py:26, qwen.py:162,171, and one Python call chain per expert)
disappears from the step.  The activation of layer l+1 is
``layer_norm(MoE_l(x_l) + x_l)``, the reference's two-layer protocol
(pdscope_compare.py:609-705), fused into the combine kernel
(PDX_LAYER_OUT_NORM): it keeps every layer's input at unit scale, as
the synthetic configs specify (without it the random residual stream grows
layer by layer until the last layers compute on inf/NaN).

Also here: seeded synthetic workloads standing in for the BASELINE configs
(weights ~N(0, 0.02), activations ~N(0, 1); no checkpoint or dataset is used).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .runtime import LN_EPS, ExpertSlab, _ptr, _stream


@dataclass
class StageBuffers:
    """Per-layer device buffers of the staged (route / pack / FFN / combine) path."""
    logits: torch.Tensor
    selected: torch.Tensor
    weights: torch.Tensor
    counts: torch.Tensor
    offsets: torch.Tensor
    tokens: torch.Tensor
    positions: torch.Tensor
    packed_w: torch.Tensor
    inverse: torch.Tensor
    active: torch.Tensor


class ResidentMoEStack:
    """``layers`` MoE layers with all experts resident; one slab per layer."""

    def __init__(self, gates, slabs, top_k=8, normalize=True):
        if len(gates) != len(slabs) or not gates:
            raise ValueError("one router per expert slab is required")
        self.gates, self.slabs = list(gates), list(slabs)
        self.experts, self.hidden = self.gates[0].shape
        self.inter = self.slabs[0].inter
        self.top_k, self.normalize = top_k, normalize
        self.device = self.gates[0].device
        self._graphs = {}
        self._bufs = {}

    @property
    def num_layers(self):
        return len(self.gates)

    # -- buffers ----------------------------------------------------------------
    def buffers(self, t_count, mode=_lib.FFN_AUTO):
        key = (t_count, mode)
        b = self._bufs.get(key)
        if b is not None:
            return b
        dev, L, E, H, k = self.device, self.num_layers, self.experts, self.hidden, self.top_k
        bf, i32 = dict(dtype=torch.bfloat16, device=dev), dict(dtype=torch.int32, device=dev)
        # acts[0] is the step input (never overwritten); layers alternate acts[1], acts[2]
        acts = [torch.zeros((t_count, H), **bf) for _ in range(3)]
        n = t_count * k
        # every layer's expert counts in one [L, E] block, so one copy moves them all
        counts = torch.zeros((L, E), **i32)
        stages = [StageBuffers(logits=torch.empty((t_count, E), **bf),
                               selected=torch.empty((t_count, k), dtype=torch.int64, device=dev),
                               weights=torch.empty((t_count, k), **bf), counts=counts[l],
                               offsets=torch.empty(E + 1, **i32), tokens=torch.empty(n, **i32),
                               positions=torch.empty(n, **i32), packed_w=torch.empty(n, **bf),
                               inverse=torch.empty(n, **i32), active=torch.empty(E + 1, **i32))
                  for l in range(L)]
        rows = torch.empty((n, H), **bf)  # expert outputs of the current layer (staged path)
        ws_layer = lib.pdx_layer_workspace_bytes(t_count, H, E, k, self.inter, mode)
        ws_stage = max(lib.pdx_route_workspace_bytes(t_count, E), lib.pdx_pack_workspace_bytes(t_count, k, E),
                       lib.pdx_ffn_workspace_bytes(n, E, H, self.inter, mode))
        ws = torch.empty(max(ws_layer, ws_stage), dtype=torch.uint8, device=dev)
        b = dict(acts=acts, stages=stages, ws=ws, rows=rows, counts=counts,
                 counts_host=torch.zeros((L, E), dtype=torch.int32).pin_memory(), counts_ready=torch.cuda.Event())
        self._bufs[key] = b
        return b

    @staticmethod
    def _act_in(acts, l):
        return acts[0] if l == 0 else acts[1 + (l - 1) % 2]

    @staticmethod
    def _act_out(acts, l):
        return acts[1 + l % 2]

    # -- fused path: one C-ABI call per layer -------------------------------------
    def _step_fused(self, t_count, mode, counts_to_host=False):
        b = self.buffers(t_count, mode)
        acts, stages, ws = b["acts"], b["stages"], b["ws"]
        s = _stream()
        for l in range(self.num_layers):
            st = stages[l]
            x_in, x_out = self._act_in(acts, l), self._act_out(acts, l)
            check(lib.pdx_moe_layer(_ptr(x_in), _ptr(self.gates[l]), t_count, self.hidden, self.experts,
                                    self.top_k, int(self.normalize), ctypes.byref(self.slabs[l].struct), self.inter,
                                    _ptr(x_in), _ptr(x_out), _ptr(st.logits), _ptr(st.selected),
                                    _ptr(st.weights), _ptr(st.counts), mode | _lib.LAYER_OUT_NORM, _ptr(ws),
                                    ws.numel(), s))
        if counts_to_host:
            # one device-to-host copy of every layer's counts into pinned memory,
            # inside the step (and its graph): no per-layer host synchronisation
            b["counts_host"].copy_(b["counts"], non_blocking=True)

    # -- staged path: route, pack, FFN, combine as separate calls --------------------
    def route_and_pack(self, l, t_count, mode=_lib.FFN_AUTO):
        b = self.buffers(t_count, mode)
        st, ws, s = b["stages"][l], b["ws"], _stream()
        x = self._act_in(b["acts"], l)
        check(lib.pdx_route_topk(_ptr(x), _ptr(self.gates[l]), t_count, self.hidden, self.experts, self.top_k,
                                 int(self.normalize), _ptr(st.logits), _ptr(st.selected), _ptr(st.weights),
                                 _ptr(ws), ws.numel(), s))
        check(lib.pdx_pack(_ptr(st.selected), _ptr(st.weights), t_count, self.top_k, self.experts, _ptr(st.counts),
                           _ptr(st.offsets), _ptr(st.tokens), _ptr(st.positions), _ptr(st.packed_w),
                           _ptr(st.inverse), _ptr(st.active), _ptr(ws), ws.numel(), s))

    def ffn(self, l, t_count, mode=_lib.FFN_AUTO):
        b = self.buffers(t_count, mode)
        st, ws = b["stages"][l], b["ws"]
        n = t_count * self.top_k
        check(lib.pdx_moe_ffn_grouped(_ptr(self._act_in(b["acts"], l)), t_count, _ptr(st.tokens),
                                      _ptr(st.offsets), _ptr(st.active), self.experts, n,
                                      ctypes.byref(self.slabs[l].struct), self.hidden, self.inter, _ptr(b["rows"]),
                                      mode, _ptr(ws), ws.numel(), _stream()))

    def combine(self, l, t_count, mode=_lib.FFN_AUTO):
        """Weighted combine fused with the next-layer norm."""
        b = self.buffers(t_count, mode)
        st = b["stages"][l]
        x_in, x_out = self._act_in(b["acts"], l), self._act_out(b["acts"], l)
        check(lib.pdx_combine_layernorm(_ptr(b["rows"]), _ptr(st.weights), _ptr(st.inverse), t_count, self.top_k,
                                        self.hidden, _ptr(x_in), ctypes.c_float(LN_EPS), _ptr(x_out), _stream()))

    def _step_staged(self, t_count, mode):
        for l in range(self.num_layers):
            self.route_and_pack(l, t_count, mode)
            self.ffn(l, t_count, mode)
            self.combine(l, t_count, mode)

    # -- public step --------------------------------------------------------------------
    def input(self, t_count, mode=_lib.FFN_AUTO):
        return self.buffers(t_count, mode)["acts"][0]

    def output(self, t_count, mode=_lib.FFN_AUTO):
        return self._act_out(self.buffers(t_count, mode)["acts"], self.num_layers - 1)

    def step(self, t_count, mode=_lib.FFN_AUTO, *, graph=True, counts_to_host=False):
        """Run every layer on ``input(t_count)``; result in ``output(t_count)``.

        With ``counts_to_host`` the step ends with one asynchronous copy of every
        layer's routed-token counts into pinned host memory (``expert_counts``
        reads them once the step has finished)."""
        if not graph:
            self._step_fused(t_count, mode, counts_to_host)
        else:
            key = ("fused", t_count, mode, counts_to_host)
            g = self._graphs.get(key)
            if g is None:
                self._step_fused(t_count, mode, counts_to_host)  # warm: device attributes, tensor maps
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._step_fused(t_count, mode, counts_to_host)
                self._graphs[key] = g
            g.replay()
        if counts_to_host:
            self.buffers(t_count, mode)["counts_ready"].record()

    def expert_counts(self, t_count, mode=_lib.FFN_AUTO):
        """[L, E] int32 pinned host tensor of the last ``step(..., counts_to_host=True)``:
        waits for that step's copy (not for the whole device).  Valid until the
        next such step."""
        b = self.buffers(t_count, mode)
        b["counts_ready"].synchronize()
        return b["counts_host"]

    def ffn_graph(self, t_count, mode=_lib.FFN_AUTO):
        """CUDA graph of the grouped FFN of every layer on the current packing."""
        key = ("ffn", t_count, mode)
        g = self._graphs.get(key)
        if g is None:
            for l in range(self.num_layers):
                self.ffn(l, t_count, mode)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for l in range(self.num_layers):
                    self.ffn(l, t_count, mode)
            self._graphs[key] = g
        return g

    def stage_once(self, t_count, mode=_lib.FFN_AUTO):
        """One staged step (fills every layer's packing for ffn_graph)."""
        self._step_staged(t_count, mode)

    def stage_times_us(self, t_count, mode=_lib.FFN_AUTO, layers=8, repeats=3):
        """Mean device time per layer of each stage of the staged path, from CUDA
        events on the current stream: route (logits + top-k), pack, FFN, combine
        (with the stack's next-layer norm fused in)."""
        b = self.buffers(t_count, mode)
        st_ws, s = b["ws"], _stream()
        names = ("route", "pack", "ffn", "combine")
        tot = dict.fromkeys(names, 0.0)
        n = 0
        for _ in range(repeats):
            for l in range(min(layers, self.num_layers)):
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
                st = b["stages"][l]
                x = self._act_in(b["acts"], l)
                ev[0].record()
                check(lib.pdx_route_topk(_ptr(x), _ptr(self.gates[l]), t_count, self.hidden, self.experts,
                                         self.top_k, int(self.normalize), _ptr(st.logits), _ptr(st.selected),
                                         _ptr(st.weights), _ptr(st_ws), st_ws.numel(), s))
                ev[1].record()
                check(lib.pdx_pack(_ptr(st.selected), _ptr(st.weights), t_count, self.top_k, self.experts,
                                   _ptr(st.counts), _ptr(st.offsets), _ptr(st.tokens), _ptr(st.positions),
                                   _ptr(st.packed_w), _ptr(st.inverse), _ptr(st.active), _ptr(st_ws),
                                   st_ws.numel(), s))
                ev[2].record()
                self.ffn(l, t_count, mode)
                ev[3].record()
                self.combine(l, t_count, mode)
                ev[4].record()
                torch.cuda.synchronize(self.device)
                for i, name in enumerate(names):
                    tot[name] += ev[i].elapsed_time(ev[i + 1]) * 1e3
                n += 1
        return {name: tot[name] / n for name in names}

    def release_graphs(self):
        self._graphs.clear()


class ExpertLoadTracker:
    """Routed-token totals per (layer, expert), fed from the pinned count
    copies of ``ResidentMoEStack.step(..., counts_to_host=True)``.

    The reference derives its static hot table (hot/qwen.txt, read by
    load_hot_profile, expertbench/pdscope_runtime.py:62-72, which fixes the
    resident set AdaptSched plans around) from a routing profile of this
    kind; ``hot_sets`` / ``write_hot_file`` turn the totals into that table,
    hottest first with ties to the lower expert id.
    """

    def __init__(self, layers, experts):
        self.totals = np.zeros((layers, experts), np.int64)
        self.steps = 0

    def add(self, counts):
        self.totals += np.asarray(counts.numpy() if hasattr(counts, "numpy") else counts, dtype=np.int64)
        self.steps += 1

    def hot_sets(self, per_layer):
        order = np.argsort(-self.totals, axis=1, kind="stable")
        return [order[l, :per_layer].tolist() for l in range(self.totals.shape[0])]

    def write_hot_file(self, path, per_layer):
        from .offload import write_hot_file
        write_hot_file(path, self.hot_sets(per_layer))


# ---------------------------------------------------------------------------
# Synthetic workloads (seeded, no checkpoint or dataset)
# ---------------------------------------------------------------------------

QWEN3_30B = dict(hidden=2048, experts=128, inter=768, top_k=8, layers=48)
QWEN3_235B = dict(hidden=4096, experts=128, inter=1536, top_k=8, layers=94)

# Zipf(s=1.1) router skew: a dedicated hidden coordinate carries a constant
# activation and gate[e, 0] = -ALPHA * s * log(rank_e), so the logits gain a
# per-expert offset without changing route() itself.
ZIPF_S = 1.1
ZIPF_ALPHA = 0.75  # top-16 experts take ~75% of assignments (measured and reported by bench.py)


def build_stack(layers, hidden, experts, inter, top_k=8, device="cuda", seed=0, zipf=False):
    gen = torch.Generator(device=device).manual_seed(seed)
    gates, slabs = [], []
    for l in range(layers):
        gate = torch.randn(experts, hidden, device=device, generator=gen) * 0.02
        if zipf:
            perm = torch.randperm(experts, device=device, generator=gen)
            ranks = torch.empty(experts, device=device)
            ranks[perm] = torch.arange(1, experts + 1, device=device, dtype=torch.float32)
            gate[:, 0] = -ZIPF_ALPHA * ZIPF_S * torch.log(ranks)
        gates.append(gate.to(torch.bfloat16))
        slabs.append(ExpertSlab.allocate(experts, hidden, inter, device, generator=gen))
    return ResidentMoEStack(gates, slabs, top_k=top_k)


def prefill_lengths(count=8, lo=256, hi=4096, seed=0):
    """Ragged prefill batch: ``count`` sequence lengths ~U[lo, hi] (seeded)."""
    rng = np.random.default_rng(seed)
    return [int(v) for v in rng.integers(lo, hi + 1, size=count)]


def activations(t_count, hidden, device="cuda", seed=1, zipf=False):
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(t_count, hidden, device=device, generator=gen)
    if zipf:
        x[:, 0] = 1.0
    return x.to(torch.bfloat16)


def expert_bytes(hidden, inter):
    return 3 * hidden * inter * 2
