"""Offload mode: a per-layer hot set resident in HBM, every other expert in
pinned host memory, fetched over the host link by the copy engine.

Reference path being replaced (nezha-Anonymous/PDScope):
  * ExpertExecutor.load / finish_load            expertbench/executor.py:333-390
    (H2D copy of one expert's three tensors into a cache or staging slot on a
    load stream; completion gated by an event)
  * demand pipeline                              expertbench/pdscope_runtime.py:361-383
  * next-layer prefetch                          expertbench/pdscope_runtime.py:392-399
  * gate-fallback predictor                      expertbench/pdscope_runtime.py:245-249
    (route the CURRENT activation with the NEXT layer's gate)
  * the hot table                                load_hot_profile, pdscope_runtime.py:62-72

B200 design.  One device slot pool = [hot slots of every layer | cache ring].
Each expert slot holds gate_proj | up_proj | down_proj back to back (the
reference's cache-slot layout, executor.py:323-331), so one expert is ONE
contiguous 9 MiB copy.  Per layer:

1. route + pack with this layer's gate, and route + pack of the same
   activation with the next layer's gate (the predictor); both expert-count
   vectors come back in one pinned device-to-host copy and one host sync
   (the reference syncs once per layer for grouping, pdscope_runtime.py:26);
2. hot experts use their fixed slots; experts already in the cache ring
   (earlier demand or prefetch) use theirs; the rest are demand-copied on the
   copy-engine stream, in chunks;
3. the next layer's predicted experts are queued on the same copy stream
   right after this layer's demand copies, so the copy engine keeps streaming
   while this layer computes and while the host waits for the next routing;
4. the grouped FFN runs as one launch over the ready experts, then one launch
   per demand chunk, each waiting only for its own chunk's copy event, so
   copies and tensor-core work overlap chunk by chunk; one combine at the end.

A cache slot is overwritten only after the event of its last reader
completed, and never while the current layer holds it (the reference's
"complete only after the event" rule, expertbench/cache.py:1-6, and its
live-consumer assertion, pdscope_runtime.py:376-377).
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import ExpertWeights, check, lib
from .runtime import LN_EPS, _ptr, _stream


@dataclass
class SlotState:
    key: tuple | None = None       # (layer, expert) held, or None
    ready: object = None           # event: the copy into the slot finished
    last_use: object = None        # event: the last compute that read the slot finished
    prefetched: bool = False       # filled by the predictor and not yet read


class CacheRing:
    """LRU assignment of device cache slots to (layer, expert) keys.

    Host bookkeeping only (events are opaque objects handed in and out).  A
    slot held by the current layer (``pinned``) is never evicted; an evicted
    slot is returned with the event its new copy must wait for (its last
    reader), so a copy never overwrites weights a kernel may still read."""

    def __init__(self, n_slots):
        if n_slots < 1:
            raise ValueError("offload needs at least one cache slot")
        self.slots = [SlotState() for _ in range(n_slots)]
        self.where = {}                                        # key -> slot index
        self.lru = OrderedDict((i, None) for i in range(n_slots))  # least recently used first

    def __len__(self):
        return len(self.slots)

    def lookup(self, key):
        return self.where.get(key)

    def touch(self, idx):
        self.lru.move_to_end(idx)

    def acquire(self, key, pinned):
        """Slot for ``key`` outside ``pinned``: (index, last reader event of its
        previous content, whether that content was an unread prefetch)."""
        if key in self.where:
            raise ValueError(f"{key} already has a cache slot")
        for idx in self.lru:
            if idx in pinned:
                continue
            st = self.slots[idx]
            if st.key is not None:
                del self.where[st.key]
            prev, wasted = st.last_use, st.key is not None and st.prefetched
            st.key, st.ready, st.last_use, st.prefetched = key, None, None, False
            self.where[key] = idx
            self.lru.move_to_end(idx)
            return idx, prev, wasted
        raise RuntimeError("every cache slot is held by the current layer; enlarge the cache ring")


@dataclass
class OffloadStats:
    """Ledger counters (the reference's ``h2d_bytes_completed`` and hit accounting)."""
    h2d_bytes: int = 0
    demand_copies: int = 0
    prefetch_copies: int = 0
    prefetch_used: int = 0         # prefetched slots later read by their layer
    prefetch_wasted: int = 0       # prefetched slots evicted unread
    cache_hits: int = 0            # non-hot experts found in the ring (any origin)
    hot_hits: int = 0
    warm_hits: int = 0             # static-tier experts (fixed cache slots)
    expert_uses: int = 0           # (layer, expert) pairs computed
    layers: int = 0

    def as_dict(self):
        return dict(self.__dict__)


def zipf_hot_sets(gates, count):
    """The ``count`` experts of each layer with the largest router offset on
    the Zipf coordinate (hidden column 0), hottest first: a hot table by Zipf
    rank (the order a hot file lists them in)."""
    out = []
    for g in gates:
        bias = g[:, 0].float().cpu()
        out.append(torch.argsort(bias, descending=True, stable=True)[:count].tolist())
    return out


def write_hot_file(path, hot):
    """Hot table in the reference's text format (hot/qwen.txt, read by
    load_hot_profile, pdscope_runtime.py:62-72): one ``layer,expert`` row per
    line, no header, hottest first across layers -- rank 0 of every layer,
    then rank 1, ... -- so that a global budget of the first N rows spreads
    over the layers."""
    with open(path, "w") as f:
        for r in range(max((len(h) for h in hot), default=0)):
            for l, hs in enumerate(hot):
                if r < len(hs):
                    f.write(f"{l},{hs[r]}\n")


def load_hot_file(path, per_layer, layers):
    """First ``per_layer`` rows of each layer of a ``layer,expert`` hot file."""
    hot = [[] for _ in range(layers)]
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line or not line[0].isdigit():
                continue
            l, e = (int(v) for v in line.split(","))
            if l < layers and len(hot[l]) < per_layer:
                hot[l].append(e)
    return hot


class OffloadMoEStack:
    """MoE layers whose experts live in pinned host memory, except a hot set.

    ``gates``: list of [E, H] BF16 CUDA routers.  ``host_experts``: pinned CPU
    BF16 tensor [L, E, 3*I*H] (per expert gate_proj | up_proj | down_proj).
    ``hot``: per layer, the expert ids kept resident.  ``warm``: optional, per
    layer, further experts given fixed cache slots (a static cache tier, the
    reference's 'static' ExpertCache policy, filled from the next rows of the
    hot table); they are copies of host experts, never evicted.
    ``cache_slots``: size of the LRU cache ring (demand + prefetch + reuse).
    ``chunk``: demand experts per FFN launch.
    """

    def __init__(self, gates, host_experts, hot, *, hidden, inter, cache_slots, top_k=8, normalize=True,
                 prefetch=True, chunk=16, warm=None):
        self.gates = list(gates)
        self.L = len(self.gates)
        self.E = self.gates[0].shape[0]
        self.H, self.I, self.k, self.normalize = hidden, inter, top_k, normalize
        if host_experts.device.type != "cpu" or not host_experts.is_pinned():
            raise ValueError("host experts must be a pinned CPU tensor (copy-engine transfers)")
        if host_experts.dtype != torch.bfloat16 or tuple(host_experts.shape) != (self.L, self.E, 3 * inter * hidden):
            raise ValueError("host experts must be BF16 [layers, experts, 3*inter*hidden]")
        self.host = host_experts
        self.per = 3 * inter * hidden
        self.dev = self.gates[0].device
        self.hot = [list(h) for h in hot]
        self.warm = [list(w) for w in warm] if warm is not None else [[] for _ in range(self.L)]
        n_hot = sum(len(h) for h in self.hot)
        n_fixed = n_hot + sum(len(w) for w in self.warm)
        self.pool = torch.empty((n_fixed + cache_slots) * self.per, dtype=torch.bfloat16, device=self.dev)
        self.hot_slot, self.warm_keys = {}, set()
        s = 0
        for l in range(self.L):
            for e in self.hot[l] + self.warm[l]:
                if (l, e) in self.hot_slot:
                    raise ValueError(f"expert {e} of layer {l} listed twice in the hot/warm tiers")
                self.hot_slot[(l, e)] = s
                if e in self.warm[l]:
                    self.warm_keys.add((l, e))
                self.pool[s * self.per:(s + 1) * self.per].copy_(self.host[l, e])
                s += 1
        self.ring0 = n_fixed
        n_hot = n_fixed
        self.ring = CacheRing(cache_slots)
        self.copy_stream = torch.cuda.Stream(device=self.dev)
        self.prefetch, self.chunk = prefetch, max(1, chunk)
        self.stats = OffloadStats()
        base = self.pool.data_ptr()
        self._weights = dict(gate=base, up=base + inter * hidden * 2, down=base + 2 * inter * hidden * 2,
                             gate_stride=self.per, up_stride=self.per, down_stride=self.per,
                             num_slots=n_hot + cache_slots)
        i32 = dict(dtype=torch.int32)
        # slot tables and active lists: host staging (pinned) + device copies.
        # Rewritten only after the per-layer host sync, when earlier copies out of
        # them have completed.
        self.table_host = torch.zeros((self.L, self.E), **i32).pin_memory()
        self.table_dev = torch.zeros((self.L, self.E), **i32, device=self.dev)
        self.max_launch = 1 + -(-self.E // self.chunk)
        self.active_host = torch.zeros((self.max_launch, self.E + 1), **i32).pin_memory()
        self.active_dev = torch.zeros((self.max_launch, self.E + 1), **i32, device=self.dev)
        self.counts_host = torch.zeros((2, self.E), **i32).pin_memory()
        self._bufs = {}
        torch.cuda.synchronize(self.dev)

    # ---- buffers (grow-free per token count) ------------------------------------------
    def _buffers(self, t):
        b = self._bufs.get(t)
        if b is not None:
            return b
        dev, E, H, k = self.dev, self.E, self.H, self.k
        bf, i32 = dict(dtype=torch.bfloat16, device=dev), dict(dtype=torch.int32, device=dev)
        n = t * k

        def routing():
            return dict(logits=torch.empty((t, E), **bf), sel=torch.empty((t, k), dtype=torch.int64, device=dev),
                        w=torch.empty((t, k), **bf), offsets=torch.empty(E + 1, **i32),
                        tokens=torch.empty(n, **i32), positions=torch.empty(n, **i32),
                        packed_w=torch.empty(n, **bf), inverse=torch.empty(n, **i32),
                        active=torch.empty(E + 1, **i32))
        counts = torch.empty((2, E), **i32)
        ws = max(lib.pdx_route_workspace_bytes(t, E), lib.pdx_pack_workspace_bytes(t, k, E),
                 lib.pdx_ffn_workspace_bytes(n, E, H, self.I, _lib.FFN_AUTO))
        b = dict(cur=routing(), nxt=routing(), counts=counts, rows=torch.empty((n, H), **bf),
                 acts=[torch.empty((t, H), **bf) for _ in range(2)],
                 ws=torch.empty(ws, dtype=torch.uint8, device=dev))
        self._bufs[t] = b
        return b

    # ---- device steps ---------------------------------------------------------------
    def _route_pack(self, x, gate, r, counts, ws):
        t = x.shape[0]
        s = _stream()
        check(lib.pdx_route_topk(_ptr(x), _ptr(gate), t, self.H, self.E, self.k, int(self.normalize),
                                 _ptr(r["logits"]), _ptr(r["sel"]), _ptr(r["w"]), _ptr(ws), ws.numel(), s))
        check(lib.pdx_pack(_ptr(r["sel"]), _ptr(r["w"]), t, self.k, self.E, _ptr(counts), _ptr(r["offsets"]),
                           _ptr(r["tokens"]), _ptr(r["positions"]), _ptr(r["packed_w"]), _ptr(r["inverse"]),
                           _ptr(r["active"]), _ptr(ws), ws.numel(), s))

    def _ffn(self, l, x, r, active_row, rows, ws):
        t = x.shape[0]
        wt = ExpertWeights(slot_of_expert=self.table_dev[l].data_ptr(), **self._weights)
        check(lib.pdx_moe_ffn_grouped(_ptr(x), t, _ptr(r["tokens"]), _ptr(r["offsets"]),
                                      _ptr(self.active_dev[active_row]), self.E, t * self.k, ctypes.byref(wt),
                                      self.H, self.I, _ptr(rows), _lib.FFN_AUTO, _ptr(ws), ws.numel(), _stream()))

    # ---- copies -----------------------------------------------------------------------
    def _copy_in(self, key, pinned, prefetched):
        idx, prev, wasted = self.ring.acquire(key, pinned)
        if wasted:
            self.stats.prefetch_wasted += 1
        slot = self.ring0 + idx
        l, e = key
        cs = self.copy_stream
        if prev is not None:
            cs.wait_event(prev)   # the slot's last reader must finish first
        with torch.cuda.stream(cs):
            self.pool[slot * self.per:(slot + 1) * self.per].copy_(self.host[l, e], non_blocking=True)
        st = self.ring.slots[idx]
        st.prefetched = prefetched
        self.stats.h2d_bytes += self.per * 2
        if prefetched:
            self.stats.prefetch_copies += 1
        else:
            self.stats.demand_copies += 1
        return idx

    def _mark_ready(self, idxs):
        ev = torch.cuda.Event()
        ev.record(self.copy_stream)
        for i in idxs:
            self.ring.slots[i].ready = ev
        return ev

    # ---- one layer --------------------------------------------------------------------
    def forward_layer(self, l, x, out, residual=None, norm=False):
        """out = residual + MoE_l(x) (residual may be None), or with ``norm``
        layer_norm(MoE_l(x) + residual), the stack's next-layer activation."""
        t = x.shape[0]
        b = self._buffers(t)
        comp = torch.cuda.current_stream(self.dev)
        ws = b["ws"]
        cur, nxt = b["cur"], b["nxt"]
        predict = self.prefetch and l + 1 < self.L
        self._route_pack(x, self.gates[l], cur, b["counts"][0], ws)
        if predict:
            self._route_pack(x, self.gates[l + 1], nxt, b["counts"][1], ws)
        self.counts_host.copy_(b["counts"], non_blocking=True)
        comp.synchronize()   # the per-layer grouping sync
        counts = self.counts_host.numpy()
        needed = np.nonzero(counts[0])[0].tolist()
        self.stats.layers += 1
        self.stats.expert_uses += len(needed)

        pinned, ready, waits, demand = set(), [], [], []
        table = self.table_host[l].numpy()
        for e in needed:
            hs = self.hot_slot.get((l, e))
            if hs is not None:
                table[e] = hs
                ready.append(e)
                if (l, e) in self.warm_keys:
                    self.stats.warm_hits += 1
                else:
                    self.stats.hot_hits += 1
                continue
            idx = self.ring.lookup((l, e))
            if idx is not None:
                st = self.ring.slots[idx]
                self.stats.cache_hits += 1
                if st.prefetched:
                    self.stats.prefetch_used += 1
                    st.prefetched = False
                self.ring.touch(idx)
                pinned.add(idx)
                table[e] = self.ring0 + idx
                ready.append(e)
                if st.ready is not None:
                    waits.append(st.ready)
                continue
            demand.append(e)
        # demand copies, one event per chunk
        chunks = []
        for c0 in range(0, len(demand), self.chunk):
            part = demand[c0:c0 + self.chunk]
            idxs = []
            for e in part:   # each slot joins the live set at once: a later copy cannot take it
                idxs.append(self._copy_in((l, e), pinned, prefetched=False))
                pinned.add(idxs[-1])
            for e, i in zip(part, idxs):
                table[e] = self.ring0 + i
            chunks.append((part, self._mark_ready(idxs)))
        # predicted experts of the next layer, queued behind the demand copies
        if predict:
            issued = []
            for e in np.nonzero(counts[1])[0].tolist():
                key = (l + 1, e)
                if key in self.hot_slot or self.ring.lookup(key) is not None:
                    continue
                if len(pinned) + len(issued) >= len(self.ring):
                    break
                issued.append(self._copy_in(key, pinned | set(issued), prefetched=True))
            if issued:
                self._mark_ready(issued)
        # active lists: row 0 = ready experts, row 1+c = demand chunk c
        act = self.active_host.numpy()
        lists = [ready] + [p for p, _ in chunks]
        for i, lst in enumerate(lists):
            act[i, 0] = len(lst)
            act[i, 1:1 + len(lst)] = lst
        self.table_dev[l].copy_(self.table_host[l], non_blocking=True)
        self.active_dev[:len(lists)].copy_(self.active_host[:len(lists)], non_blocking=True)
        for ev in waits:
            comp.wait_event(ev)
        rows = b["rows"]
        if ready:
            self._ffn(l, x, cur, 0, rows, ws)
        for c, (_, ev) in enumerate(chunks):
            comp.wait_event(ev)
            self._ffn(l, x, cur, 1 + c, rows, ws)
        if norm:
            check(lib.pdx_combine_layernorm(_ptr(rows), _ptr(cur["w"]), _ptr(cur["inverse"]), t, self.k, self.H,
                                            _ptr(residual), ctypes.c_float(LN_EPS), _ptr(out), _stream()))
        else:
            check(lib.pdx_combine(_ptr(rows), _ptr(cur["w"]), _ptr(cur["inverse"]), t, self.k, self.H,
                                  _ptr(residual), _ptr(out), _stream()))
        done = torch.cuda.Event()
        done.record(comp)
        for idx in pinned:
            self.ring.slots[idx].last_use = done
        return out

    def forward(self, x):
        """Every layer on ``x`` [T, H]; layer l+1's input is
        layer_norm(MoE_l(x_l) + x_l) (the next-layer activation of the resident
        stack).  Returns a buffer owned by the stack (valid until the next call
        with the same token count)."""
        b = self._buffers(x.shape[0])
        h = x
        for l in range(self.L):
            out = b["acts"][l % 2]
            self.forward_layer(l, h, out, residual=h, norm=True)
            h = out
        return h


class NativeOffloadMoEStack:
    """OffloadMoEStack with the per-layer orchestration in C++
    (``pdx_offload_*``): same placement policy, copies and launches, no Python
    on the per-layer path.  Arguments as OffloadMoEStack, plus ``max_tokens``
    (the largest batch a call may carry; sizes the device workspace)."""

    def __init__(self, gates, host_experts, hot, *, hidden, inter, cache_slots, top_k=8, normalize=True,
                 prefetch=True, chunk=16, warm=None, max_tokens=4096):
        self.gates = list(gates)
        self.L, self.E = len(self.gates), self.gates[0].shape[0]
        self.H, self.I, self.k = hidden, inter, top_k
        if host_experts.device.type != "cpu" or not host_experts.is_pinned():
            raise ValueError("host experts must be a pinned CPU tensor (copy-engine transfers)")
        if host_experts.dtype != torch.bfloat16 or tuple(host_experts.shape) != (self.L, self.E, 3 * inter * hidden):
            raise ValueError("host experts must be BF16 [layers, experts, 3*inter*hidden]")
        self.host = host_experts
        self.dev = self.gates[0].device
        warm = warm if warm is not None else [[] for _ in range(self.L)]
        fixed = [list(h) + list(w) for h, w in zip(hot, warm)]
        hot_n = {len(h) for h in hot}
        if len(hot_n) > 1:
            raise ValueError("the native engine needs the same hot-set size in every layer")
        self._gate_ptrs = (ctypes.c_void_p * self.L)(*[g.data_ptr() for g in self.gates])
        self._fixed_count = (ctypes.c_int32 * self.L)(*[len(f) for f in fixed])
        flat = [e for f in fixed for e in f]
        self._fixed = (ctypes.c_int32 * max(1, len(flat)))(*flat)
        self.cfg = _lib.OffloadConfig(layers=self.L, experts=self.E, hidden=hidden, inter=inter, top_k=top_k,
                                      normalize=int(normalize), gates=self._gate_ptrs,
                                      host_experts=host_experts.data_ptr(), fixed_count=self._fixed_count,
                                      fixed_experts=self._fixed, hot_per_layer=hot_n.pop() if hot_n else 0,
                                      chunk=chunk, prefetch=int(prefetch), cache_slots=cache_slots,
                                      max_tokens=max_tokens)
        pool_bytes = lib.pdx_offload_pool_bytes(ctypes.byref(self.cfg))
        ws_bytes = lib.pdx_offload_workspace_bytes(ctypes.byref(self.cfg))
        if not pool_bytes or not ws_bytes:
            check(_lib.PDX_ERR_INVALID)
        self.pool = torch.empty(pool_bytes, dtype=torch.uint8, device=self.dev)
        self.ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.dev)
        h = ctypes.c_void_p()
        check(lib.pdx_offload_create(ctypes.byref(self.cfg), _ptr(self.pool), _ptr(self.ws), ws_bytes,
                                     ctypes.byref(h)))
        self._h = h
        self._acts = {}

    @property
    def stats(self):
        st = _lib.OffloadStats()
        check(lib.pdx_offload_get_stats(self._h, ctypes.byref(st)))
        return OffloadStats(**{name: getattr(st, name) for name, _ in _lib.OffloadStats._fields_})

    def forward_layer(self, l, x, out, residual=None, norm=False):
        check(lib.pdx_offload_forward_layer(self._h, l, _ptr(x), x.shape[0], _ptr(residual), int(norm), _ptr(out),
                                            _stream()))
        return out

    def forward(self, x):
        """Every layer on ``x``; layer l+1's input is layer_norm(MoE_l(x_l) + x_l)."""
        t = x.shape[0]
        acts = self._acts.get(t)
        if acts is None:
            acts = self._acts[t] = [torch.empty_like(x) for _ in range(2)]
        h = x
        for l in range(self.L):
            self.forward_layer(l, h, acts[l % 2], residual=h, norm=True)
            h = acts[l % 2]
        return h

    def close(self):
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.dev)
            lib.pdx_offload_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PinnedHostBuffer:
    """Page-locked host memory of exactly ``nbytes``: a plain allocation
    registered with cudaHostRegister.  (torch's pinned allocator rounds each
    block up to a power of two, which would nearly double a 54 GiB expert
    store.)  ``close()`` unregisters it; the tensor must not be used after."""

    def __init__(self, nbytes):
        self.tensor = torch.empty(int(nbytes), dtype=torch.uint8)
        torch.cuda.check_error(torch.cuda.cudart().cudaHostRegister(self.tensor.data_ptr(), int(nbytes), 0))
        self._registered = True

    def close(self):
        if getattr(self, "_registered", False):
            self._registered = False
            torch.cuda.check_error(torch.cuda.cudart().cudaHostUnregister(self.tensor.data_ptr()))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def measure_h2d_gbs(device, nbytes=1 << 30, repeats=5):
    """Pinned host -> device copy bandwidth on a dedicated stream (GB/s, best of
    ``repeats``), the host-link roofline of offload mode."""
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=device)
    s = torch.cuda.Stream(device=device)
    best = 0.0
    for _ in range(repeats):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        with torch.cuda.stream(s):
            dst.copy_(src, non_blocking=True)
        e1.record(s)
        s.synchronize()
        best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9)
    del src, dst
    return best
