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
import math
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


class LedgerPlacer:
    """Device slot placement driven by an ExpertCache-style ticket ledger.

    The reference keeps expert residency in ``ExpertCache``
    (expertbench/cache.py:353-647): ``on_demand`` declares a layer's routed
    experts, ``begin_load`` reserves a copy (evicting by its own policy) and
    returns a ticket in the 'cache' pool or a 'demand_staging' slot,
    ``submit`` / ``complete_load`` bracket the transfer (the byte closure
    h2d_bytes_submitted == h2d_bytes_completed, :552-574), ``acquire`` /
    ``release`` bracket the compute, ``end_demand`` closes the layer and
    ``take_retired`` hands back the tickets whose memory may be reused.  This
    class maps those tickets onto device slots and keeps the ledger's calls
    in that order, while the copies and kernels themselves run ahead on the
    device (ordered by events): a transfer is reported complete, and a use
    released, only once its event has finished.

    ``ledger``: the ExpertCache (or an object with its API); ``key_of(layer,
    expert)`` and ``demand_of(request, step, layer)`` build its key and demand
    ids.  Slots: ``cache_slots`` cache-pool slots then one slot per staging
    slot of the ledger.  ``device``: copy issue and event queries --
    ``copy(key, slot, after) -> event`` (a copy into ``slot`` that starts after
    the event ``after``), ``done(event) -> bool`` and ``wait(event)`` (host).
    CUDA-free, so the reference's own ledger can drive it on any host.
    """

    def __init__(self, ledger, *, key_of, demand_of, cache_slots, device, request="offload"):
        self.ledger, self.key_of, self.demand_of, self.device = ledger, key_of, demand_of, device
        self.request = request
        self.n_cache = cache_slots
        self.free = list(range(cache_slots - 1, -1, -1))
        self.slot_of = {}            # ticket -> slot
        self.copy_event = {}         # ticket -> event of its submitted, not yet completed transfer
        self.last_use = {}           # slot -> event of its last reader
        self.open = None             # (identity, use handles, done event) of the layer awaiting its close
        self.identity = None         # demand id of the layer being placed
        self.prefetch_skipped = 0

    # -- tickets and slots --------------------------------------------------------
    def _slot_for(self, ticket):
        if ticket.pool == "demand_staging":
            slot = self.n_cache + ticket.slot
        else:
            if not self.free:
                raise RuntimeError("ledger admitted more cache copies than the device pool has slots")
            slot = self.free.pop()
        self.slot_of[ticket] = slot
        return slot

    def _load(self, key, origin):
        ticket = self.ledger.begin_load(key, origin=origin)
        if ticket in self.slot_of:             # a repeated reservation returns the live ticket
            return ticket, False
        self._retire()                         # the reservation's evictions free their slots now
        slot = self._slot_for(ticket)
        self.copy_event[ticket] = self.device.copy(key, slot, self.last_use.get(slot))
        self.ledger.submit(ticket)
        return ticket, True

    def _complete(self, ticket, wait):
        ev = self.copy_event.get(ticket)
        if ev is None:
            return True
        if not self.device.done(ev):
            if not wait:
                return False
            self.device.wait(ev)
        self.ledger.complete_load(ticket)
        del self.copy_event[ticket]
        return True

    def _retire(self):
        for ticket in self.ledger.take_retired():
            slot = self.slot_of.pop(ticket, None)
            self.copy_event.pop(ticket, None)
            if slot is not None and slot < self.n_cache:
                self.free.append(slot)

    def load_initial(self, keys):
        """The initial hotset (origin 'initial'), loaded before the first demand."""
        for key in keys:
            ticket, _ = self._load(key, "initial")
            self._complete(ticket, wait=True)

    # -- one layer ------------------------------------------------------------------
    def close_layer(self):
        """Closes the open layer once its compute event finished: release its
        uses, end its demand, complete finished transfers, recycle slots."""
        if self.open is None:
            return
        identity, handles, done = self.open
        self.device.wait(done)
        for h in handles:
            self.ledger.release(h)
        self.ledger.end_demand(identity)
        self.open = None
        for ticket in list(self.copy_event):
            self._complete(ticket, wait=False)
        self._retire()

    def place_layer(self, step, layer, counts, predicted=(), probabilities=None):
        """Slots for this layer's routed experts ``counts`` {expert: tokens} and
        prefetch copies of ``predicted`` (next-layer experts).  Returns
        (slot of each routed expert, {expert: copy event} of the routed experts
        whose transfers are still in flight, demand experts, prefetched
        experts).  ``probabilities``: at a decode step (one token), the
        token's full softmax over the layer's experts, handed to a
        score-keeping ledger right after the demand is declared and before
        any load -- the order the reference's DecodeScoreLayerCache requires
        (update_decode_scores, expertbench/cache.py:903-929)."""
        self.close_layer()
        identity = self.identity = self.demand_of(self.request, step, layer)
        keys = {e: self.key_of(layer, e) for e in counts}
        self.ledger.on_demand(identity, {keys[e]: int(n) for e, n in counts.items()})
        if probabilities is not None and step > 0 and hasattr(self.ledger, "update_decode_scores"):
            self.ledger.update_decode_scores(identity, [float(v) for v in probabilities])
        slots, pending, demand = {}, {}, []
        for e in sorted(counts):
            key = keys[e]
            view = self.ledger.lookup(key)
            if view is None:
                ticket, _ = self._load(key, "demand")
                demand.append(e)
            else:
                ticket = view.ticket
            slots[e] = self.slot_of[ticket]
            if ticket in self.copy_event:
                pending[e] = self.copy_event[ticket]
        issued = []
        for e in predicted:
            key = self.key_of(layer + 1, e)
            if self.ledger.lookup(key) is not None:
                continue
            try:
                self._load(key, "prefetch")
            except Exception as exc:           # CapacityBlocked: no evictable cache bytes for speculation
                if type(exc).__name__ != "CapacityBlocked":
                    raise
                self.prefetch_skipped += 1
                continue
            issued.append(e)
        return slots, pending, demand, issued

    def begin_compute(self, layer, counts, done):
        """The layer's compute is enqueued (``done`` = its completion event):
        the transfers it reads complete (host wait), its uses are acquired,
        and its slots are marked read until ``done``."""
        handles = []
        for e in sorted(counts):
            key = self.key_of(layer, e)
            ticket = self.ledger.lookup(key).ticket
            self._complete(ticket, wait=True)
            handles.append(self.ledger.acquire(key))
            self.last_use[self.slot_of[ticket]] = done
        self.open = (self.identity, handles, done)

    def drain(self):
        """Closes the open layer and completes every transfer still in flight
        (the ledger's byte closure holds afterwards)."""
        self.close_layer()
        for ticket in list(self.copy_event):
            self._complete(ticket, wait=True)
        self._retire()


class _CopyEngine:
    """LedgerPlacer's device side for an OffloadMoEStack: one cudaMemcpyAsync
    of the expert's 9 MiB slot from pinned host memory on the copy stream,
    after the slot's last reader, and an event per copy."""

    def __init__(self, stack):
        self.stack = stack

    def copy(self, key, slot, after):
        st = self.stack
        l, e = (key.layer, key.expert) if hasattr(key, "layer") else key
        cs = st.copy_stream
        if after is not None:
            cs.wait_event(after)
        with torch.cuda.stream(cs):
            st.pool[slot * st.per:(slot + 1) * st.per].copy_(st.host[l, e], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(cs)
        return ev

    def done(self, ev):
        return ev.query()

    def wait(self, ev):
        ev.synchronize()


class TicketLedger:
    """A small ticket ledger with ExpertCache's call protocol, for hosts
    without the reference package: cache slots of equal size, demand-staging
    fallback when the cache has no evictable entry, byte counters with the
    same names.  Keys are (layer, expert) tuples and demand ids (request,
    step, layer) tuples; ``CapacityBlocked`` is raised as the reference does
    when speculation finds no evictable room.

    ``policy``: "lru" evicts the least recently demanded entry.  "score"
    keeps the decode score of the reference's DecodeScoreLayerCache
    (expertbench/cache.py:852-966): scores start at zero, and each decode
    layer step's ``update_decode_scores`` sets, for every expert of the
    layer, s = 0.5 s + 0.5 p if the expert is among the 2*top_k most probable
    (ties to the lower id) and s = 0.5 s otherwise, in binary64; during decode
    steps (step > 0) the victim is the evictable entry of least (score, key),
    during prefill the least recently demanded one.  Unlike the reference's
    class, the cache is one pool for all layers, not fixed per-layer quotas."""

    class CapacityBlocked(RuntimeError):
        pass

    @dataclass(frozen=True)
    class Ticket:
        generation: int
        key: tuple
        pool: str
        slot: object

    @dataclass
    class View:
        ticket: object
        state: str

    def __init__(self, cache_slots, staging_slots, nbytes, initial_hotset=(), *, policy="lru", top_k=None):
        if policy not in ("lru", "score"):
            raise ValueError(f"unknown ledger policy {policy!r}")
        if policy == "score" and not (isinstance(top_k, int) and top_k >= 1):
            raise ValueError("the score policy needs the router's top_k")
        self.cache_slots, self.staging_slots, self.nbytes = cache_slots, staging_slots, nbytes
        self.policy, self.top_k = policy, top_k
        self._scores = {}            # layer -> [float] per expert
        self._scored = None          # demand id whose scores are current
        self.initial_hotset = frozenset(initial_hotset)
        self._entries = {}           # key -> dict(ticket, ready, submitted, users)
        self._lru = OrderedDict()    # cache keys, least recent first
        self._staging_busy = set()
        self._retired = []
        self._gen = 0
        self._active = None          # (identity, remaining keys)
        self._stats = dict(h2d_bytes_submitted=0, h2d_bytes_completed=0, gpu_completed_experts=0, evictions=0,
                           demand_loads_submitted=0, prefetch_loads_submitted=0, initial_loads_submitted=0,
                           score_updates=0)

    def stats(self):
        return dict(self._stats)

    def lookup(self, key):
        ent = self._entries.get(key)
        if ent is None:
            return None
        return TicketLedger.View(ent["ticket"], "in_use" if ent["users"] else "ready" if ent["ready"] else "loading")

    def on_demand(self, identity, counts):
        if self._active is not None:
            raise RuntimeError("another layer-step demand is active")
        self._active = (identity, set(counts))
        for key in counts:
            if key in self._lru:
                self._lru.move_to_end(key)

    def _evictable(self, key):
        ent = self._entries[key]
        return ent["ready"] and not ent["users"] and not (self._active and key in self._active[1])

    def update_decode_scores(self, identity, probabilities):
        """The decode step's full softmax over the layer's experts (one token).
        With the LRU policy the scores are kept too when ``top_k`` is given
        (observed, not used: the reference's observe_only mode)."""
        if self.top_k is None:
            return
        if self._active is None or self._active[0] != identity or identity[1] == 0:
            raise RuntimeError("score update requires the current decode demand")
        if self._scored == identity:
            raise RuntimeError("the scores of this demand were updated already")
        values = [float(v) for v in probabilities]
        if any(not (0.0 <= v <= 1.0) for v in values) or abs(math.fsum(values) - 1.0) > 1e-5:
            raise RuntimeError("score update requires the full softmax probabilities")
        layer = identity[2]
        prev = self._scores.get(layer) or [0.0] * len(values)
        if len(prev) != len(values):
            raise RuntimeError("probability vector length differs from the layer's expert count")
        order = sorted(range(len(values)), key=lambda i: (-values[i], i))
        chosen = set(order[:min(2 * self.top_k, len(values))])
        self._scores[layer] = [0.5 * prev[i] + (0.5 * values[i] if i in chosen else 0.0)
                               for i in range(len(values))]
        self._scored = identity
        self._stats["score_updates"] += 1

    def score_values(self, layer):
        return tuple(self._scores.get(layer, ()))

    def _victim(self):
        candidates = (k for k in self._lru if self._evictable(k))
        if self.policy == "score" and self._active is not None and self._active[0][1] > 0:
            scores = self._scores
            return min(candidates, default=None,
                       key=lambda k: (scores.get(k[0], ())[k[1]] if k[1] < len(scores.get(k[0], ())) else 0.0, k))
        return next(candidates, None)

    def begin_load(self, key, *, origin="demand", admit=True):
        if key in self._entries:
            return self._entries[key]["ticket"]
        cached = sum(1 for k in self._entries if self._entries[k]["ticket"].pool == "cache")
        victim = None
        if cached >= self.cache_slots:
            victim = self._victim()
        if cached < self.cache_slots or victim is not None:
            if victim is not None:
                self._retired.append(self._entries.pop(victim)["ticket"])
                del self._lru[victim]
                self._stats["evictions"] += 1
            pool, slot = "cache", None
            self._lru[key] = None
        elif origin == "demand":
            free = [i for i in range(self.staging_slots) if i not in self._staging_busy]
            if not free:
                raise TicketLedger.CapacityBlocked("demand staging busy")
            pool, slot = "demand_staging", free[0]
            self._staging_busy.add(slot)
        else:
            raise TicketLedger.CapacityBlocked("no evictable cache bytes")
        self._gen += 1
        t = TicketLedger.Ticket(self._gen, key, pool, slot)
        self._entries[key] = dict(ticket=t, ready=False, submitted=False, users=set(), origin=origin)
        return t

    def submit(self, ticket):
        ent = self._entries[ticket.key]
        if ent["ticket"] != ticket or ent["submitted"]:
            raise RuntimeError("stale or repeated submission")
        ent["submitted"] = True
        self._stats["h2d_bytes_submitted"] += self.nbytes
        self._stats[ent["origin"] + "_loads_submitted"] += 1

    def complete_load(self, ticket):
        ent = self._entries[ticket.key]
        if ent["ticket"] != ticket or not ent["submitted"] or ent["ready"]:
            raise RuntimeError("completion needs one submitted, incomplete transfer")
        ent["ready"] = True
        self._stats["h2d_bytes_completed"] += self.nbytes

    def acquire(self, key):
        ent = self._entries[key]
        if not ent["ready"]:
            raise RuntimeError("weights are not ready")
        self._gen += 1
        ent["users"].add(self._gen)
        return (key, self._gen)

    def release(self, handle):
        key, serial = handle
        ent = self._entries[key]
        ent["users"].remove(serial)
        if not ent["users"]:
            self._active[1].discard(key)
            self._stats["gpu_completed_experts"] += 1
            if ent["ticket"].pool == "demand_staging":
                self._staging_busy.discard(ent["ticket"].slot)
                self._retired.append(self._entries.pop(key)["ticket"])

    def end_demand(self, identity):
        if self._active is None or self._active[0] != identity or self._active[1]:
            raise RuntimeError("cannot finish layer: some experts have not completed")
        self._active = None

    def take_retired(self):
        out, self._retired = self._retired, []
        return out


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
                 prefetch=True, chunk=16, warm=None, ledger=None, key_of=None, demand_of=None, request="offload"):
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
        self.placer = None
        self._step = -1
        if ledger is not None:
            self._init_ledger(ledger, hot, warm, key_of, demand_of, request, prefetch, chunk)
            return
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

    def _init_ledger(self, ledger, hot, warm, key_of, demand_of, request, prefetch, chunk):
        """Residency kept by a ticket ledger (ExpertCache's API): its cache pool
        and staging slots are the device pool, its initial hotset the hot
        table; LedgerPlacer maps tickets to slots."""
        if warm:
            raise ValueError("with a ledger, residency beyond the hot set is the ledger's own policy")
        slot_bytes = self.per * 2
        n_cache = getattr(ledger, "cache_slots", None) or ledger.cache_bytes // slot_bytes
        n_stage = getattr(ledger, "staging_slots", None) or len(ledger.staging_slot_bytes)
        n_slots = n_cache + n_stage
        self.pool = torch.empty(n_slots * self.per, dtype=torch.bfloat16, device=self.dev)
        self.copy_stream = torch.cuda.Stream(device=self.dev)
        self.prefetch, self.chunk = prefetch, max(1, chunk)
        self.stats = OffloadStats()
        key_of = key_of or (lambda l, e: (l, e))
        demand_of = demand_of or (lambda r, s, l: (r, s, l))
        self.placer = LedgerPlacer(ledger, key_of=key_of, demand_of=demand_of, cache_slots=n_cache,
                                   device=_CopyEngine(self), request=request)
        self.ledger = ledger
        base = self.pool.data_ptr()
        self._weights = dict(gate=base, up=base + self.I * self.H * 2, down=base + 2 * self.I * self.H * 2,
                             gate_stride=self.per, up_stride=self.per, down_stride=self.per, num_slots=n_slots)
        i32 = dict(dtype=torch.int32)
        self.table_host = torch.zeros((self.L, self.E), **i32).pin_memory()
        self.table_dev = torch.zeros((self.L, self.E), **i32, device=self.dev)
        self.max_launch = 1 + -(-self.E // self.chunk)
        self.active_host = torch.zeros((self.max_launch, self.E + 1), **i32).pin_memory()
        self.active_dev = torch.zeros((self.max_launch, self.E + 1), **i32, device=self.dev)
        self.counts_host = torch.zeros((2, self.E), **i32).pin_memory()
        # one decode token's logits, for a ledger that keeps decode scores
        self.scores_wanted = hasattr(ledger, "update_decode_scores")
        self.logits_host = torch.zeros((1, self.E), dtype=torch.bfloat16).pin_memory()
        self._bufs = {}
        self.placer.load_initial([key_of(l, e) for l, hs in enumerate(hot) for e in hs])
        torch.cuda.synchronize(self.dev)

    def finish(self):
        """Ledger mode: close the last layer and complete every transfer in
        flight (the ledger's byte closure holds afterwards)."""
        if self.placer is not None:
            self.placer.drain()

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
        scores = self.placer is not None and self.scores_wanted and t == 1
        if scores:
            self.logits_host.copy_(cur["logits"], non_blocking=True)
        comp.synchronize()   # the per-layer grouping sync
        counts = self.counts_host.numpy()
        needed = np.nonzero(counts[0])[0].tolist()
        self.stats.layers += 1
        self.stats.expert_uses += len(needed)
        if self.placer is not None:
            # the decode token's full softmax (the native probabilities a score ledger keeps)
            probs = torch.softmax(self.logits_host[0].double(), 0).tolist() if scores else None
            return self._forward_layer_ledger(l, x, out, residual, norm, counts, needed, predict, b, comp, probs)

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

    def _forward_layer_ledger(self, l, x, out, residual, norm, counts, needed, predict, b, comp, probs=None):
        """forward_layer's placement and launches when a ledger keeps residency."""
        t = x.shape[0]
        cur = {e: int(counts[0][e]) for e in needed}
        predicted = np.nonzero(counts[1])[0].tolist() if predict else []
        slots, pending, demand, issued = self.placer.place_layer(self._step, l, cur, predicted, probs)
        self.stats.demand_copies += len(demand)
        self.stats.prefetch_copies += len(issued)
        self.stats.h2d_bytes += (len(demand) + len(issued)) * self.per * 2
        self.stats.cache_hits += len(cur) - len(demand)
        table = self.table_host[l].numpy()
        for e, s in slots.items():
            table[e] = s
        demand_set = set(demand)
        ready = [e for e in needed if e not in demand_set]
        chunks = [demand[c0:c0 + self.chunk] for c0 in range(0, len(demand), self.chunk)]
        act = self.active_host.numpy()
        lists = [ready] + chunks
        for i, lst in enumerate(lists):
            act[i, 0] = len(lst)
            act[i, 1:1 + len(lst)] = lst
        self.table_dev[l].copy_(self.table_host[l], non_blocking=True)
        self.active_dev[:len(lists)].copy_(self.active_host[:len(lists)], non_blocking=True)
        rows, ws, cur_r = b["rows"], b["ws"], b["cur"]
        for e in ready:                      # cached experts whose transfers are still landing
            if e in pending:
                comp.wait_event(pending[e])
        if ready:
            self._ffn(l, x, cur_r, 0, rows, ws)
        for c, part in enumerate(chunks):
            for e in part:
                comp.wait_event(pending[e])
            self._ffn(l, x, cur_r, 1 + c, rows, ws)
        if norm:
            check(lib.pdx_combine_layernorm(_ptr(rows), _ptr(cur_r["w"]), _ptr(cur_r["inverse"]), t, self.k, self.H,
                                            _ptr(residual), ctypes.c_float(LN_EPS), _ptr(out), _stream()))
        else:
            check(lib.pdx_combine(_ptr(rows), _ptr(cur_r["w"]), _ptr(cur_r["inverse"]), t, self.k, self.H,
                                  _ptr(residual), _ptr(out), _stream()))
        done = torch.cuda.Event()
        done.record(comp)
        self.placer.begin_compute(l, cur, done)
        return out

    def forward(self, x):
        """Every layer on ``x`` [T, H]; layer l+1's input is
        layer_norm(MoE_l(x_l) + x_l) (the next-layer activation of the resident
        stack).  Returns a buffer owned by the stack (valid until the next call
        with the same token count)."""
        self._step += 1
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

    _PLACES = {_lib.PLACE_HOT: "hot", _lib.PLACE_WARM: "static", _lib.PLACE_CACHE: "cache",
               _lib.PLACE_LOADING: "cache_loading", _lib.PLACE_DEMAND: "demand"}

    def trace_row(self, step, *, diagnostics=True):
        """The reference's per-layer row (the dict PDScopeCudaRuntime.forward
        returns, expertbench/pdscope_runtime.py:492-512) for the last
        forward_layer call, built from the native engine's own trace
        (pdx_offload_last_trace): token counts, the decision the engine
        executed (every routed expert on the GPU: resident, cached or copied
        on demand), the prefetch ledger and the routing fingerprints."""
        tr = _lib.OffloadTrace()
        E = self.E
        counts = (ctypes.c_int32 * (2 * E))()
        place = (ctypes.c_int32 * E)()
        pre = (ctypes.c_int32 * E)()
        dem = (ctypes.c_int32 * E)()
        check(lib.pdx_offload_last_trace(self._h, ctypes.byref(tr), counts, place, pre, dem))
        layer, t = tr.layer, tr.tokens
        cur = {e: counts[e] for e in range(E) if counts[e] > 0}
        nxt = {e: counts[E + e] for e in range(E) if counts[E + e] > 0}
        placements = {e: self._PLACES[place[e]] for e in cur}
        demand = [dem[i] for i in range(tr.demand)]
        resident = sorted((e for e in cur if place[e] != _lib.PLACE_DEMAND), key=lambda e: (-cur[e], e))
        issued = [pre[i] for i in range(tr.prefetch_issued)]
        phase = "prefill" if step == 0 else "decode"
        decision = dict(phase=phase, mode="offload_native", cpu_queue=[], gpu_resident_queue=resident,
                        on_demand_queue=demand, prefetch_queue=issued, unload_queue=[],
                        placements={e: "gpu" for e in sorted(cur)}, slot_kind=placements)
        sha, nsha = None, None
        if diagnostics:
            from .runtime import tensor_hash
            sel = torch.empty((t, self.k), dtype=torch.int64, device=self.dev)
            check(lib.pdx_offload_copy_selected(self._h, 0, t, _ptr(sel), _stream()))
            sha = tensor_hash(sel)
            if layer + 1 < self.L and nxt:
                check(lib.pdx_offload_copy_selected(self._h, 1, t, _ptr(sel), _stream()))
                nsha = tensor_hash(sel)
        return dict(phase=phase, step=step, layer=layer, token_counts=cur, dispatch="compact", decision=decision,
                    prefetch_issued=issued, prefetch_capacity_skipped=tr.prefetch_skipped,
                    next_prediction_counts=nxt, predictor="next_layer_gate_on_current_activation",
                    scheduler="native_offload_engine", selected_sha256=sha, next_selected_sha256=nsha,
                    ready_at_reveal=tr.hot + tr.warm + tr.cache_ready, loading_at_reveal=tr.cache_loading,
                    counters=dict(h2d_bytes_completed=tr.h2d_bytes, demand_copies=tr.demand,
                                  prefetch_copies=tr.prefetch_issued, prefetch_used=tr.prefetch_used,
                                  gpu_completed_experts=tr.routed_experts, cpu_completed_experts=0),
                    ping_pong_slots=[], merge_mode="fused", demand_chunks=tr.demand_chunks,
                    pipeline="copy-engine demand chunks, then next-layer prefetch on the same copy stream",
                    measured_performance=False)

    def forward(self, x, *, step=None, rows=None):
        """Every layer on ``x``; layer l+1's input is layer_norm(MoE_l(x_l) + x_l).
        With ``rows`` (a list) and ``step``, appends each layer's trace row."""
        t = x.shape[0]
        acts = self._acts.get(t)
        if acts is None:
            acts = self._acts[t] = [torch.empty_like(x) for _ in range(2)]
        h = x
        for l in range(self.L):
            self.forward_layer(l, h, acts[l % 2], residual=h, norm=True)
            if rows is not None:
                rows.append(self.trace_row(step if step is not None else 0))
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
