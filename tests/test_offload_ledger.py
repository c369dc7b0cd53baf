"""Offload placement driven by an ExpertCache ticket ledger (CPU, no GPU).

LedgerPlacer keeps the reference ledger's call protocol -- on_demand,
begin_load / submit / complete_load, acquire / release, end_demand,
take_retired (expertbench/cache.py:353-647) -- while mapping its tickets onto
device slots.  Here a simulated copy engine stands in for the GPU: every
copy writes the expert's key into its slot, and events finish late (only
when waited for, or on a later query), as transfers do.  Over many layer
steps with demand misses, evictions, staging and prefetch, every routed
expert must find its own weights in its slot, no copy may land in a slot the
open layer reads, and the ledger's byte closure must hold:
h2d_bytes_submitted == h2d_bytes_completed == copies x expert bytes
(cache.py:552-574).  The reference's own ExpertCache runs when its source
tree is present; the package's TicketLedger always runs.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

REF = Path("/root/reference")
L, E, K, NB = 4, 16, 4, 1000


class Event:
    def __init__(self):
        self.queries = 0
        self.finished = False


class FakeDevice:
    """Copies land at once in ``memory``; their events report finished only
    from their second query on (or when waited for)."""

    def __init__(self, n_slots):
        self.memory = [None] * n_slots
        self.copies = 0
        self.protected = set()       # slots the open layer reads

    def copy(self, key, slot, after):
        assert slot not in self.protected, "a copy landed in a slot the open layer reads"
        if after is not None:
            assert after.finished, "a copy started before the slot's last reader finished"
        self.memory[slot] = key
        self.copies += 1
        return Event()

    def done(self, ev):
        ev.queries += 1
        if ev.queries >= 2:
            ev.finished = True
        return ev.finished

    def wait(self, ev):
        ev.finished = True


def _run(ledger, key_of, demand_of, cache_slots, staging_slots, hot):
    from pdscope_b200.offload import LedgerPlacer
    dev = FakeDevice(cache_slots + staging_slots)
    placer = LedgerPlacer(ledger, key_of=key_of, demand_of=demand_of, cache_slots=cache_slots, device=dev)
    placer.load_initial([key_of(l, e) for l in range(L) for e in hot[l]])
    rng = np.random.default_rng(0)
    routed_total = 0
    for step in range(8):
        tokens = 1 if step else 6
        for l in range(L):
            sel = np.argsort(-rng.random((tokens, E)), axis=1)[:, :K]
            ids, n = np.unique(sel, return_counts=True)
            counts = {int(e): int(c) for e, c in zip(ids, n)}
            predicted = [int(e) for e in np.unique(np.argsort(-rng.random((tokens, E)), axis=1)[:, :K])] \
                if l + 1 < L else []
            dev.protected = set()
            slots, pending, demand, issued = placer.place_layer(step, l, counts, predicted)
            assert set(slots) == set(counts)
            assert len(set(slots.values())) == len(slots)
            for e, s in slots.items():
                assert dev.memory[s] == key_of(l, e), (step, l, e)
            done = Event()
            dev.protected = set(slots.values())
            placer.begin_compute(l, counts, done)
            done.finished = True          # the layer's kernels finish before the next placement
            dev.protected = set()
            routed_total += len(counts)
    placer.drain()
    return dev, placer, routed_total


def _check_closure(stats, dev, routed_total):
    assert stats["h2d_bytes_submitted"] == stats["h2d_bytes_completed"] == dev.copies * NB
    assert stats["gpu_completed_experts"] == routed_total


def test_ticket_ledger_protocol_and_byte_closure():
    from pdscope_b200.offload import TicketLedger
    hot = [[0, 1, 2] for _ in range(L)]
    ledger = TicketLedger(cache_slots=20, staging_slots=2, nbytes=NB)
    dev, placer, routed = _run(ledger, lambda l, e: (l, e), lambda r, s, l: (r, s, l), 20, 2, hot)
    st = ledger.stats()
    _check_closure(st, dev, routed)
    assert st["evictions"] > 0 and st["prefetch_loads_submitted"] > 0


def test_reference_expert_cache_drives_the_placement():
    if not (REF / "expertbench" / "cache.py").exists():
        pytest.skip("reference source tree not present")
    sys.path.insert(0, str(REF))
    try:
        from expertbench.cache import DemandID, ExpertCache, ExpertKey
    finally:
        sys.path.remove(str(REF))
    hot = [[0, 1, 2] for _ in range(L)]
    keys = {ExpertKey(l, e, "bf16"): NB for l in range(L) for e in range(E)}
    cache_slots, staging = 20, 2
    ledger = ExpertCache(keys, cache_slots * NB, [NB] * staging, policy="LRU",
                         initial_hotset=[ExpertKey(l, e, "bf16") for l in range(L) for e in hot[l]])
    dev, placer, routed = _run(ledger, lambda l, e: ExpertKey(l, e, "bf16"), DemandID, cache_slots, staging, hot)
    st = ledger.stats()
    _check_closure(st, dev, routed)
    assert st.get("evictions", 0) > 0
    assert st.get("prefetch_loads_submitted", 0) + placer.prefetch_skipped > 0
    assert ledger.active_demand is None


def _run_scored(ledger, key_of, demand_of, cache_slots, staging_slots, hot, steps=8):
    """Prefill (6 tokens) then one-token decode steps whose routing comes from
    a seeded softmax; every decode layer step hands the full softmax to the
    ledger through LedgerPlacer.place_layer(..., probabilities)."""
    from pdscope_b200.offload import LedgerPlacer
    dev = FakeDevice(cache_slots + staging_slots)
    placer = LedgerPlacer(ledger, key_of=key_of, demand_of=demand_of, cache_slots=cache_slots, device=dev)
    placer.load_initial([key_of(l, e) for l in range(L) for e in hot[l]])
    rng = np.random.default_rng(7)
    history = {l: [] for l in range(L)}
    for step in range(steps):
        tokens = 1 if step else 6
        for l in range(L):
            logits = rng.standard_normal((tokens, E))
            p = np.exp(logits - logits.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            sel = np.argsort(-p, axis=1, kind="stable")[:, :K]
            ids, n = np.unique(sel, return_counts=True)
            counts = {int(e): int(c) for e, c in zip(ids, n)}
            probs = p[0].tolist() if step else None
            if probs is not None:
                history[l].append(p[0])
            slots, _, _, _ = placer.place_layer(step, l, counts, (), probs)
            for e, s in slots.items():
                assert dev.memory[s] == key_of(l, e), (step, l, e)
            done = Event()
            dev.protected = set(slots.values())
            placer.begin_compute(l, counts, done)
            done.finished = True
            dev.protected = set()
    placer.drain()
    return dev, history


def _expected_scores(history):
    """Decode score after each update: s = 0.5 s + 0.5 p on the 2k most
    probable experts (ties to the lower id), s = 0.5 s elsewhere."""
    s = np.zeros(E)
    for p in history:
        chosen = np.zeros(E, bool)
        chosen[sorted(range(E), key=lambda i: (-p[i], i))[:2 * K]] = True
        s = np.array([0.5 * s[i] + (0.5 * p[i] if chosen[i] else 0.0) for i in range(E)])
    return s


def test_score_ledger_keeps_the_decode_score():
    from pdscope_b200.offload import TicketLedger
    hot = [[0, 1, 2] for _ in range(L)]
    ledger = TicketLedger(cache_slots=18, staging_slots=2, nbytes=NB, policy="score", top_k=K)
    dev, history = _run_scored(ledger, lambda l, e: (l, e), lambda r, s, l: (r, s, l), 18, 2, hot)
    st = ledger.stats()
    assert st["h2d_bytes_submitted"] == st["h2d_bytes_completed"] == dev.copies * NB
    assert st["score_updates"] == 7 * L and st["evictions"] > 0
    for l in range(L):
        assert ledger.score_values(l) == tuple(_expected_scores(history[l]))


def test_score_ledger_evicts_the_least_scored_entry():
    """At a decode step the victim is the evictable entry of least score."""
    from pdscope_b200.offload import TicketLedger
    led = TicketLedger(cache_slots=2, staging_slots=1, nbytes=NB, policy="score", top_k=1)
    for key in ((0, 0), (0, 1)):
        t = led.begin_load(key, origin="initial")
        led.submit(t)
        led.complete_load(t)
    ident = ("r", 1, 0)
    led.on_demand(ident, {(0, 2): 1})
    led.update_decode_scores(ident, [0.1, 0.6, 0.3])   # expert 0 stays out of the top 2k = 2
    t = led.begin_load((0, 2))
    assert t.pool == "cache" and led.take_retired()[0].key == (0, 0)
    assert led.score_values(0) == (0.0, 0.3, 0.15)


def test_reference_decode_score_cache_drives_the_placement():
    """The reference's own DecodeScoreLayerCache (cache.py:852-966) through
    the placer: same scores as the package's score ledger on the same
    routing, byte closure, every routed expert in its own slot."""
    if not (REF / "expertbench" / "cache.py").exists():
        pytest.skip("reference source tree not present")
    sys.path.insert(0, str(REF))
    try:
        from expertbench.cache import DecodeScoreLayerCache, DemandID, ExpertKey
    finally:
        sys.path.remove(str(REF))
    hot = [[0, 1, 2] for _ in range(L)]
    keys = {ExpertKey(l, e, "bf16"): NB for l in range(L) for e in range(E)}
    initial = [ExpertKey(l, e, "bf16") for l in range(L) for e in hot[l]]
    # per-layer quotas fixed by the initial set; one grouped launch reads a
    # layer's routed experts together, so staging holds a whole prefill miss set
    ledger = DecodeScoreLayerCache(keys, len(initial) * NB, [NB] * E, top_k=K, initial_hotset=initial)
    dev, history = _run_scored(ledger, lambda l, e: ExpertKey(l, e, "bf16"), DemandID, len(initial), E, hot)
    st = ledger.stats()
    assert st["h2d_bytes_submitted"] == st["h2d_bytes_completed"] == dev.copies * NB
    assert st["score_updates"] == 7 * L
    for l in range(L):
        assert ledger.score_values(l) == tuple(_expected_scores(history[l]))
