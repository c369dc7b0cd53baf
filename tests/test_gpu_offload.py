"""Offload mode on the device: experts in pinned host memory, a hot set and a
small cache ring in HBM.  The output of every step must equal the all-resident
stack's output bit for bit (same kernels, same split-K plan; only the expert
slot table differs), through prefill and decode steps that force demand
chunks, prefetch hits and evictions."""
import pytest
import torch

pytestmark = pytest.mark.gpu

L, E, H, I, K = 4, 16, 256, 128, 4


@pytest.fixture(scope="module")
def stacks():
    from pdscope_b200.offload import OffloadMoEStack, zipf_hot_sets
    from pdscope_b200.stack import build_stack
    res = build_stack(L, H, E, I, top_k=K, seed=5, zipf=True)
    host = torch.stack([s.storage.view(E, -1).cpu() for s in res.slabs]).pin_memory()
    hot = zipf_hot_sets(res.gates, 4)
    off = OffloadMoEStack(res.gates, host, hot, hidden=H, inter=I, cache_slots=14, top_k=K, chunk=3)
    return res, off


def _resident(res, x):
    t = x.shape[0]
    res.input(t).copy_(x)
    res.step(t, graph=False)
    return res.output(t).clone()


@pytest.mark.parametrize("t_count", [1, 7, 96])
def test_offload_matches_resident(stacks, t_count):
    from pdscope_b200.stack import activations
    res, off = stacks
    for step in range(3):
        x = activations(t_count, H, seed=300 + 10 * t_count + step, zipf=True)
        want = _resident(res, x)
        got = off.forward(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (t_count, step)
    from pdscope_b200.runtime import raise_device_error
    raise_device_error()


def test_offload_ledger(stacks):
    from pdscope_b200.stack import activations
    _, off = stacks
    before = off.stats.as_dict()
    for step in range(6):
        off.forward(activations(1, H, seed=900 + step, zipf=True))
    torch.cuda.synchronize()
    s = off.stats.as_dict()
    d = {k: s[k] - before[k] for k in s}
    assert d["layers"] == 6 * L
    # every non-hot expert use is either a ring hit or a demand copy
    assert d["expert_uses"] == d["hot_hits"] + d["warm_hits"] + d["cache_hits"] + d["demand_copies"]
    assert d["h2d_bytes"] == (d["demand_copies"] + d["prefetch_copies"]) * 3 * H * I * 2
    assert d["prefetch_copies"] > 0


def test_offload_rejects_pageable_host():
    from pdscope_b200.offload import OffloadMoEStack
    g = [torch.zeros(E, H, dtype=torch.bfloat16, device="cuda")]
    with pytest.raises(ValueError, match="pinned"):
        OffloadMoEStack(g, torch.zeros(1, E, 3 * H * I, dtype=torch.bfloat16), [[0]], hidden=H, inter=I,
                        cache_slots=4, top_k=K)


def test_offload_warm_tier_matches_resident(stacks):
    """A static cache tier (fixed slots for the next experts by rank) changes
    where weights come from, not the result."""
    from pdscope_b200.offload import OffloadMoEStack, zipf_hot_sets
    from pdscope_b200.stack import activations
    res, off = stacks
    ranked = zipf_hot_sets(res.gates, 7)
    warm_stack = OffloadMoEStack(res.gates, off.host, [r[:3] for r in ranked], hidden=H, inter=I, cache_slots=12,
                                 top_k=K, chunk=2, warm=[r[3:] for r in ranked])
    for t_count in (1, 50):
        x = activations(t_count, H, seed=700 + t_count, zipf=True)
        want = _resident(res, x)
        got = warm_stack.forward(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), t_count
    assert warm_stack.stats.warm_hits > 0


def _fresh(res, native, **kw):
    from pdscope_b200.offload import NativeOffloadMoEStack, OffloadMoEStack, zipf_hot_sets
    host = torch.stack([s.storage.view(E, -1).cpu() for s in res.slabs]).pin_memory()
    ranked = zipf_hot_sets(res.gates, 6)
    cls = NativeOffloadMoEStack if native else OffloadMoEStack
    extra = dict(max_tokens=128) if native else {}
    return cls(res.gates, host, [r[:4] for r in ranked], hidden=H, inter=I, cache_slots=14, top_k=K, chunk=3,
               warm=[r[4:] for r in ranked], **extra, **kw)


def test_native_engine_matches_python_and_resident(stacks):
    """The C++ host engine: same outputs as the resident stack, and the same
    placement decisions (ledger counters) as the Python orchestration."""
    from pdscope_b200.stack import activations
    res, _ = stacks
    nat, py = _fresh(res, True), _fresh(res, False)
    for step, t_count in enumerate((1, 7, 96, 1, 1, 33)):
        x = activations(t_count, H, seed=1200 + step, zipf=True)
        want = _resident(res, x)
        a = nat.forward(x).clone()
        b = py.forward(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(a.view(torch.int16), want.view(torch.int16)), (step, t_count)
        assert torch.equal(b.view(torch.int16), want.view(torch.int16)), (step, t_count)
    assert nat.stats.as_dict() == py.stats.as_dict()
    nat.close()


def test_native_engine_rejects_bad_calls(stacks):
    res, _ = stacks
    nat = _fresh(res, True)
    x = torch.zeros(200, H, dtype=torch.bfloat16, device="cuda")   # above max_tokens
    with pytest.raises(ValueError):
        nat.forward_layer(0, x, torch.empty_like(x))
    with pytest.raises(ValueError):
        nat.forward_layer(L, x[:4], torch.empty_like(x[:4]))        # layer out of range
    nat.close()


def test_native_engine_trace_rows(stacks):
    """The C++ engine reports each layer as the reference's row
    (pdscope_runtime.py:492-512): routed counts equal the device routing,
    every routed expert is placed exactly once (hot / static / cache / demand),
    the row's prefetch ledger and H2D bytes add up to the engine's counters,
    and selected_sha256 fingerprints the routing the reference would hash."""
    import hashlib
    from pdscope_b200.runtime import pack, route
    from pdscope_b200.stack import activations
    res, _ = stacks
    nat = _fresh(res, True)
    before = nat.stats.as_dict()
    rows = []
    for step, t_count in enumerate((12, 1, 1, 1)):
        x = activations(t_count, H, seed=1500 + step, zipf=True)
        rows_before = len(rows)
        nat.forward(x, step=step, rows=rows)
        torch.cuda.synchronize()
        r0 = rows[rows_before]
        assert r0["layer"] == 0 and r0["phase"] == ("prefill" if step == 0 else "decode")
        sel = route(x, res.gates[0], K, True).selected
        counts = torch.bincount(sel.flatten(), minlength=E).tolist()
        assert r0["token_counts"] == {e: c for e, c in enumerate(counts) if c}
        assert r0["selected_sha256"] == hashlib.sha256(sel.cpu().contiguous().view(torch.uint8).numpy()
                                                       .tobytes()).hexdigest()
        nsel = route(x, res.gates[1], K, True).selected
        ncounts = torch.bincount(nsel.flatten(), minlength=E).tolist()
        assert r0["next_prediction_counts"] == {e: c for e, c in enumerate(ncounts) if c}
    assert len(rows) == 4 * L
    s = nat.stats.as_dict()
    d = {k: s[k] - before[k] for k in s}
    for r in rows:
        dec = r["decision"]
        routed = set(r["token_counts"])
        assert set(dec["gpu_resident_queue"]) | set(dec["on_demand_queue"]) == routed
        assert not set(dec["gpu_resident_queue"]) & set(dec["on_demand_queue"])
        assert dec["cpu_queue"] == [] and set(dec["slot_kind"]) == routed
        assert r["counters"]["h2d_bytes_completed"] == (len(dec["on_demand_queue"]) + len(r["prefetch_issued"])) \
            * 3 * H * I * 2
    assert sum(r["counters"]["h2d_bytes_completed"] for r in rows) == d["h2d_bytes"]
    assert sum(len(r["decision"]["on_demand_queue"]) for r in rows) == d["demand_copies"]
    assert sum(len(r["prefetch_issued"]) for r in rows) == d["prefetch_copies"]
    assert sum(r["counters"]["prefetch_used"] for r in rows) == d["prefetch_used"]
    assert rows[-1]["next_prediction_counts"] == {} and rows[-1]["next_selected_sha256"] is None
    nat.close()


def test_offload_through_a_ticket_ledger(stacks):
    """Residency kept by a ticket ledger with ExpertCache's protocol
    (expertbench/cache.py:353-647; the reference's own ExpertCache drives the
    same LedgerPlacer in tests/test_offload_ledger.py): outputs stay equal to
    the all-resident stack through demand copies, evictions and prefetches,
    and the ledger's byte closure holds (h2d_bytes_submitted ==
    h2d_bytes_completed == every copy issued, cache.py:552-574)."""
    from pdscope_b200.offload import OffloadMoEStack, TicketLedger, zipf_hot_sets
    from pdscope_b200.stack import activations
    res, off = stacks
    hot = zipf_hot_sets(res.gates, 2)
    nbytes = 3 * H * I * 2
    ledger = TicketLedger(cache_slots=18, staging_slots=2, nbytes=nbytes,
                          initial_hotset=[(l, e) for l, hs in enumerate(hot) for e in hs])
    st = OffloadMoEStack(res.gates, off.host, hot, hidden=H, inter=I, cache_slots=0, top_k=K, chunk=3,
                         ledger=ledger)
    for step, t_count in enumerate((12, 1, 1, 40, 1, 1, 7)):
        x = activations(t_count, H, seed=1700 + step, zipf=True)
        want = _resident(res, x)
        got = st.forward(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (step, t_count)
    st.finish()
    s = ledger.stats()
    copies = st.stats.demand_copies + st.stats.prefetch_copies + len(ledger.initial_hotset)
    assert s["h2d_bytes_submitted"] == s["h2d_bytes_completed"] == copies * nbytes
    assert s["evictions"] > 0 and st.stats.prefetch_copies > 0
    assert s["gpu_completed_experts"] == st.stats.expert_uses


def test_offload_through_a_decode_score_ledger(stacks):
    """The score-keeping ledger (the reference DecodeScoreLayerCache's decode
    rule: EMA of the token's top-2k softmax probabilities, least score
    evicted at decode steps): each one-token step hands the full softmax of
    every layer to the ledger before any load; outputs stay equal to the
    all-resident stack, the byte closure holds, and every decode layer step
    updated the scores once."""
    from pdscope_b200.offload import OffloadMoEStack, TicketLedger, zipf_hot_sets
    from pdscope_b200.stack import activations
    res, off = stacks
    hot = zipf_hot_sets(res.gates, 2)
    nbytes = 3 * H * I * 2
    ledger = TicketLedger(cache_slots=12, staging_slots=4, nbytes=nbytes, policy="score", top_k=K,
                          initial_hotset=[(l, e) for l, hs in enumerate(hot) for e in hs])
    st = OffloadMoEStack(res.gates, off.host, hot, hidden=H, inter=I, cache_slots=0, top_k=K, chunk=3,
                         ledger=ledger)
    steps = (10, 1, 1, 1, 1, 1, 1)
    for step, t_count in enumerate(steps):
        x = activations(t_count, H, seed=1900 + step, zipf=True)
        want = _resident(res, x)
        got = st.forward(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (step, t_count)
    st.finish()
    s = ledger.stats()
    copies = st.stats.demand_copies + st.stats.prefetch_copies + len(ledger.initial_hotset)
    assert s["h2d_bytes_submitted"] == s["h2d_bytes_completed"] == copies * nbytes
    assert s["score_updates"] == L * (len(steps) - 1)
    assert s["evictions"] > 0
    for l in range(L):
        sc = ledger.score_values(l)
        assert len(sc) == E and all(0.0 <= v <= 1.0 for v in sc) and sum(sc) > 0.0
