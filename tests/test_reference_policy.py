"""AdaptSched, unchanged, on the B200 cost table (CPU, no GPU needed).

The reference's own ``FileCosts`` (benchmarks/pdscope_compare.py:55-85) must
accept pdscope_b200/cost_table_b200.json, and its ``plan_pdscope``
(expertbench/pdscope_policy.py:72-223), fed by that table with every expert
resident in HBM, must keep every routed expert on the GPU in both phases --
the decision the resident runtime executes.  The runtime's planner call
(pdscope_b200.runtime.PDScopeCudaRuntime._decision) is checked against a
direct call with the arguments the reference's forward passes
(expertbench/pdscope_runtime.py:270-280).

These tests import the reference from its source tree and are skipped where
it is absent (the GPU box never has it); ``TableCosts`` is checked against
FileCosts point for point.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = Path("/root/reference")
TABLE = ROOT / "pdscope_b200" / "cost_table_b200.json"

pytestmark = pytest.mark.skipif(not (REF / "expertbench" / "pdscope_policy.py").exists(),
                                reason="reference source tree not present")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, str(REF))
    try:
        from benchmarks.pdscope_compare import FileCosts
        from expertbench.pdscope_policy import plan_pdscope
        yield FileCosts, plan_pdscope
    finally:
        sys.path.remove(str(REF))


def _routing_counts(tokens, seed, experts=128, k=8):
    rng = np.random.default_rng(seed)
    sel = np.argsort(-rng.random((tokens, experts)), axis=1)[:, :k]
    ids, n = np.unique(sel, return_counts=True)
    return {int(e): int(c) for e, c in zip(ids, n)}


def test_file_costs_accepts_the_b200_table(ref):
    FileCosts, _ = ref
    from pdscope_b200.costs import TableCosts
    fc, tc = FileCosts(TABLE), TableCosts(TABLE)
    assert fc.loads == [1, 4, 16, 64, 128, 256, 1024, 4096]
    for n in (1, 2, 3, 4, 7, 16, 100, 128, 300, 1024, 2500, 4096):
        a, b = fc.for_load(n), tc.for_load(n)
        assert a.keys() == b.keys()
        for key in a:
            assert a[key] == pytest.approx(b[key], rel=1e-12), (n, key)


@pytest.mark.parametrize("phase,tokens", [("decode", 1), ("prefill", 16), ("prefill", 512), ("prefill", 4096)])
def test_plan_keeps_resident_experts_on_gpu(ref, phase, tokens):
    FileCosts, plan_pdscope = ref
    costs = FileCosts(TABLE)
    cur = _routing_counts(tokens, 1 + tokens)
    nxt = _routing_counts(tokens, 2 + tokens)
    d = plan_pdscope(cur, nxt, current_layer=5, phase=phase, current_gpu_ids=list(cur), next_gpu_ids=list(nxt),
                     costs=costs, attention_ms=0., hit_rate=0., prefetch_slots=0, top_k=8)
    assert d["cpu_queue"] == []
    assert sorted(d["gpu_resident_queue"]) == sorted(cur)
    assert d["on_demand_queue"] == [] and d["prefetch_queue"] == [] and d["unload_queue"] == []
    if phase == "decode":
        assert d["cpu_balance_target"] == 0      # n_c = argmin max((k-n) t_g, n t_c) is 0 on the B200


def test_runtime_calls_the_planner_as_the_reference_does(ref):
    FileCosts, plan_pdscope = ref
    from pdscope_b200.runtime import PDScopeCudaRuntime
    costs = FileCosts(TABLE)
    calls = []

    def recording(*args, **kwargs):
        calls.append((args, kwargs))
        return plan_pdscope(*args, **kwargs)
    rt = PDScopeCudaRuntime({3: object()}, plan=recording, costs=costs)
    cur, nxt = _routing_counts(64, 9), _routing_counts(64, 10)
    got = rt._decision(cur, nxt, layer=3, phase="prefill", top_k=8, attention_ms=0.25, hit_rate=0.5)
    want = plan_pdscope(cur, nxt, current_layer=3, phase="prefill", current_gpu_ids=list(cur),
                        next_gpu_ids=list(nxt), costs=costs, attention_ms=0.25, hit_rate=0.5, prefetch_slots=0,
                        top_k=8, cpu_balance_target_override=None, joint_next=True, record_checks=False,
                        trusted=True, compute_formula_target=True)
    assert got == want
    (args, kwargs), = calls
    assert args == (cur, nxt)
    assert kwargs["costs"] is costs and kwargs["trusted"] is True and kwargs["record_checks"] is False


def test_runtime_without_planner_runs_every_expert_on_gpu():
    from pdscope_b200.runtime import PDScopeCudaRuntime
    rt = PDScopeCudaRuntime({0: object()})
    rt.plan = None                                   # no planner importable in this process
    cur = _routing_counts(16, 3)
    d = rt._decision(cur, {}, layer=0, phase="prefill", top_k=8, attention_ms=0., hit_rate=0.)
    assert d["cpu_queue"] == [] and sorted(d["gpu_resident_queue"]) == sorted(cur)
    assert d["placements"] == {e: "gpu" for e in sorted(cur)}


def test_reference_load_hot_profile_reads_our_hot_file(tmp_path, ref):
    """write_hot_file's table is the reference's hot/qwen.txt format: its own
    load_hot_profile (expertbench/pdscope_runtime.py:62-72) accepts it and
    takes the hottest rows first."""
    sys.path.insert(0, str(REF))
    try:
        from expertbench.cache import ExpertKey
        from expertbench.pdscope_runtime import load_hot_profile
    finally:
        sys.path.remove(str(REF))
    from pdscope_b200.stack import ExpertLoadTracker
    tracker = ExpertLoadTracker(48, 128)
    rng = np.random.default_rng(0)
    tracker.add(rng.integers(0, 50, size=(48, 128)))
    path = tmp_path / "hot.txt"
    tracker.write_hot_file(path, 16)
    masters = {ExpertKey(l, e, "bf16"): None for l in range(48) for e in range(128)}
    keys, meta = load_hot_profile(path, masters, 48 * 4)
    hot = tracker.hot_sets(16)
    assert meta["entries"] == 48 * 16
    assert [(k.layer, k.expert) for k in keys] == [(l, hot[l][r]) for r in range(4) for l in range(48)]
