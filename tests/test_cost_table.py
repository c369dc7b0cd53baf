"""The committed B200 cost table (pdscope_b200/cost_table_b200.json, written by
``python -m pdscope_b200.costs`` on a B200) passes the checks the reference's
FileCosts applies (benchmarks/pdscope_compare.py:62-71) and interpolates like
FileCosts.for_load (:77-85)."""
import bisect
import json
from pathlib import Path

import pytest

from pdscope_b200.costs import LOADS, validate

TABLE = Path(__file__).resolve().parents[1] / "pdscope_b200" / "cost_table_b200.json"


def test_table_schema():
    table = json.loads(TABLE.read_text())
    assert validate(table) == list(LOADS)
    assert table["schema_version"] == 1


def _for_load(table, n):
    pts = {int(k): v for k, v in table["points"].items()}
    loads = sorted(pts)
    if n in pts:
        return pts[n]
    hi = bisect.bisect_left(loads, n)
    lo, up = loads[hi - 1], loads[hi]
    r = (n - lo) / (up - lo)
    return {k: pts[lo][k] + r * (pts[up][k] - pts[lo][k]) for k in pts[lo]}


def test_table_interpolates_inside_domain():
    table = json.loads(TABLE.read_text())
    mid = _for_load(table, 2000)
    lo, hi = table["points"]["1024"], table["points"]["4096"]
    for key in ("cpu_ms", "gpu_ms", "h2d_ms"):
        assert min(lo[key], hi[key]) <= mid[key] <= max(lo[key], hi[key])


def test_validate_rejects_bad_tables():
    with pytest.raises(ValueError, match="kind"):
        validate({"kind": "other", "points": {}})
    with pytest.raises(ValueError, match="domain"):
        validate({"kind": "pdscope_cost_table", "points": {"1": {}, "64": {}}})
