"""Offload-mode host logic on CPU: the cache-ring ledger and the hot-table format.

The ring is the B200 form of the reference's slot ledger (expertbench/cache.py
begin_load/acquire/release, :505-626): a slot is handed out only outside the
current layer's live set, and its new copy waits for the last reader of its old
content."""
import pytest

import torch

from pdscope_b200.offload import CacheRing, load_hot_file, write_hot_file, zipf_hot_sets


def test_ring_lru_and_pinning():
    ring = CacheRing(3)
    got = [ring.acquire(("L0", e), pinned=set())[0] for e in range(3)]
    assert sorted(got) == [0, 1, 2]
    ring.slots[got[0]].last_use = "ev0"
    ring.touch(got[0])                       # expert 0 becomes most recently used
    idx, prev, wasted = ring.acquire(("L0", 9), pinned={got[1]})
    assert idx == got[2] and prev is None and not wasted   # LRU outside the pinned set
    assert ring.lookup(("L0", 2)) is None and ring.lookup(("L0", 9)) == idx
    idx2, prev2, _ = ring.acquire(("L0", 10), pinned={got[1], idx})
    assert idx2 == got[0] and prev2 == "ev0"              # new copy must wait for the old reader


def test_ring_all_pinned_raises():
    ring = CacheRing(2)
    a, _, _ = ring.acquire((0, 0), set())
    b, _, _ = ring.acquire((0, 1), set())
    with pytest.raises(RuntimeError, match="enlarge the cache ring"):
        ring.acquire((0, 2), {a, b})
    with pytest.raises(ValueError):
        ring.acquire((0, 0), set())
    with pytest.raises(ValueError):
        CacheRing(0)


def test_ring_counts_unread_prefetch():
    ring = CacheRing(1)
    i, _, _ = ring.acquire((1, 5), set())
    ring.slots[i].prefetched = True
    _, _, wasted = ring.acquire((1, 6), set())
    assert wasted


def test_hot_file_round_trip(tmp_path):
    hot = [[5, 1, 7], [2, 0, 3]]
    p = tmp_path / "hot.txt"
    write_hot_file(p, hot)
    lines = p.read_text().splitlines()
    # the reference's hot/qwen.txt format: no header, hottest rank of every layer first
    assert lines == ["0,5", "1,2", "0,1", "1,0", "0,7", "1,3"]
    assert load_hot_file(p, 2, 2) == [[5, 1], [2, 0]]
    assert load_hot_file(p, 3, 1) == [[5, 1, 7]]


def test_zipf_hot_sets_hottest_first(tmp_path):
    """The hot table lists each layer's experts by Zipf rank, so the first N
    rows of the file are the N hottest (load_hot_profile reads the head)."""
    ranks = torch.tensor([3, 1, 4, 2, 5, 6, 8, 7], dtype=torch.float32)
    g = torch.zeros(8, 4)
    g[:, 0] = -0.825 * torch.log(ranks)          # rank 1 -> largest offset
    hot = zipf_hot_sets([g.to(torch.bfloat16)], 8)
    assert hot == [[1, 3, 0, 2, 4, 5, 7, 6]]
    p = tmp_path / "hot.txt"
    write_hot_file(p, hot)
    assert load_hot_file(p, 3, 1) == [[1, 3, 0]]
