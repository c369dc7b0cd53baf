"""Expert-parallel exchange logic on CPU: world_size 2 over gloo.

The device kernels are replaced by the oracle (HostOps below, row by row so
each row's arithmetic is independent of batching); everything else -- the
dispatch layout, the two exchange forms (padded and exact), the regrouping of
received rows by local expert and the combine map -- is the product code of
pdscope_b200/expert_parallel.py.  Each rank's EP output must equal the
single-process oracle layer on that rank's tokens bit for bit.
"""
import os
import socket
import types

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import moe_oracle as mo

E, K, H, I = 16, 4, 64, 32


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class HostOps:
    """Oracle-backed stand-ins for the sm_100a kernels (test only)."""

    def __init__(self, wg, wu, wd, first_expert):
        self.wg, self.wu, self.wd, self.first = wg, wu, wd, first_expert

    def route(self, x, gate, top_k, normalize):
        _, sel, w = mo.route(_bits(x), _bits(gate), top_k, normalize)
        return torch.from_numpy(sel), _bf16(w)

    def pack(self, sel, w, experts):
        p = mo.compact_expert_groups(sel.numpy(), _bits(w), experts)
        nz = np.nonzero(p["counts"])[0]
        active = np.zeros(experts + 1, np.int32)
        active[0] = len(nz)
        active[1:1 + len(nz)] = nz
        return types.SimpleNamespace(counts=torch.from_numpy(p["counts"]), offsets=torch.from_numpy(p["offsets"]),
                                     tokens=torch.from_numpy(p["tokens"]), positions=torch.from_numpy(p["positions"]),
                                     weights=_bf16(p["weights"]), inverse=torch.from_numpy(p["inverse"]),
                                     active=torch.from_numpy(active))

    def gather(self, x, tokens):
        return x[tokens.long()].contiguous()

    def dispatch(self, x, p, top_k, experts, ranks, capacity):
        el = experts // ranks
        send = torch.zeros((ranks * capacity, x.shape[1]), dtype=x.dtype)
        inv = torch.zeros(x.shape[0] * top_k, dtype=torch.int32)
        off = p.offsets.numpy()
        for row in range(x.shape[0] * top_k):
            e = int(np.searchsorted(off, row, side="right") - 1)
            d = e // el
            pos = row - off[d * el]
            assert pos < capacity
            send[d * capacity + pos] = x[int(p.tokens[row])]
            inv[int(p.positions[row])] = d * capacity + pos
        return send, inv

    def layout(self, recv_counts, ranks, el, capacity, rows_cap):
        rc = recv_counts.numpy().reshape(ranks, el)
        blk = np.zeros((ranks, el), np.int64)
        run = 0
        for s in range(ranks):
            run = s * capacity if capacity > 0 else run
            for l in range(el):
                blk[s, l] = run
                run += rc[s, l]
        offsets = np.zeros(el + 1, np.int32)
        perm = []
        for l in range(el):
            offsets[l] = len(perm)
            for s in range(ranks):
                perm.extend(range(blk[s, l], blk[s, l] + rc[s, l]))
        offsets[el] = len(perm)
        nz = [l for l in range(el) if offsets[l + 1] > offsets[l]]
        active = np.zeros(el + 1, np.int32)
        active[0] = len(nz)
        active[1:1 + len(nz)] = nz
        return types.SimpleNamespace(offsets=offsets, active=active, perm=np.array(perm, np.int64), experts=el)

    def regroup(self, recv, lay):
        out = torch.zeros_like(recv)
        n = int(lay.offsets[-1])
        out[:n] = recv[torch.from_numpy(lay.perm[:n])]
        return out

    def ungroup(self, grouped, lay):
        out = torch.zeros_like(grouped)
        n = int(lay.offsets[-1])
        out[torch.from_numpy(lay.perm[:n])] = grouped[:n]
        return out

    def ffn(self, rows_in, lay, slab, mode=0):
        xb = _bits(rows_in)
        y = np.zeros_like(xb)
        for a in range(int(lay.active[0])):
            l = int(lay.active[1 + a])
            e = self.first + l
            for r in range(int(lay.offsets[l]), int(lay.offsets[l + 1])):
                y[r:r + 1] = mo.expert_forward(xb[r:r + 1], self.wg[e], self.wu[e], self.wd[e])
        return _bf16(y)

    def combine(self, y, y_rows, weights, inverse, residual):
        t_count, k = weights.shape
        yb = mo.bf16_to_f32(_bits(y))
        w = mo.bf16_to_f32(_bits(weights))
        inv = inverse.numpy().reshape(t_count, k)
        acc = np.zeros((t_count, y.shape[1]), np.float32)
        for s in range(k):
            acc = (acc + mo.bf16_round(yb[inv[:, s]] * w[:, s:s + 1])).astype(np.float32)
        return _bf16(mo.f32_to_bf16(acc))


def _reference_rows(x_bits, gate, wg, wu, wd):
    """Single-process layer on one rank's tokens, FFN row by row."""
    _, sel, w = mo.route(x_bits, gate, K, True)
    p = mo.compact_expert_groups(sel, w, E)
    rows = np.zeros((x_bits.shape[0] * K, H), np.uint16)
    off = p["offsets"]
    for e in range(E):
        for r in range(off[e], off[e + 1]):
            rows[r:r + 1] = mo.expert_forward(x_bits[p["tokens"][r:r + 1]], wg[e], wu[e], wd[e])
    return mo.combine(rows, p, x_bits.shape[0], K)


def _worker(rank, world, port, tokens, mode, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pdscope_b200.expert_parallel import ExpertParallelMoE, TorchDistExchange
        _, gate, wg, wu, wd = mo.synthetic_layer(31, 1, H, E, I)
        x = mo.synthetic_layer(100 + rank, tokens, H, E, I)[0]
        el = E // world
        slab = types.SimpleNamespace(num_slots=el)
        layer = ExpertParallelMoE(_bf16(gate), slab, rank=rank, world=world, exchange=TorchDistExchange(),
                                  top_k=K, ops=HostOps(wg, wu, wd, rank * el))
        out = layer.forward(_bf16(x), mode=mode)
        ref = _reference_rows(x, gate, wg, wu, wd)
        q.put((rank, bool(np.array_equal(_bits(out), ref))))
    except Exception as exc:  # report, then let the parent fail the test
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,tokens,mode", [(2, 5, "padded"), (2, 13, "exact"), (2, 40, None),
                                              (4, 6, "padded"), (4, 11, "exact")])
def test_expert_parallel_gloo(world, tokens, mode):
    """2 and 4 ranks (EL = 8 and 4 local experts; at 4 ranks min(k, EL) = k
    bounds the padded capacity)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tokens, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {r: True for r in range(world)}, results


def _lost_rank_worker(rank, world, port, q):
    """Rank 1 serves layer 0 and then leaves (between layers, before layer 1's
    count exchange, with nothing of its own in flight); rank 0 goes on to
    layer 1 and must get an error from the exchange, not wait forever."""
    import datetime
    import time
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    from pdscope_b200.expert_parallel import ExpertParallelMoE, TorchDistExchange
    _, gate, wg, wu, wd = mo.synthetic_layer(31, 1, H, E, I)
    x = mo.synthetic_layer(100 + rank, 4, H, E, I)[0]
    el = E // world
    layer = ExpertParallelMoE(_bf16(gate), types.SimpleNamespace(num_slots=el), rank=rank, world=world,
                              exchange=TorchDistExchange(), top_k=K, ops=HostOps(wg, wu, wd, rank * el))
    layer.forward(_bf16(x), mode="padded")                  # layer 0 on both ranks
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)                                         # gone without a goodbye
    t0 = time.monotonic()
    try:
        layer.forward(_bf16(x), mode="padded")              # layer 1: the peer never joins
        q.put((rank, "no error"))
    except Exception as exc:
        q.put((rank, ("raised", time.monotonic() - t0, type(exc).__name__)))
    q.close()
    q.join_thread()
    os._exit(0)


def test_lost_rank_raises_on_the_survivor():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lost_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "left"
    outcome = results[0]
    assert isinstance(outcome, tuple) and outcome[0] == "raised", outcome
    assert outcome[1] < 40.0, outcome          # within the process-group timeout (10 s) plus slack


def test_capacity_bound():
    """The padded block must hold every row a rank can send one destination:
    T tokens x min(k, EL) distinct experts per token."""
    from pdscope_b200.expert_parallel import ExpertParallelMoE
    slab = types.SimpleNamespace(num_slots=8)
    layer = ExpertParallelMoE(torch.zeros(16, 8, dtype=torch.bfloat16), slab, rank=0, world=2, top_k=4)
    assert layer.capacity(10) == 10 * 4
    layer = ExpertParallelMoE(torch.zeros(16, 8, dtype=torch.bfloat16), types.SimpleNamespace(num_slots=2),
                              rank=0, world=8, top_k=4)
    assert layer.capacity(10) == 10 * 2
