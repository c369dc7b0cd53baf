"""Expert parallelism for the MoE layer: experts sharded over GPUs.

The reference is single-GPU (one process, experts resident or offloaded).
This module serves the same layer with the 128 experts split evenly over the
ranks of a process group -- expert e on rank e // EL, EL = E / ranks -- and
one NCCL all-to-all each way over NVLink.  Each rank owns its own tokens;
routing is replicated (every rank holds the router).

Per layer on every rank:
  1. route + pack locally (all E experts)                     pdx_route_topk, pdx_pack
  2. dispatch: packed rows for rank d are the contiguous range of experts
     [d*EL, (d+1)*EL); all-to-all of the per-expert counts, then of the rows
  3. the received rows are regrouped by local expert (every source's rows of
     expert l made contiguous), so each local expert's weights are streamed
     once per layer however many ranks sent it rows; one grouped FFN; the
     results are put back in the receive layout      pdx_ep_layout, pdx_ep_regroup,
                                                      pdx_moe_ffn_grouped, pdx_ep_ungroup
  4. all-to-all of the unweighted rows back, weighted combine in slot order
                                                      pdx_ep_combine
Two exchange forms:
  * padded (decode, T <= 256 per rank): every (source, destination) block has the fixed
    capacity T*min(k, EL) rows, so sizes never leave the device (no host sync;
    the whole step can be captured in a CUDA graph);
  * exact (prefill): the counts are read back to size an exact all-to-all
    (one host sync per layer, like the reference's grouping sync).
Arithmetic per row is identical to the single-GPU layer, so outputs match it
bit for bit (the same rows meet the same weights; combine order is slot order).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lib
from .runtime import LN_EPS, ExpertSlab, Packed, _ptr, _stream, pack as _pack, residual_layernorm

PADDED_MAX_TOKENS = 256


@dataclass
class Layout:
    """Regrouped receive buffer: local expert l's rows from all sources at
    [offsets[l], offsets[l+1]); perm[g] = receive-buffer row of regrouped row g."""
    offsets: torch.Tensor   # int32 [EL+1]
    active: torch.Tensor    # int32 [EL+1]
    perm: torch.Tensor      # int32 [rows_cap]
    experts: int            # EL


class DeviceOps:
    """The sm_100a kernels used by ExpertParallelMoE (libpdx_moe)."""

    def route(self, x, gate, top_k, normalize):
        t_count, hidden = x.shape
        experts = gate.shape[0]
        dev = x.device
        logits = torch.empty((t_count, experts), dtype=torch.bfloat16, device=dev)
        sel = torch.empty((t_count, top_k), dtype=torch.int64, device=dev)
        w = torch.empty((t_count, top_k), dtype=torch.bfloat16, device=dev)
        ws = torch.empty(lib.pdx_route_workspace_bytes(t_count, experts), dtype=torch.uint8, device=dev)
        check(lib.pdx_route_topk(_ptr(x), _ptr(gate), t_count, hidden, experts, top_k, int(normalize), _ptr(logits),
                                 _ptr(sel), _ptr(w), _ptr(ws), ws.numel(), _stream()))
        return sel, w

    def pack(self, sel, w, experts):
        return _pack(sel, w, experts)

    def gather(self, x, tokens):
        rows = tokens.numel()
        out = torch.empty((rows, x.shape[1]), dtype=x.dtype, device=x.device)
        check(lib.pdx_gather_rows(_ptr(x), _ptr(tokens), rows, x.shape[1], _ptr(out), _stream()))
        return out

    def dispatch(self, x, p, top_k, experts, ranks, capacity):
        t_count, hidden = x.shape
        # rows past a block's count are sent but never read (the receiver's layout
        # comes from the counts), so the buffer needs no clearing
        send = torch.empty((ranks * capacity, hidden), dtype=x.dtype, device=x.device)
        inv_ep = torch.empty(t_count * top_k, dtype=torch.int32, device=x.device)
        check(lib.pdx_ep_dispatch(_ptr(x), _ptr(p.tokens), _ptr(p.positions), _ptr(p.offsets), t_count, top_k,
                                  hidden, experts, ranks, capacity, _ptr(send), _ptr(inv_ep), _stream()))
        return send, inv_ep

    def layout(self, recv_counts, ranks, local_experts, capacity, rows_cap):
        dev = recv_counts.device
        lay = Layout(offsets=torch.empty(local_experts + 1, dtype=torch.int32, device=dev),
                     active=torch.empty(local_experts + 1, dtype=torch.int32, device=dev),
                     perm=torch.empty(max(rows_cap, 1), dtype=torch.int32, device=dev), experts=local_experts)
        check(lib.pdx_ep_layout(_ptr(recv_counts), ranks, local_experts, capacity, rows_cap, _ptr(lay.offsets),
                                _ptr(lay.active), _ptr(lay.perm), _stream()))
        return lay

    def regroup(self, recv, lay):
        out = torch.empty_like(recv)
        check(lib.pdx_ep_regroup(_ptr(recv), _ptr(lay.perm), _ptr(lay.offsets), lay.experts, recv.shape[0],
                                 recv.shape[1], _ptr(out), _stream()))
        return out

    def ungroup(self, grouped, lay):
        out = torch.empty_like(grouped)
        check(lib.pdx_ep_ungroup(_ptr(grouped), _ptr(lay.perm), _ptr(lay.offsets), lay.experts, grouped.shape[0],
                                 grouped.shape[1], _ptr(out), _stream()))
        return out

    def ffn(self, rows_in, lay, slab, mode=_lib.FFN_AUTO):
        rows, hidden = rows_in.shape
        y = torch.empty_like(rows_in)
        ws = torch.empty(lib.pdx_ffn_workspace_bytes(rows, lay.experts, hidden, slab.inter, mode),
                         dtype=torch.uint8, device=rows_in.device)
        check(lib.pdx_moe_ffn_grouped(_ptr(rows_in), rows, None, _ptr(lay.offsets), _ptr(lay.active), lay.experts,
                                      rows, ctypes.byref(slab.struct), hidden, slab.inter, _ptr(y), mode, _ptr(ws),
                                      ws.numel(), _stream()))
        return y

    def combine(self, y, y_rows, weights, inverse, residual):
        t_count, k = weights.shape
        out = torch.empty((t_count, y.shape[1]), dtype=torch.bfloat16, device=y.device)
        check(lib.pdx_ep_combine(_ptr(y), y_rows, _ptr(weights), _ptr(inverse), t_count, k, y.shape[1],
                                 _ptr(residual), _ptr(out), _stream()))
        return out


class TorchDistExchange:
    """All-to-all over a torch.distributed process group (NCCL on GPUs).

    BF16 payloads travel as raw bytes (a uint8 view keeps dim 0, so row splits
    still apply) so every backend can carry them."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_to_all(self, inp, out_rows=None, in_splits=None, out_splits=None):
        shape = (out_rows if out_rows is not None else inp.shape[0],) + tuple(inp.shape[1:])
        out = torch.empty(shape, dtype=inp.dtype, device=inp.device)
        a = out.view(torch.uint8) if out.dtype == torch.bfloat16 else out
        b = inp.view(torch.uint8) if inp.dtype == torch.bfloat16 else inp
        self.dist.all_to_all_single(a, b, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                    group=self.group)
        return out


@dataclass
class Dispatched:
    """State of one layer between the exchanges on one rank."""
    t_count: int
    weights: torch.Tensor
    packed: Packed
    mode: str
    capacity: int
    send: torch.Tensor
    inverse: torch.Tensor
    send_splits: list | None = None


class ExpertParallelMoE:
    """One MoE layer whose experts are sharded over the ranks of a group.

    ``gate`` [E, H] is the full router (replicated); ``local_slab`` holds this
    rank's EL = E / world experts in slots 0..EL-1 (global expert rank*EL + l
    in slot l).
    """

    def __init__(self, gate, local_slab, *, rank, world, exchange=None, top_k=8, normalize=True, ops=None):
        self.gate, self.slab = gate, local_slab
        self.experts, self.hidden = gate.shape
        if self.experts % world:
            raise ValueError("experts must divide evenly over the ranks")
        self.local = self.experts // world
        if local_slab.num_slots < self.local:
            raise ValueError("local slab holds fewer experts than this rank owns")
        self.rank, self.world = rank, world
        self.top_k, self.normalize = top_k, normalize
        self.exchange = exchange
        self.ops = ops or DeviceOps()

    def capacity(self, t_count):
        return t_count * min(self.top_k, self.local)

    # ---- phase 1: route, pack, lay out the send buffer --------------------------
    def dispatch(self, x, mode=None):
        t_count = x.shape[0]
        mode = mode or ("padded" if t_count <= PADDED_MAX_TOKENS else "exact")
        sel, w = self.ops.route(x, self.gate, self.top_k, self.normalize)
        p = self.ops.pack(sel, w, self.experts)
        if mode == "padded":
            cap = self.capacity(t_count)
            send, inv = self.ops.dispatch(x, p, self.top_k, self.experts, self.world, cap)
            return Dispatched(t_count, w, p, mode, cap, send, inv)
        send = self.ops.gather(x, p.tokens)
        return Dispatched(t_count, w, p, mode, 0, send, p.inverse)

    # ---- phase 2: experts of this rank on the received rows -----------------------
    def compute(self, recv, recv_counts, capacity):
        """Regroup by local expert, one grouped FFN, back to the receive layout."""
        if recv.shape[0] == 0:
            return recv
        lay = self.ops.layout(recv_counts, self.world, self.local, capacity, recv.shape[0])
        self.last_active = lay.active
        grouped = self.ops.regroup(recv, lay)
        mode = _lib.FFN_GEMV if capacity > 0 else _lib.FFN_AUTO   # decode: weight-streaming path
        y = self.ops.ffn(grouped, lay, self.slab, mode)
        return self.ops.ungroup(y, lay)

    # ---- phase 3: weighted combine of the returned rows -----------------------------
    def finish(self, d, back, residual=None):
        return self.ops.combine(back, back.shape[0], d.weights, d.inverse, residual)

    # ---- padded exchange over NVLink peer memory ----------------------------------------
    def forward_p2p(self, x, peer, layer, residual=None, norm=False, marks=None):
        """The padded layer with the exchange done by peer stores and flags
        (pdx_ep_dispatch_p2p ... pdx_ep_wait_back) instead of all-to-alls.
        With ``norm`` the output is layer_norm(MoE(x) + residual).  ``marks``
        (a list) receives (stage, CUDA event) pairs recorded after each stage."""
        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))
        t_count, hidden = x.shape
        cap = self.capacity(t_count)
        if cap > peer.cap_max:
            raise ValueError("batch larger than the peer exchange was sized for")
        if (hidden, self.local, self.world, self.rank) != (peer.H, peer.EL, peer.R, peer.rank) or \
                not 0 <= layer < peer.L:
            raise ValueError("peer exchange regions were sized for another layer shape, group or layer count")
        R, EL, k, dev = self.world, self.local, self.top_k, x.device
        mark("start")
        sel, w = self.ops.route(x, self.gate, k, self.normalize)
        p = self.ops.pack(sel, w, self.experts)
        mark("route_pack")
        lay = ctypes.byref(peer.structs[layer])
        inv = torch.empty(t_count * k, dtype=torch.int32, device=dev)
        s = _stream()
        check(lib.pdx_ep_dispatch_p2p(_ptr(x), _ptr(p.tokens), _ptr(p.positions), _ptr(p.offsets), t_count, k, hidden,
                                      self.experts, R, self.rank, cap, lay, _ptr(inv), s))
        mark("dispatch")
        rows_cap = R * cap
        ly = Layout(offsets=torch.empty(EL + 1, dtype=torch.int32, device=dev),
                    active=torch.empty(EL + 1, dtype=torch.int32, device=dev),
                    perm=torch.empty(rows_cap, dtype=torch.int32, device=dev), experts=EL)
        check(lib.pdx_ep_layout_p2p(R, self.rank, EL, cap, rows_cap, lay, _ptr(ly.offsets), _ptr(ly.active),
                                    _ptr(ly.perm), s))
        self.last_active = ly.active   # this rank's active local experts (a graph replay refreshes it)
        mark("layout_wait")
        grouped = torch.empty((rows_cap, hidden), dtype=x.dtype, device=dev)
        check(lib.pdx_ep_regroup(ctypes.c_void_p(peer.local(layer, "recv")), _ptr(ly.perm), _ptr(ly.offsets), EL,
                                 rows_cap, hidden, _ptr(grouped), s))
        mark("regroup")
        y = self.ops.ffn(grouped, ly, self.slab, _lib.FFN_GEMV)
        mark("ffn")
        check(lib.pdx_ep_return_p2p(_ptr(y), _ptr(ly.perm), _ptr(ly.offsets), EL, rows_cap, hidden, R, self.rank, cap,
                                    lay, s))
        mark("return")
        check(lib.pdx_ep_wait_back(R, self.rank, lay, s))
        mark("wait_back")
        out = torch.empty((t_count, hidden), dtype=torch.bfloat16, device=dev)
        back = ctypes.c_void_p(peer.local(layer, "back"))
        if norm:
            check(lib.pdx_ep_combine_layernorm(back, rows_cap, _ptr(w), _ptr(inv), t_count, k, hidden, _ptr(residual),
                                               ctypes.c_float(LN_EPS), _ptr(out), s))
        else:
            check(lib.pdx_ep_combine(back, rows_cap, _ptr(w), _ptr(inv), t_count, k, hidden, _ptr(residual),
                                     _ptr(out), s))
        mark("combine")
        return out

    # ---- the whole layer over the exchange -------------------------------------------
    def forward(self, x, residual=None, mode=None):
        ex = self.exchange
        d = self.dispatch(x, mode)
        recv_counts = ex.all_to_all(d.packed.counts)
        if d.mode == "padded":
            recv = ex.all_to_all(d.send)
            y = self.compute(recv, recv_counts, d.capacity)
            back = ex.all_to_all(y)
        else:
            sc = d.packed.counts.view(self.world, self.local).sum(1).tolist()   # host sync (sizes)
            rc = recv_counts.view(self.world, self.local).sum(1).tolist()
            recv = ex.all_to_all(d.send, out_rows=sum(rc), in_splits=sc, out_splits=rc)
            y = self.compute(recv, recv_counts, 0)
            back = ex.all_to_all(y, out_rows=sum(sc), in_splits=rc, out_splits=sc)
        return self.finish(d, back, residual)


def local_slab_of(full_slab, rank, world):
    """Slots [rank*EL, (rank+1)*EL) of a full-layer slab as a rank-local slab (a view)."""
    el = full_slab.num_slots // world
    per = 3 * full_slab.inter * full_slab.hidden
    return ExpertSlab(full_slab.storage[rank * el * per:(rank + 1) * el * per], full_slab.hidden, full_slab.inter)


class PeerExchange:
    """Exchange regions of every layer mapped into every rank of the group
    (CUDA IPC), for the padded exchange over NVLink peer memory
    (pdx_ep_*_p2p).  Per layer: recv / back blocks [R][C][H] BF16 for up to
    ``max_tokens`` tokens per rank, per-source expert counts and flags; a local
    step counter and two ticket words per layer.  Collective construction and
    ``close`` (every rank calls both)."""

    def __init__(self, layers, max_tokens, *, world, rank, local_experts, hidden, top_k, device, group=None):
        import torch.distributed as dist
        self.L, self.R, self.rank, self.EL, self.H = layers, world, rank, local_experts, hidden
        self.cap_max = max_tokens * min(top_k, local_experts)
        a = lambda n: (n + 255) // 256 * 256
        blk = a(self.R * self.cap_max * hidden * 2)
        self.off = dict(recv=0, back=blk, cnt=2 * blk, rflag=2 * blk + a(self.R * self.EL * 4),
                        bflag=2 * blk + a(self.R * self.EL * 4) + a(self.R * 8))
        self.per_layer = self.off["bflag"] + a(self.R * 8)
        ptr = ctypes.c_void_p()
        check(lib.pdx_p2p_alloc(self.per_layer * layers, ctypes.byref(ptr)))
        self.base = ptr.value
        handle = ctypes.create_string_buffer(64)
        check(lib.pdx_ipc_handle(self.base, handle))
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.peer_base, self._opened = [], []
        for r in range(world):
            if r == rank:
                self.peer_base.append(self.base)
                continue
            q = ctypes.c_void_p()
            check(lib.pdx_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(q)))
            self.peer_base.append(q.value)
            self._opened.append(q.value)
        tbl = torch.empty((layers, 5, world), dtype=torch.int64)
        for l in range(layers):
            for i, key in enumerate(("recv", "back", "cnt", "rflag", "bflag")):
                for r in range(world):
                    tbl[l, i, r] = self.peer_base[r] + l * self.per_layer + self.off[key]
        self.tbl = tbl.to(device)
        self.step = torch.zeros(layers, dtype=torch.int64, device=device)
        self.ticket = torch.zeros((layers, 2), dtype=torch.int32, device=device)
        self.structs = []
        for l in range(layers):
            t = self.tbl[l]
            self.structs.append(_lib.P2PLayer(recv=t[0].data_ptr(), back=t[1].data_ptr(), cnt=t[2].data_ptr(),
                                              rflag=t[3].data_ptr(), bflag=t[4].data_ptr(),
                                              step=self.step[l].data_ptr(), ticket=self.ticket[l].data_ptr()))
        self.group = group
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def local(self, layer, key):
        return self.base + layer * self.per_layer + self.off[key]

    def close(self):
        """Unmap the peers' regions and free this rank's (collective)."""
        import torch.distributed as dist
        if self.base is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for q in self._opened:
            lib.pdx_ipc_close(q)
        self._opened = []
        dist.barrier(group=self.group)
        lib.pdx_p2p_free(self.base)
        self.base = None


class ExpertParallelStack:
    """``layers`` expert-parallel MoE layers driven as one step on every rank.

    Layer l+1's input is ``layer_norm(MoE_l(x_l) + x_l)`` (the resident
    stack's next-layer activation).  ``step`` replays one CUDA graph per batch size holding every
    layer's kernels and NCCL exchanges (padded exchange only: all ranks must
    use the same batch size).
    """

    def __init__(self, gates, local_slabs, *, rank, world, exchange, top_k=8, peer=None):
        self.layers = [ExpertParallelMoE(g, s, rank=rank, world=world, exchange=exchange, top_k=top_k)
                       for g, s in zip(gates, local_slabs)]
        self.hidden = gates[0].shape[1]
        self.device = gates[0].device
        self.peer = peer          # PeerExchange: padded layers exchange over peer memory
        self._graphs, self._io = {}, {}

    def io(self, t_count):
        if t_count not in self._io:
            self._io[t_count] = (torch.zeros((t_count, self.hidden), dtype=torch.bfloat16, device=self.device),
                                 torch.zeros((t_count, self.hidden), dtype=torch.bfloat16, device=self.device))
        return self._io[t_count]

    def _run(self, t_count, mode):
        x, out = self.io(t_count)
        h = x
        for i, layer in enumerate(self.layers):
            if mode == "padded" and self.peer is not None:
                h = layer.forward_p2p(h, self.peer, i, residual=h, norm=True)
            else:
                y = layer.forward(h, residual=None, mode=mode)
                h = residual_layernorm(y, h, out=y)
        out.copy_(h)

    def step(self, t_count, *, graph=True):
        mode = "padded" if t_count <= PADDED_MAX_TOKENS else "exact"
        if not graph or mode == "exact":
            self._run(t_count, mode)
            return
        g = self._graphs.get(t_count)
        if g is None:
            self._run(t_count, mode)          # warm: workspaces, device attributes
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._run(t_count, mode)
            self._graphs[t_count] = g
        g.replay()

    def local_active_experts(self):
        """Per layer, how many of this rank's experts received rows in the
        last step (synchronises the device)."""
        return [int(layer.last_active[0].item()) for layer in self.layers]

    def release_graphs(self):
        """Drop the captured graphs (they hold NCCL work; release before
        destroying the process group)."""
        self._graphs.clear()

    def stage_times_us(self, t_count, layers=8, repeats=3):
        """Mean device time per layer of each stage of the peer-exchange
        decode layer (route+pack, dispatch, layout incl. the wait for every
        source's flag, regroup, FFN, return, wait for the returned blocks,
        combine), from CUDA events recorded between the stages of eager
        layers on this rank.  Every rank must call it (the stages wait on one
        another)."""
        if self.peer is None:
            raise ValueError("stage timing covers the peer-memory exchange")
        x, _ = self.io(t_count)
        tot, n = {}, 0
        for _ in range(repeats):
            h = x
            for i, layer in enumerate(self.layers[:layers]):
                marks = []
                h = layer.forward_p2p(h, self.peer, i, residual=h, norm=True, marks=marks)
                torch.cuda.synchronize(self.device)
                for (_, a), (name, b) in zip(marks, marks[1:]):
                    tot[name] = tot.get(name, 0.0) + a.elapsed_time(b) * 1e3
                n += 1
        return {name: v / n for name, v in tot.items()}
