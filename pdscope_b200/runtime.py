"""Host-side mirror of PDScope's MoE expert path over the sm_100a kernels.

Same names, argument meaning and error behaviour as the reference
(nezha-Anonymous/PDScope); every numeric step runs in libpdx_moe.so:

* ``Routing``, ``route``            expertbench/adapters/qwen.py:132-152
* ``expert_groups``                 expertbench/adapters/qwen.py:155-174
* ``compact_expert_groups``         expertbench/pdscope_runtime.py:16-39
* ``expert_forward``                expertbench/adapters/qwen.py:87-90
* ``PdxGpuBackend``                 the ExpertExecutor.gpu_backend hook,
                                    expertbench/executor.py:178, 476-477
* ``PDScopeCudaRuntime.forward``    expertbench/pdscope_runtime.py:208-512
                                    (HBM-resident experts)

Tensors are torch CUDA tensors (BF16 activations and weights); torch is used
for device memory and streams only.  Kernels run on the caller's current
stream.
"""
from __future__ import annotations

import ctypes
import hashlib
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import ExpertWeights, check, lib

PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


class _Workspace:
    """Grow-only scratch buffers, one per (device, purpose)."""

    def __init__(self):
        self._bufs = {}

    def get(self, device, nbytes, tag="default"):
        key = (device.index if device.index is not None else torch.cuda.current_device(), tag)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


_WS = _Workspace()


def _require_cuda_bf16(name, t, ndim=None):
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda" or t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be a BF16 CUDA tensor")
    if ndim is not None and t.ndim != ndim:
        raise ValueError(f"{name} must have {ndim} dimensions")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def raise_device_error():
    """Synchronise the current stream and turn a device error word into an exception."""
    code = _lib.device_error(_stream())
    if code == _lib.PDX_DEVERR_BAD_EXPERT:
        raise ValueError("expert ID outside configured range")
    if code == _lib.PDX_DEVERR_BAD_SLOT:
        raise ValueError("expert slot outside the weight slab")
    if code:
        raise _lib.PdxError(f"device error {code} (bounded wait expired)")


# ---------------------------------------------------------------------------
# a1: routing
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class Routing:
    logits: object
    selected: object
    weights: object
    probabilities: object = None


def route(inputs, gate, top_k, normalize, *, capture_probabilities=False):
    """Qwen3's native gate order on the B200 (qwen.py:140-152).

    logits = F.linear(inputs, gate) (exact dot products rounded once to BF16);
    selected/weights = renormalised top-k of the FP32 softmax.
    ``capture_probabilities`` returns the FP32 softmax of the logits as a
    diagnostic, as the reference does.
    """
    if inputs.ndim != 2 or inputs.shape[1] != gate.shape[1] or inputs.dtype != gate.dtype:
        raise ValueError("router input shape/dtype mismatch")
    if (type(top_k) is not int or not 0 < top_k <= gate.shape[0] or type(normalize) is not bool
            or type(capture_probabilities) is not bool):
        raise ValueError("invalid routing parameters")
    _require_cuda_bf16("inputs", inputs, 2)
    _require_cuda_bf16("gate", gate, 2)
    t_count, hidden = inputs.shape
    experts = gate.shape[0]
    dev = inputs.device
    logits = torch.empty((t_count, experts), dtype=torch.bfloat16, device=dev)
    selected = torch.empty((t_count, top_k), dtype=torch.int64, device=dev)
    weights = torch.empty((t_count, top_k), dtype=torch.bfloat16, device=dev)
    ws_bytes = lib.pdx_route_workspace_bytes(t_count, experts)
    ws = _WS.get(dev, ws_bytes, "route")
    check(lib.pdx_route_topk(_ptr(inputs), _ptr(gate), t_count, hidden, experts, top_k, int(normalize),
                             _ptr(logits), _ptr(selected), _ptr(weights), _ptr(ws), ws.numel(), _stream()))
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32) if capture_probabilities else None
    return Routing(logits, selected, weights, probs)


def topk_from_logits(logits, top_k, normalize):
    """Softmax/top-k/renormalise on given BF16 logits (qwen.py:148-152 alone)."""
    _require_cuda_bf16("logits", logits, 2)
    t_count, experts = logits.shape
    selected = torch.empty((t_count, top_k), dtype=torch.int64, device=logits.device)
    weights = torch.empty((t_count, top_k), dtype=torch.bfloat16, device=logits.device)
    check(lib.pdx_topk_from_logits(_ptr(logits), t_count, experts, top_k, int(normalize), _ptr(selected),
                                   _ptr(weights), _stream()))
    return selected, weights


# ---------------------------------------------------------------------------
# a2/a3: packing
# ---------------------------------------------------------------------------


@dataclass
class Packed:
    """Device-side packed layout of one layer's routed assignments."""
    counts: torch.Tensor      # int32 [E]
    offsets: torch.Tensor     # int32 [E+1]
    tokens: torch.Tensor      # int32 [T*k]
    positions: torch.Tensor   # int32 [T*k]
    weights: torch.Tensor     # bf16  [T*k]
    inverse: torch.Tensor     # int32 [T*k]
    active: torch.Tensor      # int32 [E+1]


def pack(selected, weights, experts):
    """Stable slot-major counting sort (pdscope_runtime.py:25-31) on the device."""
    if selected.ndim != 2:
        raise ValueError("selected must be [T, k]")
    n, k = selected.shape
    if n < 1 or k < 1:
        raise ValueError("empty expert routing")
    if selected.dtype != torch.int64 or selected.device.type != "cuda" or not selected.is_contiguous():
        raise ValueError("selected must be a contiguous int64 CUDA tensor")
    _require_cuda_bf16("weights", weights, 2)
    dev = selected.device
    i32 = dict(dtype=torch.int32, device=dev)
    out = Packed(counts=torch.empty(experts, **i32), offsets=torch.empty(experts + 1, **i32),
                 tokens=torch.empty(n * k, **i32), positions=torch.empty(n * k, **i32),
                 weights=torch.empty(n * k, dtype=torch.bfloat16, device=dev),
                 inverse=torch.empty(n * k, **i32), active=torch.empty(experts + 1, **i32))
    ws_bytes = lib.pdx_pack_workspace_bytes(n, k, experts)
    ws = _WS.get(dev, ws_bytes, "pack")
    check(lib.pdx_pack(_ptr(selected), _ptr(weights), n, k, experts, _ptr(out.counts), _ptr(out.offsets),
                       _ptr(out.tokens), _ptr(out.positions), _ptr(out.weights), _ptr(out.inverse),
                       _ptr(out.active), _ptr(ws), ws.numel(), _stream()))
    return out


def compact_expert_groups(routing, experts=128):
    """Group true IDs in native slot/token order (pdscope_runtime.py:16-39).

    Returns ``(groups, cpu_indices)`` with ``groups[e] = (tokens int64 [n_e] on
    the device, weights bf16 [n_e])`` and ``cpu_indices[e]`` the same tokens on
    the host -- one device-to-host copy of the counts and token order, as in
    the reference.
    """
    n, k = routing.selected.shape
    if n < 1 or k < 1:
        raise ValueError("empty expert routing")
    p = pack(routing.selected, routing.weights, experts)
    counts = p.counts.cpu()  # synchronises the stream
    raise_device_error()
    tokens = p.tokens.long()
    tokens_cpu = tokens.cpu()
    groups, cpu_indices, start = {}, {}, 0
    for e, count in enumerate(counts.tolist()):
        if count:
            end = start + count
            groups[e] = (tokens[start:end], p.weights[start:end])
            cpu_indices[e] = tokens_cpu[start:end]
            start = end
    return groups, cpu_indices


def expert_groups(routing, *, mode="generic"):
    """Deterministic expert-ID order and native top-k-slot/token order (qwen.py:155-174)."""
    if mode not in ("generic", "single_token"):
        raise ValueError("unsupported expert grouping mode")
    if mode == "single_token":
        if routing.selected.ndim != 2 or routing.selected.shape[0] != 1:
            raise ValueError("single-token grouping requires exactly one token")
        ids = routing.selected.detach().cpu()[0].tolist()
        if not ids or len(set(ids)) != len(ids):
            raise ValueError("single-token grouping requires distinct selected expert IDs")
        tokens = torch.zeros((1,), dtype=torch.long, device=routing.selected.device)
        return [(expert, tokens, routing.weights[0, slot:slot + 1])
                for slot, expert in sorted(enumerate(ids), key=lambda pair: pair[1])]
    experts = int(routing.logits.shape[1]) if routing.logits is not None else 128
    groups, _ = compact_expert_groups(routing, experts)
    return [(e, t, w) for e, (t, w) in sorted(groups.items())]


# ---------------------------------------------------------------------------
# a5: expert FFN
# ---------------------------------------------------------------------------


def expert_forward(inputs, tensors):
    """Native expert formula (qwen.py:87-90) for one expert on the B200.

    ``tensors`` holds BF16 CUDA ``gate_proj`` [I,H], ``up_proj`` [I,H] and
    ``down_proj`` [H,I]; the result is the unweighted [n,H] BF16 output with the
    reference's rounding points.
    """
    _require_cuda_bf16("inputs", inputs, 2)
    g, u, d = (tensors[name] for name in PROJECTIONS)
    for name, t in zip(PROJECTIONS, (g, u, d)):
        _require_cuda_bf16(name, t, 2)
    inter, hidden = g.shape
    if inputs.shape[1] != hidden or u.shape != g.shape or d.shape != (hidden, inter):
        raise ValueError("invalid expert input shape")
    n = inputs.shape[0]
    out = torch.empty((n, hidden), dtype=torch.bfloat16, device=inputs.device)
    ws_bytes = lib.pdx_expert_ffn_workspace_bytes(n, hidden, inter)
    ws = _WS.get(inputs.device, ws_bytes, "expert")
    check(lib.pdx_expert_ffn(_ptr(inputs), n, _ptr(g), _ptr(u), _ptr(d), hidden, inter, _ptr(out), _ptr(ws),
                             ws.numel(), _stream()))
    return out


class PdxGpuBackend:
    """Drop-in for ``ExpertExecutor.gpu_backend`` (executor.py:178, 476-477).

    ``executor.gpu_backend = PdxGpuBackend()`` makes every GPU expert of the
    reference's executor run on the sm_100a kernels; the call happens on the
    executor's compute stream, weights are the borrowed cache-slot views and
    are not retained.
    """

    def __init__(self):
        self.calls = 0

    def __call__(self, key, inputs, tensors):
        self.calls += 1
        return expert_forward(inputs, tensors)


# ---------------------------------------------------------------------------
# a7: combine
# ---------------------------------------------------------------------------


def combine(rows, weights, inverse, residual=None):
    """Deterministic fused merge (pdscope_runtime.py:454-464).

    ``rows`` [T*k, H] unweighted expert outputs in packed order, ``weights``
    the [T, k] routing weights, ``inverse`` [T*k] the packed row of each
    (token, slot).
    """
    _require_cuda_bf16("rows", rows, 2)
    _require_cuda_bf16("weights", weights, 2)
    t_count, k = weights.shape
    hidden = rows.shape[1]
    out = torch.empty((t_count, hidden), dtype=torch.bfloat16, device=rows.device)
    if residual is not None:
        _require_cuda_bf16("residual", residual, 2)
    check(lib.pdx_combine(_ptr(rows), _ptr(weights), _ptr(inverse), t_count, k, hidden, _ptr(residual),
                          _ptr(out), _stream()))
    return out


LN_EPS = 1e-5


def residual_layernorm(y, residual, eps=LN_EPS, out=None):
    """Next-layer activation of a multi-layer stack as the reference's
    two-layer protocol forms it (benchmarks/pdscope_compare.py:609-705):
    ``layer_norm(y.float() + residual.float(), (H,)).to(bf16)``.  ``out`` may
    be ``y`` or ``residual``."""
    _require_cuda_bf16("y", y, 2)
    _require_cuda_bf16("residual", residual, 2)
    if y.shape != residual.shape:
        raise ValueError("y and residual shapes differ")
    t_count, hidden = y.shape
    if out is None:
        out = torch.empty_like(y)
    check(lib.pdx_residual_layernorm(_ptr(y), _ptr(residual), t_count, hidden, ctypes.c_float(eps), _ptr(out),
                                     _stream()))
    return out


# ---------------------------------------------------------------------------
# Weight placement
# ---------------------------------------------------------------------------


class ExpertSlab:
    """Experts of one layer (or several) in equal BF16 slots [gate | up | down].

    This is the layout of the reference's ExpertExecutor cache slab
    (executor.py:219-227, 323-331): slot s holds gate_proj [I,H], up_proj [I,H]
    and down_proj [H,I] back to back.  ``slot_of_expert`` (int32 CUDA [E],
    optional) maps expert ids to slots.
    """

    def __init__(self, storage, hidden, inter, slot_of_expert=None):
        _require_cuda_bf16("storage", storage)
        per_slot = 3 * inter * hidden
        if storage.numel() % per_slot:
            raise ValueError("slab does not hold whole expert slots")
        self.storage = storage.view(-1)
        self.hidden, self.inter = hidden, inter
        self.num_slots = storage.numel() // per_slot
        self.slot_of_expert = slot_of_expert
        base = self.storage.data_ptr()
        self.struct = ExpertWeights(gate=base, up=base + inter * hidden * 2, down=base + 2 * inter * hidden * 2,
                                    gate_stride=per_slot, up_stride=per_slot, down_stride=per_slot,
                                    num_slots=self.num_slots,
                                    slot_of_expert=slot_of_expert.data_ptr() if slot_of_expert is not None else None)

    @classmethod
    def allocate(cls, num_slots, hidden, inter, device, std=0.02, generator=None):
        """Random-init slab (weights ~N(0, std)) generated on the device."""
        storage = torch.empty(num_slots * 3 * inter * hidden, dtype=torch.bfloat16, device=device)
        step = 3 * inter * hidden
        for s in range(num_slots):
            chunk = torch.randn(step, dtype=torch.float32, device=device, generator=generator)
            storage[s * step:(s + 1) * step] = (chunk * std).to(torch.bfloat16)
        return cls(storage, hidden, inter)

    @classmethod
    def from_tensors(cls, experts, device=None):
        """Pack a list of {gate_proj, up_proj, down_proj} dicts into a slab."""
        g0 = experts[0]["gate_proj"]
        inter, hidden = g0.shape
        device = device or g0.device
        storage = torch.empty(len(experts) * 3 * inter * hidden, dtype=torch.bfloat16, device=device)
        view = storage.view(len(experts), 3 * inter * hidden)
        for s, ex in enumerate(experts):
            view[s, :inter * hidden] = ex["gate_proj"].reshape(-1)
            view[s, inter * hidden:2 * inter * hidden] = ex["up_proj"].reshape(-1)
            view[s, 2 * inter * hidden:] = ex["down_proj"].reshape(-1)
        return cls(storage, hidden, inter)

    def expert_tensors(self, slot):
        """Views of one slot as the reference's {gate_proj, up_proj, down_proj} dict."""
        i, h = self.inter, self.hidden
        flat = self.storage[slot * 3 * i * h:(slot + 1) * 3 * i * h]
        return dict(gate_proj=flat[:i * h].view(i, h), up_proj=flat[i * h:2 * i * h].view(i, h),
                    down_proj=flat[2 * i * h:].view(h, i))


# ---------------------------------------------------------------------------
# Whole layer
# ---------------------------------------------------------------------------


@dataclass
class LayerOutputs:
    out: torch.Tensor
    logits: torch.Tensor
    selected: torch.Tensor
    weights: torch.Tensor
    counts: torch.Tensor


class ResidentMoELayer:
    """One MoE layer whose experts are all resident in HBM.

    ``forward`` runs route -> pack -> grouped FFN -> combine in one C-ABI call
    with no host synchronisation.
    """

    def __init__(self, gate, slab, top_k=8, normalize=True):
        _require_cuda_bf16("gate", gate, 2)
        if gate.shape[1] != slab.hidden:
            raise ValueError("router and expert hidden sizes differ")
        self.gate, self.slab = gate, slab
        self.experts, self.hidden = gate.shape
        self.inter = slab.inter
        self.top_k, self.normalize = top_k, normalize

    def workspace_bytes(self, t_count, mode=_lib.FFN_AUTO):
        return lib.pdx_layer_workspace_bytes(t_count, self.hidden, self.experts, self.top_k, self.inter, mode)

    def forward(self, x, residual=None, *, mode=_lib.FFN_AUTO, outputs=None, workspace=None):
        _require_cuda_bf16("x", x, 2)
        t_count = x.shape[0]
        dev = x.device
        if outputs is None:
            outputs = LayerOutputs(
                out=torch.empty((t_count, self.hidden), dtype=torch.bfloat16, device=dev),
                logits=torch.empty((t_count, self.experts), dtype=torch.bfloat16, device=dev),
                selected=torch.empty((t_count, self.top_k), dtype=torch.int64, device=dev),
                weights=torch.empty((t_count, self.top_k), dtype=torch.bfloat16, device=dev),
                counts=torch.empty(self.experts, dtype=torch.int32, device=dev))
        if workspace is None:
            workspace = _WS.get(dev, self.workspace_bytes(t_count, mode), "layer")
        check(lib.pdx_moe_layer(_ptr(x), _ptr(self.gate), t_count, self.hidden, self.experts, self.top_k,
                                int(self.normalize), ctypes.byref(self.slab.struct), self.inter, _ptr(residual),
                                _ptr(outputs.out), _ptr(outputs.logits), _ptr(outputs.selected),
                                _ptr(outputs.weights), _ptr(outputs.counts), mode, _ptr(workspace),
                                workspace.numel(), _stream()))
        return outputs


def tensor_hash(tensor):
    return hashlib.sha256(tensor.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


class PDScopeCudaRuntime:
    """Layer-level drop-in for ``PDScopeCudaRuntime.forward`` with HBM-resident experts.

    ``layers`` maps layer index -> ExpertSlab (slot e = expert e, or an
    explicit ``slot_of_expert``).  ``forward`` keeps the reference signature
    and return value ``(output, Routing, row)``; ``row`` carries the keys the
    reference harness reads (pdscope_compare.py:412-420).  With every expert
    resident the placement decision is all-GPU: no CPU queue, no demand
    staging, no prefetch.
    """

    def __init__(self, layers, *, top_k=8, merge="fused", dispatch="compact", demand_slots=2,
                 input_pregather=False, graph_output_pool=False, diagnostics=True):
        if merge not in ("reference", "fused"):
            raise ValueError("invalid merge mode")
        if dispatch not in ("reference", "compact"):
            raise ValueError("invalid dispatch mode")
        if type(demand_slots) is not int or demand_slots not in (2, 3, 4):
            raise ValueError("invalid demand staging depth")
        self.layers = dict(layers)
        self.top_k = top_k
        self.merge, self.dispatch, self.demand_slots = merge, dispatch, demand_slots
        self.input_pregather, self.graph_output_pool = bool(input_pregather), bool(graph_output_pool)
        self.diagnostics = diagnostics
        self.forwards = 0

    def forward(self, inputs, gate, *, layer, step, request="pdscope", next_gate=None, top_k=8, normalize=True,
                attention_ms=0., prefetch=True):
        if (inputs.ndim != 2 or (step > 0 and inputs.shape[0] != 1)
                or (step == 0 and inputs.shape[0] < 2) or layer not in self.layers):
            raise ValueError("invalid prefill/decode activation or layer")
        phase = "prefill" if step == 0 else "decode"
        slab = self.layers[layer]
        moe = ResidentMoELayer(gate, slab, top_k=top_k, normalize=normalize)
        res = moe.forward(inputs)
        routing = Routing(res.logits, res.selected, res.weights)
        counts_list = res.counts.cpu().tolist()  # synchronises, as the reference's grouping does
        raise_device_error()
        counts = {e: n for e, n in enumerate(counts_list) if n}
        if sum(counts.values()) != inputs.shape[0] * top_k:
            raise AssertionError("lost or duplicated routed expert")
        self.forwards += 1
        resident = sorted(counts)
        decision = dict(mode="gpu_resident", phase=phase, cpu_queue=[], gpu_resident_queue=resident,
                        on_demand_queue=[], prefetch_queue=[], placements={e: "gpu" for e in resident})
        row = dict(phase=phase, step=step, layer=layer, token_counts=counts, dispatch=self.dispatch,
                   decision=decision, prefetch_issued=[], prefetch_capacity_skipped=[],
                   merge_mode=self.merge, input_pregather=self.input_pregather,
                   demand_slots=self.demand_slots, graph_output_pool=self.graph_output_pool,
                   selected_sha256=tensor_hash(res.selected) if self.diagnostics else None,
                   backend="pdx_moe sm_100a", measured_performance=False)
        return res.out, routing, row
