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
                                    (HBM-resident experts; AdaptSched's
                                    plan_pdscope decides the placement)

Tensors are torch CUDA tensors (BF16 activations and weights); torch is used
for device memory and streams only.  Kernels run on the caller's current
stream.
"""
from __future__ import annotations

import ctypes
import hashlib
from collections import Counter
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


@dataclass(frozen=True)
class ExpertKey:
    """Expert identity handed to CPU backends; the fields of the reference's
    ``ExpertKey`` (expertbench/cache.py:32-35)."""
    layer: int
    expert: int
    representation: str = "bf16"


def _reference_planner():
    """AdaptSched's ``plan_pdscope`` (expertbench/pdscope_policy.py:72) when the
    reference package is importable in this process, else None."""
    try:
        from expertbench.pdscope_policy import plan_pdscope
    except ImportError:
        return None
    return plan_pdscope


class PDScopeCudaRuntime:
    """Layer-level drop-in for ``PDScopeCudaRuntime.forward`` with HBM-resident experts.

    ``layers`` maps layer index -> ExpertSlab (slot e = expert e, or an
    explicit ``slot_of_expert``).  ``forward`` keeps the reference's signature,
    checks and return value ``(output, Routing, row)``
    (expertbench/pdscope_runtime.py:208-512); ``row`` carries the keys the
    reference harness reads (benchmarks/pdscope_compare.py:412-420).

    Placement follows the reference: every layer asks the AdaptSched planner
    ``plan`` (the signature of ``plan_pdscope``, pdscope_policy.py:72) with the
    arguments the reference passes (pdscope_runtime.py:270-280) -- this
    layer's routed counts, the next layer's predicted counts (the next gate
    on the current activation, :245-248, when ``prefetch`` and ``next_gate``
    are given), the resident ids, the cost table ``costs`` (``for_load(n)``,
    e.g. FileCosts over pdscope_b200/cost_table_b200.json) -- and executes
    its decision: ``gpu_resident_queue`` in one grouped FFN launch, the
    ``cpu_queue`` experts through ``cpu_backend(key, rows)`` (the reference's
    CPU backend duck type, executor.py:513-530) or, without one, the torch
    CPU ``expert_forward`` over ``masters[layer][e]`` (gate, up, down host
    tensors), their rows uploaded into their packed places before the merge.
    With every expert resident the planner has nothing to demand-load or
    prefetch; a decision that asks for either is rejected.  ``plan=None``
    uses the reference's ``plan_pdscope`` if it is importable, otherwise the
    all-GPU decision (row ``planner`` says which).  ``merge`` 'fused' and
    'reference' both run the deterministic slot-order combine (the reference
    documents the two as the same math in a different accumulation order,
    :456-459).
    """

    def __init__(self, layers, *, top_k=8, merge="fused", dispatch="compact", demand_slots=2,
                 input_pregather=False, graph_output_pool=False, diagnostics=True, plan=None, costs=None,
                 decode_costs=None, cpu_backend=None, masters=None, speculative_slots=0, decode_cpu_target=None):
        if merge not in ("reference", "fused"):
            raise ValueError("invalid merge mode")
        if dispatch not in ("reference", "compact"):
            raise ValueError("invalid dispatch mode")
        if type(demand_slots) is not int or demand_slots not in (2, 3, 4):
            raise ValueError("invalid demand staging depth")
        if type(speculative_slots) is not int or not 0 <= speculative_slots <= 128:
            raise ValueError("invalid PDScope cache contract")
        if cpu_backend is not None and not callable(cpu_backend):
            raise ValueError("CPU backend must be an explicit synchronous callable")
        if (decode_cpu_target is not None
                and (type(decode_cpu_target) is not int or not 0 <= decode_cpu_target <= 8)):
            raise ValueError("invalid decode CPU balance target")
        self.layers = dict(layers)
        self.top_k = top_k
        self.merge, self.dispatch, self.demand_slots = merge, dispatch, demand_slots
        self.input_pregather, self.graph_output_pool = bool(input_pregather), bool(graph_output_pool)
        self.diagnostics = diagnostics
        self.plan = plan if plan is not None else _reference_planner()
        self.planner_name = ("plan_pdscope" if plan is None and self.plan is not None else
                             getattr(plan, "__name__", "caller planner") if plan is not None else "none")
        if self.plan is not None and costs is None:
            from .costs import TableCosts
            costs = TableCosts()
        self.costs = costs
        self.decode_costs = decode_costs if decode_costs is not None else costs
        self.cpu_backend, self.masters = cpu_backend, masters
        self.speculative_slots = speculative_slots
        self.decode_cpu_target = decode_cpu_target
        self.forecasts = {}
        self.prediction_counts = {phase: dict(hits=0, total=0) for phase in ("prefill", "decode")}
        self.forwards = 0
        self.completed = dict(gpu_completed_experts=0, cpu_completed_experts=0)

    def _decision(self, counts, next_counts, *, layer, phase, top_k, attention_ms, hit_rate):
        resident = list(counts)                 # every expert of every layer is resident in HBM
        next_resident = list(next_counts)
        if self.plan is None:
            gpu = sorted(counts, key=lambda e: (-counts[e], e))
            return dict(phase=phase, mode="all_resident", cpu_queue=[], gpu_resident_queue=gpu,
                        on_demand_queue=[], prefetch_queue=[], unload_queue=[],
                        placements={e: "gpu" for e in sorted(counts)})
        return self.plan(counts, next_counts, current_layer=layer, phase=phase, current_gpu_ids=resident,
                         next_gpu_ids=next_resident,
                         costs=self.decode_costs if phase == "decode" else self.costs,
                         attention_ms=attention_ms, hit_rate=hit_rate, prefetch_slots=self.speculative_slots,
                         top_k=top_k,
                         cpu_balance_target_override=(self.decode_cpu_target if phase == "decode" else None),
                         joint_next=True, record_checks=False, trusted=True,
                         compute_formula_target=(self.decode_cpu_target is None))

    def _cpu_expert(self, layer, e, rows):
        key = ExpertKey(layer, e)
        if self.cpu_backend is not None:
            out = self.cpu_backend(key, rows)
        elif self.masters is not None:
            g, u, d = self.masters[layer][e]
            with torch.inference_mode():
                out = torch.nn.functional.linear(torch.nn.functional.silu(torch.nn.functional.linear(rows, g))
                                                 * torch.nn.functional.linear(rows, u), d)
        else:
            raise ValueError("the decision places experts on the CPU but neither a CPU backend nor host "
                             "master weights were given")
        if (not isinstance(out, torch.Tensor) or out.device.type != "cpu" or out.dtype != torch.bfloat16
                or out.shape != rows.shape):
            raise ValueError("CPU backend must return completed unweighted CPU BF16 input-shaped output")
        return out

    def forward(self, inputs, gate, *, layer, step, request="pdscope", next_gate=None, top_k=8, normalize=True,
                attention_ms=0., prefetch=True):
        if (inputs.ndim != 2 or (step > 0 and inputs.shape[0] != 1)
                or (step == 0 and inputs.shape[0] < 2) or layer not in self.layers):
            raise ValueError("invalid prefill/decode activation or layer")
        phase = "prefill" if step == 0 else "decode"
        slab = self.layers[layer]
        _require_cuda_bf16("inputs", inputs, 2)
        experts, hidden = gate.shape
        t_count = inputs.shape[0]
        dev = inputs.device
        routing = route(inputs, gate, top_k, normalize)
        p = pack(routing.selected, routing.weights, experts)
        offsets = p.offsets.cpu()                # synchronises, as the reference's grouping does (:26)
        raise_device_error()
        counts = {e: int(offsets[e + 1] - offsets[e]) for e in range(experts) if offsets[e + 1] > offsets[e]}
        prior = self.forecasts.pop((request, step, layer), None)
        if prior:
            self.prediction_counts[phase]["hits"] += len(set(prior) & set(counts))
            self.prediction_counts[phase]["total"] += len(prior)
        observed = self.prediction_counts[phase]
        hit_rate = observed["hits"] / observed["total"] if observed["total"] else 0.
        next_routing, next_counts = None, {}
        if prefetch and next_gate is not None:
            # layer-local ids of the TARGET gate on the CURRENT activation (:245-248)
            next_routing = route(inputs, next_gate, top_k, normalize)
            next_counts = dict(Counter(next_routing.selected.cpu().flatten().tolist()))
        decision = self._decision(counts, next_counts, layer=layer, phase=phase, top_k=top_k,
                                  attention_ms=attention_ms, hit_rate=hit_rate)
        if decision["on_demand_queue"] or decision["prefetch_queue"]:
            raise AssertionError("every expert is resident: nothing can be demand-loaded or prefetched")
        gpu_ids = sorted(decision["gpu_resident_queue"])
        cpu_ids = sorted(decision["cpu_queue"])
        if set(gpu_ids) & set(cpu_ids) or set(gpu_ids) | set(cpu_ids) != set(counts):
            raise AssertionError("demand partition failed")
        rows_total = t_count * top_k
        y = torch.empty((rows_total, hidden), dtype=torch.bfloat16, device=dev)
        if gpu_ids:
            active = torch.zeros(experts + 1, dtype=torch.int32)
            active[0] = len(gpu_ids)
            active[1:1 + len(gpu_ids)] = torch.tensor(gpu_ids, dtype=torch.int32)
            active = active.to(dev, non_blocking=True)
            ws = _WS.get(dev, lib.pdx_ffn_workspace_bytes(rows_total, experts, hidden, slab.inter, _lib.FFN_AUTO),
                         "ffn")
            check(lib.pdx_moe_ffn_grouped(_ptr(inputs), t_count, _ptr(p.tokens), _ptr(p.offsets), _ptr(active),
                                          experts, rows_total, ctypes.byref(slab.struct), hidden, slab.inter,
                                          _ptr(y), _lib.FFN_AUTO, _ptr(ws), ws.numel(), _stream()))
        if cpu_ids:
            tokens_cpu = p.tokens.cpu().long()
            x_cpu = inputs.cpu()
            for e in cpu_ids:
                a, b = int(offsets[e]), int(offsets[e + 1])
                y[a:b].copy_(self._cpu_expert(layer, e, x_cpu[tokens_cpu[a:b]]))
        out = combine(y, routing.weights, p.inverse)
        raise_device_error()
        self.completed["gpu_completed_experts"] += len(gpu_ids)
        self.completed["cpu_completed_experts"] += len(cpu_ids)
        if len(gpu_ids) + len(cpu_ids) != len(counts) or sum(counts.values()) != rows_total:
            raise AssertionError("lost or duplicated routed expert")
        self.forwards += 1
        row = dict(phase=phase, step=step, layer=layer, token_counts=counts, dispatch=self.dispatch,
                   decision=decision, planner=self.planner_name, prefetch_issued=[], prefetch_capacity_skipped=[],
                   next_prediction_counts=next_counts, causal_hit_counts=dict(observed),
                   predictor="next_layer_gate_on_current_activation",
                   merge_mode=self.merge, input_pregather=self.input_pregather,
                   demand_slots=self.demand_slots, graph_output_pool=self.graph_output_pool,
                   ping_pong_slots=[], counters=dict(gpu_completed_experts=len(gpu_ids),
                                                     cpu_completed_experts=len(cpu_ids)),
                   selected_sha256=tensor_hash(routing.selected) if self.diagnostics else None,
                   next_selected_sha256=(tensor_hash(next_routing.selected)
                                         if self.diagnostics and next_routing is not None else None),
                   backend="pdx_moe sm_100a", measured_performance=False)
        return out, routing, row
