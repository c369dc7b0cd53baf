"""The reference's CPU layer path, restated with torch CPU ops -- BASELINE ONLY.

Timed by ``bench.py`` (``cpu_baseline`` and ``--impl reference``) on the host
cores of the GPU box.  It follows, op for op, what the reference runs when an
expert is placed on the CPU with ``cpu_backend=None``:

1. ``route``                 expertbench/adapters/qwen.py:140-152
2. ``compact_expert_groups`` expertbench/pdscope_runtime.py:16-39
3. per-expert ``expert_forward`` on CPU tensors
                             expertbench/executor.py:513-530 -> qwen.py:87-90
4. fused merge ``index_add_`` expertbench/pdscope_runtime.py:454-464

The ktransformers AVX2 kernel the reference can also use is a third-party
project that is not vendored, so it is not part of this baseline.
"""
from __future__ import annotations

import time

import torch
import torch.nn.functional as F


def route(inputs, gate, top_k, normalize):
    logits = F.linear(inputs, gate)
    probabilities = F.softmax(logits, dim=-1, dtype=torch.float32)
    weights, selected = torch.topk(probabilities, top_k, dim=-1)
    if normalize:
        weights = weights / weights.sum(dim=-1, keepdim=True)
    return logits, selected, weights.to(inputs.dtype)


def compact_expert_groups(selected, weights, experts):
    n, k = selected.shape
    flat = selected.T.contiguous().view(-1)
    counts = torch.bincount(flat, minlength=experts).tolist()
    order = torch.argsort(flat, stable=True)
    tokens = order.remainder(n)
    positions = tokens * k + torch.div(order, n, rounding_mode="floor")
    w = weights.reshape(-1)[positions]
    groups, start = {}, 0
    for e, count in enumerate(counts):
        if count:
            groups[e] = (tokens[start:start + count], w[start:start + count])
            start += count
    return groups


def expert_forward(inputs, gate_proj, up_proj, down_proj):
    return F.linear(F.silu(F.linear(inputs, gate_proj)) * F.linear(inputs, up_proj), down_proj)


def layer_forward(inputs, gate, experts, top_k=8, normalize=True):
    """One MoE layer on the CPU; ``experts[e]`` = (gate_proj, up_proj, down_proj)."""
    with torch.inference_mode():
        _, selected, weights = route(inputs, gate, top_k, normalize)
        groups = compact_expert_groups(selected, weights, gate.shape[0])
        output = torch.zeros_like(inputs)
        keep = sorted(groups)
        parts = [expert_forward(inputs[groups[e][0]], *experts[e]) for e in keep]
        index = torch.cat([groups[e][0] for e in keep])
        weight = torch.cat([groups[e][1] for e in keep])[:, None]
        output.index_add_(0, index, torch.cat(parts, dim=0).to(output.dtype) * weight)
        return output, len(keep)


def make_layer(hidden, experts, inter, seed):
    """Random-init CPU layer (BF16; weights ~N(0, 0.02))."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    gate = (torch.randn(experts, hidden, generator=g) * 0.02).to(torch.bfloat16)
    ex = []
    for _ in range(experts):
        ex.append(tuple((torch.randn(shape, generator=g) * 0.02).to(torch.bfloat16)
                        for shape in ((inter, hidden), (inter, hidden), (hidden, inter))))
    return gate, ex


def stack_step(x, layers, num_layers, top_k=8, normalize=True):
    """One step of a ``num_layers``-deep stack on the CPU: layer l uses
    ``layers[l % len(layers)]`` and the next activation is formed as the
    reference's two-layer protocol does (benchmarks/pdscope_compare.py:609-705,
    ``x = F.layer_norm(out.float() + x.float(), (H,)).to(bf16)``).  Returns the
    last activation and the active experts of every layer."""
    active = []
    with torch.inference_mode():
        for l in range(num_layers):
            gate, ex = layers[l % len(layers)]
            out, n_active = layer_forward(x, gate, ex, top_k, normalize)
            active.append(n_active)
            x = F.layer_norm(out.float() + x.float(), (x.shape[1],)).to(torch.bfloat16)
    return x, active


def time_layers(layers, tokens, hidden, threads, repeats=1, seed=7):
    """Seconds per layer (mean) and active experts per layer for a token batch."""
    torch.set_num_threads(threads)
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16)
    total, active = 0.0, []
    for _ in range(repeats):
        for gate, ex in layers:
            t0 = time.perf_counter()
            out, n_active = layer_forward(x, gate, ex)
            total += time.perf_counter() - t0
            active.append(n_active)
            x = (x.float() + out.float()).to(torch.bfloat16)
    return total / (repeats * len(layers)), active
