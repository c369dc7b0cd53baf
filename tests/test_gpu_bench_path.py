"""Parity of exactly what bench.py times.

* Routing against the reference's own device route (F.linear/softmax/topk,
  expertbench/adapters/qwen.py:147-152, on the B200) over whole rows at the
  benchmarked batch sizes: every cuBLAS logit is within the error bound of an
  FP32 accumulation of the exact one, ids agree on at least 99% of rows, and
  every row whose ids differ is a near-tie (the two experts the routings
  order differently are closer on the exact logits than their two error
  bounds together).
* The CUDA-graph replay of the multi-layer step (ResidentMoEStack.step with
  graph=True, the timed path) against the eager step, bit for bit, over
  several replays with new inputs.
* The config-3 prefill grouped FFN at full size (12,450 tokens, Zipf(1.1)
  router skew, auto path = token-tiled tcgen05 GEMM) against the oracle's
  expert_forward (qwen.py:87-90) on sampled rows: rows of the largest
  segment, every expert's tail tile and every one-row expert.  Tolerance
  rtol/atol 2e-2 and FP32 relative L2 <= 0.02 (pdscope_compare.py:692-695).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

H, E, I, K = 2048, 128, 768, 8


def _zipf_gate(gen, device="cuda"):
    from pdscope_b200.stack import ZIPF_ALPHA, ZIPF_S
    gate = torch.randn(E, H, device=device, generator=gen) * 0.02
    perm = torch.randperm(E, device=device, generator=gen)
    ranks = torch.empty(E, device=device)
    ranks[perm] = torch.arange(1, E + 1, device=device, dtype=torch.float32)
    gate[:, 0] = -ZIPF_ALPHA * ZIPF_S * torch.log(ranks)
    return gate.to(torch.bfloat16)


@pytest.mark.parametrize("tokens,zipf", [(1, False), (64, False), (512, False), (12450, True)])
def test_route_full_row_agreement_vs_device_reference(tokens, zipf):
    from pdscope_b200.agreement import route_agreement
    from pdscope_b200.stack import activations
    gen = torch.Generator(device="cuda").manual_seed(7000 + tokens)
    if zipf:
        gate = _zipf_gate(gen)
    else:
        gate = (torch.randn(E, H, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    x = activations(tokens, H, seed=8000 + tokens, zipf=zipf)
    a = route_agreement(x, gate, K, True)
    print(f"route agreement T={tokens}: {a}")
    assert a["logit_diffs_within_fp32_bound"]               # cuBLAS's logits within FP32-accumulation error
    assert a["ids_equal_where_logits_equal"]                 # identical logits -> identical ids
    assert a["weights_equal_where_logits_equal"]             # ... and identical BF16 weights
    assert a["all_differing_rows_near_ties"], a              # every id difference is a near-tie
    assert a["ids_equal_frac"] >= 0.99


@pytest.mark.parametrize("tokens,layers", [(1, 4), (64, 4), (12450, 2)])
def test_stack_graph_replay_bit_equal_to_eager(tokens, layers):
    """The timed path: one CUDA graph per multi-layer step, replayed with new
    inputs, equals the eager step bit for bit."""
    from pdscope_b200.stack import activations, build_stack
    zipf = tokens > 1000
    stack = build_stack(layers, H, E, I, K, seed=11, zipf=zipf)
    x_in = stack.input(tokens)
    for rep in range(3):
        x = activations(tokens, H, seed=900 + rep, zipf=zipf)
        x_in.copy_(x)
        stack.step(tokens, graph=False)
        eager = stack.output(tokens).clone()
        x_in.copy_(x)
        stack.step(tokens, graph=True)
        torch.cuda.synchronize()
        graphed = stack.output(tokens).clone()
        assert torch.isfinite(eager.float()).all()
        assert torch.equal(graphed, eager), f"replay {rep}: graph and eager steps differ"
    from pdscope_b200.runtime import raise_device_error
    raise_device_error()
    stack.release_graphs()


def test_config3_prefill_ffn_at_size_vs_oracle():
    """12,450 Zipf-routed tokens (the benchmarked prefill) through the auto FFN
    path; sampled rows against the oracle."""
    from pdscope_b200 import _lib
    from pdscope_b200.runtime import ExpertSlab, pack, raise_device_error, route
    from pdscope_b200.stack import activations, prefill_lengths
    from tests.gpu_util import to_bits
    tokens = sum(prefill_lengths(8, seed=0))
    assert tokens == 12450
    gen = torch.Generator(device="cuda").manual_seed(31)
    gate = _zipf_gate(gen)
    slab = ExpertSlab.allocate(E, H, I, "cuda", generator=gen)
    x = activations(tokens, H, seed=77, zipf=True)
    r = route(x, gate, K, True)
    p = pack(r.selected, r.weights, E)
    rows = tokens * K
    mode = _lib.FFN_AUTO
    ws = torch.empty(_lib.lib.pdx_ffn_workspace_bytes(rows, E, H, I, mode), dtype=torch.uint8, device="cuda")
    y = torch.empty((rows, H), dtype=torch.bfloat16, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.lib.pdx_moe_ffn_grouped(
        ctypes.c_void_p(x.data_ptr()), tokens, ctypes.c_void_p(p.tokens.data_ptr()),
        ctypes.c_void_p(p.offsets.data_ptr()), ctypes.c_void_p(p.active.data_ptr()), E, rows,
        ctypes.byref(slab.struct), H, I, ctypes.c_void_p(y.data_ptr()), mode, ctypes.c_void_p(ws.data_ptr()),
        ws.numel(), s))
    torch.cuda.synchronize()
    raise_device_error()
    counts = p.counts.cpu().numpy()
    offsets = p.offsets.cpu().numpy()
    toks = p.tokens.cpu().numpy()
    top16 = np.sort(counts)[::-1][:16].sum() / counts.sum()
    assert top16 > 0.6                      # the Zipf skew is in effect
    biggest = int(np.argmax(counts))
    assert counts[biggest] > 4096           # a segment of many 128-row tiles
    sample = {}
    n = counts[biggest]
    picks = np.unique(np.concatenate([np.arange(0, 128), np.linspace(0, n - 1, 128).astype(int),
                                      np.arange(max(0, n - 130), n)]))
    sample[biggest] = picks
    ones = 0
    for e in range(E):
        c = int(counts[e])
        if c == 0 or e == biggest:
            continue
        ones += c == 1
        tail0 = (c - 1) // 128 * 128          # first row of the expert's last 128-row tile
        sample[e] = np.unique(np.concatenate([np.arange(tail0, c)[-16:], [0]]))
    x_bits = to_bits(x)
    y_bits = to_bits(y)
    storage = slab.storage.view(E, 3 * I * H)
    worst_l2 = 0.0
    for e, local in sample.items():
        w = to_bits(storage[e])
        g, u, d = w[:I * H].reshape(I, H), w[I * H:2 * I * H].reshape(I, H), w[2 * I * H:].reshape(H, I)
        prow = offsets[e] + local
        xr = x_bits[toks[prow]]
        exp = mo.expert_forward(xr, g, u, d)
        got = y_bits[prow]
        np.testing.assert_allclose(mo.bf16_to_f32(got), mo.bf16_to_f32(exp), rtol=2e-2, atol=2e-2)
        l2 = mo.error_metrics(mo.bf16_to_f32(got), mo.reference_fp32(xr, g, u, d))["relative_l2"]
        worst_l2 = max(worst_l2, l2)
    assert worst_l2 <= 0.02
    print(f"config-3 FFN: {len(sample)} experts sampled, {ones} one-row experts, largest segment {n} rows, "
          f"worst FP32 relative L2 {worst_l2:.4f}")


def test_graph_step_copies_counts_to_host_for_the_policy():
    """The whole-step graph ends with one async copy of every layer's expert
    counts into pinned host memory; the counts equal the device's, feed the
    load tracker (the hot table the reference's load_hot_profile reads), and
    the step's output is unchanged by the copy."""
    from pdscope_b200.stack import ExpertLoadTracker, activations, build_stack
    layers, tokens = 4, 64
    stack = build_stack(layers, H, E, I, K, seed=5)
    tracker = ExpertLoadTracker(layers, E)
    want_total = torch.zeros((layers, E), dtype=torch.int64)
    for rep in range(3):
        stack.input(tokens).copy_(activations(tokens, H, seed=40 + rep))
        stack.step(tokens, graph=False)
        eager = stack.output(tokens).clone()
        stack.step(tokens, counts_to_host=True)
        host = stack.expert_counts(tokens)
        torch.cuda.synchronize()
        device = stack.buffers(tokens)["counts"].cpu()
        assert torch.equal(host, device)
        assert (host.sum(dim=1) == tokens * K).all()
        assert torch.equal(stack.output(tokens), eager)
        tracker.add(host)
        want_total += device.long()
    assert np.array_equal(tracker.totals, want_total.numpy()) and tracker.steps == 3
    hot = tracker.hot_sets(4)
    for l in range(layers):
        top = np.sort(want_total[l].numpy())[::-1][:4]
        assert sorted(want_total[l].numpy()[hot[l]].tolist(), reverse=True) == top.tolist()
    stack.release_graphs()
