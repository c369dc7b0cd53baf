"""The PDScopeCudaRuntime.forward drop-in and the ExpertExecutor.gpu_backend hook,
exercised with the reference's two-layer protocol (pdscope_compare.py:609-705):
a 16-token prefill then four 1-token decodes over layers 0 and 1, activation
seed 20261011, next activation layer_norm(out + x)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup():
    from tests.gpu_util import to_dev
    from pdscope_b200.runtime import ExpertSlab
    hidden, experts, inter = 2048, 128, 768
    layers, gates, host = {}, {}, {}
    for layer in (0, 1):
        x, gate, wg, wu, wd = mo.synthetic_layer(50 + layer, 1, hidden, experts, inter)
        host[layer] = (gate, wg, wu, wd)
        gates[layer] = to_dev(gate)
        layers[layer] = ExpertSlab.from_tensors([dict(gate_proj=to_dev(wg[e]), up_proj=to_dev(wu[e]),
                                                      down_proj=to_dev(wd[e])) for e in range(experts)])
    return layers, gates, host


def test_two_layer_protocol(setup):
    from tests.gpu_util import to_bits
    from pdscope_b200 import PDScopeCudaRuntime
    layers, gates, host = setup
    core = PDScopeCudaRuntime(layers, merge="fused", dispatch="compact")
    gen = torch.Generator(device="cpu").manual_seed(20261011)
    rows = []
    for step, n in enumerate((16, 1, 1, 1, 1)):
        x = torch.randn((n, 2048), generator=gen).to(torch.bfloat16).cuda()
        for layer in (0, 1):
            out, routing, row = core.forward(x, gates[layer], layer=layer, step=step,
                                             next_gate=gates.get(layer + 1), attention_ms=0.)
            gate, wg, wu, wd = host[layer]
            xb = to_bits(x)
            logits, sel, w = mo.route(xb, gate, 8, True)
            assert np.array_equal(routing.selected.cpu().numpy(), sel)          # :672-674 (torch.equal)
            assert np.abs(to_bits(routing.weights).astype(int) - w.astype(int)).max() <= 1
            ref32 = mo.moe_layer_fp32(xb, sel, w, wg, wu, wd)
            m = mo.error_metrics(mo.bf16_to_f32(to_bits(out)), ref32)
            assert m["finite"] and m["relative_l2"] <= 0.02                     # :692-695
            assert row["phase"] == ("prefill" if step == 0 else "decode")
            assert sum(row["token_counts"].values()) == n * 8
            for key in ("merge_mode", "demand_slots", "input_pregather", "graph_output_pool", "decision",
                        "token_counts"):
                assert key in row
            assert row["decision"]["cpu_queue"] == []
            rows.append(row)
            x = F.layer_norm(out.float() + x.float(), (2048,)).to(torch.bfloat16)
    assert core.forwards == 10


def test_runtime_rejects_like_reference(setup):
    from pdscope_b200 import PDScopeCudaRuntime
    layers, gates, _ = setup
    core = PDScopeCudaRuntime(layers)
    x1 = torch.zeros((1, 2048), dtype=torch.bfloat16, device="cuda")
    x2 = torch.zeros((2, 2048), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        core.forward(x1, gates[0], layer=0, step=0)      # prefill needs >= 2 tokens
    with pytest.raises(ValueError):
        core.forward(x2, gates[0], layer=0, step=1)      # decode is one token
    with pytest.raises(ValueError):
        core.forward(x2, gates[0], layer=7, step=0)      # unknown layer
    with pytest.raises(ValueError):
        PDScopeCudaRuntime(layers, merge="other")


def test_gpu_backend_hook(setup):
    """PdxGpuBackend is the ExpertExecutor.gpu_backend callable: (key, x, tensors) -> y."""
    from tests.gpu_util import f32, torch_expert_forward
    from pdscope_b200 import PdxGpuBackend
    layers, _, _ = setup
    backend = PdxGpuBackend()
    tensors = layers[0].expert_tensors(5)
    x = torch.randn((3, 2048), device="cuda").to(torch.bfloat16)
    y = backend(("layer0", 5), x, tensors)
    ref = torch_expert_forward(x, tensors["gate_proj"], tensors["up_proj"], tensors["down_proj"])
    np.testing.assert_allclose(f32(y), f32(ref), rtol=2e-2, atol=2e-2)
    assert backend.calls == 1


def test_runtime_executes_a_mixed_decision(setup):
    """A planner decision that puts experts on the CPU (as AdaptSched does when
    the CPU is faster for them) is executed as planned: those experts run
    through the CPU backend duck type (executor.py:513-530, ``backend(key, x)``)
    and their rows join the GPU experts' rows in the merge."""
    from tests.gpu_util import to_bits
    from pdscope_b200 import PDScopeCudaRuntime
    layers, gates, host = setup
    gate, wg, wu, wd = host[0]
    masters = {e: tuple(torch.from_numpy(np.ascontiguousarray(w[e]).view(np.int16)).view(torch.bfloat16)
                        for w in (wg, wu, wd)) for e in range(128)}
    seen = []

    def cpu_backend(key, x):
        seen.append((key.layer, key.expert, x.shape[0]))
        g, u, d = masters[key.expert]
        return F.linear(F.silu(F.linear(x, g)) * F.linear(x, u), d)

    def planner(cur, nxt, **kw):
        order = sorted(cur, key=lambda e: (-cur[e], e))
        cpu, gpu = order[:2], order[2:]
        return dict(phase=kw["phase"], mode="prefill", cpu_queue=cpu, gpu_resident_queue=gpu, on_demand_queue=[],
                    prefetch_queue=[], unload_queue=[], placements={e: "gpu" if e in gpu else "cpu" for e in cur})

    core = PDScopeCudaRuntime(layers, plan=planner, costs=object(), cpu_backend=cpu_backend)
    x = torch.randn((24, 2048), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).cuda()
    out, routing, row = core.forward(x, gates[0], layer=0, step=0)
    xb = to_bits(x)
    ref, _, sel, w, _, _ = mo.moe_layer(xb, gate, wg, wu, wd, 8)
    assert np.array_equal(routing.selected.cpu().numpy(), sel)
    np.testing.assert_allclose(mo.bf16_to_f32(to_bits(out)), mo.bf16_to_f32(ref), rtol=2e-2, atol=2e-2)
    cpu_ids = row["decision"]["cpu_queue"]
    assert len(cpu_ids) == 2 and sorted(e for _, e, _ in seen) == sorted(cpu_ids)
    assert all(n == row["token_counts"][e] for _, e, n in seen)
    assert row["counters"] == dict(gpu_completed_experts=len(row["token_counts"]) - 2, cpu_completed_experts=2)
    assert row["planner"] == "planner"


def test_runtime_rejects_demand_on_resident_experts(setup):
    from pdscope_b200 import PDScopeCudaRuntime
    layers, gates, _ = setup

    def planner(cur, nxt, **kw):
        return dict(cpu_queue=[], gpu_resident_queue=[], on_demand_queue=sorted(cur), prefetch_queue=[])
    core = PDScopeCudaRuntime(layers, plan=planner, costs=object())
    x = torch.randn((4, 2048), device="cuda").to(torch.bfloat16)
    with pytest.raises(AssertionError):
        core.forward(x, gates[0], layer=0, step=0)


def test_runtime_next_gate_prediction(setup):
    """With prefetch and a next gate the runtime routes the current activation
    through the next layer's gate (pdscope_runtime.py:245-248) and hands those
    counts to the planner."""
    from pdscope_b200 import PDScopeCudaRuntime
    from pdscope_b200.runtime import route
    layers, gates, _ = setup
    got = []

    def planner(cur, nxt, **kw):
        got.append(dict(nxt))
        return dict(cpu_queue=[], gpu_resident_queue=sorted(cur), on_demand_queue=[], prefetch_queue=[])
    core = PDScopeCudaRuntime(layers, plan=planner, costs=object())
    x = torch.randn((1, 2048), device="cuda").to(torch.bfloat16)
    _, _, row = core.forward(x, gates[0], layer=0, step=3, next_gate=gates[1])
    want = route(x, gates[1], 8, True).selected[0].tolist()
    assert got[0] == {e: 1 for e in want} == row["next_prediction_counts"]
    core.forward(x, gates[0], layer=0, step=4, next_gate=gates[1], prefetch=False)
    assert got[1] == {}


def test_gpu_backend_under_the_executor_protocol(setup):
    """PdxGpuBackend called exactly as ExpertExecutor.gpu calls its gpu_backend
    (executor.py:454-488): weights are views into one flat uint8 cache slot
    (the load path's views, :343-349), filled by a copy on a load stream and
    fenced by its event (:350-360); the call runs on the compute stream after
    wait_stream, under inference_mode, with record_stream on its inputs; the
    result is read after the compute event completes (finish_gpu, :490-511)."""
    from tests.gpu_util import to_bits
    from pdscope_b200 import PdxGpuBackend
    layers, _, host = setup
    _, wg, wu, wd = host[1]
    e = 17
    master = [torch.from_numpy(np.ascontiguousarray(w[e]).view(np.int16)).view(torch.bfloat16).pin_memory()
              for w in (wg, wu, wd)]
    nbytes = sum(t.numel() * 2 for t in master)
    flat = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    load_stream, compute_stream = torch.cuda.Stream(), torch.cuda.Stream()
    views, off = {}, 0
    with torch.cuda.stream(load_stream):
        for name, t in zip(("gate_proj", "up_proj", "down_proj"), master):
            size = t.numel() * 2
            views[name] = flat[off:off + size].view(torch.bfloat16).view(t.shape)
            views[name].copy_(t, non_blocking=True)
            off += size
        loaded = torch.cuda.Event()
        loaded.record(load_stream)
    loaded.synchronize()                                   # finish_load(wait=True)
    backend = PdxGpuBackend()
    x = torch.randn((5, 2048), device="cuda").to(torch.bfloat16)
    with torch.cuda.stream(compute_stream), torch.inference_mode():
        compute_stream.wait_stream(torch.cuda.current_stream())
        flat.record_stream(compute_stream)
        x.record_stream(compute_stream)
        y = backend(("layer1", e), x, views)
        done = torch.cuda.Event()
        done.record(compute_stream)
    done.synchronize()                                     # finish_gpu(wait=True)
    want = mo.expert_forward(to_bits(x), wg[e], wu[e], wd[e])
    np.testing.assert_allclose(mo.bf16_to_f32(to_bits(y)), mo.bf16_to_f32(want), rtol=2e-2, atol=2e-2)
    assert backend.calls == 1
