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
