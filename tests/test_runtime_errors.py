"""The Python mirror rejects invalid arguments the way the reference does
(ValueError with the reference's message) before any device work, so these
run on the CPU.  References: route -- expertbench/adapters/qwen.py:142-146;
expert_groups -- qwen.py:157-164; compact_expert_groups --
expertbench/pdscope_runtime.py:24; PDScopeCudaRuntime.forward --
pdscope_runtime.py:214-216."""
import pytest
import torch

from pdscope_b200 import runtime


def _bf16(*shape):
    return torch.zeros(*shape, dtype=torch.bfloat16)


@pytest.mark.parametrize("inputs,gate", [(_bf16(4), _bf16(8, 16)),          # inputs not 2-D
                                         (_bf16(4, 12), _bf16(8, 16)),      # hidden mismatch
                                         (torch.zeros(4, 16), _bf16(8, 16))])  # dtype mismatch
def test_route_rejects_shapes(inputs, gate):
    with pytest.raises(ValueError, match="router input shape/dtype mismatch"):
        runtime.route(inputs, gate, 2, True)


@pytest.mark.parametrize("top_k,normalize,capture", [(0, True, False), (9, True, False), (2.0, True, False),
                                                     (2, 1, False), (2, True, 1)])
def test_route_rejects_parameters(top_k, normalize, capture):
    with pytest.raises(ValueError, match="invalid routing parameters"):
        runtime.route(_bf16(4, 16), _bf16(8, 16), top_k, normalize, capture_probabilities=capture)


def test_expert_groups_rejects_mode_and_shapes():
    r = runtime.Routing(None, torch.zeros(2, 2, dtype=torch.int64), _bf16(2, 2))
    with pytest.raises(ValueError, match="unsupported expert grouping mode"):
        runtime.expert_groups(r, mode="fancy")
    with pytest.raises(ValueError, match="single-token grouping requires exactly one token"):
        runtime.expert_groups(r, mode="single_token")
    dup = runtime.Routing(None, torch.tensor([[3, 3]]), _bf16(1, 2))
    with pytest.raises(ValueError, match="distinct selected expert IDs"):
        runtime.expert_groups(dup, mode="single_token")


def test_single_token_grouping_order_on_cpu():
    """Decode grouping sorts the slots by expert id and keeps each slot's weight
    (pure index work, no kernel)."""
    sel = torch.tensor([[7, 2, 5]])
    w = torch.tensor([[0.5, 0.3, 0.2]], dtype=torch.bfloat16)
    groups = runtime.expert_groups(runtime.Routing(None, sel, w), mode="single_token")
    assert [e for e, _, _ in groups] == [2, 5, 7]
    assert [float(g[2]) for g in groups] == [float(w[0, 1]), float(w[0, 2]), float(w[0, 0])]
    assert all(g[1].tolist() == [0] for g in groups)


def test_compact_groups_rejects_empty():
    r = runtime.Routing(None, torch.zeros(0, 8, dtype=torch.int64), _bf16(0, 8))
    with pytest.raises(ValueError, match="empty expert routing"):
        runtime.compact_expert_groups(r)


def test_layer_runtime_rejects_bad_activation():
    rt = runtime.PDScopeCudaRuntime({0: None})
    with pytest.raises(ValueError, match="invalid prefill/decode activation or layer"):
        rt.forward(_bf16(3, 16), _bf16(8, 16), layer=0, step=1)      # decode with 3 tokens
    with pytest.raises(ValueError, match="invalid prefill/decode activation or layer"):
        rt.forward(_bf16(1, 16), _bf16(8, 16), layer=0, step=0)      # prefill with 1 token
    with pytest.raises(ValueError, match="invalid prefill/decode activation or layer"):
        rt.forward(_bf16(4, 16), _bf16(8, 16), layer=5, step=0)      # unknown layer
    with pytest.raises(ValueError, match="invalid merge mode"):
        runtime.PDScopeCudaRuntime({}, merge="atomic")
