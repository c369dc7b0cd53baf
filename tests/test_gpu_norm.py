"""The synthetic stack's next-layer activation, layer_norm(y + x) (the
reference's two-layer protocol, benchmarks/pdscope_compare.py:609-705:
``x = F.layer_norm(out.float() + x.float(), (H,)).to(torch.bfloat16)``),
against torch on the device: within one BF16 ulp, nearly all bit-equal."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,hidden", [(1, 2048), (7, 256), (512, 2048), (300, 4096), (3, 8192)])
def test_residual_layernorm_matches_torch(tokens, hidden):
    from pdscope_b200.runtime import residual_layernorm
    gen = torch.Generator(device="cuda").manual_seed(tokens + hidden)
    y = (torch.randn(tokens, hidden, device="cuda", generator=gen) * 0.3).to(torch.bfloat16)
    x = torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16)
    want = F.layer_norm(y.float() + x.float(), (hidden,)).to(torch.bfloat16)
    got = residual_layernorm(y, x)
    ulp = (got.view(torch.int16).int() - want.view(torch.int16).int()).abs()
    assert int(ulp.max()) <= 1
    assert (ulp == 0).float().mean().item() > 0.99
    # in place over y (the stacks write the norm over the MoE output)
    y2 = y.clone()
    residual_layernorm(y2, x, out=y2)
    assert torch.equal(y2, got)


def test_residual_layernorm_rejects_bad_shapes():
    from pdscope_b200.runtime import residual_layernorm
    a = torch.zeros(2, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="multiple of 8"):
        residual_layernorm(a, a)               # H not a multiple of 8 (unsupported)
    b = torch.zeros(2, 16, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        residual_layernorm(b, torch.zeros(3, 16, dtype=torch.bfloat16, device="cuda"))


def test_stack_activations_stay_finite():
    """48 random-init layers: every layer's input stays at unit scale."""
    from pdscope_b200.stack import activations, build_stack
    stack = build_stack(48, 256, 16, 128, top_k=4, seed=3, zipf=True)
    t = 96
    stack.input(t).copy_(activations(t, 256, seed=4, zipf=True))
    stack.step(t, graph=False)
    out = stack.output(t).float()
    assert torch.isfinite(out).all()
    assert 0.5 < out.pow(2).mean().sqrt().item() < 2.0


@pytest.mark.parametrize("tokens,mode", [(1, 0), (33, 0), (300, 0), (300, 1)])
def test_fused_combine_norm_bit_identical(tokens, mode):
    """PDX_LAYER_OUT_NORM / pdx_combine_layernorm == combine (no residual) then
    residual_layernorm, bit for bit."""
    import ctypes
    from pdscope_b200 import _lib
    from pdscope_b200.runtime import ExpertSlab, ResidentMoELayer, combine, pack, residual_layernorm, route
    gen = torch.Generator(device="cuda").manual_seed(tokens)
    hidden, experts, inter = 512, 16, 256
    slab = ExpertSlab.allocate(experts, hidden, inter, "cuda", generator=gen)
    gate = (torch.randn(experts, hidden, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    x = torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16)
    layer = ResidentMoELayer(gate, slab, top_k=4)
    two_step = residual_layernorm(layer.forward(x, mode=mode).out, x)
    fused = layer.forward(x, residual=x, mode=mode | _lib.LAYER_OUT_NORM).out
    assert torch.equal(fused, two_step)
    # the standalone entry point over packed expert rows
    r = route(x, gate, 4, True)
    p = pack(r.selected, r.weights, experts)
    rows = torch.randn(tokens * 4, hidden, device="cuda", generator=gen).to(torch.bfloat16)
    want = residual_layernorm(combine(rows, r.weights, p.inverse), x)
    got = torch.empty_like(x)
    _lib.check(_lib.lib.pdx_combine_layernorm(
        ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(r.weights.data_ptr()), ctypes.c_void_p(p.inverse.data_ptr()),
        tokens, 4, hidden, ctypes.c_void_p(x.data_ptr()), ctypes.c_float(1e-5), ctypes.c_void_p(got.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    assert torch.equal(got, want)
