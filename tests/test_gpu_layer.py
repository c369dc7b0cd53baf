"""GPU parity of the whole layer: route -> pack -> grouped FFN -> combine.

Contract (pdscope_compare.py:670-695 restated): routing ids equal the oracle
bit for bit; layer output within rtol/atol 2e-2 of the oracle's BF16 layer and
FP32 relative L2 <= 0.02 against the all-FP32 layer on the same routing.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

RTOL = ATOL = 2e-2


@pytest.fixture(scope="module")
def pdx():
    import pdscope_b200
    return pdscope_b200


def _layer(pdx, x, gate, wg, wu, wd, k, mode=0, residual=None):
    from tests.gpu_util import to_dev
    from pdscope_b200.runtime import ExpertSlab, ResidentMoELayer
    experts = gate.shape[0]
    slab = ExpertSlab.from_tensors([dict(gate_proj=to_dev(wg[e]), up_proj=to_dev(wu[e]), down_proj=to_dev(wd[e]))
                                    for e in range(experts)])
    layer = ResidentMoELayer(to_dev(gate), slab, top_k=k)
    res = layer.forward(to_dev(x), residual=to_dev(residual) if residual is not None else None, mode=mode)
    torch.cuda.synchronize()
    from pdscope_b200.runtime import raise_device_error
    raise_device_error()
    return res, layer, slab


def _check_layer(res, x, gate, wg, wu, wd, k):
    from tests.gpu_util import to_bits
    out, logits, sel, w, packed, rows = mo.moe_layer(x, gate, wg, wu, wd, k)
    assert np.array_equal(to_bits(res.logits), logits)
    assert np.array_equal(res.selected.cpu().numpy(), sel)
    d = np.abs(to_bits(res.weights).astype(np.int32) - w.astype(np.int32))
    assert d.max() <= 1
    assert np.array_equal(res.counts.cpu().numpy(), packed["counts"])
    got = mo.bf16_to_f32(to_bits(res.out))
    np.testing.assert_allclose(got, mo.bf16_to_f32(out), rtol=RTOL, atol=ATOL)
    ref32 = mo.moe_layer_fp32(x, sel, w, wg, wu, wd)
    assert mo.error_metrics(got, ref32)["relative_l2"] <= 0.02
    return got


@pytest.mark.parametrize("mode", (0, 1, 2, 3, 4, 5, 6))
def test_small_layer_golden(pdx, golden, mode):
    """The golden small layer (E=16, k=4, H=256, I=128, T=32)."""
    x, gate, wg, wu, wd = mo.synthetic_layer(4242, 32, 256, 16, 128)
    res, _, _ = _layer(pdx, x, gate, wg, wu, wd, 4, mode)
    got = _check_layer(res, x, gate, wg, wu, wd, 4)
    np.testing.assert_allclose(got, mo.bf16_to_f32(golden["layer_fused_out"]), rtol=RTOL, atol=ATOL)
    assert mo.error_metrics(got, golden["layer_fp32_out"])["relative_l2"] <= 0.02


@pytest.mark.parametrize("tokens", (1, 512))
def test_qwen3_layer_config1(pdx, tokens):
    """H=2048, E=128, I=768, k=8 at decode T=1 and prefill T=512."""
    x, gate, wg, wu, wd = mo.synthetic_layer(0, tokens, 2048, 128, 768)
    res, _, _ = _layer(pdx, x, gate, wg, wu, wd, 8)
    _check_layer(res, x, gate, wg, wu, wd, 8)


@pytest.mark.parametrize("tokens", (2, 8, 63, 64, 65, 100))
def test_layer_ragged_sizes(pdx, tokens):
    x, gate, wg, wu, wd = mo.synthetic_layer(77 + tokens, tokens, 512, 32, 256)
    res, _, _ = _layer(pdx, x, gate, wg, wu, wd, 8)
    _check_layer(res, x, gate, wg, wu, wd, 8)


@pytest.mark.parametrize("tokens", (1, 8, 64))
def test_layer_single_launch_decode_matches_staged(pdx, tokens):
    """pdx_moe_layer at decode batches: the single-launch FFN, whose tickets and
    counters the fused top-k + pack kernel clears, equals the staged FFN bit
    for bit, on repeated calls with one workspace."""
    from tests.gpu_util import to_dev
    x, gate, wg, wu, wd = mo.synthetic_layer(500 + tokens, tokens, 2048, 128, 768)
    res, layer, _ = _layer(pdx, x, gate, wg, wu, wd, 8, mode=6)
    staged = res.out.clone()
    _check_layer(res, x, gate, wg, wu, wd, 8)
    xd = to_dev(x)
    for _ in range(3):
        again = layer.forward(xd, mode=1)
        torch.cuda.synchronize()
        assert torch.equal(again.out, staged)
    from pdscope_b200.runtime import raise_device_error
    raise_device_error()


def test_layer_residual(pdx):
    x, gate, wg, wu, wd = mo.synthetic_layer(9, 20, 256, 16, 128)
    resid = mo.f32_to_bf16(np.random.default_rng(3).standard_normal((20, 256), dtype=np.float32))
    from tests.gpu_util import to_bits
    res, _, _ = _layer(pdx, x, gate, wg, wu, wd, 4, residual=resid)
    out = mo.moe_layer(x, gate, wg, wu, wd, 4)[0]
    exp = mo.bf16_to_f32(resid) + mo.bf16_to_f32(out)
    np.testing.assert_allclose(mo.bf16_to_f32(to_bits(res.out)), exp, rtol=RTOL, atol=ATOL)


def test_layer_vs_reference_torch_path(pdx):
    """Against the reference's own GPU arithmetic (torch route + expert_forward +
    fused index_add merge) on the B200, same inputs."""
    from tests.gpu_util import f32, to_dev, torch_expert_forward, torch_route
    x, gate, wg, wu, wd = mo.synthetic_layer(11, 256, 2048, 128, 768)
    res, _, _ = _layer(pdx, x, gate, wg, wu, wd, 8)
    xd, gd = to_dev(x), to_dev(gate)
    _, sel, w = torch_route(xd, gd, 8, True)
    out = torch.zeros_like(xd)
    for e in torch.unique(sel).tolist():
        slots, toks = torch.where((sel == e).T)
        y = torch_expert_forward(xd[toks], to_dev(wg[e]), to_dev(wu[e]), to_dev(wd[e]))
        out.index_add_(0, toks, (y * w[toks, slots, None]).to(torch.bfloat16))
    np.testing.assert_allclose(f32(res.out), f32(out), rtol=RTOL, atol=ATOL)


def test_full_size_properties(pdx):
    """Size-independent properties at a prefill size: determinism and token
    permutation equivariance (each row's arithmetic is independent of the
    others), both bit-exact."""
    from tests.gpu_util import to_dev
    from pdscope_b200.runtime import ExpertSlab, ResidentMoELayer
    tokens, hidden, experts, inter = 4096, 2048, 128, 768
    gen = torch.Generator(device="cuda").manual_seed(0)
    slab = ExpertSlab.allocate(experts, hidden, inter, "cuda", generator=gen)
    gate = (torch.randn(experts, hidden, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    x = torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16)
    layer = ResidentMoELayer(gate, slab)
    a = layer.forward(x)
    out_a = a.out.clone()
    b = layer.forward(x)
    assert torch.equal(out_a, b.out)
    perm = torch.randperm(tokens, device="cuda", generator=gen)
    c = layer.forward(x[perm].contiguous())
    assert torch.equal(c.out, out_a[perm])
    assert torch.equal(c.selected, a.selected[perm])
    # CTA-pair prefill tiles: deterministic and equivariant too, and equal to
    # the single-CTA tiles up to BF16 rounding of the FFN rows
    e1 = layer.forward(x, mode=5).out.clone()
    e2 = layer.forward(x[perm].contiguous(), mode=5).out
    assert torch.equal(e2, e1[perm])
    f = layer.forward(x, mode=4).out
    assert (e1 == f).float().mean().item() > 0.999
    # decode path at a batch of 64: same properties
    xs = x[:64].contiguous()
    d1 = layer.forward(xs).out.clone()
    p = torch.randperm(64, device="cuda", generator=gen)
    d2 = layer.forward(xs[p].contiguous()).out
    assert torch.equal(d2, d1[p])
    torch.cuda.synchronize()
    from pdscope_b200.runtime import raise_device_error
    raise_device_error()
