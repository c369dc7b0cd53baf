"""GPU parity of routing (qwen.py:140-152) against the oracle and torch on the B200."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

# 65..4096 and 12450: split-K tiled router (2-4 K splits); 18944 = 296 whole tiles: one split
ROUTE_T = (1, 3, 16, 17, 64, 65, 256, 1000, 1024, 4096, 12450, 18944)


@pytest.fixture(scope="module")
def pdx():
    import pdscope_b200
    return pdscope_b200


def test_torch_topk_tie_order_on_device():
    """Pin the oracle's tie rule on the reference's own device op: a tie at the
    k boundary is won by the lower index; inside the selection equal values come
    in descending index order."""
    v = torch.tensor([[0.1, 0.5, 0.3, 0.5, 0.3, 0.5, 0.2, 0.3]], device="cuda")
    _, i = torch.topk(v, 5, dim=-1)
    assert i.tolist() == [[5, 3, 1, 4, 2]]
    gen = torch.Generator(device="cuda").manual_seed(0)
    for k in (1, 2, 4, 8):
        probs = torch.rand(4096, 128, device="cuda", generator=gen)
        probs = (probs * 16).floor() / 16  # many exact ties
        _, sel = torch.topk(probs, k, dim=-1)
        _, ora = mo.topk_torch_cuda(probs.cpu().numpy(), k)
        assert np.array_equal(sel.cpu().numpy(), ora)


@pytest.mark.parametrize("tokens", ROUTE_T)
def test_topk_from_logits_matches_oracle(pdx, tokens):
    from tests.gpu_util import to_bits, to_dev
    x, gate = mo.synthetic_router(1000 + tokens, tokens)
    logits = mo.router_logits(x, gate)
    sel, w = pdx.topk_from_logits(to_dev(logits), 8, True)
    o_sel, o_w = mo.route_from_logits(logits, 8, True)
    assert np.array_equal(sel.cpu().numpy(), o_sel)
    wb = to_bits(w)
    diff = np.abs(wb.astype(np.int32) - o_w.astype(np.int32))
    assert diff.max() <= 1            # numpy exp vs CUDA expf: at most one BF16 ulp
    assert (diff == 0).mean() > 0.999


@pytest.mark.parametrize("tokens", (1, 16, 256, 4096))
@pytest.mark.parametrize("normalize", (True, False))
def test_topk_bit_exact_vs_torch_on_same_logits(pdx, tokens, normalize):
    """Same logits -> the reference's own CUDA softmax/topk/renorm, bit for bit."""
    from tests.gpu_util import torch_route, to_dev
    x, gate = mo.synthetic_router(2000 + tokens, tokens)
    xd, gd = to_dev(x), to_dev(gate)
    logits, t_sel, t_w = torch_route(xd, gd, 8, normalize)
    sel, w = pdx.topk_from_logits(logits.contiguous(), 8, normalize)
    assert torch.equal(sel, t_sel)
    assert torch.equal(w, t_w)


@pytest.mark.parametrize("tokens", ROUTE_T)
def test_route_matches_oracle(pdx, tokens):
    from tests.gpu_util import to_bits, to_dev
    x, gate = mo.synthetic_router(3000 + tokens, tokens)
    r = pdx.route(to_dev(x), to_dev(gate), 8, True)
    logits, o_sel, o_w = mo.route(x, gate, 8, True)
    assert np.array_equal(to_bits(r.logits), logits)          # exact dot products, one rounding
    assert np.array_equal(r.selected.cpu().numpy(), o_sel)    # bit-exact ids
    d = np.abs(to_bits(r.weights).astype(np.int32) - o_w.astype(np.int32))
    assert d.max() <= 1 and (d == 0).mean() > 0.999


@pytest.mark.parametrize("tokens", (16, 1024, 4096))
def test_route_vs_torch_cublas(pdx, tokens):
    """Against the reference run on the B200 (cuBLAS logits): ids agree wherever
    the BF16 logits agree; the rate of one-ulp cuBLAS logit differences is small."""
    from tests.gpu_util import torch_route, to_dev
    x, gate = mo.synthetic_router(4000 + tokens, tokens)
    xd, gd = to_dev(x), to_dev(gate)
    t_logits, t_sel, t_w = torch_route(xd, gd, 8, True)
    r = pdx.route(xd, gd, 8, True)
    same = (r.logits == t_logits).all(dim=1)
    assert (r.logits != t_logits).float().mean().item() < 5e-3
    assert torch.equal(r.selected[same], t_sel[same])
    assert torch.equal(r.weights[same], t_w[same])


def test_route_golden_reference_rows(pdx, golden):
    """Against the reference's own CPU output: ids on tie-free rows, weights exact."""
    from tests.gpu_util import to_bits, to_dev
    for tokens in (1, 16, 64, 256, 1024, 4096):
        x, gate = mo.synthetic_router(20261012 + tokens, tokens)
        r = pdx.route(to_dev(x), to_dev(gate), 8, True)
        ours = to_bits(r.logits)
        ref_sel = golden[f"route_T{tokens}_selected"].astype(np.int64)
        key = f"route_T{tokens}_logits"
        same = (golden[key] == ours).all(axis=1) if key in golden else np.ones(tokens, bool)
        rows = same & mo.tie_free_rows(ours, 8)
        assert np.array_equal(r.selected.cpu().numpy()[rows], ref_sel[rows])
        w = to_bits(r.weights)
        assert (w == golden[f"route_T{tokens}_weights"]).all(axis=1).mean() > 0.99


def test_route_other_shapes(pdx):
    """E, k, H away from the Qwen3 defaults (E not a multiple of 8, k=1, odd T)."""
    from tests.gpu_util import to_bits, to_dev
    for (tokens, hidden, experts, k) in ((5, 64, 20, 3), (33, 256, 16, 4), (9, 512, 200, 1), (7, 2048, 64, 8),
                                         (300, 512, 200, 4), (130, 256, 16, 4), (97, 1024, 130, 8)):
        x, gate = mo.synthetic_router(5000 + tokens, tokens, hidden, experts)
        for normalize in (True, False):
            r = pdx.route(to_dev(x), to_dev(gate), k, normalize)
            logits, o_sel, o_w = mo.route(x, gate, k, normalize)
            assert np.array_equal(to_bits(r.logits), logits)
            assert np.array_equal(r.selected.cpu().numpy(), o_sel)
            d = np.abs(to_bits(r.weights).astype(np.int32) - o_w.astype(np.int32))
            assert d.max() <= 1


def test_route_rejects_like_reference(pdx):
    from tests.gpu_util import to_dev
    x, gate = mo.synthetic_router(1, 4)
    xd, gd = to_dev(x), to_dev(gate)
    with pytest.raises(ValueError, match="routing parameters"):
        pdx.route(xd, gd, 0, True)
    with pytest.raises(ValueError, match="routing parameters"):
        pdx.route(xd, gd, 8, 1)
    with pytest.raises(ValueError, match="shape/dtype"):
        pdx.route(xd[:, :100], gd, 8, True)
