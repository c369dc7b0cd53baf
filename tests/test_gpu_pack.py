"""GPU parity of packing (compact_expert_groups, pdscope_runtime.py:16-39)."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pdx():
    import pdscope_b200
    return pdscope_b200


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _pack_np(pdx, sel, w_bits, experts):
    from tests.gpu_util import to_bits, to_dev
    p = pdx.pack(torch.from_numpy(sel).cuda(), to_dev(w_bits), experts)
    return dict(counts=p.counts.cpu().numpy(), offsets=p.offsets.cpu().numpy(), tokens=p.tokens.cpu().numpy(),
                positions=p.positions.cpu().numpy(), weights=to_bits(p.weights), inverse=p.inverse.cpu().numpy(),
                active=p.active.cpu().numpy())


def _check_against_oracle(got, sel, w_bits, experts):
    exp = mo.compact_expert_groups(sel, w_bits, experts)
    for key in ("counts", "offsets", "tokens", "positions", "weights", "inverse"):
        assert np.array_equal(got[key], exp[key]), key
    nz = np.nonzero(exp["counts"])[0]
    assert got["active"][0] == len(nz)
    assert np.array_equal(got["active"][1:1 + len(nz)], nz)


@pytest.mark.parametrize("tokens", (1, 16, 64, 256, 1024, 4096))
def test_pack_on_reference_routing_golden(pdx, golden, tokens):
    """Bit-exact against the reference's own grouping of its own routing."""
    sel = golden[f"route_T{tokens}_selected"].astype(np.int64)
    w = golden[f"route_T{tokens}_weights"]
    got = _pack_np(pdx, sel, w, 128)
    assert np.array_equal(got["counts"], golden[f"route_T{tokens}_counts"])
    key = f"route_T{tokens}_group_tokens"
    if key in golden:
        assert np.array_equal(got["tokens"], golden[key])
        assert np.array_equal(got["weights"], golden[f"route_T{tokens}_group_weights"])
    else:
        assert _sha(got["tokens"]) == bytes(golden[key + "_sha256"]).decode()
        assert _sha(got["weights"]) == bytes(golden[f"route_T{tokens}_group_weights_sha256"]).decode()
    _check_against_oracle(got, sel, w, 128)


@pytest.mark.parametrize("tokens,k,experts", [(1, 8, 128), (3, 2, 8), (65, 8, 128), (1000, 4, 16),
                                              (1025, 8, 128), (17000, 8, 128), (36864, 8, 128),
                                              (50, 6, 1000)])
def test_pack_random_and_large(pdx, tokens, k, experts):
    """Single-CTA and multi-CTA paths, ragged sizes, up to the EP prefill scale."""
    rng = np.random.default_rng(tokens * 7 + k)
    # distinct experts per token, skewed popularity (Zipf-like)
    pop = 1.0 / np.arange(1, experts + 1) ** 1.1
    sel = np.stack([rng.choice(experts, size=k, replace=False, p=pop / pop.sum()) for _ in range(tokens)])
    sel = sel.astype(np.int64)
    w = mo.f32_to_bf16(rng.random((tokens, k), dtype=np.float32))
    got = _pack_np(pdx, sel, w, experts)
    _check_against_oracle(got, sel, w, experts)


def test_pack_duplicates_and_empty_experts(pdx):
    """Same expert twice for one token and experts with no tokens (arbitrary ids)."""
    sel = np.array([[5, 5, 0], [0, 5, 5], [7, 7, 7]], np.int64)
    w = mo.f32_to_bf16(np.arange(9, dtype=np.float32).reshape(3, 3) / 9)
    got = _pack_np(pdx, sel, w, 8)
    _check_against_oracle(got, sel, w, 8)


def test_compact_expert_groups_api(pdx, golden):
    """The host-facing groups dict equals the oracle's per-expert split."""
    from tests.gpu_util import to_bits, to_dev
    from pdscope_b200.runtime import Routing
    sel = golden["route_T256_selected"].astype(np.int64)
    w = golden["route_T256_weights"]
    r = Routing(None, torch.from_numpy(sel).cuda(), to_dev(w))
    groups, cpu_idx = pdx.compact_expert_groups(r)
    exp = mo.compact_expert_groups(sel, w, 128)
    off = exp["offsets"]
    assert set(groups) == set(np.nonzero(exp["counts"])[0].tolist())
    for e, (t, ww) in groups.items():
        assert t.dtype == torch.int64 and t.is_cuda
        assert np.array_equal(t.cpu().numpy(), exp["tokens"][off[e]:off[e + 1]])
        assert np.array_equal(to_bits(ww), exp["weights"][off[e]:off[e + 1]])
        assert torch.equal(cpu_idx[e], t.cpu())
    generic = pdx.expert_groups(Routing(torch.zeros(256, 128, dtype=torch.bfloat16, device="cuda"),
                                        r.selected, r.weights))
    assert [g[0] for g in generic] == sorted(groups)


def test_pack_rejects_out_of_range_ids(pdx):
    from tests.gpu_util import to_dev
    from pdscope_b200.runtime import Routing
    sel = torch.tensor([[0, 1], [2, 200]], dtype=torch.int64, device="cuda")
    w = to_dev(np.zeros((2, 2), np.uint16))
    with pytest.raises(ValueError, match="outside configured range"):
        pdx.compact_expert_groups(Routing(None, sel, w), experts=128)
    # the context stays usable afterwards
    sel_ok = torch.tensor([[0, 1], [2, 3]], dtype=torch.int64, device="cuda")
    groups, _ = pdx.compact_expert_groups(Routing(None, sel_ok, w), experts=128)
    assert sorted(groups) == [0, 1, 2, 3]


def test_single_token_grouping(pdx, golden):
    from tests.gpu_util import to_bits, to_dev
    x, gate = mo.synthetic_router(777, 1)
    r = pdx.route(to_dev(x), to_dev(gate), 8, True)
    st = pdx.expert_groups(r, mode="single_token")
    assert [e for e, _, _ in st] == golden["single_token_experts"].tolist()
    assert np.array_equal(np.concatenate([to_bits(w) for _, _, w in st]), golden["single_token_weights"])
