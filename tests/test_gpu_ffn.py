"""GPU parity of the expert FFN (expert_forward, qwen.py:87-90): streaming GEMV
(decode) and tcgen05 grouped GEMM (prefill) against the oracle.

Tolerance: BF16 outputs within rtol 2e-2 / atol 2e-2 of the oracle's BF16
restatement, and FP32-accumulate relative L2 <= 0.02 against reference_fp32
(the reference's own bound, pdscope_compare.py:692-695)."""
import ctypes

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


def _expert(seed, hidden, inter):
    rng = np.random.default_rng(seed)
    g = mo.f32_to_bf16(rng.standard_normal((inter, hidden), dtype=np.float32) * 0.02)
    u = mo.f32_to_bf16(rng.standard_normal((inter, hidden), dtype=np.float32) * 0.02)
    d = mo.f32_to_bf16(rng.standard_normal((hidden, inter), dtype=np.float32) * 0.02)
    return g, u, d


def _check_rows(actual_bits, x, g, u, d):
    exp = mo.expert_forward(x, g, u, d)
    a = mo.bf16_to_f32(actual_bits)
    np.testing.assert_allclose(a, mo.bf16_to_f32(exp), rtol=RTOL, atol=ATOL)
    ref32 = mo.reference_fp32(x, g, u, d)
    assert mo.error_metrics(a, ref32)["relative_l2"] <= 0.02
    # nearly all elements bit-identical to the BF16 restatement
    return (actual_bits == exp).mean()


@pytest.mark.parametrize("n", (1, 3, 8, 9, 64, 65, 200, 1000))
@pytest.mark.parametrize("shape", ((256, 128), (2048, 768)))
def test_expert_forward(pdx, n, shape):
    from tests.gpu_util import to_bits, to_dev
    hidden, inter = shape
    g, u, d = _expert(n + hidden, hidden, inter)
    x = mo.f32_to_bf16(np.random.default_rng(n).standard_normal((n, hidden), dtype=np.float32))
    y = pdx.expert_forward(to_dev(x), dict(gate_proj=to_dev(g), up_proj=to_dev(u), down_proj=to_dev(d)))
    frac = _check_rows(to_bits(y), x, g, u, d)
    assert frac > 0.9


def test_expert_forward_vs_torch_on_device(pdx):
    """Against the reference's own GPU expert_forward (cuBLAS) on the B200."""
    from tests.gpu_util import f32, to_dev, torch_expert_forward
    g, u, d = _expert(5, 2048, 768)
    for n in (1, 7, 300):
        x = to_dev(mo.f32_to_bf16(np.random.default_rng(n).standard_normal((n, 2048), dtype=np.float32)))
        gd, ud, dd = to_dev(g), to_dev(u), to_dev(d)
        ours = pdx.expert_forward(x, dict(gate_proj=gd, up_proj=ud, down_proj=dd))
        ref = torch_expert_forward(x, gd, ud, dd)
        np.testing.assert_allclose(f32(ours), f32(ref), rtol=RTOL, atol=ATOL)


def _grouped_case(pdx, tokens, experts, k, hidden, inter, mode, seed, slot_perm=False, zipf=False, check=True,
                  prepacked=False):
    from tests.gpu_util import to_bits, to_dev
    from pdscope_b200 import _lib
    from pdscope_b200.runtime import ExpertSlab
    x, gate, wg, wu, wd = mo.synthetic_layer(seed, tokens, hidden, experts, inter)
    if zipf:  # Zipf(1.1) router skew through hidden column 0: a few experts take most rows
        ranks = np.random.default_rng(seed).permutation(experts) + 1
        gate = gate.copy()
        x = x.copy()
        gate[:, 0] = mo.f32_to_bf16((-0.75 * 1.1 * np.log(ranks)).astype(np.float32))
        x[:, 0] = mo.f32_to_bf16(np.ones(tokens, np.float32))
    _, sel, w = mo.route(x, gate, k, True)
    packed = mo.compact_expert_groups(sel, w, experts)
    slab = ExpertSlab.from_tensors([dict(gate_proj=to_dev(wg[e]), up_proj=to_dev(wu[e]), down_proj=to_dev(wd[e]))
                                    for e in range(experts)])
    slot_of = None
    if slot_perm:  # experts stored in a shuffled slot order, as a cache ledger would
        perm = np.random.default_rng(seed).permutation(experts)
        order = np.argsort(perm)  # slot s holds expert perm[s]
        storage = slab.storage.view(experts, -1)[torch.from_numpy(perm).cuda()].contiguous()
        slot_of = torch.from_numpy(order.astype(np.int32)).cuda()
        slab = ExpertSlab(storage.view(-1), hidden, inter, slot_of_expert=slot_of)
    rows = tokens * k
    y = torch.empty((rows, hidden), dtype=torch.bfloat16, device="cuda")
    dev = {key: torch.from_numpy(packed[key]).cuda() for key in ("tokens", "offsets")}
    nz = np.nonzero(packed["counts"])[0]
    active = torch.from_numpy(np.concatenate([[len(nz)], nz, np.zeros(experts - len(nz), int)]).astype(np.int32)).cuda()
    ws_bytes = _lib.lib.pdx_ffn_workspace_bytes(rows, experts, hidden, inter, mode)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    xd = to_dev(x)
    tok_ptr = ctypes.c_void_p(dev["tokens"].data_ptr())
    x_rows = tokens
    if prepacked:  # rows already in packed order (tokens == NULL), as the expert-parallel exchange hands them over
        xd = xd[dev["tokens"].long()].contiguous()
        tok_ptr, x_rows = None, rows
    _lib.check(_lib.lib.pdx_moe_ffn_grouped(
        ctypes.c_void_p(xd.data_ptr()), x_rows, tok_ptr,
        ctypes.c_void_p(dev["offsets"].data_ptr()), ctypes.c_void_p(active.data_ptr()), experts, rows,
        ctypes.byref(slab.struct), hidden, inter, ctypes.c_void_p(y.data_ptr()), mode,
        ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert _lib.device_error(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    got = to_bits(y)
    if not check:
        return got
    exp = np.zeros_like(got)
    off = packed["offsets"]
    for e in nz:
        a, b = off[e], off[e + 1]
        exp[a:b] = mo.expert_forward(x[packed["tokens"][a:b]], wg[e], wu[e], wd[e])
    np.testing.assert_allclose(mo.bf16_to_f32(got), mo.bf16_to_f32(exp), rtol=RTOL, atol=ATOL)
    assert (got == exp).mean() > 0.9
    return got


@pytest.mark.parametrize("mode", (1, 2, 3, 4, 5, 6))
@pytest.mark.parametrize("tokens", (1, 5, 64, 300))
def test_grouped_ffn_small_shape(pdx, mode, tokens):
    _grouped_case(pdx, tokens, 16, 4, 256, 128, mode, 100 + tokens)


@pytest.mark.parametrize("mode", (1, 2, 3, 5))
def test_grouped_ffn_slot_mapping(pdx, mode):
    """Experts located through slot_of_expert (the executor's cache-slot ledger)."""
    a = _grouped_case(pdx, 40, 16, 4, 256, 128, mode, 7, slot_perm=False)
    b = _grouped_case(pdx, 40, 16, 4, 256, 128, mode, 7, slot_perm=True)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("mode,tokens", ((1, 1), (1, 8), (1, 64), (1, 130), (3, 64), (2, 130), (2, 512), (5, 130),
                                         (5, 512)))
def test_grouped_ffn_qwen3_shape(pdx, mode, tokens):
    _grouped_case(pdx, tokens, 128, 8, 2048, 768, mode, 200 + tokens)


@pytest.mark.parametrize("tokens,experts,k,hidden,inter,zipf", (
    (1, 128, 8, 2048, 768, False), (2, 128, 8, 2048, 768, False), (8, 128, 8, 2048, 768, False),
    (16, 64, 8, 1024, 512, False), (17, 128, 8, 2048, 768, False), (33, 32, 8, 512, 256, False),
    (64, 128, 8, 2048, 768, False), (64, 16, 4, 256, 128, True), (40, 8, 8, 512, 256, True),
    (65, 128, 8, 2048, 768, False), (130, 128, 8, 2048, 768, True), (512, 128, 8, 2048, 768, False),
    (300, 16, 4, 256, 128, True)))
def test_single_launch_decode_matches_staged(pdx, tokens, experts, k, hidden, inter, zipf):
    """The decode FFN in one launch (mode 1 with T <= 64: gate/up on the whole
    token matrix, down in the same launch behind per-expert h counters)
    against the staged form (mode 6: row gather, then one launch per
    projection).  Same weight tiles, K slices and slice order, so the rows are
    bit-identical; the single launch runs twice in a row on one workspace (its
    tickets and counters are cleared before every launch).  Cases cover split-K
    in either projection (few active experts), Zipf-skewed experts with more
    rows than one down tile, every token on every expert, and T not a multiple
    of 16; past 64 tokens the single launch tiles the gate/up GEMM over the
    gathered rows (config 1 at T = 512 among them)."""
    a = _grouped_case(pdx, tokens, experts, k, hidden, inter, 6, 300 + tokens, zipf=zipf)
    b = _grouped_case(pdx, tokens, experts, k, hidden, inter, 1, 300 + tokens, zipf=zipf)
    c = _grouped_case(pdx, tokens, experts, k, hidden, inter, 1, 300 + tokens, zipf=zipf)
    assert np.array_equal(a, b)
    assert np.array_equal(b, c)


@pytest.mark.parametrize("tokens,experts", ((8, 128), (64, 16), (200, 128)))
def test_single_launch_prepacked_rows(pdx, tokens, experts):
    """Rows handed over already in packed order (tokens == NULL, the
    expert-parallel exchange's form): the single launch tiles them directly
    and matches the staged form bit for bit."""
    a = _grouped_case(pdx, tokens, experts, 8, 2048, 768, 6, 700 + tokens, prepacked=True)
    b = _grouped_case(pdx, tokens, experts, 8, 2048, 768, 1, 700 + tokens, prepacked=True)
    assert np.array_equal(a, b)


def test_ffn_paths_agree(pdx):
    """The three FFN paths (weight-streaming tcgen05, token-tiled tcgen05, SIMT)
    are independent implementations of the same rows."""
    outs = [mo.bf16_to_f32(_grouped_case(pdx, 96, 32, 8, 512, 256, m, 31)) for m in (1, 2, 3)]
    for a in outs[1:]:
        assert np.abs(outs[0] - a).max() <= 2e-2


@pytest.mark.parametrize("tokens", (1, 2, 16))
def test_stream_split_k_deterministic(pdx, tokens):
    """Few experts -> split-K with a fixed-order reduction: repeated runs are
    bit-identical."""
    a = _grouped_case(pdx, tokens, 64, 8, 1024, 512, 1, 900 + tokens)
    b = _grouped_case(pdx, tokens, 64, 8, 1024, 512, 1, 900 + tokens)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("tokens", (700, 3000))
def test_pair_tiles_match_single(pdx, tokens):
    """CTA-pair 256 x 256 tiles (mode 5) against single-CTA 128 x 256 tiles
    (mode 4) on a Zipf-skewed prefill at the Qwen3-30B-A3B shape: segments of
    thousands of rows, ragged tails and one-row experts.  Each output element
    takes the same K-ordered sequence of MMAs on both paths."""
    a = _grouped_case(pdx, tokens, 128, 8, 2048, 768, 4, 55 + tokens, zipf=True, check=False)
    b = _grouped_case(pdx, tokens, 128, 8, 2048, 768, 5, 55 + tokens, zipf=True, check=False)
    np.testing.assert_allclose(mo.bf16_to_f32(a), mo.bf16_to_f32(b), rtol=RTOL, atol=ATOL)
    assert (a == b).mean() > 0.999


def test_pair_tiles_zipf_oracle(pdx):
    """CTA-pair path against the oracle on a skewed batch."""
    _grouped_case(pdx, 400, 16, 8, 512, 256, 5, 77, zipf=True)
