"""Expert-parallel device path on one GPU: R ranks simulated in one process.

Each simulated rank runs the product phases of ExpertParallelMoE (dispatch ->
regroup + grouped FFN -> combine) with the sm_100a kernels; the all-to-all is
done by slicing the ranks' buffers exactly as the NCCL exchange lays them
out.  Results must match the single-GPU layer on the same tokens: bit for bit
on the exact (prefill) exchange, and within the BF16 tolerance (2e-2) on the
padded (decode) exchange, whose split-K plan may group the K sum differently.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(ranks, experts, hidden, inter, tokens, seed):
    from pdscope_b200.expert_parallel import ExpertParallelMoE, local_slab_of
    from pdscope_b200.runtime import ExpertSlab, ResidentMoELayer
    gen = torch.Generator(device="cuda").manual_seed(seed)
    slab = ExpertSlab.allocate(experts, hidden, inter, "cuda", generator=gen)
    gate = (torch.randn(experts, hidden, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    xs = [torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16) for _ in range(ranks)]
    layers = [ExpertParallelMoE(gate, local_slab_of(slab, r, ranks), rank=r, world=ranks) for r in range(ranks)]
    single = ResidentMoELayer(gate, slab)
    return layers, single, xs


def _simulate(layers, xs, mode):
    R = len(layers)
    EL = layers[0].local
    ds = [layers[r].dispatch(xs[r], mode) for r in range(R)]
    rc = [torch.cat([ds[s].packed.counts[r * EL:(r + 1) * EL] for s in range(R)]) for r in range(R)]
    outs = []
    if mode == "padded":
        C = ds[0].capacity
        recv = [torch.cat([ds[s].send[r * C:(r + 1) * C] for s in range(R)]) for r in range(R)]
        ys = [layers[r].compute(recv[r], rc[r], C) for r in range(R)]
        back = [torch.cat([ys[r][s * C:(s + 1) * C] for r in range(R)]) for s in range(R)]
    else:
        off = [d.packed.offsets.cpu().tolist() for d in ds]
        blocks = [[(off[s][r * EL], off[s][(r + 1) * EL]) for r in range(R)] for s in range(R)]
        recv = [torch.cat([ds[s].send[a:b] for s, (a, b) in ((s, blocks[s][r]) for s in range(R))]) for r in range(R)]
        ys = [layers[r].compute(recv[r], rc[r], 0) for r in range(R)]
        back = []
        for s in range(R):
            parts = []
            for r in range(R):
                start = sum(blocks[q][r][1] - blocks[q][r][0] for q in range(s))
                n = blocks[s][r][1] - blocks[s][r][0]
                parts.append(ys[r][start:start + n])
            back.append(torch.cat(parts))
    for s in range(R):
        outs.append(layers[s].finish(ds[s], back[s]))
    return outs


@pytest.mark.parametrize("ranks,tokens,mode", [(2, 1, "padded"), (4, 8, "padded"), (8, 64, "padded"),
                                                (2, 300, "exact"), (4, 1000, "exact")])
def test_expert_parallel_matches_single_gpu(ranks, tokens, mode):
    from pdscope_b200.runtime import raise_device_error
    layers, single, xs = _setup(ranks, 128, 2048, 768, tokens, seed=ranks * 100 + tokens)
    outs = _simulate(layers, xs, mode)
    torch.cuda.synchronize()
    raise_device_error()
    for s in range(ranks):
        ref = single.forward(xs[s]).out
        if mode == "exact":
            assert torch.equal(outs[s], ref)
        else:
            np.testing.assert_allclose(outs[s].float().cpu().numpy(), ref.float().cpu().numpy(), rtol=2e-2, atol=2e-2)
            assert (outs[s] == ref).float().mean().item() > 0.95
