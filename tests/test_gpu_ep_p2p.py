"""Expert-parallel exchange over NVLink peer memory on 2 GPUs (one process per
GPU): the peer-store exchange (pdx_ep_dispatch_p2p ... pdx_ep_wait_back) must
give the same layer outputs, bit for bit, as the NCCL all-to-all exchange,
eagerly and replayed from a CUDA graph.  Needs two GPUs; skipped on one."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

L, E, H, I, K, T = 3, 16, 256, 128, 4, 8


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    peer = None
    try:
        from pdscope_b200.expert_parallel import ExpertParallelStack, PeerExchange, TorchDistExchange
        from pdscope_b200.runtime import ExpertSlab
        from pdscope_b200.stack import activations
        el = E // world
        g_gate = torch.Generator(device=dev).manual_seed(0)
        g_w = torch.Generator(device=dev).manual_seed(100 + rank)
        gates = [(torch.randn(E, H, device=dev, generator=g_gate) * 0.02).to(torch.bfloat16) for _ in range(L)]
        slabs = [ExpertSlab.allocate(el, H, I, dev, generator=g_w) for _ in range(L)]
        ref = ExpertParallelStack(gates, slabs, rank=rank, world=world, exchange=TorchDistExchange(), top_k=K)
        peer = PeerExchange(L, T, world=world, rank=rank, local_experts=el, hidden=H, top_k=K, device=dev)
        p2p = ExpertParallelStack(gates, slabs, rank=rank, world=world, exchange=TorchDistExchange(), top_k=K,
                                  peer=peer)
        ok = True
        for step in range(3):
            x = activations(T, H, device=dev, seed=10 + 7 * step + rank)
            for st in (ref, p2p):
                st.io(T)[0].copy_(x)
            ref.step(T, graph=False)
            p2p.step(T, graph=(step > 0))      # eager, then captured and replayed
            torch.cuda.synchronize(dev)
            ok &= torch.equal(ref.io(T)[1], p2p.io(T)[1])
        from pdscope_b200.runtime import raise_device_error
        raise_device_error()
        p2p.release_graphs()
        q.put((rank, bool(ok)))
    except Exception as exc:   # report; the parent fails the test
        q.put((rank, repr(exc)))
    finally:
        if peer is not None:
            try:
                peer.close()
            except Exception:
                pass
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_matches_nccl_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}, results
