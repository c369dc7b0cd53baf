"""pdx_pack_static: packing for callers that cannot allocate device memory.

Callers such as a plugin whose host process owns the device's memory, an FFI
caller without a device allocator, or a latency-critical path that cannot
take cudaMalloc's synchronisation, pack through pdx_pack_static, which keeps
its scratch in a fixed device array instead of a caller workspace.  This test
calls it through the C ABI and requires the same outputs, bit for bit, as
pdx_pack with a workspace, on two calls in a row (the second reuses the
array the first left behind).  It lives in its own file so a run that stops
at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FIELDS = ("counts", "offsets", "tokens", "positions", "packed_w", "inverse", "active")


def _routing(seed, tokens, k, experts):
    g = torch.Generator(device="cpu").manual_seed(seed)
    scores = torch.rand(tokens, experts, generator=g)
    sel = torch.topk(scores, k, dim=-1).indices.to(torch.int64)
    w = torch.rand(tokens, k, generator=g).to(torch.bfloat16)
    return sel.cuda(), w.cuda()


def _outputs(tokens, k, experts):
    n = tokens * k
    i32 = dict(dtype=torch.int32, device="cuda")
    return dict(counts=torch.full((experts,), -7, **i32), offsets=torch.full((experts + 1,), -7, **i32),
                tokens=torch.full((n,), -7, **i32), positions=torch.full((n,), -7, **i32),
                packed_w=torch.zeros(n, dtype=torch.bfloat16, device="cuda"),
                inverse=torch.full((n,), -7, **i32), active=torch.full((experts + 1,), -7, **i32))


def _ptrs(o):
    return [ctypes.c_void_p(o[f].data_ptr()) for f in FIELDS]


def test_pack_static_matches_workspace_pack():
    from pdscope_b200 import _lib
    lib = _lib.lib
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the first two calls take the multi-CTA path (T*k > 1024), which uses the
    # scratch; then the single-CTA path (T*k <= 1024, no scratch), and a shape
    # whose histograms fill the array exactly (ceil(T*k/4096) * E == 65536)
    for seed, tokens, k, experts in ((1, 1500, 8, 128), (2, 2300, 6, 96), (3, 64, 8, 128), (4, 32768, 8, 1024)):
        sel, w = _routing(seed, tokens, k, experts)
        ref, got = _outputs(tokens, k, experts), _outputs(tokens, k, experts)
        ws = torch.empty(lib.pdx_pack_workspace_bytes(tokens, k, experts), dtype=torch.uint8, device="cuda")
        _lib.check(lib.pdx_pack(ctypes.c_void_p(sel.data_ptr()), ctypes.c_void_p(w.data_ptr()), tokens, k,
                                experts, *_ptrs(ref), ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream))
        _lib.check(lib.pdx_pack_static(ctypes.c_void_p(sel.data_ptr()), ctypes.c_void_p(w.data_ptr()), tokens, k,
                                       experts, *_ptrs(got), stream))
        torch.cuda.synchronize()
        assert _lib.device_error(stream) == 0
        for f in FIELDS:
            assert torch.equal(ref[f], got[f]), f
        n_active = int(got["active"][0])
        assert n_active == int((got["counts"] > 0).sum())
        assert torch.equal(torch.sort(got["inverse"]).values, torch.arange(tokens * k, device="cuda",
                                                                           dtype=torch.int32))


def test_pack_static_rejects_sizes_beyond_its_array():
    from pdscope_b200 import _lib
    null = ctypes.c_void_p(16)
    # ceil(200000*8/4096) * 1024 > 65536 histogram entries
    st = _lib.lib.pdx_pack_static(null, null, 200000, 8, 1024, null, null, null, null, null, null, null,
                                  ctypes.c_void_p(0))
    assert st == _lib.PDX_ERR_UNSUPPORTED
    assert "exceeds" in _lib.last_error()
