"""Failure detection of the expert-parallel peer exchange on one GPU, without
faulting anything: the flag waits of k_ep_layout_p2p and k_ep_wait_back run
against flags that nothing sets.  Each wait gives up after its limit
(shortened here with pdx_set_flag_wait_limit_ns), raises
PDX_DEVERR_WAIT_TIMEOUT, leaves the layout empty and returns, so the context
stays usable; the same region then completes normally once the flags are
set.  The reference's analogue is its run guard's deadline
(benchmarks/pdscope_compare.py:153-161)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

R, EL, H, T, K = 2, 4, 256, 3, 4


def _region(device="cuda"):
    """One layer's exchange region with every 'peer' entry pointing at this
    GPU's own zeroed buffers (no other rank exists)."""
    from pdscope_b200 import _lib
    cap = T * min(K, EL)
    z = lambda n, dt: torch.zeros(n, dtype=dt, device=device)
    bufs = dict(recv=z(R * cap * H, torch.bfloat16), back=z(R * cap * H, torch.bfloat16),
                cnt=z(R * EL, torch.int32), rflag=z(R, torch.int64), bflag=z(R, torch.int64))
    tbl = torch.tensor([[bufs[k].data_ptr()] * R for k in ("recv", "back", "cnt", "rflag", "bflag")],
                       dtype=torch.int64, device=device)
    step = z(1, torch.int64)
    ticket = z(2, torch.int32)
    lay = _lib.P2PLayer(recv=tbl[0].data_ptr(), back=tbl[1].data_ptr(), cnt=tbl[2].data_ptr(),
                        rflag=tbl[3].data_ptr(), bflag=tbl[4].data_ptr(), step=step.data_ptr(),
                        ticket=ticket.data_ptr())
    return cap, bufs, tbl, step, ticket, lay


def test_flag_waits_time_out_and_leave_an_empty_layout():
    from pdscope_b200 import _lib
    lib = _lib.lib
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert _lib.device_error(s) == 0
    cap, bufs, tbl, step, ticket, lay = _region()
    offsets = torch.full((EL + 1,), -7, dtype=torch.int32, device="cuda")
    active = torch.full((EL + 1,), -7, dtype=torch.int32, device="cuda")
    perm = torch.full((R * cap,), -7, dtype=torch.int32, device="cuda")
    _lib.check(lib.pdx_set_flag_wait_limit_ns(50_000_000))            # 50 ms
    try:
        _lib.check(lib.pdx_ep_layout_p2p(R, 0, EL, cap, R * cap, ctypes.byref(lay), offsets.data_ptr(),
                                         active.data_ptr(), perm.data_ptr(), s))
        assert _lib.device_error(s) == _lib.PDX_DEVERR_WAIT_TIMEOUT
        assert int(active[0]) == 0                                     # nothing downstream runs
        assert offsets.tolist() == [0] * (EL + 1)
        assert (perm == -7).all()                                      # nothing written past the empty layout
        _lib.check(lib.pdx_ep_wait_back(R, 0, ctypes.byref(lay), s))
        assert _lib.device_error(s) == _lib.PDX_DEVERR_WAIT_TIMEOUT
        assert int(step[0]) == 1                                       # the layer still closes its step
        assert _lib.device_error(s) == 0                               # the error word was cleared

        # the context is still usable: the same region completes once both
        # sources' flags reach the next step and their counts are in place
        counts = torch.tensor([1, 0, 2, 0, 0, 3, 0, 1], dtype=torch.int32, device="cuda")   # [source][expert]
        bufs["cnt"].copy_(counts)
        bufs["rflag"].fill_(2)
        _lib.check(lib.pdx_ep_layout_p2p(R, 0, EL, cap, R * cap, ctypes.byref(lay), offsets.data_ptr(),
                                         active.data_ptr(), perm.data_ptr(), s))
        assert _lib.device_error(s) == 0
        per_expert = counts.view(R, EL).sum(0).tolist()               # rows of each local expert
        assert offsets.tolist() == [0] + list(torch.tensor(per_expert).cumsum(0).tolist())
        assert active[:1 + sum(c > 0 for c in per_expert)].tolist() == \
            [sum(c > 0 for c in per_expert)] + [l for l in range(EL) if per_expert[l] > 0]
        # regrouped rows: each local expert's rows from source 0, then source 1
        # (source s's block starts at s * cap, its experts back to back)
        want = []
        blk = [[0] * EL for _ in range(R)]
        for src in range(R):
            run = src * cap
            for l in range(EL):
                blk[src][l] = run
                run += int(counts[src * EL + l])
        for l in range(EL):
            for src in range(R):
                want.extend(range(blk[src][l], blk[src][l] + int(counts[src * EL + l])))
        assert perm[:len(want)].tolist() == want
        bufs["bflag"].fill_(2)
        _lib.check(lib.pdx_ep_wait_back(R, 0, ctypes.byref(lay), s))
        assert _lib.device_error(s) == 0
        assert int(step[0]) == 2
    finally:
        _lib.check(lib.pdx_set_flag_wait_limit_ns(0))


def test_flag_wait_limit_bounds():
    from pdscope_b200 import _lib
    with pytest.raises(ValueError):
        _lib.check(_lib.lib.pdx_set_flag_wait_limit_ns(61_000_000_000))
    _lib.check(_lib.lib.pdx_set_flag_wait_limit_ns(0))
