"""ctypes binding of libpdx_moe.so (the C ABI in include/pdx_moe.h).

The shared library is the only compute path: if it is missing or cannot be
loaded this module raises at import time; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("PDX_MOE_LIB", _PKG / "libpdx_moe.so"))

PDX_OK = 0
PDX_ERR_INVALID = 1
PDX_ERR_UNSUPPORTED = 2
PDX_ERR_WORKSPACE = 3
PDX_ERR_CUDA = 4
PDX_ERR_DEVICE = 5

PDX_DEVERR_NONE = 0
PDX_DEVERR_WAIT_TIMEOUT = 1
PDX_DEVERR_BAD_EXPERT = 2
PDX_DEVERR_BAD_SLOT = 3

FFN_AUTO, FFN_GEMV, FFN_GEMM, FFN_SIMT, FFN_GEMM_1CTA, FFN_GEMM_PAIR, FFN_GEMV_STAGED = 0, 1, 2, 3, 4, 5, 6
LAYER_OUT_NORM = 0x100   # OR into pdx_moe_layer's mode: out = layer_norm(MoE(x) + residual)

ABI_VERSION = 1

c_i64 = ctypes.c_int64
c_i32 = ctypes.c_int32
c_vp = ctypes.c_void_p
c_sz = ctypes.c_size_t


class ExpertWeights(ctypes.Structure):
    """struct pdx_expert_weights."""
    _fields_ = [("gate", c_vp), ("up", c_vp), ("down", c_vp),
                ("gate_stride", c_i64), ("up_stride", c_i64), ("down_stride", c_i64),
                ("num_slots", c_i64), ("slot_of_expert", c_vp)]


class OffloadConfig(ctypes.Structure):
    """pdx_offload_config."""
    _fields_ = [("layers", c_i32), ("experts", c_i32), ("hidden", c_i32), ("inter", c_i32), ("top_k", c_i32),
                ("normalize", c_i32), ("gates", ctypes.POINTER(c_vp)), ("host_experts", c_vp),
                ("fixed_count", ctypes.POINTER(c_i32)), ("fixed_experts", ctypes.POINTER(c_i32)),
                ("hot_per_layer", c_i32), ("chunk", c_i32), ("prefetch", c_i32), ("cache_slots", c_i64),
                ("max_tokens", c_i64)]


class OffloadStats(ctypes.Structure):
    """pdx_offload_stats."""
    _fields_ = [(name, c_i64) for name in ("h2d_bytes", "demand_copies", "prefetch_copies", "prefetch_used",
                                           "prefetch_wasted", "cache_hits", "hot_hits", "warm_hits",
                                           "expert_uses", "layers")]


class OffloadTrace(ctypes.Structure):
    """pdx_offload_trace."""
    _fields_ = [(name, c_i32) for name in ("layer", "routed_experts", "hot", "warm", "cache_ready", "cache_loading",
                                           "demand", "demand_chunks", "prefetch_issued", "prefetch_used",
                                           "prefetch_skipped")] + [("tokens", c_i64), ("h2d_bytes", c_i64)]


PLACE_NONE, PLACE_HOT, PLACE_WARM, PLACE_CACHE, PLACE_LOADING, PLACE_DEMAND = 0, 1, 2, 3, 4, 5


class P2PLayer(ctypes.Structure):
    """pdx_p2p_layer."""
    _fields_ = [("recv", c_vp), ("back", c_vp), ("cnt", c_vp), ("rflag", c_vp), ("bflag", c_vp), ("step", c_vp),
                ("ticket", c_vp)]


# name -> (restype, argtypes)
SIGNATURES = {
    "pdx_last_error": (ctypes.c_char_p, []),
    "pdx_abi_version": (ctypes.c_int, []),
    "pdx_launch_count": (ctypes.c_uint64, []),
    "pdx_route_workspace_bytes": (c_sz, [c_i64, c_i64]),
    "pdx_route_topk": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp,
                                      c_vp, c_sz, c_vp]),
    "pdx_topk_from_logits": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "pdx_pack_workspace_bytes": (c_sz, [c_i64, c_i32, c_i64]),
    "pdx_pack": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i32, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                c_vp, c_sz, c_vp]),
    "pdx_pack_static": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i32, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                       c_vp]),
    "pdx_gather_rows": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp]),
    "pdx_ffn_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64, c_i64, c_i32]),
    "pdx_moe_ffn_grouped": (ctypes.c_int, [c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64,
                                           ctypes.POINTER(ExpertWeights), c_i64, c_i64, c_vp, c_i32, c_vp,
                                           c_sz, c_vp]),
    "pdx_expert_ffn_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64]),
    "pdx_expert_ffn": (ctypes.c_int, [c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_sz, c_vp]),
    "pdx_combine": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, c_i32, c_i64, c_vp, c_vp, c_vp]),
    "pdx_residual_layernorm": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i64, ctypes.c_float, c_vp, c_vp]),
    "pdx_combine_layernorm": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, c_i32, c_i64, c_vp, ctypes.c_float, c_vp,
                                             c_vp]),
    "pdx_layer_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64, c_i32, c_i64, c_i32]),
    "pdx_moe_layer": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_i32,
                                     ctypes.POINTER(ExpertWeights), c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                     c_i32, c_vp, c_sz, c_vp]),
    "pdx_ep_dispatch": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i64, c_i64, c_i32, c_i64, c_vp, c_vp,
                                       c_vp]),
    "pdx_ep_layout": (ctypes.c_int, [c_vp, c_i32, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "pdx_ep_regroup": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "pdx_ep_ungroup": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "pdx_ep_combine": (ctypes.c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i32, c_i64, c_vp, c_vp, c_vp]),
    "pdx_ep_combine_layernorm": (ctypes.c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i32, c_i64, c_vp, ctypes.c_float,
                                                c_vp, c_vp]),
    "pdx_device_error": (ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_uint32)]),
    "pdx_p2p_alloc": (ctypes.c_int, [c_sz, ctypes.POINTER(c_vp)]),
    "pdx_p2p_free": (ctypes.c_int, [c_vp]),
    "pdx_ipc_handle": (ctypes.c_int, [c_vp, c_vp]),
    "pdx_ipc_open": (ctypes.c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "pdx_ipc_close": (ctypes.c_int, [c_vp]),
    "pdx_ep_dispatch_p2p": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i64, c_i64, c_i32, c_i32, c_i64,
                                           ctypes.POINTER(P2PLayer), c_vp, c_vp]),
    "pdx_ep_layout_p2p": (ctypes.c_int, [c_i32, c_i32, c_i64, c_i64, c_i64, ctypes.POINTER(P2PLayer), c_vp, c_vp,
                                         c_vp, c_vp]),
    "pdx_ep_return_p2p": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_i32, c_i64,
                                         ctypes.POINTER(P2PLayer), c_vp]),
    "pdx_ep_wait_back": (ctypes.c_int, [c_i32, c_i32, ctypes.POINTER(P2PLayer), c_vp]),
    "pdx_set_flag_wait_limit_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "pdx_offload_pool_bytes": (c_sz, [ctypes.POINTER(OffloadConfig)]),
    "pdx_offload_workspace_bytes": (c_sz, [ctypes.POINTER(OffloadConfig)]),
    "pdx_offload_create": (ctypes.c_int, [ctypes.POINTER(OffloadConfig), c_vp, c_vp, c_sz, ctypes.POINTER(c_vp)]),
    "pdx_offload_forward_layer": (ctypes.c_int, [c_vp, c_i32, c_vp, c_i64, c_vp, c_i32, c_vp, c_vp]),
    "pdx_offload_get_stats": (ctypes.c_int, [c_vp, ctypes.POINTER(OffloadStats)]),
    "pdx_offload_destroy": (None, [c_vp]),
    "pdx_offload_last_trace": (ctypes.c_int, [c_vp, ctypes.POINTER(OffloadTrace), c_vp, c_vp, c_vp, c_vp]),
    "pdx_offload_copy_selected": (ctypes.c_int, [c_vp, c_i32, c_i64, c_vp, c_vp]),
}


class PdxError(RuntimeError):
    """A CUDA or device-side failure reported by libpdx_moe."""


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"libpdx_moe.so not found at {LIB_PATH}; build it with "
                          "`python -m pdscope_b200.build` (the CUDA path has no fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.pdx_abi_version() != ABI_VERSION:
        raise ImportError("libpdx_moe.so ABI version mismatch; rebuild it")
    return lib


lib = _load()


def last_error() -> str:
    msg = lib.pdx_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Map a pdx_status to the reference's exception types."""
    if status == PDX_OK:
        return
    msg = last_error()
    if status == PDX_ERR_INVALID:
        raise ValueError(msg)
    if status == PDX_ERR_UNSUPPORTED:
        raise ValueError("unsupported by the sm_100a kernels: " + msg)
    if status == PDX_ERR_WORKSPACE:
        raise RuntimeError("workspace: " + msg)
    raise PdxError(msg)


def device_error(stream_handle) -> int:
    """Synchronise the stream, then read and clear the device error word."""
    code = ctypes.c_uint32(0)
    status = lib.pdx_device_error(stream_handle, ctypes.byref(code))
    if status not in (PDX_OK, PDX_ERR_DEVICE):
        check(status)
    return int(code.value)
