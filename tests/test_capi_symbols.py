"""CPU checks of the C-ABI library: it loads, exports every declared symbol,
and rejects invalid arguments before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "pdx_moe.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pdx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_path():
    names = declared_functions()
    for required in ("pdx_route_topk", "pdx_topk_from_logits", "pdx_pack", "pdx_gather_rows",
                     "pdx_moe_ffn_grouped", "pdx_expert_ffn", "pdx_combine", "pdx_moe_layer",
                     "pdx_device_error", "pdx_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from pdscope_b200 import _lib
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # the binding table covers the header exactly
    assert set(_lib.SIGNATURES) == set(declared_functions())
    assert _lib.lib.pdx_abi_version() == _lib.ABI_VERSION


def test_python_constants_match_header():
    """The integer constants the bindings mirror (status codes, device error
    codes, FFN modes, the layer flag) have the header's values."""
    from pdscope_b200 import _lib
    text = (ROOT / "include" / "pdx_moe.h").read_text()
    consts = {m.group(1): int(m.group(2), 0)
              for m in re.finditer(r"\b(PDX_[A-Z0-9_]+)\s*(?:=\s*|\s+)(0x[0-9a-fA-F]+|\d+)u?\b", text)}
    mirrored = {}
    for name, value in consts.items():
        for py_name in (name, name[len("PDX_"):]):
            if hasattr(_lib, py_name):
                mirrored[name] = (getattr(_lib, py_name), value)
    for required in ("PDX_OK", "PDX_ERR_DEVICE", "PDX_DEVERR_BAD_SLOT", "PDX_FFN_GEMM_1CTA", "PDX_LAYER_OUT_NORM"):
        assert required in mirrored, required
    assert all(py == c for py, c in mirrored.values()), mirrored


def test_workspace_queries_are_monotone():
    from pdscope_b200 import _lib
    from pdscope_b200._lib import lib
    a = lib.pdx_layer_workspace_bytes(1, 2048, 128, 8, 768, 0)
    b = lib.pdx_layer_workspace_bytes(512, 2048, 128, 8, 768, 0)
    c = lib.pdx_layer_workspace_bytes(512, 2048, 128, 8, 768, 2)
    d = lib.pdx_layer_workspace_bytes(4096, 2048, 128, 8, 768, 0)
    assert 0 < a < b < d and 0 < c < d
    # auto mode sizes for the path it runs: the weight-streaming path up to 48
    # rows per expert (T=512 here), the token-tiled GEMM beyond
    assert b == lib.pdx_layer_workspace_bytes(512, 2048, 128, 8, 768, 1)
    assert d == lib.pdx_layer_workspace_bytes(4096, 2048, 128, 8, 768, 2)
    assert lib.pdx_pack_workspace_bytes(4096, 8, 128) >= 8 * 128 * 4
    assert lib.pdx_route_workspace_bytes(64, 128) >= 64 * 128 * 2
    # prefill sizes also hold the split-K router partials (up to 4 x T x E FP64)
    assert lib.pdx_route_workspace_bytes(4096, 128) >= 4 * 4096 * 128 * 8
    # auto FFN workspace for rows = T*k also covers T <= 64 (decode path), e.g. 16 tokens x 8
    for rows in (128, 512):
        assert lib.pdx_ffn_workspace_bytes(rows, 128, 2048, 768, 0) >= lib.pdx_ffn_workspace_bytes(rows, 128, 2048,
                                                                                                      768, 1)
    # the decode path's query covers the single launch (both forms) and the
    # staged form (mode 6) it may fall back to, at every rows / experts mix
    for rows, experts in ((8, 128), (64, 128), (512, 128), (4096, 128), (300, 16), (2048, 1024)):
        one = lib.pdx_ffn_workspace_bytes(rows, experts, 2048, 768, _lib.FFN_GEMV)
        staged = lib.pdx_ffn_workspace_bytes(rows, experts, 2048, 768, _lib.FFN_GEMV_STAGED)
        assert one >= staged >= rows * 768 * 2


def test_validation_errors_without_device():
    """Contract violations return PDX_ERR_INVALID (the reference's ValueError)."""
    from pdscope_b200 import _lib
    lib = _lib.lib
    null = ctypes.c_void_p(0)
    # T = 0: 'empty expert routing'
    st = lib.pdx_route_topk(null, null, 0, 2048, 128, 8, 1, null, null, null, null, 0, null)
    assert st == _lib.PDX_ERR_INVALID and "empty" in _lib.last_error()
    # top_k > E: 'invalid routing parameters'
    st = lib.pdx_route_topk(null, null, 4, 2048, 8, 9, 1, null, null, null, null, 0, null)
    assert st == _lib.PDX_ERR_INVALID and "routing parameters" in _lib.last_error()
    # top_k beyond the kernels' range is UNSUPPORTED, not silently wrong
    st = lib.pdx_route_topk(null, null, 4, 2048, 128, 33, 1, null, null, null, null, 0, null)
    assert st == _lib.PDX_ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        _lib.check(_lib.PDX_ERR_INVALID)
    # pack with null outputs
    st = lib.pdx_pack(null, null, 4, 8, 128, null, null, null, null, null, null, null, null, 0, null)
    assert st == _lib.PDX_ERR_INVALID
    # combine with top_k = 0
    st = lib.pdx_combine(null, null, null, 4, 0, 2048, null, null, null)
    assert st == _lib.PDX_ERR_INVALID
    # layer: unsupported hidden size for the tcgen05 path
    w = _lib.ExpertWeights()
    st = lib.pdx_moe_layer(null, null, 4, 2040, 128, 8, 1, ctypes.byref(w), 768, null, null, null, null, null,
                           null, 2, null, 0, null)
    assert st in (_lib.PDX_ERR_UNSUPPORTED, _lib.PDX_ERR_INVALID)


def test_expert_ffn_rejects_empty_input():
    from pdscope_b200 import _lib
    null = ctypes.c_void_p(0)
    st = _lib.lib.pdx_expert_ffn(ctypes.c_void_p(16), 0, ctypes.c_void_p(16), ctypes.c_void_p(16),
                                 ctypes.c_void_p(16), 2048, 768, ctypes.c_void_p(16), null, 0, null)
    assert st == _lib.PDX_ERR_INVALID
