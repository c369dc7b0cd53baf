"""B200-native (sm_100a) MoE expert execution path for PDScope.

The compute lives in ``libpdx_moe.so`` (C ABI: include/pdx_moe.h); this
package binds it (``_lib``) and mirrors the reference's Python interface
(``runtime``).
"""
from . import _lib  # noqa: F401  (fails loudly if the CUDA library is missing)
from .runtime import (PDScopeCudaRuntime, PdxGpuBackend, ExpertSlab, ResidentMoELayer, Routing,  # noqa: F401
                      combine, compact_expert_groups, expert_forward, expert_groups, pack, route,
                      topk_from_logits)
