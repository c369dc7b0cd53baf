"""B200-native (sm_100a) MoE expert execution path for PDScope.

The compute lives in ``libpdx_moe.so`` (C ABI: include/pdx_moe.h); ``_lib``
binds it and ``runtime`` mirrors the reference's Python interface.  Importing
the package itself does not load the library (so ``pdscope_b200.build`` can
rebuild it); the first use of any runtime name loads it and raises if it is
missing -- there is no fallback.
"""
_RUNTIME_NAMES = ("PDScopeCudaRuntime", "PdxGpuBackend", "ExpertSlab", "ResidentMoELayer", "Routing", "combine",
                  "compact_expert_groups", "expert_forward", "expert_groups", "pack", "route", "topk_from_logits")


def __getattr__(name):
    if name in _RUNTIME_NAMES:
        from . import runtime
        return getattr(runtime, name)
    raise AttributeError(name)
