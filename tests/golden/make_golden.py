"""Generate golden vectors by running the reference's own Python path on CPU.

Run once in a container where the reference checkout exists:

    python tests/golden/make_golden.py /path/to/PDScope

It imports the reference's ``route``, ``expert_groups``, ``expert_forward``,
``reference_fp32`` (expertbench/adapters/qwen.py) and ``compact_expert_groups``
(expertbench/pdscope_runtime.py), feeds them seeded numpy inputs (regenerated
bit-identically by the tests from the seeds stored here) and writes the
outputs to ``golden_v1.npz`` beside this script.  Large outputs are stored as
SHA-256 digests of their canonical little-endian bytes; small ones in full.

The reference is NOT needed to run the tests; only this generator uses it.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import moe_oracle as mo  # noqa: E402


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def to_torch_bf16(bits):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def from_torch_bf16(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


route_inputs = mo.synthetic_router


def main(ref_root):
    sys.path.insert(0, str(Path(ref_root).resolve()))
    import torch
    from expertbench.adapters.qwen import route, expert_groups, expert_forward, reference_fp32
    from expertbench.pdscope_runtime import compact_expert_groups

    torch.set_num_threads(1)
    out = {}
    meta = dict(generator="tests/golden/make_golden.py", torch=torch.__version__,
                reference_functions=["expertbench/adapters/qwen.py:route",
                                     "expertbench/adapters/qwen.py:expert_groups",
                                     "expertbench/adapters/qwen.py:expert_forward",
                                     "expertbench/adapters/qwen.py:reference_fp32",
                                     "expertbench/pdscope_runtime.py:compact_expert_groups"],
                cases={})

    # --- route at the Qwen3-30B-A3B router shape (H=2048, E=128, k=8) -------------
    for tokens in (1, 16, 64, 256, 1024, 4096):
        seed = 20261012 + tokens
        x, gate = route_inputs(seed, tokens)
        r = route(to_torch_bf16(x), to_torch_bf16(gate), 8, True)
        logits = from_torch_bf16(r.logits)
        sel = r.selected.numpy().astype(np.int64)
        w = from_torch_bf16(r.weights)
        key = f"route_T{tokens}"
        meta["cases"][key] = dict(seed=seed, tokens=tokens, hidden=2048, experts=128, top_k=8)
        out[f"{key}_selected"] = sel.astype(np.uint8)
        out[f"{key}_weights"] = w
        if tokens <= 256:
            out[f"{key}_logits"] = logits
        else:
            out[f"{key}_logits_sha256"] = np.frombuffer(sha(logits).encode(), dtype=np.uint8)
        # grouping on the reference routing (pdscope_compare.py:583-606 contract)
        groups, cpu_idx = compact_expert_groups(r)
        generic = expert_groups(r)
        if set(groups) != {e for e, _, _ in generic}:
            raise AssertionError("reference compact/generic expert sets differ")
        experts_sorted = sorted(groups)
        counts = np.zeros(128, np.int32)
        tok_cat, w_cat = [], []
        for e in experts_sorted:
            t_e, w_e = groups[e]
            counts[e] = t_e.numel()
            tok_cat.append(t_e.numpy())
            w_cat.append(from_torch_bf16(w_e))
            g_e = [g for g in generic if g[0] == e][0]
            if not (torch.equal(g_e[1], t_e) and torch.equal(g_e[2], w_e)
                    and torch.equal(cpu_idx[e], t_e)):
                raise AssertionError("reference compact/generic order differs")
        tok_cat = np.concatenate(tok_cat).astype(np.int32)
        w_cat = np.concatenate(w_cat)
        out[f"{key}_counts"] = counts
        if tokens <= 256:
            out[f"{key}_group_tokens"] = tok_cat
            out[f"{key}_group_weights"] = w_cat
        else:
            out[f"{key}_group_tokens_sha256"] = np.frombuffer(sha(tok_cat).encode(), dtype=np.uint8)
            out[f"{key}_group_weights_sha256"] = np.frombuffer(sha(w_cat).encode(), dtype=np.uint8)

    # single-token grouping (decode path, qwen.py:159-167)
    x, gate = route_inputs(777, 1)
    r = route(to_torch_bf16(x), to_torch_bf16(gate), 8, True)
    st = expert_groups(r, mode="single_token")
    out["single_token_experts"] = np.array([e for e, _, _ in st], np.int32)
    out["single_token_weights"] = np.concatenate([from_torch_bf16(w) for _, _, w in st])
    meta["cases"]["single_token"] = dict(seed=777, tokens=1)

    # --- whole small layer: E=16, k=4, H=256, I=128, T=32 -------------------------
    seed, tokens, hidden, experts, inter, k = 4242, 32, 256, 16, 128, 4
    x, gate, wg, wu, wd = mo.synthetic_layer(seed, tokens, hidden, experts, inter)
    xt = to_torch_bf16(x)
    r = route(xt, to_torch_bf16(gate), k, True)
    groups, _ = compact_expert_groups(r, experts=experts)
    parts, parts32 = {}, {}
    for e, (t_e, _) in groups.items():
        tensors = dict(gate_proj=to_torch_bf16(wg[e]), up_proj=to_torch_bf16(wu[e]),
                       down_proj=to_torch_bf16(wd[e]))
        parts[e] = expert_forward(xt[t_e], tensors)
        parts32[e] = reference_fp32(xt[t_e], tensors)
    keep = sorted(groups)
    index = torch.cat([groups[e][0] for e in keep])
    weight = torch.cat([groups[e][1] for e in keep])[:, None]
    rows = torch.cat([parts[e] for e in keep], dim=0)
    fused = torch.zeros_like(xt)
    fused.index_add_(0, index, rows.to(fused.dtype) * weight)          # pdscope_runtime.py:461-464
    fp32 = torch.zeros(xt.shape, dtype=torch.float32)
    rows32 = torch.cat([parts32[e] for e in keep], dim=0)
    fp32.index_add_(0, index, rows32 * weight.float())                 # harness.py:86-87
    out["layer_logits"] = from_torch_bf16(r.logits)
    out["layer_selected"] = r.selected.numpy().astype(np.uint8)
    out["layer_weights"] = from_torch_bf16(r.weights)
    out["layer_rows"] = from_torch_bf16(rows)
    out["layer_rows_fp32"] = rows32.numpy()
    out["layer_fused_out"] = from_torch_bf16(fused)
    out["layer_fp32_out"] = fp32.numpy()
    meta["cases"]["layer"] = dict(seed=seed, tokens=tokens, hidden=hidden, experts=experts,
                                  inter=inter, top_k=k,
                                  inputs="oracle.moe_oracle.synthetic_layer(seed, ...)")

    np.savez_compressed(HERE / "golden_v1.npz", **out)
    (HERE / "golden_v1.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "golden_v1.npz", sum(v.nbytes for v in out.values()), "bytes raw")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
