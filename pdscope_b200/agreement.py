"""Routing agreement between ``pdx_route_topk`` and the reference's own route
run on the same device.

The reference routes with ``F.linear`` (cuBLAS, FP32 accumulation in an
unspecified order, one BF16 rounding), an FP32 softmax, ``torch.topk`` and a
renormalisation (expertbench/adapters/qwen.py:147-152).  The kernels here
compute the exact dot products and round once.  An FP32 accumulation of H
products is within gamma_H * sum|x_h g_h| (gamma_H ~ H * 2^-24) of the exact
sum, so after both are rounded to BF16 they differ by at most that bound plus
one BF16 ulp.  Ids can then differ only where two candidates of a row are
within their two error bounds of each other.  ``route_agreement`` measures
this on given inputs: full-row id equality, set equality, whether every logit
difference stays inside the bound, and for every row whose ids differ
whether the first two experts the routings order differently are such a
near-tie on the exact logits.

This is a measurement aid for benchmarks and tests; nothing on the product
path calls it.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def device_reference_route(x, gate, top_k, normalize):
    """The body of the reference's route() (qwen.py:147-152) with torch on x's device."""
    logits = F.linear(x, gate)
    probs = F.softmax(logits, dim=-1, dtype=torch.float32)
    w, sel = torch.topk(probs, top_k, dim=-1)
    if normalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return logits, sel, w.to(x.dtype)


def _bf16_ulp(v):
    """Spacing of BF16 values at |v| (8 significant bits)."""
    m = v.abs().clamp_min(torch.finfo(torch.float32).tiny)
    _, e = torch.frexp(m)
    return torch.ldexp(torch.ones_like(m), (e - 8).to(torch.int32))


def route_agreement(x, gate, top_k=8, normalize=True):
    """Compare pdx routing with the reference's device routing on (x, gate)."""
    from .runtime import route
    r = route(x, gate, top_k, normalize)
    t_logits, t_sel, t_w = device_reference_route(x, gate, top_k, normalize)
    ours, theirs = r.selected, t_sel
    ids_equal = (ours == theirs).all(dim=1)
    sets_equal = (ours.sort(dim=1).values == theirs.sort(dim=1).values).all(dim=1)
    lo, lt = r.logits.float(), t_logits.float()
    hidden = x.shape[1]
    # error bound of an FP32-accumulated BF16 logit against the exact one
    abs_sum = x.float().abs() @ gate.float().abs().T
    err = hidden * 2.0 ** -24 * abs_sum + _bf16_ulp(torch.maximum(lo.abs(), lt.abs()))
    within = bool(((lo - lt).abs() <= err).all())
    diff_ulps = (lo - lt).abs() / _bf16_ulp(torch.maximum(lo.abs(), lt.abs()))
    logit_rows = (lo != lt).any(dim=1)
    same_logit_rows = ~logit_rows
    weights_equal = bool(torch.equal(r.weights[same_logit_rows], t_w[same_logit_rows]))
    ids_on_same_logits = bool(torch.equal(ours[same_logit_rows], theirs[same_logit_rows]))
    bad = (~ids_equal).nonzero().flatten()
    gaps, near = [], []
    if bad.numel():
        o, t = ours[bad], theirs[bad]
        first = (o != t).int().argmax(dim=1)
        a = o.gather(1, first[:, None]).squeeze(1)
        b = t.gather(1, first[:, None]).squeeze(1)
        la = lo[bad].gather(1, a[:, None]).squeeze(1)
        lb = lo[bad].gather(1, b[:, None]).squeeze(1)
        ea = err[bad].gather(1, a[:, None]).squeeze(1)
        eb = err[bad].gather(1, b[:, None]).squeeze(1)
        gap = (la - lb).abs()
        gaps = (gap / _bf16_ulp(torch.maximum(la.abs(), lb.abs()))).tolist()
        near = (gap <= ea + eb).tolist()
    rows = int(x.shape[0])
    return dict(rows=rows, ids_equal=int(ids_equal.sum()), sets_equal=int(sets_equal.sum()),
                ids_equal_frac=float(ids_equal.float().mean()),
                rows_with_logit_diff=int(logit_rows.sum()),
                logit_elements_differ_frac=float((lo != lt).float().mean()),
                max_logit_diff_ulps=float(diff_ulps.max()) if diff_ulps.numel() else 0.0,
                logit_diffs_within_fp32_bound=within,
                differing_rows=len(gaps), max_gap_ulps_of_differing=max(gaps) if gaps else 0.0,
                all_differing_rows_near_ties=all(near),
                ids_equal_where_logits_equal=ids_on_same_logits,
                weights_equal_where_logits_equal=weights_equal)
