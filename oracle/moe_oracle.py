"""CPU oracle for the PDScope per-layer MoE expert path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of the reference's hot path so
that the CUDA kernels in ``pdscope_b200`` can be checked against it.  It is
imported only by ``tests/``, by ``__graft_entry__.smoke()`` and by the
``cpu_baseline`` leg of ``bench.py``; it is never part of the product path.

Reference functions restated here (paths inside nezha-Anonymous/PDScope):

* ``route``                 expertbench/adapters/qwen.py:140-152
* ``expert_groups``         expertbench/adapters/qwen.py:155-174
* ``compact_expert_groups`` expertbench/pdscope_runtime.py:16-39
* ``expert_forward``        expertbench/adapters/qwen.py:87-90
* ``reference_fp32``        expertbench/adapters/qwen.py:93-98
* fused merge               expertbench/pdscope_runtime.py:454-464
* ``error_metrics``         benchmarks/harness.py:33-42

BF16 tensors are carried as ``uint16`` arrays of raw bits.

Rounding contract (why each step is written the way it is):

* Router logits.  The reference computes ``F.linear(x, gate)`` in BF16, i.e. an
  FP32-accumulated dot product rounded once to BF16; the accumulation order is
  whatever cuBLAS picks and is not part of the contract.  The oracle takes the
  mathematically exact dot product (FP64 accumulation of exact BF16xBF16
  products) rounded once to BF16 with round-to-nearest-even.  The CUDA kernel
  does the same, so both agree bit for bit; cuBLAS differs from both by one
  BF16 ulp on a small fraction of logits (measured and reported by the GPU
  tests, never hidden).
* Softmax.  ``F.softmax(logits, dim=-1, dtype=float32)`` on CUDA runs PyTorch's
  warp-per-row softmax: lane ``l`` holds elements ``l + 32*i``, sums them in
  ``i`` order, then an xor-butterfly over offsets 16, 8, 4, 2, 1; each
  probability is ``exp(x - max) / sum`` in FP32.  The oracle reproduces that
  order exactly; only ``exp`` itself comes from numpy instead of CUDA's
  ``expf`` (both are within 2 ulp, so the BF16 routing weights can differ by
  one BF16 ulp in rare cases).
* Top-k.  ``torch.topk`` on CUDA selects by value descending, lower expert
  index winning a tie at the k boundary, and orders the selection with
  PyTorch's unstable 32-wide bitonic sort, so equal values come out in that
  network's order (pinned on the B200).  The oracle restates both steps
  (``topk_torch_cuda``).
* Renormalisation.  ``weights.sum(-1)`` over k FP32 values uses PyTorch's
  reduction tree (``block_x_reduce``: lanes of width ``last_pow2(k)``, each
  lane summing its strided elements, then shfl_down with offsets 1, 2, 4 ...).
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------
# BF16 <-> float helpers (IEEE-754 binary32 truncated to 16 bits)
# ----------------------------------------------------------------------------


def bf16_to_f32(bits):
    """Raw BF16 bits (uint16) -> float32, exact."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """float32 -> BF16 bits, round to nearest even (NaN -> canonical qNaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = 0x7FC0
    return rounded


def f64_to_bf16(x):
    """float64 -> BF16 bits with a single round-to-nearest-even step.

    Rounds directly at BF16's 8-bit significand (no intermediate float32
    rounding, so no double rounding).  Subnormal results use the fixed BF16
    subnormal spacing 2**-133; results beyond the BF16 range become +-inf.
    """
    x = np.asarray(x, dtype=np.float64)
    _, e = np.frexp(x)
    e = np.maximum(e.astype(np.int64) - 1, -126)
    ulp = np.ldexp(1.0, (e - 7).astype(np.int32))
    with np.errstate(over="ignore", invalid="ignore"):
        q = np.rint(x / ulp) * ulp
        f = q.astype(np.float32)
    return (np.ascontiguousarray(f).view(np.uint32) >> 16).astype(np.uint16)


def bf16_round(x):
    """float32 array -> float32 array holding the BF16-rounded values."""
    return bf16_to_f32(f32_to_bf16(x))


# ----------------------------------------------------------------------------
# a1: route  (expertbench/adapters/qwen.py:140-152)
# ----------------------------------------------------------------------------


def router_logits(x_bits, gate_bits):
    """BF16 logits = RNE_bf16(exact x . gate^T); [T,H] x [E,H] -> [T,E] bits."""
    x = bf16_to_f32(x_bits).astype(np.float64)
    g = bf16_to_f32(gate_bits).astype(np.float64)
    return f64_to_bf16(x @ g.T)


def _next_pow2(n):
    p = 1
    while p < n:
        p <<= 1
    return p


def _last_pow2(n):
    p = 1
    while p * 2 <= n:
        p <<= 1
    return p


def softmax_fp32(logit_bits):
    """F.softmax(logits, dim=-1, dtype=float32) in PyTorch's CUDA warp order."""
    l32 = bf16_to_f32(logit_bits)
    t_count, e_count = l32.shape
    width = _next_pow2(e_count)
    lanes = min(width, 32)
    iters = width // lanes
    padded = np.full((t_count, width), -np.inf, dtype=np.float32)
    padded[:, :e_count] = l32
    # element index = lane + it * lanes  ->  view [T, iters, lanes]
    grid = padded.reshape(t_count, iters, lanes)
    row_max = grid.max(axis=(1, 2)).astype(np.float32)
    with np.errstate(invalid="ignore"):
        ex = np.exp((grid - row_max[:, None, None]).astype(np.float32)).astype(np.float32)
    lane_sum = np.zeros((t_count, lanes), dtype=np.float32)
    for it in range(iters):
        lane_sum = (lane_sum + ex[:, it, :]).astype(np.float32)
    lane_idx = np.arange(lanes)
    offset = lanes // 2
    while offset > 0:
        lane_sum = (lane_sum + lane_sum[:, lane_idx ^ offset]).astype(np.float32)
        offset //= 2
    total = lane_sum[:, :1]
    probs = (ex.reshape(t_count, width) / total).astype(np.float32)
    return probs[:, :e_count]


def _bitonic32_desc(keys, vals):
    """PyTorch's small bitonic key/value sort (sort size 32, descending, GT
    comparator, unstable), as used by torch.topk(sorted=True) for k <= 32.

    ``keys`` [T, n] float32 and ``vals`` [T, n] int64 in gather order, n <= 32;
    positions >= n are invalid and always sort to the end.  Compare-exchange of
    (a, b = a | stride): cond = (K[a] > K[b] and valid[a]) or not valid[b];
    exchange when cond == dir, dir = bit `size` of a while building bitonic
    runs, False in the final merge.
    """
    t_count, n = keys.shape
    size = 32
    K = np.zeros((t_count, size), np.float32)
    V = np.full((t_count, size), -1, np.int64)
    ok = np.zeros((t_count, size), bool)
    K[:, :n], V[:, :n], ok[:, :n] = keys, vals, True
    pos = np.arange(size)

    def step(stride, dirs):
        a = pos[(pos & stride) == 0]
        b = a | stride
        cond = ((K[:, a] > K[:, b]) & ok[:, a]) | ~ok[:, b]
        do = cond == dirs[None, :]
        for arr in (K, V, ok):
            xa, xb = arr[:, a].copy(), arr[:, b].copy()
            arr[:, a] = np.where(do, xb, xa)
            arr[:, b] = np.where(do, xa, xb)

    s = 2
    while s < size:
        stride = s // 2
        while stride > 0:
            a = pos[(pos & stride) == 0]
            step(stride, (a & s) != 0)
            stride //= 2
        s *= 2
    stride = size // 2
    while stride > 0:
        step(stride, np.zeros(size // 2, bool))
        stride //= 2
    return K[:, :n], V[:, :n]


def topk_torch_cuda(values, k):
    """torch.topk(values, k) (sorted) as it runs on CUDA, restated.

    1. Selection (gatherTopK): every value strictly above the k-th largest, in
       index order, then values equal to the k-th largest in index order until
       k are taken -- so a tie at the k boundary is won by the lower index.
    2. Order: PyTorch's 32-wide bitonic sort (descending, unstable) of that
       gather order; equal values come out in the network's order, e.g.
       [.1,.5,.3,.5,.3,.5,.2,.3], k=5 -> [5,3,1,4,2] (pinned on the B200).
    """
    if k > 32:
        raise ValueError("the restated bitonic order covers k <= 32")
    t_count, e_count = values.shape
    idx = np.broadcast_to(np.arange(e_count), values.shape)
    chosen = np.lexsort((idx, -values.astype(np.float64)), axis=-1)[:, :k]
    cv = np.take_along_axis(values, chosen, axis=1).astype(np.float32)
    kth = cv[:, -1:]
    gather = np.lexsort((chosen, (cv == kth).astype(np.int8)), axis=-1)
    g_idx = np.take_along_axis(chosen, gather, axis=1).astype(np.int64)
    g_val = np.take_along_axis(cv, gather, axis=1)
    if k == 1:
        return g_val, g_idx
    vals, sel = _bitonic32_desc(g_val, g_idx)
    return vals, sel


def torch_sum_lastdim(v):
    """weights.sum(dim=-1) for a small FP32 row, in PyTorch's reduction tree."""
    t_count, k = v.shape
    width = min(_last_pow2(k), 32)
    vt0 = 4
    lanes = np.zeros((t_count, width), dtype=np.float32)
    for lane in range(width):
        acc = [np.zeros(t_count, dtype=np.float32) for _ in range(vt0)]
        elems = list(range(lane, k, width))
        pos = 0
        while pos + vt0 <= len(elems):
            for i in range(vt0):
                acc[i] = (acc[i] + v[:, elems[pos + i]]).astype(np.float32)
            pos += vt0
        for i, e in enumerate(elems[pos:]):
            acc[i] = (acc[i] + v[:, e]).astype(np.float32)
        total = acc[0]
        for i in range(1, vt0):
            total = (total + acc[i]).astype(np.float32)
        lanes[:, lane] = total
    offset = 1
    while offset < width:
        shifted = np.zeros_like(lanes)
        shifted[:, : width - offset] = lanes[:, offset:]
        lanes = (lanes + shifted).astype(np.float32)
        offset <<= 1
    return lanes[:, 0]


def route_from_logits(logit_bits, top_k, normalize):
    """Softmax, top-k and optional renormalisation; returns (ids int64, w bf16 bits)."""
    if not 0 < top_k <= logit_bits.shape[1]:
        raise ValueError("invalid routing parameters")
    probs = softmax_fp32(logit_bits)
    weights, selected = topk_torch_cuda(probs, top_k)
    if normalize:
        denom = torch_sum_lastdim(weights)
        weights = (weights / denom[:, None]).astype(np.float32)
    return selected, f32_to_bf16(weights)


def route(x_bits, gate_bits, top_k, normalize):
    """qwen.route restated: returns (logits bits, selected int64, weights bits)."""
    if x_bits.ndim != 2 or x_bits.shape[1] != gate_bits.shape[1]:
        raise ValueError("router input shape/dtype mismatch")
    logits = router_logits(x_bits, gate_bits)
    selected, weights = route_from_logits(logits, top_k, normalize)
    return logits, selected, weights


# ----------------------------------------------------------------------------
# a2 / a3: grouping  (qwen.py:155-174, pdscope_runtime.py:16-39)
# ----------------------------------------------------------------------------


def compact_expert_groups(selected, weight_bits, experts=128):
    """Stable slot-major counting sort of the routed (token, slot) pairs.

    Returns a dict with the packed layout used by the CUDA path:
      counts[E] int32, offsets[E+1] int32 (exclusive prefix),
      tokens[T*k] int32  (order % T       -- pdscope_runtime.py:29),
      positions[T*k] int32 (t*k + order//T -- pdscope_runtime.py:29),
      weights[T*k] bf16 bits (weights.reshape(-1)[positions] -- :31),
      inverse[T*k] int32 (inverse[t*k+s] = packed row of assignment (t, s)).
    """
    n, k = selected.shape
    if n < 1 or k < 1:
        raise ValueError("empty expert routing")
    flat = np.ascontiguousarray(selected.T).reshape(-1)
    if flat.min() < 0 or flat.max() >= experts:
        raise ValueError("expert ID outside configured range")
    counts = np.bincount(flat, minlength=experts).astype(np.int32)
    order = np.argsort(flat, kind="stable")
    tokens = (order % n).astype(np.int32)
    positions = (tokens.astype(np.int64) * k + order // n).astype(np.int32)
    weights = np.asarray(weight_bits).reshape(-1)[positions]
    offsets = np.zeros(experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    inverse = np.empty(n * k, dtype=np.int32)
    inverse[positions] = np.arange(n * k, dtype=np.int32)
    return dict(counts=counts, offsets=offsets, tokens=tokens, positions=positions,
                weights=weights, inverse=inverse)


def expert_groups(selected, weight_bits):
    """Generic per-expert (expert, tokens, weights) list in native order.

    Same order as ``torch.where((selected == e).T)``: slot-major, then token.
    """
    groups = []
    for expert in sorted(set(selected.reshape(-1).tolist())):
        slots, tokens = np.nonzero((selected == expert).T)
        groups.append((expert, tokens.astype(np.int64), weight_bits[tokens, slots]))
    return groups


def expert_groups_single_token(selected, weight_bits):
    """qwen.expert_groups(mode='single_token'): one token, sorted by expert id."""
    if selected.shape[0] != 1:
        raise ValueError("single-token grouping requires exactly one token")
    ids = selected[0].tolist()
    if len(set(ids)) != len(ids):
        raise ValueError("single-token grouping requires distinct selected expert IDs")
    return [(e, np.zeros(1, np.int64), weight_bits[0, s:s + 1])
            for s, e in sorted(enumerate(ids), key=lambda p: p[1])]


# ----------------------------------------------------------------------------
# a5: expert FFN  (qwen.py:87-98)
# ----------------------------------------------------------------------------


def expert_forward(x_bits, gate_bits, up_bits, down_bits):
    """F.linear(silu(F.linear(x,Wg)) * F.linear(x,Wu), Wd) with BF16 roundings.

    Each F.linear rounds its FP32 accumulation once to BF16; SiLU is computed
    in FP32 from the BF16 gate and rounded; the product of two BF16 tensors is
    rounded; the down projection rounds once.  Returns BF16 bits [n, H].
    """
    x = bf16_to_f32(x_bits)
    g = bf16_round(x @ bf16_to_f32(gate_bits).T)
    u = bf16_round(x @ bf16_to_f32(up_bits).T)
    s = bf16_round(g / (np.float32(1) + np.exp(-g)))
    h = bf16_round(s * u)
    return f32_to_bf16(h @ bf16_to_f32(down_bits).T)


def reference_fp32(x_bits, gate_bits, up_bits, down_bits):
    """qwen.reference_fp32: all-FP32 SwiGLU, float32 result [n, H]."""
    x = bf16_to_f32(x_bits).astype(np.float64)
    g = x @ bf16_to_f32(gate_bits).astype(np.float64).T
    u = x @ bf16_to_f32(up_bits).astype(np.float64).T
    h = (g / (1.0 + np.exp(-g))) * u
    return (h @ bf16_to_f32(down_bits).astype(np.float64).T).astype(np.float32)


# ----------------------------------------------------------------------------
# a7: combine  (pdscope_runtime.py:454-464)
# ----------------------------------------------------------------------------


def combine(rows_bits, packed, n_tokens, k):
    """Deterministic fused merge used by the CUDA path.

    out[t] = RNE_bf16( sum_s  float(bf16(y[inverse[t*k+s]] * w[t,s])) ), the
    per-row BF16 product matching ``rows.to(bf16) * weight`` (:464) and the sum
    accumulated in FP32 over slots s = 0..k-1 with one final rounding.
    """
    y = bf16_to_f32(rows_bits)
    w = bf16_to_f32(packed["weights"])  # in packed order
    prod = bf16_round(y * w[:, None])
    inv = packed["inverse"].reshape(n_tokens, k)
    acc = np.zeros((n_tokens, y.shape[1]), dtype=np.float32)
    for s in range(k):
        acc = (acc + prod[inv[:, s]]).astype(np.float32)
    return f32_to_bf16(acc)


def combine_reference_order(rows_bits, packed, n_tokens):
    """The reference's own merge as ``index_add_`` computes it on CPU.

    ``output.index_add_(0, index, rows.to(bf16) * weight)`` (:461-464): the
    per-row product is a BF16 multiply; CPU ``index_add_`` on BF16 then
    accumulates in FP32 in packed-row order and rounds once (verified against
    the golden fixture bit for bit).  On CUDA the same call uses BF16 atomics
    whose order is not fixed, so only tolerance-level agreement is defined
    there.
    """
    y = bf16_to_f32(rows_bits)
    w = bf16_to_f32(packed["weights"])
    prod = bf16_round(y * w[:, None])
    acc = np.zeros((n_tokens, y.shape[1]), dtype=np.float32)
    for row, tok in enumerate(packed["tokens"]):
        acc[tok] = (acc[tok] + prod[row]).astype(np.float32)
    return f32_to_bf16(acc)


def combine_fp32(rows_f32, packed, n_tokens):
    """FP32 merge of FP32 rows (harness.py:86-87 style), for relative-L2 checks."""
    w = bf16_to_f32(packed["weights"])
    out = np.zeros((n_tokens, rows_f32.shape[1]), dtype=np.float64)
    np.add.at(out, packed["tokens"], rows_f32.astype(np.float64) * w[:, None])
    return out.astype(np.float32)


# ----------------------------------------------------------------------------
# Whole layer
# ----------------------------------------------------------------------------


def moe_layer(x_bits, gate_bits, w_gate, w_up, w_down, top_k=8, normalize=True):
    """route -> compact grouping -> per-expert FFN -> deterministic combine.

    ``w_gate``/``w_up`` are [E, I, H] and ``w_down`` [E, H, I] BF16 bits.
    Returns (out bits [T,H], logits, selected, weights, packed, rows bits).
    """
    n, _ = x_bits.shape
    experts = gate_bits.shape[0]
    logits, selected, weights = route(x_bits, gate_bits, top_k, normalize)
    packed = compact_expert_groups(selected, weights, experts)
    rows = np.zeros((n * top_k, x_bits.shape[1]), dtype=np.uint16)
    off = packed["offsets"]
    for e in range(experts):
        a, b = off[e], off[e + 1]
        if a == b:
            continue
        rows[a:b] = expert_forward(x_bits[packed["tokens"][a:b]], w_gate[e], w_up[e], w_down[e])
    out = combine(rows, packed, n, top_k)
    return out, logits, selected, weights, packed, rows


def moe_layer_fp32(x_bits, selected, weight_bits, w_gate, w_up, w_down):
    """FP32 layer reference on fixed routing (harness.py:86-87)."""
    n, k = selected.shape
    packed = compact_expert_groups(selected, weight_bits, w_gate.shape[0])
    rows = np.zeros((n * k, x_bits.shape[1]), dtype=np.float32)
    off = packed["offsets"]
    for e in range(w_gate.shape[0]):
        a, b = off[e], off[e + 1]
        if a != b:
            rows[a:b] = reference_fp32(x_bits[packed["tokens"][a:b]], w_gate[e], w_up[e], w_down[e])
    return combine_fp32(rows, packed, n)


def error_metrics(actual, reference):
    """benchmarks/harness.py:33-42 restated on float arrays."""
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    r = np.asarray(reference, dtype=np.float64).reshape(-1)
    delta = a - r
    norm = float(np.linalg.norm(r))
    rms = float(np.sqrt(np.mean(r * r))) if r.size else 0.0
    return dict(relative_l2=float(np.linalg.norm(delta)) / max(norm, 1e-12),
                max_abs_over_reference_rms=float(np.abs(delta).max()) / max(rms, 1e-12) if r.size else 0.0,
                max_abs=float(np.abs(delta).max()) if r.size else 0.0, reference_rms=rms,
                finite=bool(np.isfinite(a).all() and np.isfinite(r).all()))


# ----------------------------------------------------------------------------
# Seeded synthetic inputs (weights ~N(0,0.02), x ~N(0,1))
# ----------------------------------------------------------------------------


def synthetic_layer(seed, tokens, hidden, experts, inter, weight_std=0.02):
    """Deterministic numpy inputs for one layer (BF16 bits)."""
    rng = np.random.default_rng(seed)
    x = f32_to_bf16(rng.standard_normal((tokens, hidden), dtype=np.float32))
    gate = f32_to_bf16(rng.standard_normal((experts, hidden), dtype=np.float32) * weight_std)
    wg = f32_to_bf16(rng.standard_normal((experts, inter, hidden), dtype=np.float32) * weight_std)
    wu = f32_to_bf16(rng.standard_normal((experts, inter, hidden), dtype=np.float32) * weight_std)
    wd = f32_to_bf16(rng.standard_normal((experts, hidden, inter), dtype=np.float32) * weight_std)
    return x, gate, wg, wu, wd


def synthetic_router(seed, tokens, hidden=2048, experts=128):
    """Seeded (x, gate) BF16 bits for routing cases: gate ~N(0,0.02), x ~N(0,1)."""
    rng = np.random.default_rng(seed)
    gate = f32_to_bf16(rng.standard_normal((experts, hidden), dtype=np.float32) * 0.02)
    x = f32_to_bf16(rng.standard_normal((tokens, hidden), dtype=np.float32))
    return x, gate


def tie_free_rows(logit_bits, top_k):
    """Rows whose top-(k+1) logits are pairwise distinct (tie order irrelevant)."""
    l32 = bf16_to_f32(logit_bits)
    top = -np.sort(-l32, axis=1)[:, : top_k + 1]
    return ~(np.diff(top, axis=1) == 0).any(axis=1)
