// Routing and packing device functions (included by the unity build).
//
// route():                 expertbench/adapters/qwen.py:140-152
// compact_expert_groups(): expertbench/pdscope_runtime.py:16-39
#pragma once

#include "pdx_common.cuh"

namespace pdx {

// ---------------------------------------------------------------------------
// Softmax + top-k + renormalisation for one token, one warp.
//
// Reproduces the CUDA reference arithmetic step for step:
//  * F.softmax(logits, dtype=float32): lane l owns elements l + 32*i; the row
//    max and the sum use an xor butterfly (offsets 16..1); each lane sums its
//    own elements in i order; p = exp(x - max) / sum with IEEE division and
//    CUDA's expf (the same function the reference's kernel calls).
//  * torch.topk(p, k): the selected set is the k largest, a tie at the k
//    boundary won by the lower expert index; the returned order is that of
//    PyTorch's 32-wide bitonic sort applied to the gather order (above-k-th
//    values by index, then k-th-value ties by index), so equal values come
//    out in the network's order (behaviour pinned on the B200).
//  * w / w.sum(-1): PyTorch's small-row reduction tree (block_x_reduce) -- lane
//    j < width = last_pow2(k) holds w_j + w_{j+width}, then shfl_down by
//    1, 2, 4, ...; lane 0's total divides every weight; result RNE to BF16.
// EPL = elements per lane = max(1, next_pow2(E) / 32).
// ---------------------------------------------------------------------------
// Values form: v[i] = logit of expert lane + 32*i (-inf past E), already in registers.
template <int EPL>
__device__ __forceinline__ void warp_softmax_topk_vals(float (&v)[EPL], int E, int k, bool normalize,
                                                       int64_t* __restrict__ sel_out, uint16_t* __restrict__ w_out) {
    const uint32_t lane = lane_id();
    float m = v[0];
#pragma unroll
    for (int i = 1; i < EPL; ++i) m = fmaxf(m, v[i]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        v[i] = expf(v[i] - m);
        s += v[i];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    // probabilities (IEEE division)
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = __fdiv_rn(v[i], s);

    // top-k selection: key = float bits of p (p >= 0 -> monotone) + 1; 0 = taken
    uint32_t taken = 0;
    float my_p = 0.f;
    int my_idx = 0;
    for (int r = 0; r < k; ++r) {
        uint32_t best_key = 0;
        int best_i = 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const int idx = static_cast<int>(lane) + 32 * i;
            const uint32_t key = (idx < E && !((taken >> i) & 1u)) ? (__float_as_uint(v[i]) + 1u) : 0u;
            if (key > best_key) { best_key = key; best_i = i; }  // strict: lower i wins ties
        }
        const uint32_t win_key = __reduce_max_sync(0xffffffffu, best_key);
        const uint32_t cand = (best_key == win_key && best_key != 0u) ? lane + 32u * best_i : 0xffffffffu;
        const uint32_t win_idx = __reduce_min_sync(0xffffffffu, cand);
        const uint32_t owner = win_idx & 31u;
        const int owner_i = static_cast<int>(win_idx >> 5);
        float p_sel = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i)
            if (i == owner_i) p_sel = v[i];
        p_sel = __shfl_sync(0xffffffffu, p_sel, owner);
        if (lane == owner) taken |= 1u << owner_i;
        if (static_cast<int>(lane) == r) { my_p = p_sel; my_idx = static_cast<int>(win_idx); }
    }
    float denom = 1.f;
    if (normalize) {
        int width = 1;
        while (width * 2 <= k) width <<= 1;
        float second = __shfl_down_sync(0xffffffffu, my_p, width);
        float a = my_p;
        if (static_cast<int>(lane) + width < k) a = a + second;
        for (int off = 1; off < width; off <<= 1) a += __shfl_down_sync(0xffffffffu, a, off);
        denom = __shfl_sync(0xffffffffu, a, 0);
    }
    // No two selected probabilities equal: every correct sort gives the
    // selection order, so the bitonic ordering below is only needed with ties.
    {
        const float next_p = __shfl_down_sync(0xffffffffu, my_p, 1);
        const bool tie_here = static_cast<int>(lane) + 1 < k && next_p == my_p;
        if (!__any_sync(0xffffffffu, tie_here)) {
            if (static_cast<int>(lane) < k) {
                sel_out[lane] = my_idx;
                w_out[lane] = f2bits(normalize ? __fdiv_rn(my_p, denom) : my_p);
            }
            return;
        }
    }
    // ---- order the selection as torch.topk(sorted=True) returns it on CUDA ----
    // (1) gather order: values above the k-th largest in index order, then the
    //     values equal to it in index order;
    const float kth = __shfl_sync(0xffffffffu, my_p, k - 1);
    int g = 0;
    for (int j = 0; j < k; ++j) {
        const float pj = __shfl_sync(0xffffffffu, my_p, j);
        const int ij = __shfl_sync(0xffffffffu, my_idx, j);
        const int cj = pj == kth, cr = my_p == kth;
        if (cj < cr || (cj == cr && ij < my_idx)) ++g;
    }
    float key = 0.f;
    int val = -1;
    bool ok = false;
    for (int j = 0; j < k; ++j) {
        const int gj = __shfl_sync(0xffffffffu, g, j);
        const float pj = __shfl_sync(0xffffffffu, my_p, j);
        const int ij = __shfl_sync(0xffffffffu, my_idx, j);
        if (gj == static_cast<int>(lane)) { key = pj; val = ij; ok = true; }
    }
    // (2) PyTorch's 32-wide bitonic key/value sort (descending, unstable): one
    //     position per lane, compare-exchange of (a, a|stride) where
    //     cond = (K[a] > K[b] && valid[a]) || !valid[b], exchanged when
    //     cond == dir (dir = bit `size` of a while building, false when merging).
    if (k > 1) {
        for (int size = 2; size <= 32; size <<= 1) {
            for (int st = size >> 1; st > 0; st >>= 1) {
                const bool dir = size < 32 && ((lane & ~static_cast<uint32_t>(st)) & static_cast<uint32_t>(size)) != 0;
                const float ko = __shfl_xor_sync(0xffffffffu, key, st);
                const int vo = __shfl_xor_sync(0xffffffffu, val, st);
                const bool oko = __shfl_xor_sync(0xffffffffu, ok ? 1 : 0, st) != 0;
                const bool lower = (lane & static_cast<uint32_t>(st)) == 0;
                const float ka = lower ? key : ko, kb = lower ? ko : key;
                const bool oka = lower ? ok : oko, okb = lower ? oko : ok;
                const bool cond = (ka > kb && oka) || !okb;
                if (cond == dir) { key = ko; val = vo; ok = oko; }
            }
        }
    }
    if (static_cast<int>(lane) < k) {
        sel_out[lane] = val;
        w_out[lane] = f2bits(normalize ? __fdiv_rn(key, denom) : key);
    }
}


template <int EPL>
__device__ __forceinline__ void warp_softmax_topk(const uint16_t* __restrict__ logits_row, int E, int k,
                                                  bool normalize, int64_t* __restrict__ sel_out,
                                                  uint16_t* __restrict__ w_out) {
    const uint32_t lane = lane_id();
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int idx = static_cast<int>(lane) + 32 * i;
        v[i] = idx < E ? bits2f(logits_row[idx]) : -INFINITY;
    }
    warp_softmax_topk_vals<EPL>(v, E, k, normalize, sel_out, w_out);
}

template <int EPL>
__device__ __forceinline__ void block_topk_rows(const uint16_t* logits, int T, int E, int k, bool normalize,
                                                int64_t* selected, uint16_t* weights, int warp_begin,
                                                int warp_stride) {
    for (int t = warp_begin; t < T; t += warp_stride)
        warp_softmax_topk<EPL>(logits + static_cast<size_t>(t) * E, E, k, normalize,
                               selected + static_cast<size_t>(t) * k, weights + static_cast<size_t>(t) * k);
}

// one token by the calling warp, dispatch on E (<= 1024)
__device__ __forceinline__ void topk_row(const uint16_t* logits, int t, int E, int k, bool normalize,
                                         int64_t* selected, uint16_t* weights) {
    const uint16_t* row = logits + static_cast<size_t>(t) * E;
    int64_t* so = selected + static_cast<size_t>(t) * k;
    uint16_t* wo = weights + static_cast<size_t>(t) * k;
    if (E <= 32) warp_softmax_topk<1>(row, E, k, normalize, so, wo);
    else if (E <= 64) warp_softmax_topk<2>(row, E, k, normalize, so, wo);
    else if (E <= 128) warp_softmax_topk<4>(row, E, k, normalize, so, wo);
    else if (E <= 256) warp_softmax_topk<8>(row, E, k, normalize, so, wo);
    else if (E <= 512) warp_softmax_topk<16>(row, E, k, normalize, so, wo);
    else warp_softmax_topk<32>(row, E, k, normalize, so, wo);
}

// dispatch on E (<= 1024)
__device__ __forceinline__ void topk_rows_dispatch(const uint16_t* logits, int T, int E, int k, bool normalize,
                                                   int64_t* selected, uint16_t* weights, int warp_begin,
                                                   int warp_stride) {
    if (E <= 32)
        block_topk_rows<1>(logits, T, E, k, normalize, selected, weights, warp_begin, warp_stride);
    else if (E <= 64)
        block_topk_rows<2>(logits, T, E, k, normalize, selected, weights, warp_begin, warp_stride);
    else if (E <= 128)
        block_topk_rows<4>(logits, T, E, k, normalize, selected, weights, warp_begin, warp_stride);
    else if (E <= 256)
        block_topk_rows<8>(logits, T, E, k, normalize, selected, weights, warp_begin, warp_stride);
    else if (E <= 512)
        block_topk_rows<16>(logits, T, E, k, normalize, selected, weights, warp_begin, warp_stride);
    else
        block_topk_rows<32>(logits, T, E, k, normalize, selected, weights, warp_begin, warp_stride);
}

// ---------------------------------------------------------------------------
// Packing: stable counting sort of the slot-major flat index f = s*T + t.
// ---------------------------------------------------------------------------
struct PackOut {
    int32_t* counts;     // [E]
    int32_t* offsets;    // [E+1]
    int32_t* tokens;     // [N]
    int32_t* positions;  // [N]
    uint16_t* packed_w;  // [N]
    int32_t* inverse;    // [N]
    int32_t* active;     // [E+1]
};

__device__ __forceinline__ int flat_expert(const int64_t* selected, int T, int k, int E, int f) {
    const int t = f % T;
    const int s = f / T;
    const int64_t e = selected[static_cast<size_t>(t) * k + s];
    if (e < 0 || e >= E) {
        raise_error(PDX_DEVERR_BAD_EXPERT);
        return -1;
    }
    return static_cast<int>(e);
}

// Block histogram of flat entries [f_begin, f_end) into smem hist[E] (pre-zeroed).
__device__ __forceinline__ void block_histogram(const int64_t* selected, int T, int k, int E, int f_begin,
                                                int f_end, int* hist) {
    for (int f = f_begin + static_cast<int>(threadIdx.x); f < f_end; f += blockDim.x) {
        const int e = flat_expert(selected, T, k, E, f);
        if (e >= 0) atomicAdd(&hist[e], 1);
    }
}

// Exclusive scan of hist[0..E) by one warp (E <= 1024).  Writes excl[0..E] (excl[E]
// = total) and, when `active` is given, the ascending list of nonzero entries.
__device__ __forceinline__ void warp_exclusive_scan(const int* hist, int E, int* excl, int32_t* active_out,
                                                    int32_t* active_smem) {
    const uint32_t lane = lane_id();
    const int per = (E + 31) / 32;
    const int b = static_cast<int>(lane) * per;
    int local = 0, local_nz = 0;
    for (int i = 0; i < per; ++i)
        if (b + i < E) {
            local += hist[b + i];
            local_nz += hist[b + i] > 0;
        }
    int inc = local, inc_nz = local_nz;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, off);
        const int z = __shfl_up_sync(0xffffffffu, inc_nz, off);
        if (static_cast<int>(lane) >= off) { inc += y; inc_nz += z; }
    }
    int run = inc - local, run_nz = inc_nz - local_nz;
    for (int i = 0; i < per; ++i)
        if (b + i < E) {
            excl[b + i] = run;
            const int c = hist[b + i];
            if (c > 0) {
                if (active_out) active_out[1 + run_nz] = b + i;
                if (active_smem) active_smem[1 + run_nz] = b + i;
                ++run_nz;
            }
            run += c;
        }
    if (lane == 31) {
        excl[E] = inc;
        if (active_out) active_out[0] = inc_nz;
        if (active_smem) active_smem[0] = inc_nz;
    }
}

// Stable scatter of flat entries [f_begin, f_end) with running positions run[E]
// (smem, absolute packed row of the next entry of each expert).  warp_hist is
// smem int[NW*E].  Entries are processed in rounds of blockDim.x in flat order;
// within a round, order = (warp, lane), i.e. flat order again.
__device__ __forceinline__ void block_stable_scatter(const int64_t* selected, const uint16_t* weights, int T,
                                                     int k, int E, int f_begin, int f_end, int* run,
                                                     int* warp_hist, const PackOut& o) {
    const int tid = static_cast<int>(threadIdx.x);
    const int warp = tid >> 5;
    const int nw = static_cast<int>(blockDim.x) >> 5;
    const uint32_t lane = lane_id();
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (int base = f_begin; base < f_end; base += blockDim.x) {
        const int f = base + tid;
        const bool in_range = f < f_end;
        const int e = in_range ? flat_expert(selected, T, k, E, f) : -1;
        for (int i = tid; i < nw * E; i += blockDim.x) warp_hist[i] = 0;
        __syncthreads();
        const uint32_t peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & lt_mask);
        if (e >= 0 && rank == 0) warp_hist[warp * E + e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int before = 0;
            for (int w = 0; w < warp; ++w) before += warp_hist[w * E + e];
            const int p = run[e] + before + rank;
            const int t = f % T;
            const int s = f / T;
            const int pos = t * k + s;
            o.tokens[p] = t;
            o.positions[p] = pos;
            o.packed_w[p] = weights[pos];
            o.inverse[pos] = p;
        }
        __syncthreads();
        for (int e2 = tid; e2 < E; e2 += blockDim.x) {
            int add = 0;
            for (int w = 0; w < nw; ++w) add += warp_hist[w * E + e2];
            run[e2] += add;
        }
        __syncthreads();
    }
}

// Whole pack by one block (N = T*k <= kPackSmemMax), from shared memory: the
// routing is read from global memory once (one coalesced pass) into s_ids /
// s_w (by position t*k + s), then histogram, scan and the stable scatter run
// on shared memory, so the only global accesses on the block's critical path
// are that load and the output stores (a single CTA walking dependent L2
// reads is what makes a pack slow).  smem: hist[E], excl[E+1], warp_hist[NW*E],
// s_ids[N] ints, s_w[N] shorts.
constexpr int kPackSmemMax = 2048;
__device__ __forceinline__ void block_pack_all(const int64_t* selected, const uint16_t* weights, int T, int k,
                                               int E, int* hist, int* excl, int* warp_hist, const PackOut& o) {
    const int N = T * k;
    int* s_ids = warp_hist + (static_cast<int>(blockDim.x) >> 5) * E;
    uint16_t* s_w = reinterpret_cast<uint16_t*>(s_ids + N);
    for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
    for (int p = threadIdx.x; p < N; p += blockDim.x) {
        const int64_t e = selected[p];
        int v = static_cast<int>(e);
        if (e < 0 || e >= E) {
            raise_error(PDX_DEVERR_BAD_EXPERT);
            v = -1;
        }
        s_ids[p] = v;
        s_w[p] = weights[p];
    }
    __syncthreads();
    for (int f = threadIdx.x; f < N; f += blockDim.x) {
        const int e = s_ids[(f % T) * k + f / T];
        if (e >= 0) atomicAdd(&hist[e], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) warp_exclusive_scan(hist, E, excl, o.active, nullptr);
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        o.counts[i] = hist[i];
        o.offsets[i] = excl[i];
    }
    if (threadIdx.x == 0) o.offsets[E] = excl[E];
    __syncthreads();
    // stable scatter in flat order f = s*T + t (rounds of blockDim.x entries;
    // within a round the (warp, lane) order is the flat order)
    const int tid = static_cast<int>(threadIdx.x);
    const int warp = tid >> 5;
    const int nw = static_cast<int>(blockDim.x) >> 5;
    const uint32_t lane = lane_id();
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (int base = 0; base < N; base += blockDim.x) {
        const int f = base + tid;
        const int t = f % T, s = f / T;
        const int pos = t * k + s;
        const int e = f < N ? s_ids[pos] : -1;
        for (int i = tid; i < nw * E; i += blockDim.x) warp_hist[i] = 0;
        __syncthreads();
        const uint32_t peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & lt_mask);
        if (e >= 0 && rank == 0) warp_hist[warp * E + e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int before = 0;
            for (int w = 0; w < warp; ++w) before += warp_hist[w * E + e];
            const int p = excl[e] + before + rank;
            o.tokens[p] = t;
            o.positions[p] = pos;
            o.packed_w[p] = s_w[pos];
            o.inverse[pos] = p;
        }
        __syncthreads();
        for (int e2 = tid; e2 < E; e2 += blockDim.x) {
            int add = 0;
            for (int w = 0; w < nw; ++w) add += warp_hist[w * E + e2];
            excl[e2] += add;
        }
        __syncthreads();
    }
}

// Whole pack by one warp for N = T*k <= 32 entries (lane = flat index f, so
// lane order is the stable order): match_any groups the lanes of one expert,
// the group's first lane writes its count, one warp scan gives the segment
// starts, and lane f's packed row is start + its rank in the group -- the
// same outputs as block_pack_all without its block-wide barriers.  smem:
// hist[E], excl[E+1] ints.
__device__ __forceinline__ void warp_pack_small(const int64_t* selected, const uint16_t* weights, int T, int k,
                                                int E, int* hist, int* excl, const PackOut& o) {
    const int lane = static_cast<int>(lane_id());
    const int N = T * k;
    for (int i = lane; i < E; i += 32) hist[i] = 0;
    int e = -1, t = 0, pos = 0;
    if (lane < N) {
        t = lane % T;
        pos = t * k + lane / T;
        const int64_t v = selected[pos];
        if (v < 0 || v >= E) raise_error(PDX_DEVERR_BAD_EXPERT);
        else e = static_cast<int>(v);
    }
    __syncwarp();
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) hist[e] = __popc(peers);
    __syncwarp();
    warp_exclusive_scan(hist, E, excl, o.active, nullptr);
    __syncwarp();
    for (int i = lane; i < E; i += 32) {
        o.counts[i] = hist[i];
        o.offsets[i] = excl[i];
    }
    if (lane == 0) o.offsets[E] = excl[E];
    if (e >= 0) {
        const int p = excl[e] + rank;
        o.tokens[p] = t;
        o.positions[p] = pos;
        o.packed_w[p] = weights[pos];
        o.inverse[pos] = p;
    }
}

// Shared memory of block_pack_all, in ints, for N = T*k entries and `warps` warps.
__host__ __device__ constexpr size_t block_pack_smem_ints(int64_t E, int64_t N, int warps) {
    return static_cast<size_t>(E + E + 1 + warps * E + N + (N + 1) / 2);
}

}  // namespace pdx
