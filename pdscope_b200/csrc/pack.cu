// Packing kernels: stable counting sort of routed (token, slot) pairs.
//
// Reference: compact_expert_groups() -- expertbench/pdscope_runtime.py:16-39
// (flat = selected.T.flatten(); counts = bincount; order = argsort(stable);
// tokens = order % T; positions = tokens*k + order//T; weights[positions]).
#include "routing.cuh"

namespace pdx {

constexpr int kPackThreads = 256;
constexpr int kPackChunk = 4096;     // largest chunk (flat entries per CTA) of the multi-CTA path
constexpr int kPackMinChunk = 256;   // one scatter round of kPackThreads entries
// chunk_hist is staged in shared memory by k_pack_scan up to this many ints
constexpr int kPackScanSmemInts = 40 * 1024;

// One CTA packs everything (N = T*k up to a few thousand entries).
// dynamic smem: hist[E] + excl[E+1] + warp_hist[8*E] ints.
__global__ void __launch_bounds__(kPackThreads) k_pack_single(const int64_t* __restrict__ selected,
                                                              const uint16_t* __restrict__ weights, int T, int k,
                                                              int E, PackOut o) {
    griddep_wait();
    griddep_launch();
    extern __shared__ int smem_i[];
    int* hist = smem_i;
    int* excl = hist + E;
    int* warp_hist = excl + E + 1;
    block_pack_all(selected, weights, T, k, E, hist, excl, warp_hist, o);
}

// Phase 1: per-chunk histograms -> chunk_hist[c*E + e] (chunk = flat entries per CTA).
__global__ void __launch_bounds__(kPackThreads) k_pack_hist(const int64_t* __restrict__ selected, int T, int k,
                                                            int E, int chunk, int* __restrict__ chunk_hist) {
    extern __shared__ int smem_i[];
    int* hist = smem_i;
    for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int N = T * k;
    const int f0 = static_cast<int>(blockIdx.x) * chunk;
    const int f1 = min(N, f0 + chunk);
    block_histogram(selected, T, k, E, f0, f1, hist);
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) chunk_hist[static_cast<size_t>(blockIdx.x) * E + i] = hist[i];
}

// Phase 2 (one CTA; the path for histograms too large for k_pack_scan_scatter's
// shared memory): counts, offsets, active list and per-chunk bases
// chunk_base[c*E + e] = offsets[e] + sum_{c' < c} chunk_hist[c'*E + e].
// dynamic smem: tot[E] + excl[E+1] ints.
__global__ void __launch_bounds__(kPackThreads) k_pack_scan(int* __restrict__ chunk_hist, int chunks, int E,
                                                            PackOut o) {
    extern __shared__ int smem_i[];
    int* tot = smem_i;
    int* excl = tot + E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = 0;
        for (int c = 0; c < chunks; ++c) {
            const int v = chunk_hist[static_cast<size_t>(c) * E + e];
            chunk_hist[static_cast<size_t>(c) * E + e] = run;  // becomes the chunk-relative base
            run += v;
        }
        tot[e] = run;
    }
    __syncthreads();
    if (threadIdx.x < 32) warp_exclusive_scan(tot, E, excl, o.active, nullptr);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        o.counts[e] = tot[e];
        o.offsets[e] = excl[e];
    }
    if (threadIdx.x == 0) o.offsets[E] = excl[E];
    const int n = chunks * E;
    for (int i = threadIdx.x; i < n; i += blockDim.x) chunk_hist[i] += excl[i % E];
}

// Phases 2 + 3 in one kernel when every chunk histogram fits in shared memory
// (chunks*E <= kPackScanSmemInts): each CTA stages all histograms, derives its
// own chunk base (offsets[e] + the counts of expert e in earlier chunks) and
// scatters its chunk; CTA 0 also writes counts, offsets and the active list.
// dynamic smem: h[chunks*E] + tot[E] + excl[E+1] + run[E] + warp_hist[8*E] ints.
__global__ void __launch_bounds__(kPackThreads) k_pack_scan_scatter(const int64_t* __restrict__ selected,
                                                                    const uint16_t* __restrict__ weights, int T,
                                                                    int k, int E, int chunk, int chunks,
                                                                    const int* __restrict__ chunk_hist, PackOut o) {
    extern __shared__ int smem_i[];
    int* __restrict__ h = smem_i;
    int* __restrict__ tot = h + chunks * E;
    int* __restrict__ excl = tot + E;
    int* __restrict__ run = excl + E + 1;
    int* __restrict__ warp_hist = run + E;
    const int n = chunks * E;
    {   // staging: 16-byte loads, eight in flight per thread before their stores
        // (chunk_hist is 16-byte aligned: it starts a workspace allocation)
        const int n4 = n / 4;
        const int4* src = reinterpret_cast<const int4*>(chunk_hist);
        int4* dst = reinterpret_cast<int4*>(h);
        for (int base = 0; base < n4; base += 8 * kPackThreads) {
            int4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = base + j * kPackThreads + static_cast<int>(threadIdx.x);
                if (i < n4) v[j] = __ldg(src + i);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = base + j * kPackThreads + static_cast<int>(threadIdx.x);
                if (i < n4) dst[i] = v[j];
            }
        }
        for (int i = 4 * n4 + static_cast<int>(threadIdx.x); i < n; i += blockDim.x) h[i] = chunk_hist[i];
    }
    __syncthreads();
    const int me = static_cast<int>(blockIdx.x);
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int before = 0, after = 0;
        for (int c = 0; c < me; ++c) before += h[c * E + e];
        for (int c = me; c < chunks; ++c) after += h[c * E + e];
        tot[e] = before + after;
        run[e] = before;
    }
    __syncthreads();
    if (threadIdx.x < 32) warp_exclusive_scan(tot, E, excl, me == 0 ? o.active : nullptr, nullptr);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        run[e] += excl[e];
        if (me == 0) {
            o.counts[e] = tot[e];
            o.offsets[e] = excl[e];
        }
    }
    if (me == 0 && threadIdx.x == 0) o.offsets[E] = excl[E];
    __syncthreads();
    const int N = T * k;
    const int f0 = me * chunk;
    const int f1 = min(N, f0 + chunk);
    block_stable_scatter(selected, weights, T, k, E, f0, f1, run, warp_hist, o);
}

// Phase 3: stable scatter of each chunk from its base.
// dynamic smem: run[E] + warp_hist[8*E] ints.
__global__ void __launch_bounds__(kPackThreads) k_pack_scatter(const int64_t* __restrict__ selected,
                                                               const uint16_t* __restrict__ weights, int T, int k,
                                                               int E, int chunk, const int* __restrict__ chunk_base,
                                                               PackOut o) {
    extern __shared__ int smem_i[];
    int* run = smem_i;
    int* warp_hist = run + E;
    for (int i = threadIdx.x; i < E; i += blockDim.x) run[i] = chunk_base[static_cast<size_t>(blockIdx.x) * E + i];
    __syncthreads();
    const int N = T * k;
    const int f0 = static_cast<int>(blockIdx.x) * chunk;
    const int f1 = min(N, f0 + chunk);
    block_stable_scatter(selected, weights, T, k, E, f0, f1, run, warp_hist, o);
}

}  // namespace pdx
