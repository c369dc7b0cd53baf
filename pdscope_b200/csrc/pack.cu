// Packing kernels: stable counting sort of routed (token, slot) pairs.
//
// Reference: compact_expert_groups() -- expertbench/pdscope_runtime.py:16-39
// (flat = selected.T.flatten(); counts = bincount; order = argsort(stable);
// tokens = order % T; positions = tokens*k + order//T; weights[positions]).
#include "routing.cuh"

namespace pdx {

constexpr int kPackThreads = 256;
constexpr int kPackChunk = 4096;  // flat entries per CTA in the multi-CTA path

// One CTA packs everything (N = T*k up to a few thousand entries).
// dynamic smem: hist[E] + excl[E+1] + warp_hist[8*E] ints.
__global__ void __launch_bounds__(kPackThreads) k_pack_single(const int64_t* __restrict__ selected,
                                                              const uint16_t* __restrict__ weights, int T, int k,
                                                              int E, PackOut o) {
    extern __shared__ int smem_i[];
    int* hist = smem_i;
    int* excl = hist + E;
    int* warp_hist = excl + E + 1;
    block_pack_all(selected, weights, T, k, E, hist, excl, warp_hist, o);
}

// Phase 1: per-chunk histograms -> chunk_hist[c*E + e].
__global__ void __launch_bounds__(kPackThreads) k_pack_hist(const int64_t* __restrict__ selected, int T, int k,
                                                            int E, int* __restrict__ chunk_hist) {
    extern __shared__ int smem_i[];
    int* hist = smem_i;
    for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int N = T * k;
    const int f0 = static_cast<int>(blockIdx.x) * kPackChunk;
    const int f1 = min(N, f0 + kPackChunk);
    block_histogram(selected, T, k, E, f0, f1, hist);
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) chunk_hist[static_cast<size_t>(blockIdx.x) * E + i] = hist[i];
}

// Phase 2 (one CTA): counts, offsets, active list and per-chunk bases
// chunk_base[c*E + e] = offsets[e] + sum_{c' < c} chunk_hist[c'*E + e].
__global__ void __launch_bounds__(kPackThreads) k_pack_scan(int* __restrict__ chunk_hist, int chunks, int E,
                                                            PackOut o) {
    extern __shared__ int smem_i[];
    int* tot = smem_i;
    int* excl = tot + E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = 0;
        for (int c = 0; c < chunks; ++c) {
            const int h = chunk_hist[static_cast<size_t>(c) * E + e];
            chunk_hist[static_cast<size_t>(c) * E + e] = run;  // becomes the chunk-relative base
            run += h;
        }
        tot[e] = run;
    }
    __syncthreads();
    if (threadIdx.x < 32) warp_exclusive_scan(tot, E, excl, o.active, nullptr);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        o.counts[e] = tot[e];
        o.offsets[e] = excl[e];
        for (int c = 0; c < chunks; ++c) chunk_hist[static_cast<size_t>(c) * E + e] += excl[e];
    }
    if (threadIdx.x == 0) o.offsets[E] = excl[E];
}

// Phase 3: stable scatter of each chunk from its base.
// dynamic smem: run[E] + warp_hist[8*E] ints.
__global__ void __launch_bounds__(kPackThreads) k_pack_scatter(const int64_t* __restrict__ selected,
                                                               const uint16_t* __restrict__ weights, int T, int k,
                                                               int E, const int* __restrict__ chunk_base,
                                                               PackOut o) {
    extern __shared__ int smem_i[];
    int* run = smem_i;
    int* warp_hist = run + E;
    for (int i = threadIdx.x; i < E; i += blockDim.x) run[i] = chunk_base[static_cast<size_t>(blockIdx.x) * E + i];
    __syncthreads();
    const int N = T * k;
    const int f0 = static_cast<int>(blockIdx.x) * kPackChunk;
    const int f1 = min(N, f0 + kPackChunk);
    block_stable_scatter(selected, weights, T, k, E, f0, f1, run, warp_hist, o);
}

}  // namespace pdx
