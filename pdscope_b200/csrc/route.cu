// Router kernels: exact BF16 logits, softmax/top-k, and the fused decode tail.
//
// Reference: route() -- expertbench/adapters/qwen.py:140-152 (logits via
// F.linear, FP32 softmax, torch.topk, renormalise, cast to BF16).
#include "routing.cuh"

namespace pdx {

constexpr int kRouteTB = 8;       // tokens per CTA block
constexpr int kRouteEB = 8;       // experts per CTA block
constexpr int kRouteWarps = 8;    // warps per CTA, each owning a share of K
static_assert(kRouteWarps == kRouteTB, "the fused tail routes one token per warp");

struct RouteTail {
    int enabled;           // 1: top-k in this kernel (per token block), 0: k_topk follows
    int k;
    int normalize;
    int do_pack;           // 1: the last token block to finish also packs every token
    unsigned int* tickets; // [1 + token blocks], zeroed by the host before the launch
    int64_t* selected;
    uint16_t* weights;
    PackOut pack;
};

__device__ __forceinline__ double bits_to_f64(uint32_t b16) {
    return static_cast<double>(__uint_as_float(b16 << 16));
}

// logits[t, e] = RNE_bf16( sum_h x[t,h] * gate[e,h] ) with FP64 accumulation.
// A CTA owns an 8-token x 8-expert block.  Warp w accumulates the 256-wide K
// chunks j = w, w+8, ...; inside a chunk lane l takes elements 8l..8l+7.  A
// transpose-reduction leaves block outputs (2l, 2l+1) (row-major t*8+e) in
// lane l; the 8 warps' partials are then added in warp order.  Products of
// two BF16 values are exact in FP64 and the FP64 sum of 2048 of them is
// within a few units of 2^-53 relative, so the BF16 rounding equals that of
// the exact sum except in cases of probability ~1e-12 per logit.
__global__ void __launch_bounds__(kRouteWarps * 32) k_router_logits(const uint16_t* __restrict__ x,
                                                                     const uint16_t* __restrict__ gate, int T,
                                                                     int H, int E, uint16_t* __restrict__ logits,
                                                                     RouteTail tail) {
    __shared__ double s_part[kRouteWarps][kRouteTB * kRouteEB];
    const int warp = static_cast<int>(threadIdx.x >> 5);
    const int lane = static_cast<int>(lane_id());
    const int n_eb = (E + kRouteEB - 1) / kRouteEB;
    const int t0 = (static_cast<int>(blockIdx.x) / n_eb) * kRouteTB;
    const int e0 = (static_cast<int>(blockIdx.x) % n_eb) * kRouteEB;
    double acc[kRouteTB * kRouteEB];
#pragma unroll
    for (int i = 0; i < kRouteTB * kRouteEB; ++i) acc[i] = 0.0;
    for (int k0 = warp * 256 + lane * 8; k0 < H; k0 += kRouteWarps * 256) {
        uint4 xv[kRouteTB], gv[kRouteEB];
#pragma unroll
        for (int t = 0; t < kRouteTB; ++t)
            xv[t] = (t0 + t < T) ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + t) * H + k0))
                                 : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int e = 0; e < kRouteEB; ++e)
            gv[e] = (e0 + e < E) ? __ldg(reinterpret_cast<const uint4*>(gate + static_cast<size_t>(e0 + e) * H + k0))
                                 : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            double xd[kRouteTB], gd[kRouteEB];
#pragma unroll
            for (int t = 0; t < kRouteTB; ++t) {
                const uint32_t w = (&xv[t].x)[q >> 1];
                xd[t] = bits_to_f64((q & 1) ? (w >> 16) : (w & 0xFFFFu));
            }
#pragma unroll
            for (int e = 0; e < kRouteEB; ++e) {
                const uint32_t w = (&gv[e].x)[q >> 1];
                gd[e] = bits_to_f64((q & 1) ? (w >> 16) : (w & 0xFFFFu));
            }
#pragma unroll
            for (int t = 0; t < kRouteTB; ++t)
#pragma unroll
                for (int e = 0; e < kRouteEB; ++e) acc[t * kRouteEB + e] = fma(xd[t], gd[e], acc[t * kRouteEB + e]);
        }
    }
    // transpose-reduce 64 partial sums over 32 lanes: lane l keeps outputs 2l, 2l+1
#pragma unroll
    for (int step = 0; step < 5; ++step) {
        const int mask = 16 >> step;
        const int half = 32 >> step;
        const bool upper = (lane & mask) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const double send = upper ? acc[i] : acc[i + half];
            const double keep = upper ? acc[i + half] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
        }
    }
    s_part[warp][2 * lane] = acc[0];
    s_part[warp][2 * lane + 1] = acc[1];
    __syncthreads();
    if (threadIdx.x < kRouteTB * kRouteEB) {
        const int o = static_cast<int>(threadIdx.x);
        double sum = s_part[0][o];
#pragma unroll
        for (int w = 1; w < kRouteWarps; ++w) sum += s_part[w][o];
        const int t = t0 + o / kRouteEB;
        const int e = e0 + o % kRouteEB;
        if (t < T && e < E) logits[static_cast<size_t>(t) * E + e] = f64_to_bf16_bits(sum);
    }
    if (!tail.enabled) return;
    // ---- fused tail -------------------------------------------------------------
    // The CTA that completes a token block (its n_eb expert blocks all written)
    // routes those 8 tokens, one warp each; with do_pack, the last token block to
    // finish then packs every token.  Threadfence-reduction pattern: writers
    // fence before the ticket, the winner fences after it.
    __shared__ unsigned int s_ticket;
    const int tb = static_cast<int>(blockIdx.x) / n_eb;
    const int n_tb = (T + kRouteTB - 1) / kRouteTB;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(&tail.tickets[1 + tb], 1u);
    __syncthreads();
    if (s_ticket != static_cast<unsigned int>(n_eb - 1)) return;
    __threadfence();
    const int t = tb * kRouteTB + warp;  // kRouteWarps == kRouteTB: one token per warp
    if (t < T) topk_row(logits, t, E, tail.k, tail.normalize != 0, tail.selected, tail.weights);
    if (!tail.do_pack) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(&tail.tickets[0], 1u);
    __syncthreads();
    if (s_ticket != static_cast<unsigned int>(n_tb - 1)) return;
    __threadfence();
    extern __shared__ int smem_i[];
    int* hist = smem_i;
    int* excl = hist + E;
    int* warp_hist = excl + E + 1;
    block_pack_all(tail.selected, tail.weights, T, tail.k, E, hist, excl, warp_hist, tail.pack);
}

// Prefill-size logits: a shared-memory-tiled FP64 GEMM.  A CTA of 128 threads
// owns 64 tokens x 128 experts; K advances in chunks of 32 staged in shared
// memory as FP64 (each BF16 operand converted once per CTA, transposed so a
// thread's operands are one LDS.64 each).  Thread (tx, ty) accumulates tokens
// ty + 8i and experts tx + 16j (i, j < 8): the strided ownership makes the
// expert reads of a warp 16 consecutive doubles (conflict-free) and the token
// reads broadcasts.  The next chunk is loaded from global memory into
// registers while the current one is multiplied.  Same exact-sum contract as
// k_router_logits (FP64 accumulation of exact BF16 products, one rounding).
constexpr int kTileT = 64;
constexpr int kTileE = 128;
constexpr int kTileK = 32;
constexpr int kTileThreads = 128;
constexpr size_t kTileSmemBytes = 2 * (kTileK * kTileT + kTileK * kTileE) * sizeof(double);

// Work unit = (64-token x 128-expert tile, K range).  With splits == 1 the unit
// covers all of K and writes the rounded BF16 logits; with splits > 1 it
// writes its FP64 partial dot products to partials[split][T][E] and
// k_topk_partials adds the splits in split order before the single rounding.
// The split count balances the units over the SMs (a 64-token tile is ~1/148
// of the work at 9.5k tokens, so whole tiles alone leave SMs idle).
__global__ void __launch_bounds__(kTileThreads, 2) k_router_logits_tiled(const uint16_t* __restrict__ x,
                                                                         const uint16_t* __restrict__ gate, int T,
                                                                         int H, int E, int splits, int k_per_split,
                                                                         uint16_t* __restrict__ logits,
                                                                         double* __restrict__ partials) {
    extern __shared__ __align__(16) double smem_route[];
    double* xs = smem_route;                            // [2][kTileK][kTileT]
    double* gs = smem_route + 2 * kTileK * kTileT;      // [2][kTileK][kTileE]
    const int tid = static_cast<int>(threadIdx.x);
    const int tx = tid % 16, ty = tid / 16;
    const int n_et = (E + kTileE - 1) / kTileE;
    const int split = static_cast<int>(blockIdx.x) % splits;
    const int tile = static_cast<int>(blockIdx.x) / splits;
    const int t0 = (tile / n_et) * kTileT;
    const int e0 = (tile % n_et) * kTileE;
    const int k_begin = split * k_per_split;
    const int k_end = min(H, k_begin + k_per_split);
    // global -> register staging: x chunk = 64 rows x 32 bf16 (256 x 16 B, 2 per
    // thread); gate chunk = 128 rows x 32 bf16 (512 x 16 B, 4 per thread).  A
    // warp's 32 lanes take 32 consecutive rows of one 8-wide K segment, so the
    // transposed FP64 stores below fill 32 consecutive doubles per k (no bank
    // conflicts).
    uint4 xr[2], gr[4];
    auto load_chunk = [&](int k0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int idx = tid + r * kTileThreads;           // 0..255
            const int row = idx % kTileT, seg = idx / kTileT;  // seg 0..3: 8 bf16 (16 B) each
            const int t = t0 + row, k = k0 + seg * 8;
            xr[r] = (t < T && k < H) ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H + k))
                                     : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int idx = tid + r * kTileThreads;           // 0..511
            const int row = idx % kTileE, seg = idx / kTileE;
            const int e = e0 + row, k = k0 + seg * 8;
            gr[r] = (e < E && k < H) ? __ldg(reinterpret_cast<const uint4*>(gate + static_cast<size_t>(e) * H + k))
                                     : make_uint4(0, 0, 0, 0);
        }
    };
    auto store_chunk = [&](int buf) {
        double* xb = xs + buf * kTileK * kTileT;
        double* gb = gs + buf * kTileK * kTileE;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int idx = tid + r * kTileThreads;
            const int row = idx % kTileT, seg = idx / kTileT;
            const uint32_t w[4] = {xr[r].x, xr[r].y, xr[r].z, xr[r].w};
#pragma unroll
            for (int q = 0; q < 8; ++q)
                xb[(seg * 8 + q) * kTileT + row] = bits_to_f64((q & 1) ? (w[q >> 1] >> 16) : (w[q >> 1] & 0xFFFFu));
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int idx = tid + r * kTileThreads;
            const int row = idx % kTileE, seg = idx / kTileE;
            const uint32_t w[4] = {gr[r].x, gr[r].y, gr[r].z, gr[r].w};
#pragma unroll
            for (int q = 0; q < 8; ++q)
                gb[(seg * 8 + q) * kTileE + row] = bits_to_f64((q & 1) ? (w[q >> 1] >> 16) : (w[q >> 1] & 0xFFFFu));
        }
    };
    double acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;
    const int n_chunks = k_end > k_begin ? (k_end - k_begin + kTileK - 1) / kTileK : 0;
    if (n_chunks > 0) {
        load_chunk(k_begin);
        store_chunk(0);
    }
    __syncthreads();
    for (int c = 0; c < n_chunks; ++c) {
        const int buf = c & 1;
        if (c + 1 < n_chunks) load_chunk(k_begin + (c + 1) * kTileK);
        const double* xb = xs + buf * kTileK * kTileT;
        const double* gb = gs + buf * kTileK * kTileE;
#pragma unroll 4
        for (int kk = 0; kk < kTileK; ++kk) {
            double xv[8], gv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] = xb[kk * kTileT + ty + 8 * i];
#pragma unroll
            for (int j = 0; j < 8; ++j) gv[j] = gb[kk * kTileE + tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fma(xv[i], gv[j], acc[i][j]);
        }
        if (c + 1 < n_chunks) store_chunk(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int t = t0 + ty + 8 * i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = e0 + tx + 16 * j;
            if (e >= E) continue;
            if (splits == 1)
                logits[static_cast<size_t>(t) * E + e] = f64_to_bf16_bits(acc[i][j]);
            else
                partials[(static_cast<size_t>(split) * T + t) * E + e] = acc[i][j];
        }
    }
}

// Split-K router tail, one warp per token: logits = RNE_bf16(sum of the FP64
// partials in split order), written out, then softmax + top-k + renormalise
// on the row just written.
__global__ void __launch_bounds__(256) k_topk_partials(const double* __restrict__ partials, int splits, int T, int E,
                                                       int k, int normalize, uint16_t* __restrict__ logits,
                                                       int64_t* __restrict__ selected,
                                                       uint16_t* __restrict__ weights) {
    const int warps = static_cast<int>(blockDim.x >> 5);
    const int lane = static_cast<int>(threadIdx.x & 31);
    for (int t = static_cast<int>(blockIdx.x) * warps + static_cast<int>(threadIdx.x >> 5); t < T;
         t += static_cast<int>(gridDim.x) * warps) {
        for (int e = lane; e < E; e += 32) {
            double sum = 0.0;
            for (int sp = 0; sp < splits; ++sp) sum += partials[(static_cast<size_t>(sp) * T + t) * E + e];
            logits[static_cast<size_t>(t) * E + e] = f64_to_bf16_bits(sum);
        }
        __syncwarp();  // the row is re-read by every lane of this warp
        topk_row(logits, t, E, k, normalize != 0, selected, weights);
    }
}

// Softmax + top-k + renormalisation, one warp per token.
__global__ void __launch_bounds__(256) k_topk(const uint16_t* __restrict__ logits, int T, int E, int k,
                                              int normalize, int64_t* __restrict__ selected,
                                              uint16_t* __restrict__ weights) {
    const int warps = static_cast<int>(blockDim.x >> 5);
    const int first = static_cast<int>(blockIdx.x) * warps + static_cast<int>(threadIdx.x >> 5);
    topk_rows_dispatch(logits, T, E, k, normalize != 0, selected, weights, first, gridDim.x * warps);
}

}  // namespace pdx
