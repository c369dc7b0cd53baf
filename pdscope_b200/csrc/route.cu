// Router kernels: exact BF16 logits, softmax/top-k, and the decode-size
// top-k + pack kernel.
//
// Reference: route() -- expertbench/adapters/qwen.py:140-152 (logits via
// F.linear, FP32 softmax, torch.topk, renormalise, cast to BF16).
#include "routing.cuh"

namespace pdx {

constexpr int kRouteTB = 8;       // tokens per CTA block
constexpr int kRouteEB = 8;       // experts per CTA block
constexpr int kRouteWarps = 8;    // warps per CTA, each owning a share of K

__device__ __forceinline__ double bits_to_f64(uint32_t b16) {
    return static_cast<double>(__uint_as_float(b16 << 16));
}

// Decode sizes route in two kernels chained by programmatic dependent launch
// (no host work, no memset, no inter-CTA tickets between them): the logits
// kernel, whose CTAs load their gate rows before waiting for the kernel that
// produced x (the gate does not depend on it), and k_topk_pack, one CTA that
// routes every token and packs them from shared memory.

// logits[t, e] = RNE_bf16( sum_h x[t,h] * gate[e,h] ) with FP64 accumulation,
// 16 < T <= 64.  A CTA owns an 8-token x 8-expert block.  Warp w accumulates
// the 256-wide K chunks j = w, w+8, ...; inside a chunk lane l takes elements
// 8l..8l+7.  A transpose-reduction leaves block outputs (2l, 2l+1) (row-major
// t*8+e) in lane l; the 8 warps' partials are then added in warp order.
// Products of two BF16 values are exact in FP64 and the FP64 sum of 2048 of
// them is within a few units of 2^-53 relative, so the BF16 rounding equals
// that of the exact sum except in cases of probability ~1e-12 per logit.
__global__ void __launch_bounds__(kRouteWarps * 32) k_router_logits(const uint16_t* __restrict__ x,
                                                                     const uint16_t* __restrict__ gate, int T,
                                                                     int H, int E, uint16_t* __restrict__ logits) {
    __shared__ double s_part[kRouteWarps][kRouteTB * kRouteEB];
    const int warp = static_cast<int>(threadIdx.x >> 5);
    const int lane = static_cast<int>(lane_id());
    const int n_eb = (E + kRouteEB - 1) / kRouteEB;
    const int t0 = (static_cast<int>(blockIdx.x) / n_eb) * kRouteTB;
    const int e0 = (static_cast<int>(blockIdx.x) % n_eb) * kRouteEB;
    double acc[kRouteTB * kRouteEB];
#pragma unroll
    for (int i = 0; i < kRouteTB * kRouteEB; ++i) acc[i] = 0.0;
    int k0 = warp * 256 + lane * 8;
    // the first K chunk of the gate rows is loaded before the wait for x
    uint4 gv[kRouteEB];
#pragma unroll
    for (int e = 0; e < kRouteEB; ++e)
        gv[e] = (k0 < H && e0 + e < E) ? __ldg(reinterpret_cast<const uint4*>(gate + static_cast<size_t>(e0 + e) * H + k0))
                                       : make_uint4(0, 0, 0, 0);
    griddep_wait();
    griddep_launch();
    for (; k0 < H; k0 += kRouteWarps * 256) {
        uint4 xv[kRouteTB];
#pragma unroll
        for (int t = 0; t < kRouteTB; ++t)
            xv[t] = (t0 + t < T) ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + t) * H + k0))
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
        const int kn = k0 + kRouteWarps * 256;   // next chunk's gate rows
#pragma unroll
        for (int e = 0; e < kRouteEB; ++e)
            if (kn < H)
                gv[e] = (e0 + e < E) ? __ldg(reinterpret_cast<const uint4*>(gate + static_cast<size_t>(e0 + e) * H + kn))
                                     : make_uint4(0, 0, 0, 0);
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
}

// Decode-size router (T <= kSmallRouteT): one CTA per expert, so the 512 KiB
// of gate rows is read by E CTAs at once instead of E/8.  Thread i takes the
// 8-element K chunks i, i+256, ... of the expert's gate row (loaded before the
// wait for x) and of every token's row and accumulates the exact products in
// FP64; each token's sum is reduced over the CTA in a fixed order (xor
// butterfly inside warps, warps in order) and rounded once to BF16, as
// k_router_logits.
constexpr int kSmallRouteT = 16;
constexpr int kSmallRouteThreads = 256;
constexpr int kSmallRouteMaxChunks = 4;   // gate chunks held in registers: H <= 4 * 256 * 8

__global__ void __launch_bounds__(kSmallRouteThreads) k_router_small(const uint16_t* __restrict__ x,
                                                                     const uint16_t* __restrict__ gate, int T,
                                                                     int H, int E, uint16_t* __restrict__ logits) {
    constexpr int kWarps = kSmallRouteThreads / 32;
    __shared__ double s_part[kWarps][kSmallRouteT];
    const int warp = static_cast<int>(threadIdx.x >> 5);
    const int lane = static_cast<int>(lane_id());
    const int e = static_cast<int>(blockIdx.x);
    const uint16_t* grow = gate + static_cast<size_t>(e) * H;
    uint4 gv[kSmallRouteMaxChunks];
#pragma unroll
    for (int c = 0; c < kSmallRouteMaxChunks; ++c) {
        const int k0 = (c * kSmallRouteThreads + static_cast<int>(threadIdx.x)) * 8;
        gv[c] = k0 < H ? __ldg(reinterpret_cast<const uint4*>(grow + k0)) : make_uint4(0, 0, 0, 0);
    }
    griddep_wait();
    griddep_launch();
    double acc[kSmallRouteT];
#pragma unroll
    for (int t = 0; t < kSmallRouteT; ++t) acc[t] = 0.0;
#pragma unroll
    for (int c = 0; c < kSmallRouteMaxChunks; ++c) {
        const int k0 = (c * kSmallRouteThreads + static_cast<int>(threadIdx.x)) * 8;
        if (k0 >= H) break;
        double gd[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const uint32_t w = (&gv[c].x)[q >> 1];
            gd[q] = bits_to_f64((q & 1) ? (w >> 16) : (w & 0xFFFFu));
        }
#pragma unroll
        for (int t = 0; t < kSmallRouteT; ++t) {
            if (t < T) {
                const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H + k0));
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const uint32_t w = (&xv.x)[q >> 1];
                    acc[t] = fma(bits_to_f64((q & 1) ? (w >> 16) : (w & 0xFFFFu)), gd[q], acc[t]);
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kSmallRouteT; ++t) {
        if (t < T) {
            double v = acc[t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) s_part[warp][t] = v;
        }
    }
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < T) {
        const int t = static_cast<int>(threadIdx.x);
        double sum = s_part[0][t];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) sum += s_part[w][t];
        logits[static_cast<size_t>(t) * E + e] = f64_to_bf16_bits(sum);
    }
}

// Decode-size top-k + pack, one CTA: warp w routes tokens w, w+32, ... from
// the logits, then the CTA packs every token from shared memory
// (block_pack_all).  dynamic smem: block_pack_smem_ints(E, T*k, 32) ints.
// It also clears `zero_words` words at `zero_ptr` (the tickets and counters of
// the FFN launch that follows it), so no clearing kernel sits in the chain.
constexpr int kTopkPackThreads = 1024;
template <int EPL>
__global__ void __launch_bounds__(kTopkPackThreads) k_topk_pack(const uint16_t* __restrict__ logits, int T, int E,
                                                               int k, int normalize, int64_t* __restrict__ selected,
                                                               uint16_t* __restrict__ weights, PackOut pack,
                                                               unsigned int* __restrict__ zero_ptr, int zero_words) {
    griddep_wait();
    griddep_launch();
    for (int i = static_cast<int>(threadIdx.x); i < zero_words; i += static_cast<int>(blockDim.x)) zero_ptr[i] = 0u;
    const int warp = static_cast<int>(threadIdx.x >> 5);
    const int nw = static_cast<int>(blockDim.x >> 5);
    for (int t = warp; t < T; t += nw)
        warp_softmax_topk<EPL>(logits + static_cast<size_t>(t) * E, E, k, normalize != 0,
                               selected + static_cast<size_t>(t) * k, weights + static_cast<size_t>(t) * k);
    __syncthreads();  // this CTA's selected/weights stores are visible to its threads
    extern __shared__ int smem_tp[];
    int* hist = smem_tp;
    int* excl = hist + E;
    if (T * k <= 32) {   // a handful of assignments: one warp packs them
        if (warp == 0) warp_pack_small(selected, weights, T, k, E, hist, excl, pack);
        return;
    }
    int* warp_hist = excl + E + 1;
    block_pack_all(selected, weights, T, k, E, hist, excl, warp_hist, pack);
}

// Prefill-size router on the FP64 tensor path (mma.sync m8n8k4 .f64; tcgen05
// has no FP64 kind): exact BF16 products summed in FP64, as k_router_logits,
// with each warp instruction doing 256 FMAs (8x8x4) from register fragments.  The FP64
// tensor path has the FP64 pipe's peak (64 FMA/clk/SM) but needs an eighth of
// the issue slots and, with a 32x64 warp tile, 1/4 of the shared-memory loads
// per FMA.  Tile: 64 tokens x 128 experts per 128-thread CTA, K chunks of 32
// in double-buffered FP64 shared memory, row stride 36 doubles so the
// fragment loads (8 rows x 4 k per warp) touch every 8-byte bank twice.
// Work unit = (tile, K range).  With splits == 1 the unit covers all of K and
// writes the rounded BF16 logits; with splits > 1 it writes its FP64 partial
// dot products to partials[split][T][E] and k_topk_partials adds the splits in
// split order before the single rounding.  The split count balances the units
// over the SMs (a 64-token tile is ~1/148 of the work at 9.5k tokens, so whole
// tiles alone leave SMs idle).
constexpr int kDmT = 64;
constexpr int kDmE = 128;
constexpr int kDmK = 32;
constexpr int kDmS = 36;  // shared-memory row stride (doubles)
constexpr int kDmThreads = 128;
constexpr size_t kDmmaSmemBytes = 2 * (kDmT + kDmE) * kDmS * sizeof(double);

__device__ __forceinline__ void dmma_884(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(kDmThreads, 2) k_router_logits_dmma(const uint16_t* __restrict__ x,
                                                                     const uint16_t* __restrict__ gate, int T, int H,
                                                                     int E, int splits, int k_per_split,
                                                                     uint16_t* __restrict__ logits,
                                                                     double* __restrict__ partials) {
    extern __shared__ __align__(16) double smem_dmma[];
    double* xs = smem_dmma;                    // [2][kDmT][kDmS]
    double* gs = smem_dmma + 2 * kDmT * kDmS;  // [2][kDmE][kDmS]
    const int tid = static_cast<int>(threadIdx.x);
    const int warp = tid >> 5, lane = tid & 31;
    const int n_et = (E + kDmE - 1) / kDmE;
    const int split = static_cast<int>(blockIdx.x) % splits;
    const int tile = static_cast<int>(blockIdx.x) / splits;
    const int t0 = (tile / n_et) * kDmT;
    const int e0 = (tile % n_et) * kDmE;
    const int k_begin = split * k_per_split;
    const int k_end = min(H, k_begin + k_per_split);
    const int wm = (warp >> 1) * 32;  // warp tile: 32 tokens x 64 experts
    const int wn = (warp & 1) * 64;
    const int fr = lane >> 2, fk = lane & 3;  // fragment row (token / expert) and k of this lane

    // global -> registers: 4 lanes per 64-byte row segment (coalesced)
    uint4 xr[2], gr[4];
    auto load_chunk = [&](int k0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int idx = tid + r * kDmThreads;  // 0..255 = 64 rows x 4 segments
            const int row = idx >> 2, seg = idx & 3;
            const int t = t0 + row, k = k0 + seg * 8;
            xr[r] = (t < T && k < H) ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H + k))
                                     : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int idx = tid + r * kDmThreads;  // 0..511 = 128 rows x 4 segments
            const int row = idx >> 2, seg = idx & 3;
            const int e = e0 + row, k = k0 + seg * 8;
            gr[r] = (e < E && k < H) ? __ldg(reinterpret_cast<const uint4*>(gate + static_cast<size_t>(e) * H + k))
                                     : make_uint4(0, 0, 0, 0);
        }
    };
    auto store8 = [&](double* dst, const uint4& v) {  // 8 BF16 -> 8 doubles, 16-byte stores
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
            reinterpret_cast<double2*>(dst)[q] = make_double2(bits_to_f64(w[q] & 0xFFFFu), bits_to_f64(w[q] >> 16));
    };
    auto store_chunk = [&](int buf) {
        double* xb = xs + buf * kDmT * kDmS;
        double* gb = gs + buf * kDmE * kDmS;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int idx = tid + r * kDmThreads;
            store8(xb + (idx >> 2) * kDmS + (idx & 3) * 8, xr[r]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int idx = tid + r * kDmThreads;
            store8(gb + (idx >> 2) * kDmS + (idx & 3) * 8, gr[r]);
        }
    };

    double acc[4][8][2];
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 8; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = 0.0;

    const int n_chunks = k_end > k_begin ? (k_end - k_begin + kDmK - 1) / kDmK : 0;
    if (n_chunks > 0) {
        load_chunk(k_begin);
        store_chunk(0);
    }
    __syncthreads();
    for (int c = 0; c < n_chunks; ++c) {
        const int buf = c & 1;
        if (c + 1 < n_chunks) load_chunk(k_begin + (c + 1) * kDmK);
        const double* xb = xs + buf * kDmT * kDmS + (wm + fr) * kDmS + fk;
        const double* gb = gs + buf * kDmE * kDmS + (wn + fr) * kDmS + fk;
#pragma unroll
        for (int kq = 0; kq < kDmK / 4; ++kq) {
            double a[4], b[8];
#pragma unroll
            for (int mi = 0; mi < 4; ++mi) a[mi] = xb[mi * 8 * kDmS + kq * 4];
#pragma unroll
            for (int ni = 0; ni < 8; ++ni) b[ni] = gb[ni * 8 * kDmS + kq * 4];
#pragma unroll
            for (int mi = 0; mi < 4; ++mi)
#pragma unroll
                for (int ni = 0; ni < 8; ++ni) dmma_884(acc[mi][ni], a[mi], b[ni]);
        }
        if (c + 1 < n_chunks) store_chunk(buf ^ 1);
        __syncthreads();
    }
    // accumulator fragment: row fr (token), columns 2*fk + {0, 1} (experts)
#pragma unroll
    for (int mi = 0; mi < 4; ++mi) {
        const int t = t0 + wm + mi * 8 + fr;
        if (t >= T) continue;
#pragma unroll
        for (int ni = 0; ni < 8; ++ni) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int e = e0 + wn + ni * 8 + 2 * fk + j;
                if (e >= E) continue;
                if (splits == 1)
                    logits[static_cast<size_t>(t) * E + e] = f64_to_bf16_bits(acc[mi][ni][j]);
                else
                    partials[(static_cast<size_t>(split) * T + t) * E + e] = acc[mi][ni][j];
            }
        }
    }
}

// Split-K router tail, one warp per token: logits = RNE_bf16(sum of the FP64
// partials in split order), written out and kept in registers for the
// softmax + top-k + renormalisation of the row.
template <int EPL>
__device__ __forceinline__ void topk_partials_row(const double* __restrict__ partials, int splits, int T, int E,
                                                  int t, int k, bool normalize, uint16_t* __restrict__ logits,
                                                  int64_t* __restrict__ selected, uint16_t* __restrict__ weights) {
    const int lane = static_cast<int>(lane_id());
    double acc[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) acc[i] = 0.0;
    // four splits' partials are loaded before they are added (in split order),
    // so a many-split row costs splits/4 memory round trips, not splits
    constexpr int kBatch = 4;
    for (int sp0 = 0; sp0 < splits; sp0 += kBatch) {
        double v[kBatch][EPL];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const double* row = partials + (static_cast<size_t>(sp0 + j) * T + t) * E;
#pragma unroll
            for (int i = 0; i < EPL; ++i) {
                const int idx = lane + 32 * i;
                v[j][i] = 0.0;
                if (sp0 + j < splits && idx < E) v[j][i] = __ldg(row + idx);
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
#pragma unroll
            for (int i = 0; i < EPL; ++i)
                if (sp0 + j < splits) acc[i] += v[j][i];
    }
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int idx = lane + 32 * i;
        if (idx < E) {
            const uint16_t b = f64_to_bf16_bits(acc[i]);
            logits[static_cast<size_t>(t) * E + idx] = b;
            v[i] = bits2f(b);
        } else {
            v[i] = -INFINITY;
        }
    }
    warp_softmax_topk_vals<EPL>(v, E, k, normalize, selected + static_cast<size_t>(t) * k,
                                weights + static_cast<size_t>(t) * k);
}

// Kernels that route a whole row per warp are instantiated per EPL (elements
// per lane, next_pow2(E) / 32) and dispatched on the host, so each keeps only
// its own row in registers.
template <int EPL>
__global__ void __launch_bounds__(256) k_topk_partials(const double* __restrict__ partials, int splits, int T, int E,
                                                       int k, int normalize, uint16_t* __restrict__ logits,
                                                       int64_t* __restrict__ selected,
                                                       uint16_t* __restrict__ weights) {
    griddep_wait();
    griddep_launch();
    const int warps = static_cast<int>(blockDim.x >> 5);
    const bool nrm = normalize != 0;
    for (int t = static_cast<int>(blockIdx.x) * warps + static_cast<int>(threadIdx.x >> 5); t < T;
         t += static_cast<int>(gridDim.x) * warps)
        topk_partials_row<EPL>(partials, splits, T, E, t, k, nrm, logits, selected, weights);
}

// Softmax + top-k + renormalisation, one warp per token.
template <int EPL>
// (Also clears `zero_words` words at `zero_ptr`, spread over the CTAs: the
// tickets and counters of the decode FFN launch two kernels later.)
__global__ void __launch_bounds__(256) k_topk(const uint16_t* __restrict__ logits, int T, int E, int k,
                                              int normalize, int64_t* __restrict__ selected,
                                              uint16_t* __restrict__ weights, unsigned int* __restrict__ zero_ptr,
                                              int zero_words) {
    griddep_wait();
    griddep_launch();
    for (int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x); i < zero_words;
         i += static_cast<int>(gridDim.x * blockDim.x))
        zero_ptr[i] = 0u;
    const int warps = static_cast<int>(blockDim.x >> 5);
    const int first = static_cast<int>(blockIdx.x) * warps + static_cast<int>(threadIdx.x >> 5);
    block_topk_rows<EPL>(logits, T, E, k, normalize != 0, selected, weights, first, gridDim.x * warps);
}

// Calls f(std::integral_constant<int, EPL>) for the EPL of E (<= 1024 experts).
template <typename F>
inline auto with_epl(int64_t E, F&& f) {
    if (E <= 32) return f(std::integral_constant<int, 1>{});
    if (E <= 64) return f(std::integral_constant<int, 2>{});
    if (E <= 128) return f(std::integral_constant<int, 4>{});
    if (E <= 256) return f(std::integral_constant<int, 8>{});
    if (E <= 512) return f(std::integral_constant<int, 16>{});
    return f(std::integral_constant<int, 32>{});
}

}  // namespace pdx
