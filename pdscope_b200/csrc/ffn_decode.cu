// Weight-streaming grouped expert FFN in ONE launch: the gate/up and the down
// projection of every active expert, weights streamed by TMA as the tcgen05 M
// operand ("swap AB").
//
// Reference: expert_forward() -- expertbench/adapters/qwen.py:87-90, run per
// routed expert by ExpertExecutor.gpu (expertbench/executor.py:454-488).
//
// At decode (T <= 64 tokens) the layer is a stream of expert weights.  The
// weight-streaming path of ffn_stream.cu runs it as three kernels (row gather,
// gate/up GEMM, down GEMM), and each kernel boundary leaves HBM idle while the
// last CTAs of one kernel drain and the next kernel's CTAs ramp up.  Here:
//   * Phase 1 (gate/up) takes the WHOLE token matrix x [T, H] as the N operand
//     (N = T rounded up to 16; TMA zero-fills rows past T), so every expert's
//     tile computes all T token columns and the epilogue keeps only the
//     columns of the tokens routed to it: packed row p of expert e reads TMEM
//     column tokens[p].  The tensor core has ~10x more throughput than the
//     weight stream needs at these sizes, so the extra columns are free and
//     the gather kernel disappears.
//     (DIRECT form, T <= 64.  The PACKED form, for larger batches or rows
//     already in packed order, tiles each expert's packed rows instead, 16,
//     32 or 64 rows per tile, like phase 2.)
//   * Phase 2 (down) runs in the same persistent CTAs, on the packed h rows
//     (N = 16/32/64 rows of one expert per tile).  Its weight tiles need
//     nothing from phase 1, so the weight producer streams them right behind
//     phase 1's weights; only the h operand waits, per expert, for a counter
//     that phase 1's epilogue warps raise once their h columns are stored.
// Roles (224 threads): warp 0 streams the weight (A) tiles, warp 6 the token
// (B) tiles -- x in phase 1, h in phase 2 after the expert's h is complete --
// warp 1 issues tcgen05.mma into double-buffered TMEM, warps 2..5 are the
// epilogue (one TMEM lane quadrant each).  A and B of one ring stage are
// counted on the same full barrier, so the weight producer runs up to a ring
// ahead of a waiting h.
// Work units are (tile, K slice) of phase 1 first, then of phase 2, taken by
// the CTAs round robin, so every expert's phase-1 tiles are issued before any
// CTA can wait on them.  Split-K partial sums are added by the warp that takes
// the last ticket, in slice order 0..splits-1 (deterministic), as in
// ffn_stream.cu.  The tickets and the per-expert counters must be zero on
// entry (the launcher clears them in the kernel before this one).
// Every wait is bounded (2 s, abort flag, drain, TMEM freed), including the
// wait for another CTA's h.
#include <cuda.h>

#include "tcgen05.cuh"

namespace pdx {

constexpr int kDecMaxT = 64;        // token columns of the direct gate/up operand
constexpr int kDecStages = 5;
constexpr int kDecThreads = 224;    // A producer, MMA, 4 epilogue warps, B producer
constexpr uint32_t kDecABytes = 128 * 64 * 2;                       // one 128 x 64 weight box
constexpr uint32_t kDecStageBytes = 2 * kDecABytes + kDecMaxT * 64 * 2;  // gate | up | tokens: 40 KiB
constexpr uint32_t kDecTmemCols = 256;  // two accumulators of up to 128 columns
constexpr int kDecMaxActive = 512;
constexpr int kDecMaxRows = 1024;
// tables after the stages and barriers: phase-1 and phase-2 tile prefixes,
// segment start, row count, weight slot (per active expert), tokens (per row)
constexpr size_t kDecSmemBytes = 1024 + kDecStages * kDecStageBytes + 256 + 5 * (kDecMaxActive + 1) * 4 +
                                 kDecMaxRows * 4;

struct DecodeArgs {
    const int32_t* offsets;        // [E+1] packed segment starts
    const int32_t* active;         // [E+1] active count, then the active expert ids
    const int32_t* tokens;         // [rows] packed row -> token (DIRECT form)
    const int32_t* slot_of_expert; // NULL = identity
    int64_t num_slots;
    int64_t gate_rows_per_slot;    // TMA-map rows between consecutive slots
    int64_t up_rows_per_slot;
    int64_t down_rows_per_slot;
    int H, I, T, rows;
    int splits1, splits2;          // K slices per tile of each phase
    uint16_t* h;                   // [rows, I]
    uint16_t* y;                   // [rows, H]
    float* partials1;              // splits1 > 1: DIRECT [I/128][splits1][rows][2][128],
                                   //   PACKED [phase-1 units][2*NB][128]
    float* partials2;              // [phase-2 units][NT2][128] when splits2 > 1
    unsigned int* tickets1;        // [phase-1 tiles * 4], zero on entry
    unsigned int* tickets2;        // [phase-2 tiles * 4], zero on entry
    unsigned int* h_ready;         // [active], zero on entry
};

__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t& r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}

// Orders this thread's generic-proxy global writes before later async-proxy
// (TMA) accesses to them, here: the h rows phase 2 loads with TMA.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float swiglu_bf16(uint32_t g_bits, uint32_t u_bits) {
    const float gb = round_bf16(__uint_as_float(g_bits));
    const float ub = round_bf16(__uint_as_float(u_bits));
    const float sv = round_bf16(__fdiv_rn(gb, 1.0f + expf(-gb)));
    return sv * ub;
}

struct DecUnit {
    int phase2;  // 0: gate/up, 1: down
    int a;       // index into the active-expert tables
    int ib;      // 128-row weight block
    int nb;      // token-row block of the expert's segment (0 in the DIRECT phase 1)
    int tile;    // tile index within its phase
    int slice;
    int kb0, kb1;
};

// Exclusive prefix over the active experts of `tiles(a)` (one warp), written
// to pre[]; returns the total in every lane.
template <typename F>
__device__ __forceinline__ int warp_tile_prefix(int n_active, int* pre, F tiles) {
    const uint32_t lane = lane_id();
    const int per = (n_active + 31) / 32;
    const int b = static_cast<int>(lane) * per;
    int local = 0;
    for (int i = 0; i < per; ++i)
        if (b + i < n_active) {
            const int t = tiles(b + i);
            pre[b + i] = t;
            local += t;
        }
    int inc = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, off);
        if (static_cast<int>(lane) >= off) inc += v;
    }
    int run = inc - local;
    for (int i = 0; i < per; ++i)
        if (b + i < n_active) {
            const int t = pre[b + i];
            pre[b + i] = run;
            run += t;
        }
    return __shfl_sync(0xffffffffu, inc, 31);
}

// Largest a < n with pre[a] <= tile.
__device__ __forceinline__ int find_expert(const int* pre, int n, int tile) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// DIRECT: phase-1 B operand = x [T, H] (tm_x box NB rows), NB >= T.
// PACKED: phase-1 B operand = the packed rows (tm_x over [rows, H], box NB).
template <bool DIRECT, int NB, int NT2>
__global__ void __launch_bounds__(kDecThreads, 1)
    k_decode_ffn(const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_u,
                 const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_d,
                 const __grid_constant__ CUtensorMap tm_h, DecodeArgs args) {
    static_assert(NB % 16 == 0 && NB <= kDecMaxT && NT2 % 16 == 0 && NT2 <= 64, "token tiles");
    extern __shared__ __align__(1024) unsigned char smem_dec[];
    const uint32_t raw_addr = smem_u32(smem_dec);
    unsigned char* smem = smem_dec + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kDecStages * kDecStageBytes);
    uint64_t* empty_bar = full_bar + kDecStages;
    uint64_t* tmem_full = empty_bar + kDecStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain_bar = tmem_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* s_misc = reinterpret_cast<int*>(tmem_slot + 2);  // [0] phase-2 tiles, [1] phase-1 tiles
    int* prefix2 = reinterpret_cast<int*>(smem + kDecStages * kDecStageBytes + 256);
    int* prefix1 = prefix2 + (kDecMaxActive + 1);
    int* t_seg0 = prefix1 + (kDecMaxActive + 1);
    int* t_rows = t_seg0 + (kDecMaxActive + 1);
    int* t_slot = t_rows + (kDecMaxActive + 1);
    int* s_tok = t_slot + (kDecMaxActive + 1);

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();
    const int m1 = args.I / 128, m2 = args.H / 128;
    const int nkb1 = args.H / 64, nkb2 = args.I / 64;
    const int s1 = args.splits1, s2 = args.splits2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kDecStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 128);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_g);
        tma_prefetch_desc(&tm_u);
        tma_prefetch_desc(&tm_d);
    }
    if (warp == 6 && lane == 0) {
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_h);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kDecTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Everything above is independent of the previous kernel; from here on the
    // routing/packing results and x are read.
    griddep_wait();
    griddep_launch();
    const int n_active = min(args.active[0], kDecMaxActive);
    const int n_rows = min(args.rows, kDecMaxRows);
    if (warp == 2) {
        // per active expert: segment, rows, slot; tiles per expert of phase 1
        // (DIRECT m1, PACKED m1 * ceil(n_e / NB)) and phase 2 (m2 * ceil(n_e /
        // NT2)) -> exclusive prefixes
        for (int i = static_cast<int>(lane); i < n_active; i += 32) {
            const int e = args.active[1 + i];
            const int seg0 = args.offsets[e];
            int64_t slot = args.slot_of_expert ? args.slot_of_expert[e] : e;
            if (slot < 0 || slot >= args.num_slots) {
                raise_error(PDX_DEVERR_BAD_SLOT);
                slot = 0;  // keeps the pipeline consistent; the call is flagged invalid
            }
            t_seg0[i] = seg0;
            t_rows[i] = args.offsets[e + 1] - seg0;
            t_slot[i] = static_cast<int>(slot);
        }
        __syncwarp();
        const int tot2 = warp_tile_prefix(n_active, prefix2, [&](int a) { return m2 * ((t_rows[a] + NT2 - 1) / NT2); });
        const int tot1 = DIRECT ? n_active * m1
                                : warp_tile_prefix(n_active, prefix1,
                                                   [&](int a) { return m1 * ((t_rows[a] + NB - 1) / NB); });
        if (lane == 0) {
            s_misc[0] = tot2;
            s_misc[1] = tot1;
        }
    } else if (DIRECT && warp >= 3) {
        for (int i = static_cast<int>(threadIdx.x) - 96; i < n_rows; i += kDecThreads - 96) {
            int t = args.tokens[i];
            if (t < 0 || t >= args.T) {
                raise_error(PDX_DEVERR_BAD_EXPERT);
                t = 0;
            }
            s_tok[i] = t;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int units1 = s_misc[1] * s1;
    const int total_units = units1 + s_misc[0] * s2;

    auto decode = [&](int u) {
        DecUnit d;
        if (u < units1) {
            d.phase2 = 0;
            d.tile = u / s1;
            d.slice = u % s1;
            if (DIRECT) {
                d.a = d.tile / m1;
                d.ib = d.tile % m1;
                d.nb = 0;
            } else {
                d.a = find_expert(prefix1, n_active, d.tile);
                const int nbc = (t_rows[d.a] + NB - 1) / NB;
                const int local = d.tile - prefix1[d.a];
                d.ib = local / nbc;
                d.nb = local % nbc;
            }
            d.kb0 = (d.slice * nkb1) / s1;
            d.kb1 = ((d.slice + 1) * nkb1) / s1;
        } else {
            const int v = u - units1;
            d.phase2 = 1;
            d.tile = v / s2;
            d.slice = v % s2;
            const int lo = find_expert(prefix2, n_active, d.tile);
            d.a = lo;
            const int nbc = (t_rows[lo] + NT2 - 1) / NT2;
            const int local = d.tile - prefix2[lo];
            d.ib = local / nbc;
            d.nb = local % nbc;
            d.kb0 = (d.slice * nkb2) / s2;
            d.kb1 = ((d.slice + 1) * nkb2) / s2;
        }
        return d;
    };

    if (warp == 0) {
        // ---------------- weight (A) producer ----------------
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
                const DecUnit d = decode(u);
                const int64_t slot = t_slot[d.a];
                const int row_a0 = d.phase2 ? static_cast<int>(slot * args.down_rows_per_slot) + d.ib * 128
                                            : static_cast<int>(slot * args.gate_rows_per_slot) + d.ib * 128;
                const int row_a1 = static_cast<int>(slot * args.up_rows_per_slot) + d.ib * 128;
                const uint32_t bytes = d.phase2 ? kDecABytes + NT2 * 128u : 2 * kDecABytes + NB * 128u;
                for (int kb = d.kb0; kb < d.kb1; ++kb) {
                    if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
                    unsigned char* sa = smem + stage * kDecStageBytes;
                    mbar_arrive_expect_tx(&full_bar[stage], bytes);
                    if (d.phase2) {
                        tma_load_2d(sa, &tm_d, &full_bar[stage], kb * 64, row_a0);
                    } else {
                        tma_load_2d(sa, &tm_g, &full_bar[stage], kb * 64, row_a0);
                        tma_load_2d(sa + kDecABytes, &tm_u, &full_bar[stage], kb * 64, row_a1);
                    }
                    if (++stage == kDecStages) { stage = 0; phase ^= 1u; }
                }
            }
        }
        __syncwarp();
    } else if (warp == 6) {
        // ---------------- token (B) producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
                const DecUnit d = decode(u);
                int row_b = DIRECT ? 0 : t_seg0[d.a] + d.nb * NB;
                if (d.phase2) {
                    // this expert's h rows: wait until every phase-1 tile of it is
                    // stored (four quadrant warps per tile)
                    const unsigned int h_target =
                        4u * static_cast<unsigned int>(DIRECT ? m1 : m1 * ((t_rows[d.a] + NB - 1) / NB));
                    const unsigned int* flag = args.h_ready + d.a;
                    if (ld_acquire_gpu(flag) < h_target) {
                        const unsigned long long t0 = global_timer_ns();
                        for (uint32_t it = 1;; ++it) {
                            __nanosleep(64);
                            if (ld_acquire_gpu(flag) >= h_target) break;
                            if ((it & 63u) == 0) {
                                if (*abort_flag) { ok = false; break; }
                                if (global_timer_ns() - t0 > kWaitLimitNs) {
                                    *abort_flag = 1;
                                    raise_error(PDX_DEVERR_WAIT_TIMEOUT);
                                    ok = false;
                                    break;
                                }
                            }
                        }
                        if (!ok) break;
                    }
                    fence_proxy_async_global();
                    row_b = t_seg0[d.a] + d.nb * NT2;
                }
                for (int kb = d.kb0; kb < d.kb1; ++kb) {
                    if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
                    unsigned char* sb = smem + stage * kDecStageBytes + 2 * kDecABytes;
                    if (d.phase2)
                        tma_load_2d(sb, &tm_h, &full_bar[stage], kb * 64, row_b);
                    else
                        tma_load_2d(sb, &tm_x, &full_bar[stage], kb * 64, row_b);
                    if (++stage == kDecStages) { stage = 0; phase ^= 1u; }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc1 = bf16_idesc(128, NB);
        constexpr uint32_t idesc2 = bf16_idesc(128, NT2);
        int stage = 0;
        uint32_t phase = 0;
        int lt = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++lt) {
            const DecUnit d = decode(u);
            const int b = lt & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
            if (!mbar_wait(&tmem_empty[b], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_acc = tmem_base + static_cast<uint32_t>(b * 128);
            for (int kb = d.kb0; kb < d.kb1; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t sa = smem_u32(smem + stage * kDecStageBytes);
                    const uint64_t a0 = sw128_desc(sa);
                    const uint64_t a1 = sw128_desc(sa + kDecABytes);
                    const uint64_t bd = sw128_desc(sa + 2 * kDecABytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t acc = (kb > d.kb0 || kk > 0) ? 1u : 0u;
                        if (d.phase2) {
                            umma_bf16(d_acc, a0 + 2u * kk, bd + 2u * kk, idesc2, acc);
                        } else {
                            umma_bf16(d_acc, a0 + 2u * kk, bd + 2u * kk, idesc1, acc);
                            umma_bf16(d_acc + NB, a1 + 2u * kk, bd + 2u * kk, idesc1, acc);
                        }
                    }
                    umma_commit(&empty_bar[stage]);
                }
                __syncwarp();
                if (++stage == kDecStages) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            if (elect_one()) umma_commit(&tmem_full[b]);
            __syncwarp();
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;
        const int i_row = q * 32 + static_cast<int>(lane);  // weight row within the tile
        int lt = 0;
        for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++lt) {
            const DecUnit d = decode(u);
            const int b = lt & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
            if (!mbar_wait(&tmem_full[b], acc_phase, abort_flag)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 128);
            const int seg0 = t_seg0[d.a];
            const int ne = t_rows[d.a];
            if (!d.phase2 && !DIRECT) {
                // gate columns [0, NB), up columns [NB, 2 NB): rows seg0 + nb*NB + t
                float acc[2 * NB];
#pragma unroll
                for (int c = 0; c < 2 * NB; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(taddr + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[c + j] = __uint_as_float(r[j]);
                }
                tc_fence_before();
                mbar_arrive(&tmem_empty[b]);
                bool publish = true;
                if (s1 > 1) {
                    float* mine = args.partials1 + static_cast<size_t>(u) * 2 * NB * 128;
#pragma unroll
                    for (int c = 0; c < 2 * NB; ++c) mine[c * 128 + i_row] = acc[c];
                    __threadfence();
                    __syncwarp();
                    unsigned int prev = 0;
                    if (lane == 0) prev = atomicAdd(&args.tickets1[d.tile * 4 + q], 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    publish = prev == static_cast<unsigned int>(s1 - 1);
                    if (publish) {
                        __threadfence();
                        const float* base = args.partials1 + static_cast<size_t>(d.tile) * s1 * 2 * NB * 128;
#pragma unroll
                        for (int c = 0; c < 2 * NB; ++c) acc[c] = __ldcg(base + c * 128 + i_row);
                        for (int s = 1; s < s1; ++s) {
                            const float* p = base + static_cast<size_t>(s) * 2 * NB * 128;
#pragma unroll
                            for (int c = 0; c < 2 * NB; ++c) acc[c] += __ldcg(p + c * 128 + i_row);
                        }
                    }
                }
                if (!publish) continue;
                const int col = d.ib * 128 + i_row;
#pragma unroll
                for (int t = 0; t < NB; ++t) {
                    const int r = d.nb * NB + t;
                    if (r < ne)
                        args.h[static_cast<int64_t>(seg0 + r) * args.I + col] =
                            f2bits(swiglu_bf16(__float_as_uint(acc[t]), __float_as_uint(acc[NB + t])));
                }
                fence_proxy_async_global();
                __threadfence();
                __syncwarp();
                if (lane == 0) red_release_gpu_add(args.h_ready + d.a, 1u);
            } else if (!d.phase2) {
                // gate column tokens[p] and up column NB + tokens[p] of every routed row p
                const int col = d.ib * 128 + i_row;
                float* part = nullptr;
                if (s1 > 1)
                    part = args.partials1 +
                           (static_cast<size_t>(d.ib * s1 + d.slice) * args.rows + seg0) * 256;
                for (int r0 = 0; r0 < ne; r0 += 8) {
                    uint32_t g[8], v[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (r0 + j < ne) {
                            const int tok = s_tok[min(seg0 + r0 + j, kDecMaxRows - 1)];
                            tmem_ld1(taddr + static_cast<uint32_t>(tok), g[j]);
                            tmem_ld1(taddr + static_cast<uint32_t>(NB + tok), v[j]);
                        }
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (r0 + j < ne) {
                            if (s1 > 1) {
                                part[static_cast<size_t>(r0 + j) * 256 + i_row] = __uint_as_float(g[j]);
                                part[static_cast<size_t>(r0 + j) * 256 + 128 + i_row] = __uint_as_float(v[j]);
                            } else {
                                args.h[static_cast<int64_t>(seg0 + r0 + j) * args.I + col] =
                                    f2bits(swiglu_bf16(g[j], v[j]));
                            }
                        }
                }
                tc_fence_before();
                mbar_arrive(&tmem_empty[b]);
                if (s1 > 1) {
                    // per-warp split-K hand-off (no cross-warp barrier); the warp
                    // completing the set adds the slices in order 0..s1-1
                    __threadfence();
                    __syncwarp();
                    unsigned int prev = 0;
                    if (lane == 0) prev = atomicAdd(&args.tickets1[d.tile * 4 + q], 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev != static_cast<unsigned int>(s1 - 1)) continue;
                    __threadfence();
                    const float* base = args.partials1 + (static_cast<size_t>(d.ib * s1) * args.rows + seg0) * 256;
                    const size_t slice_stride = static_cast<size_t>(args.rows) * 256;
                    for (int r = 0; r < ne; ++r) {
                        const float* p = base + static_cast<size_t>(r) * 256 + i_row;
                        float gs = __ldcg(p), us = __ldcg(p + 128);
                        for (int s = 1; s < s1; ++s) {
                            gs += __ldcg(p + s * slice_stride);
                            us += __ldcg(p + s * slice_stride + 128);
                        }
                        args.h[static_cast<int64_t>(seg0 + r) * args.I + col] =
                            f2bits(swiglu_bf16(__float_as_uint(gs), __float_as_uint(us)));
                    }
                }
                // this warp's 32 h columns of the tile are stored: publish them
                fence_proxy_async_global();
                __threadfence();
                __syncwarp();
                if (lane == 0) red_release_gpu_add(args.h_ready + d.a, 1u);
            } else {
                float acc[NT2];
#pragma unroll
                for (int c = 0; c < NT2; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(taddr + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[c + j] = __uint_as_float(r[j]);
                }
                tc_fence_before();
                mbar_arrive(&tmem_empty[b]);
                if (s2 > 1) {
                    const int v = u - units1;
                    float* mine = args.partials2 + static_cast<size_t>(v) * NT2 * 128;
#pragma unroll
                    for (int c = 0; c < NT2; ++c) mine[c * 128 + i_row] = acc[c];
                    __threadfence();
                    __syncwarp();
                    unsigned int prev = 0;
                    if (lane == 0) prev = atomicAdd(&args.tickets2[d.tile * 4 + q], 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev != static_cast<unsigned int>(s2 - 1)) continue;
                    __threadfence();
                    const float* base = args.partials2 + static_cast<size_t>(d.tile) * s2 * NT2 * 128;
#pragma unroll
                    for (int c = 0; c < NT2; ++c) acc[c] = __ldcg(base + c * 128 + i_row);
                    for (int s = 1; s < s2; ++s) {
                        const float* p = base + static_cast<size_t>(s) * NT2 * 128;
#pragma unroll
                        for (int c = 0; c < NT2; ++c) acc[c] += __ldcg(p + c * 128 + i_row);
                    }
                }
                const int seg1 = seg0 + ne;
                const int col = d.ib * 128 + i_row;
#pragma unroll
                for (int t = 0; t < NT2; ++t) {
                    const int row = seg0 + d.nb * NT2 + t;
                    if (row < seg1) args.y[static_cast<int64_t>(row) * args.H + col] = f2bits(acc[t]);
                }
            }
        }
    }

    __syncthreads();
    if (*abort_flag) {
        if (warp == 1) {
            if (elect_one()) umma_commit(drain_bar);
            __syncwarp();
            volatile int never = 0;
            mbar_wait(drain_bar, 0, &never);
        }
        const unsigned long long t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 2000000ull) __nanosleep(1000);
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kDecTmemCols)
                     : "memory");
    }
}

}  // namespace pdx
