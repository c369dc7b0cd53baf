// Decode-path grouped expert FFN: weight-streaming tcgen05 GEMM ("swap AB").
//
// Reference: expert_forward() -- expertbench/adapters/qwen.py:87-90, run per
// routed expert by ExpertExecutor.gpu (expertbench/executor.py:454-488).
//
// At decode each active expert sees a handful of token rows, so the layer is a
// stream of expert weights (9 MiB per expert).  Here the WEIGHTS are the MMA's
// M operand (128 weight rows per tile) and the expert's tokens the N operand
// (NT = 16 or 32 columns).  TMA streams 128x64 weight boxes through a 5-stage
// shared-memory ring, one thread issues tcgen05.mma (M=128, N=NT, K=16) into
// TMEM, and four epilogue warps read the accumulators back (TMEM lane = weight
// row, column = token).  For few experts the K range of each tile is split
// over several CTAs (split-K); the partial FP32 sums go to a workspace and,
// per 32-row quadrant, the warp that takes the last ticket adds the slices in
// order 0..splits-1 -- a fixed order, so results are deterministic -- before
// the BF16 epilogue.
//   GEMM1 (SWIGLU): A = 128 gate rows and the same 128 up rows, B = gathered x
//     rows; h[t, i] = bf16(bf16(silu(bf16(g))) * bf16(u)).
//   GEMM2 (down):   A = 128 rows of Wd, B = h rows; y[t, n] = bf16(acc).
// Every wait is bounded as in k_grouped_gemm (abort flag, drain, dealloc).
#include <cuda.h>

#include "tcgen05.cuh"

namespace pdx {

constexpr int kStreamBM = 128;
constexpr int kStreamBK = 64;
constexpr int kStreamStages = 5;
constexpr int kStreamThreads = 192;
constexpr uint32_t kStreamABytes = kStreamBM * kStreamBK * 2;     // 16 KiB per weight box
constexpr uint32_t kStreamBMaxBytes = 64 * kStreamBK * 2;         // up to 64 token rows
constexpr uint32_t kStreamStageBytes = 2 * kStreamABytes + kStreamBMaxBytes;  // 40 KiB
constexpr uint32_t kStreamTmemCols = 256;
constexpr int kStreamMaxActive = 1024;
// after the stages: barriers (256 B), then four int tables over the active
// experts -- tile prefix, segment start, row count, weight slot
constexpr size_t kStreamSmemBytes =
    1024 + kStreamStages * kStreamStageBytes + 256 + 4 * (kStreamMaxActive + 1) * 4;

struct StreamArgs {
    const int32_t* offsets;
    const int32_t* active;
    const int32_t* slot_of_expert;
    int64_t num_slots;
    int64_t a0_rows_per_slot;  // weight-map rows between slots (gate or down)
    int64_t a1_rows_per_slot;  // (up)
    int K;                     // reduction length
    int m_blocks;              // 128-row weight blocks per expert
    int splits;                // K slices per tile
    uint16_t* out;
    int64_t out_ld;
    float* partials;           // [units][cols][128] when splits > 1
    unsigned int* tickets;     // [tiles * 4] (one per epilogue warp), zero on entry when splits > 1
};

template <int NT, bool SWIGLU>
__global__ void __launch_bounds__(kStreamThreads, 1)
    k_stream_gemm(const __grid_constant__ CUtensorMap tm_a0, const __grid_constant__ CUtensorMap tm_a1,
                  const __grid_constant__ CUtensorMap tm_b, StreamArgs args) {
    static_assert(NT % 16 == 0 && NT <= 64, "token tile");
    constexpr int kCols = SWIGLU ? 2 * NT : NT;
    constexpr uint32_t kABytes = SWIGLU ? 2 * kStreamABytes : kStreamABytes;
    constexpr uint32_t kBBytes = NT * kStreamBK * 2;
    extern __shared__ __align__(1024) unsigned char smem_stream[];
    const uint32_t raw_addr = smem_u32(smem_stream);
    unsigned char* smem = smem_stream + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kStreamStages * kStreamStageBytes);
    uint64_t* empty_bar = full_bar + kStreamStages;
    uint64_t* tmem_full = empty_bar + kStreamStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain_bar = tmem_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* s_misc = reinterpret_cast<int*>(tmem_slot + 2);  // [0] total tiles
    int* prefix = reinterpret_cast<int*>(smem + kStreamStages * kStreamStageBytes + 256);
    int* t_seg0 = prefix + (kStreamMaxActive + 1);
    int* t_rows = t_seg0 + (kStreamMaxActive + 1);
    int* t_slot = t_rows + (kStreamMaxActive + 1);

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();

    const int num_kb = args.K / kStreamBK;
    const int splits = args.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStreamStages; ++s) {
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
        tma_prefetch_desc(&tm_a0);
        if (SWIGLU) tma_prefetch_desc(&tm_a1);
        tma_prefetch_desc(&tm_b);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kStreamTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Everything above is independent of the previous kernel; from here on the
    // routing/packing results (and the previous FFN stage) are read.
    griddep_wait();
    griddep_launch();
    const int n_active = min(args.active[0], kStreamMaxActive);
    // tiles per active expert = m_blocks * ceil(n_e / NT) -> exclusive prefix (warp 2)
    if (warp == 2) {
        const int per = (n_active + 31) / 32;
        const int b = static_cast<int>(lane) * per;
        int local = 0;
        for (int i = 0; i < per; ++i)
            if (b + i < n_active) {
                const int e = args.active[1 + b + i];
                const int seg0 = args.offsets[e];
                const int rows = args.offsets[e + 1] - seg0;
                int64_t slot = args.slot_of_expert ? args.slot_of_expert[e] : e;
                if (slot < 0 || slot >= args.num_slots) {
                    raise_error(PDX_DEVERR_BAD_SLOT);
                    slot = 0;  // keeps the pipeline consistent; the call is flagged invalid
                }
                const int tiles = args.m_blocks * ((rows + NT - 1) / NT);
                prefix[b + i] = tiles;
                t_seg0[b + i] = seg0;
                t_rows[b + i] = rows;
                t_slot[b + i] = static_cast<int>(slot);
                local += tiles;
            }
        int inc = local;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, off);
            if (static_cast<int>(lane) >= off) inc += y;
        }
        int run = inc - local;
        for (int i = 0; i < per; ++i)
            if (b + i < n_active) {
                const int t = prefix[b + i];
                prefix[b + i] = run;
                run += t;
            }
        if (lane == 31) s_misc[0] = inc;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total_units = s_misc[0] * splits;

    // unit u -> tile u / splits (slices of one tile adjacent), slice u % splits;
    // everything needed comes from the shared tables (no global loads per unit)
    auto decode = [&](int u, int& a, int& ib, int& nb, int& kb0, int& kb1) {
        const int tile = u / splits;
        const int s = u % splits;
        int lo = 0, hi = n_active - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
        }
        a = lo;
        const int nbc = (t_rows[lo] + NT - 1) / NT;
        const int local = tile - prefix[lo];
        ib = local / nbc;
        nb = local % nbc;
        kb0 = (s * num_kb) / splits;
        kb1 = ((s + 1) * num_kb) / splits;
        return tile;
    };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
                int a, ib, nb, kb0, kb1;
                decode(u, a, ib, nb, kb0, kb1);
                const int64_t slot = t_slot[a];
                const int row_a0 = static_cast<int>(slot * args.a0_rows_per_slot) + ib * kStreamBM;
                const int row_a1 = static_cast<int>(slot * args.a1_rows_per_slot) + ib * kStreamBM;
                const int row_b = t_seg0[a] + nb * NT;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
                    unsigned char* sa = smem + stage * kStreamStageBytes;
                    mbar_arrive_expect_tx(&full_bar[stage], kABytes + kBBytes);
                    tma_load_2d(sa, &tm_a0, &full_bar[stage], kb * kStreamBK, row_a0);
                    if (SWIGLU) tma_load_2d(sa + kStreamABytes, &tm_a1, &full_bar[stage], kb * kStreamBK, row_a1);
                    tma_load_2d(sa + 2 * kStreamABytes, &tm_b, &full_bar[stage], kb * kStreamBK, row_b);
                    if (++stage == kStreamStages) { stage = 0; phase ^= 1u; }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = bf16_idesc(kStreamBM, NT);
        int stage = 0;
        uint32_t phase = 0;
        int lt = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++lt) {
            int a, ib, nb, kb0, kb1;
            decode(u, a, ib, nb, kb0, kb1);
            const int b = lt & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
            if (!mbar_wait(&tmem_empty[b], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_g = tmem_base + static_cast<uint32_t>(b * 128);
            const uint32_t d_u = d_g + NT;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t sa = smem_u32(smem + stage * kStreamStageBytes);
                    const uint64_t a0 = sw128_desc(sa);
                    const uint64_t a1 = sw128_desc(sa + kStreamABytes);
                    const uint64_t bd = sw128_desc(sa + 2 * kStreamABytes);
#pragma unroll
                    for (int kk = 0; kk < kStreamBK / 16; ++kk) {
                        const uint32_t acc = (kb > kb0 || kk > 0) ? 1u : 0u;
                        umma_bf16(d_g, a0 + 2u * kk, bd + 2u * kk, idesc, acc);
                        if (SWIGLU) umma_bf16(d_u, a1 + 2u * kk, bd + 2u * kk, idesc, acc);
                    }
                    umma_commit(&empty_bar[stage]);
                }
                __syncwarp();
                if (++stage == kStreamStages) { stage = 0; phase ^= 1u; }
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
            int a, ib, nb, kb0, kb1;
            const int tile = decode(u, a, ib, nb, kb0, kb1);
            const int b = lt & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
            if (!mbar_wait(&tmem_full[b], acc_phase, abort_flag)) break;
            tc_fence_after();
            float acc[kCols];
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 128);
#pragma unroll
            for (int c = 0; c < kCols; c += 16) {
                uint32_t r[16];
                tmem_ld16(taddr + c, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[c + j] = __uint_as_float(r[j]);
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[b]);  // accumulator is in registers; let the MMA warp reuse it
            if (splits > 1) {
                // Each epilogue warp owns 32 weight rows of the tile in every
                // slice, so the hand-off is per warp: write this slice's rows,
                // publish, take a ticket; the warp that completes the set adds
                // the slices in order 0..splits-1.  No cross-warp barrier.
                float* mine = args.partials + static_cast<size_t>(u) * kCols * kStreamBM;
#pragma unroll
                for (int c = 0; c < kCols; ++c) mine[c * kStreamBM + i_row] = acc[c];
                __threadfence();
                __syncwarp();
                unsigned int prev = 0;
                if (lane == 0) prev = atomicAdd(&args.tickets[tile * 4 + q], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev != static_cast<unsigned int>(splits - 1)) continue;
                __threadfence();
                const float* base = args.partials + static_cast<size_t>(tile) * splits * kCols * kStreamBM;
#pragma unroll
                for (int c = 0; c < kCols; ++c) acc[c] = __ldcg(base + c * kStreamBM + i_row);
                for (int s = 1; s < splits; ++s) {
                    const float* p = base + static_cast<size_t>(s) * kCols * kStreamBM;
#pragma unroll
                    for (int c = 0; c < kCols; ++c) acc[c] += __ldcg(p + c * kStreamBM + i_row);
                }
            }
            const int seg0 = t_seg0[a];
            const int seg1 = seg0 + t_rows[a];
            const int col = ib * kStreamBM + i_row;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int row = seg0 + nb * NT + t;
                if (row < seg1) {
                    float v;
                    if (SWIGLU) {
                        const float gb = round_bf16(acc[t]);
                        const float ub = round_bf16(acc[NT + t]);
                        const float sv = round_bf16(__fdiv_rn(gb, 1.0f + expf(-gb)));
                        v = sv * ub;
                    } else {
                        v = acc[t];
                    }
                    args.out[static_cast<int64_t>(row) * args.out_ld + col] = f2bits(v);
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kStreamTmemCols)
                     : "memory");
    }
}

}  // namespace pdx
