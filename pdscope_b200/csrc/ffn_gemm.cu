// Prefill-path grouped expert FFN: tcgen05 / TMEM grouped GEMM fed by TMA.
//
// Reference: expert_forward() -- expertbench/adapters/qwen.py:87-90, applied
// per expert to the rows routed to it (ExpertExecutor.gpu,
// expertbench/executor.py:454-488, on the compact grouping of
// expertbench/pdscope_runtime.py:16-39).
//
// One persistent CTA per SM walks a static schedule of output tiles over the
// ragged expert segments (tile = 128 packed rows x N columns of one expert).
//   warp 0      TMA producer: A tile [128 x 64] + B tile [256 x 64] per stage
//   warp 1      MMA issuer: tcgen05.mma.cta_group::1.kind::f16, M=128 N=256
//               K=16, FP32 accumulators in TMEM (two 256-column buffers)
//   warps 2..9  epilogue: tcgen05.ld 32x32b, BF16 rounding, row segments
//               staged through shared memory into 64-byte global stores;
//               two warps per TMEM lane quadrant, each on half of the columns
// GEMM1 (SwiGLU): B = [128 gate rows ; 128 up rows] of the expert, epilogue
//   h = bf16(bf16(silu(bf16(g))) * bf16(u)) -> h[rows, I].
// GEMM2 (down):   B = 256 rows of Wd, epilogue y = bf16(acc) -> y[rows, H].
// Rows of an A tile past the expert's segment belong to the next expert (or
// are TMA zero fill past the end); they are computed but never stored.
// Every mbarrier wait is bounded (2 s); a timeout raises the device error
// word, releases the other roles through a shared abort flag, drains the
// tensor core and frees TMEM before the CTA exits.
#include <cuda.h>

#include "tcgen05.cuh"

namespace pdx {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;   // 64 BF16 = one 128-byte swizzle row
constexpr int kGemmBN = 256;  // MMA N (B rows per stage)
constexpr int kGemmStages = 4;
constexpr int kGemmEpiWarps = 8;                          // two per TMEM lane quadrant
constexpr int kGemmThreads = 64 + 32 * kGemmEpiWarps;      // producer, MMA, epilogue
constexpr int kPairThreads = 192;                          // producer, MMA, 4 epilogue warps
constexpr uint32_t kTileABytes = kGemmBM * kGemmBK * 2;  // 16 KiB
constexpr uint32_t kTileBBytes = kGemmBN * kGemmBK * 2;  // 32 KiB
constexpr uint32_t kStageBytes = kTileABytes + kTileBBytes;
constexpr uint32_t kTmemCols = 512;  // two 256-column FP32 accumulators
constexpr int kMaxActive = 1024;
constexpr uint32_t kEpiStageBytes = 32 * 64;  // one epilogue warp's 32 rows x 32 BF16 columns
constexpr size_t kGemmSmemBytes = 1024 /*alignment slack*/ + kGemmStages * kStageBytes + 256 /*barriers*/ +
                                  4 * (kMaxActive + 1) * 4 /*tile prefix, segment start, rows, slot*/ +
                                  kGemmEpiWarps * kEpiStageBytes /*epilogue staging*/;

struct GemmArgs {
    const int32_t* offsets;
    const int32_t* active;
    const int32_t* slot_of_expert;
    int64_t num_slots;
    int64_t b0_rows_per_slot;  // B-map rows between consecutive slots
    int64_t b1_rows_per_slot;
    int K;                     // reduction length
    int n_cols;                // output columns per expert
    int swiglu;                // 1: GEMM1 with SiLU*up epilogue, 0: down projection
    uint16_t* out;
    int64_t out_ld;
};

// ---- tile schedule ------------------------------------------------------------
struct TileInfo {
    int a;  // index into the active-expert tables
    int m;
    int n;
};

__device__ __forceinline__ TileInfo decode_tile(int tile, const int* prefix, int n_active, int n_tiles) {
    int lo = 0, hi = n_active - 1;  // largest a with prefix[a] <= tile
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    const int local = tile - prefix[lo];
    TileInfo ti;
    ti.a = lo;
    ti.m = local / n_tiles;
    ti.n = local % n_tiles;
    return ti;
}

// Per-active-expert tables of a grouped GEMM (one warp): exclusive prefix of
// output tiles (row tiles of ``bm`` x ``n_tiles`` column tiles), segment start,
// row count and weight slot.  s_misc[0] = total tiles, s_misc[1] = n_active.
__device__ __forceinline__ void build_tile_tables(const GemmArgs& args, int n_active, int n_tiles, int bm,
                                                  int* prefix, int* t_seg0, int* t_rows, int* t_slot, int* s_misc) {
    const uint32_t lane = lane_id();
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
            const int tiles = ((rows + bm - 1) / bm) * n_tiles;
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
    if (lane == 31) { s_misc[0] = inc; s_misc[1] = n_active; }
}

// Orders the use of registers filled by tcgen05.ld after tcgen05.wait::ld: the
// empty asm statements follow the (volatile) wait and their outputs are what
// the conversion reads.
template <int N>
__device__ __forceinline__ void tmem_wait_pin(uint32_t (&r)[N]) {
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// One 32 x 32 BF16 slab of output through this warp's shared-memory staging
// buffer: lane r holds row r's 32 columns (packed, 16 words) and writes them
// as four 16-byte chunks (chunk q of row r at r*64 + (q ^ ((r >> 1) & 3))*16,
// conflict-free); after the warp sync, lane l stores chunk l & 3 of rows
// (l >> 2) + 8i, i = 0..3, so every four lanes write one 64-byte row segment.
// Rows >= n_valid (past the expert's segment) are not stored.
__device__ __forceinline__ void store_slab(const uint32_t (&packed)[16], unsigned char* sbuf, uint16_t* out0,
                                           int64_t ld, int col, int n_valid) {
    const uint32_t lane = lane_id();
    const uint32_t base = smem_u32(sbuf);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t a = base + lane * 64u + ((static_cast<uint32_t>(q) ^ ((lane >> 1) & 3u)) * 16u);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(packed[4 * q]), "r"(packed[4 * q + 1]),
                     "r"(packed[4 * q + 2]), "r"(packed[4 * q + 3])
                     : "memory");
    }
    __syncwarp();
    const uint32_t cc = lane & 3u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t r = (lane >> 2) + 8u * i;
        const uint32_t a = base + r * 64u + ((cc ^ ((r >> 1) & 3u)) * 16u);
        uint4 v;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
        if (static_cast<int>(r) < n_valid)
            *reinterpret_cast<uint4*>(out0 + static_cast<int64_t>(r) * ld + col + cc * 8) = v;
    }
    __syncwarp();
}

// Columns [c0, c0 + nc) of this warp's 32 accumulator rows (TMEM lanes of its
// quadrant) -> BF16 output rows out0 + r*ld, through the staging buffer so
// the global stores are whole 64-byte row segments (the row-per-lane form
// writes 16 bytes to 32 different rows per store instruction).
// swiglu: accumulator columns [0,128) hold gate, [128,256) up.
__device__ __forceinline__ void epilogue_cols_staged(int swiglu, uint32_t taddr, uint16_t* out0, int64_t ld,
                                                     int n_valid, int c0, int nc, unsigned char* sbuf) {
    if (swiglu) {
#pragma unroll 1
        for (int c = c0; c < c0 + nc; c += 32) {
            uint32_t g[32], u[32];
            tmem_ld16(taddr + c, g);
            tmem_ld16(taddr + c + 16, g + 16);
            tmem_ld16(taddr + kGemmBN / 2 + c, u);
            tmem_ld16(taddr + kGemmBN / 2 + c + 16, u + 16);
            tmem_wait_pin(g);
            tmem_wait_pin(u);
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                float hv[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const float gb = round_bf16(__uint_as_float(g[i + j]));
                    const float ub = round_bf16(__uint_as_float(u[i + j]));
                    const float sv = round_bf16(__fdiv_rn(gb, 1.0f + expf(-gb)));
                    hv[j] = sv * ub;
                }
                packed[i / 2] = static_cast<uint32_t>(f2bits(hv[0])) | (static_cast<uint32_t>(f2bits(hv[1])) << 16);
            }
            store_slab(packed, sbuf, out0, ld, c, n_valid);
        }
    } else {
#pragma unroll 1
        for (int c = c0; c < c0 + nc; c += 64) {
            uint32_t v[64];
#pragma unroll
            for (int i = 0; i < 4; ++i) tmem_ld16(taddr + c + 16 * i, v + 16 * i);
            tmem_wait_pin(v);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t packed[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2)
                    packed[i / 2] = static_cast<uint32_t>(f2bits(__uint_as_float(v[32 * h + i]))) |
                                    (static_cast<uint32_t>(f2bits(__uint_as_float(v[32 * h + i + 1]))) << 16);
                store_slab(packed, sbuf, out0, ld, c + 32 * h, n_valid);
            }
        }
    }
}


__global__ void __launch_bounds__(kGemmThreads, 1)
    k_grouped_gemm(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b0,
                   const __grid_constant__ CUtensorMap tm_b1, GemmArgs args) {
    extern __shared__ __align__(1024) unsigned char smem_gemm[];
    // 1024-byte aligned stage buffers (SWIZZLE_128B atoms)
    const uint32_t raw_addr = smem_u32(smem_gemm);
    unsigned char* smem = smem_gemm + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kGemmStages * kStageBytes);
    uint64_t* empty_bar = full_bar + kGemmStages;
    uint64_t* tmem_full = empty_bar + kGemmStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain_bar = tmem_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* s_misc = reinterpret_cast<int*>(tmem_slot + 2);  // [0] = total tiles, [1] = n_active
    int* prefix = reinterpret_cast<int*>(smem + kGemmStages * kStageBytes + 256);
    int* t_seg0 = prefix + (kMaxActive + 1);
    int* t_rows = t_seg0 + (kMaxActive + 1);
    int* t_slot = t_rows + (kMaxActive + 1);
    unsigned char* epi_stage = reinterpret_cast<unsigned char*>(t_slot + (kMaxActive + 1));  // [8][32 x 64 B]

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();

    const int out_cols_per_tile = args.swiglu ? kGemmBN / 2 : kGemmBN;
    const int n_tiles = args.n_cols / out_cols_per_tile;
    const int num_kb = args.K / kGemmBK;

    // -- setup: barriers, TMEM, tile prefix ------------------------------------
    if (threadIdx.x == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 32 * kGemmEpiWarps);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b0);
        if (args.swiglu) tma_prefetch_desc(&tm_b1);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Everything above is independent of the previous kernel; from here on the
    // routing/packing results (and the previous FFN stage) are read.
    griddep_wait();
    griddep_launch();
    const int n_active = min(args.active[0], kMaxActive);
    if (warp == 2) build_tile_tables(args, n_active, n_tiles, kGemmBM, prefix, t_seg0, t_rows, t_slot, s_misc);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total_tiles = s_misc[0];

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
                const TileInfo ti = decode_tile(tile, prefix, n_active, n_tiles);
                const int64_t slot = t_slot[ti.a];
                const int row_a = t_seg0[ti.a] + ti.m * kGemmBM;
                const int row_b0 = static_cast<int>(slot * args.b0_rows_per_slot) + ti.n * out_cols_per_tile;
                const int row_b1 = static_cast<int>(slot * args.b1_rows_per_slot) + ti.n * out_cols_per_tile;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
                    unsigned char* sa = smem + stage * kStageBytes;
                    unsigned char* sb = sa + kTileABytes;
                    mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
                    tma_load_2d(sa, &tm_a, &full_bar[stage], kb * kGemmBK, row_a);
                    if (args.swiglu) {
                        tma_load_2d(sb, &tm_b0, &full_bar[stage], kb * kGemmBK, row_b0);
                        tma_load_2d(sb + kTileBBytes / 2, &tm_b1, &full_bar[stage], kb * kGemmBK, row_b1);
                    } else {
                        tma_load_2d(sb, &tm_b0, &full_bar[stage], kb * kGemmBK, row_b0);
                    }
                    if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = bf16_idesc(kGemmBM, kGemmBN);
        int stage = 0;
        uint32_t phase = 0;
        int lt = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++lt) {
            const int b = lt & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
            if (!mbar_wait(&tmem_empty[b], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * kGemmBN);
            for (int kb = 0; kb < num_kb; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t sa = smem_u32(smem + stage * kStageBytes);
                    const uint32_t sb = sa + kTileABytes;
                    const uint64_t a0 = sw128_desc(sa), b0 = sw128_desc(sb);
#pragma unroll
                    for (int kk = 0; kk < kGemmBK / 16; ++kk)
                        umma_bf16(d_tmem, a0 + 2u * kk, b0 + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
                    umma_commit(&empty_bar[stage]);
                }
                __syncwarp();
                if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            if (elect_one()) umma_commit(&tmem_full[b]);
            __syncwarp();
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int half = (warp - 2) >> 2;  // which half of the tile's columns
        const int half_cols = (args.swiglu ? kGemmBN / 2 : kGemmBN) / 2;
        int lt = 0;
        for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++lt) {
            const int b = lt & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
            if (!mbar_wait(&tmem_full[b], acc_phase, abort_flag)) break;
            tc_fence_after();
            const TileInfo ti = decode_tile(tile, prefix, n_active, n_tiles);
            const int seg0 = t_seg0[ti.a];
            const int n_e = t_rows[ti.a];
            const int r0 = ti.m * kGemmBM + q * 32;   // first row of this warp's lane quadrant
            uint16_t* out0 = args.out + static_cast<int64_t>(seg0 + r0) * args.out_ld + ti.n * out_cols_per_tile;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * kGemmBN);
            epilogue_cols_staged(args.swiglu, taddr, out0, args.out_ld, min(32, n_e - r0), half * half_cols, half_cols,
                                 epi_stage + (warp - 2) * kEpiStageBytes);
            tc_fence_before();
            mbar_arrive(&tmem_empty[b]);
        }
    }

    // -- teardown -------------------------------------------------------------------
    __syncthreads();
    if (*abort_flag) {
        // Let in-flight TMA copies land and the tensor core finish before the
        // shared memory and TMEM of this CTA are released.
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

// ---- CTA-pair variant: 256 x 256 output tiles (tcgen05 cta_group::2) -------------
//
// A cluster of two CTAs on two SMs computes one 256-row x 256-column tile per
// step.  Each CTA stages its own 128 rows of A and half of B's 256 rows (the
// gate half or the up half in the SwiGLU GEMM, rows n0..n0+127 or
// n0+128..n0+255 of Wd in the down GEMM), so per MMA K-block a CTA moves
// 32 KiB instead of the 48 KiB of the single-CTA 128 x 256 tile: a third less
// L2-to-SM traffic per FLOP.  The even CTA (rank 0) issues the MMAs for both;
// each CTA's TMEM holds its own 128 rows of the accumulator.
//   full_bar   rank 0 only; both CTAs' TMA loads count their bytes on it
//   empty_bar  in each CTA; rank 0's MMA commits to both
//   tmem_full  in each CTA; rank 0's MMA commits to both
//   tmem_empty rank 0 only; one arrival per epilogue warp of either CTA (8)
// Each CTA's TMA loads fill only its own shared memory.  Every wait is
// bounded; a timeout sets the abort flag of both CTAs.
constexpr int kPairStages = 6;
constexpr uint32_t kPairTileA = 128 * kGemmBK * 2;  // 16 KiB: this CTA's 128 rows of A
constexpr uint32_t kPairTileB = 128 * kGemmBK * 2;  // 16 KiB: this CTA's half of B
constexpr uint32_t kPairStageBytes = kPairTileA + kPairTileB;
constexpr int kPairBM = 256;
constexpr size_t kGemmPairSmemBytes = 1024 + kPairStages * kPairStageBytes + 256 + 4 * (kMaxActive + 1) * 4 +
                                      4 * kEpiStageBytes /*epilogue staging, one buffer per epilogue warp*/;

__device__ __forceinline__ void pair_abort(volatile int* abort_flag, uint32_t peer_abort_addr) {
    *abort_flag = 1;
    st_shared_remote_u32(peer_abort_addr, 1u);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    k_grouped_gemm_pair(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b0,
                        const __grid_constant__ CUtensorMap tm_b1, GemmArgs args) {
    extern __shared__ __align__(1024) unsigned char smem_pair[];
    // identical offsets in both CTAs: the MMA reads the peer's stage at the same address
    const uint32_t raw_addr = smem_u32(smem_pair);
    unsigned char* smem = smem_pair + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
    uint64_t* empty_bar = full_bar + kPairStages;
    uint64_t* tmem_full = empty_bar + kPairStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain_bar = tmem_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* s_misc = reinterpret_cast<int*>(tmem_slot + 2);
    int* prefix = reinterpret_cast<int*>(smem + kPairStages * kPairStageBytes + 256);
    int* t_seg0 = prefix + (kMaxActive + 1);
    int* t_rows = t_seg0 + (kMaxActive + 1);
    int* t_slot = t_rows + (kMaxActive + 1);
    unsigned char* epi_stage = reinterpret_cast<unsigned char*>(t_slot + (kMaxActive + 1));  // [4][32 x 64 B]

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();
    const uint32_t crank = cluster_ctarank();
    const uint32_t peer = crank ^ 1u;
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int n_pairs = static_cast<int>(gridDim.x >> 1);
    const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<int*>(abort_flag)), peer);

    const int out_cols_per_tile = args.swiglu ? kGemmBN / 2 : kGemmBN;
    const int n_tiles = args.n_cols / out_cols_per_tile;
    const int num_kb = args.K / kGemmBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 8);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b0);
        if (args.swiglu) tma_prefetch_desc(&tm_b1);
    }
    if (warp == 1) {  // same warp in both CTAs allocates the pair's TMEM
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    griddep_wait();
    griddep_launch();
    const int n_active = min(args.active[0], kMaxActive);
    if (warp == 2) build_tile_tables(args, n_active, n_tiles, kPairBM, prefix, t_seg0, t_rows, t_slot, s_misc);
    tc_fence_before();
    cluster_sync_all();  // barriers of both CTAs initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total_tiles = s_misc[0];
    // rank 0's barriers, addressed from either CTA
    const uint32_t full0 = mapa_shared(smem_u32(full_bar), 0);
    const uint32_t tmem_empty0 = mapa_shared(smem_u32(tmem_empty), 0);

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = pair; tile < total_tiles && ok; tile += n_pairs) {
                const TileInfo ti = decode_tile(tile, prefix, n_active, n_tiles);
                const int64_t slot = t_slot[ti.a];
                const int row_a = t_seg0[ti.a] + ti.m * kPairBM + static_cast<int>(crank) * 128;
                // SwiGLU: rank 0 stages 128 gate rows (tm_b0), rank 1 the matching 128
                // up rows (tm_b1).  Down: rows n0..n0+127 / n0+128..n0+255 of Wd (tm_b0).
                const bool use_b1 = args.swiglu && crank == 1;
                int row_b;
                if (args.swiglu)
                    row_b = static_cast<int>(slot * (crank ? args.b1_rows_per_slot : args.b0_rows_per_slot)) +
                            ti.n * out_cols_per_tile;
                else
                    row_b = static_cast<int>(slot * args.b0_rows_per_slot) + ti.n * kGemmBN +
                            static_cast<int>(crank) * 128;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
                        pair_abort(abort_flag, peer_abort);
                        ok = false;
                        break;
                    }
                    unsigned char* sa = smem + stage * kPairStageBytes;
                    if (crank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * kPairStageBytes);
                    const uint32_t fb = full0 + static_cast<uint32_t>(stage) * 8u;
                    tma_load_2d_pair(sa, &tm_a, fb, kb * kGemmBK, row_a);
                    if (use_b1)
                        tma_load_2d_pair(sa + kPairTileA, &tm_b1, fb, kb * kGemmBK, row_b);
                    else
                        tma_load_2d_pair(sa + kPairTileA, &tm_b0, fb, kb * kGemmBK, row_b);
                    if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
                }
            }
            // tail: every stage's last release (a commit from rank 0) has landed
            // before this CTA's shared memory can go away
            for (int i = 0; i < kPairStages && ok; ++i) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
                    pair_abort(abort_flag, peer_abort);
                    break;
                }
                if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (rank 0 only) ----------------
        if (crank == 0) {
            constexpr uint32_t idesc = bf16_idesc(kPairBM, kGemmBN);
            const uint32_t empty_local = smem_u32(empty_bar), empty_peer = mapa_shared(empty_local, 1);
            const uint32_t tfull_local = smem_u32(tmem_full), tfull_peer = mapa_shared(tfull_local, 1);
            int stage = 0;
            uint32_t phase = 0;
            int lt = 0;
            bool ok = true;
            for (int tile = pair; tile < total_tiles && ok; tile += n_pairs, ++lt) {
                const int b = lt & 1;
                const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
                if (!mbar_wait(&tmem_empty[b], acc_phase ^ 1u, abort_flag)) {
                    pair_abort(abort_flag, peer_abort);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * kGemmBN);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
                        pair_abort(abort_flag, peer_abort);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (elect_one()) {
                        const uint32_t sa = smem_u32(smem + stage * kPairStageBytes);
                        const uint64_t a0 = sw128_desc(sa), b0 = sw128_desc(sa + kPairTileA);
#pragma unroll
                        for (int kk = 0; kk < kGemmBK / 16; ++kk)
                            umma_bf16_pair(d_tmem, a0 + 2u * kk, b0 + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
                        umma_commit_pair(empty_local + static_cast<uint32_t>(stage) * 8u);
                        umma_commit_pair(empty_peer + static_cast<uint32_t>(stage) * 8u);
                    }
                    __syncwarp();
                    if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                if (elect_one()) {
                    umma_commit_pair(tfull_local + static_cast<uint32_t>(b) * 8u);
                    umma_commit_pair(tfull_peer + static_cast<uint32_t>(b) * 8u);
                }
                __syncwarp();
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
        const int q = warp & 3;
        const int row0_in_tile = static_cast<int>(crank) * 128 + q * 32;   // this warp's first row
        int lt = 0;
        for (int tile = pair; tile < total_tiles; tile += n_pairs, ++lt) {
            const int b = lt & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(lt >> 1) & 1u;
            if (!mbar_wait(&tmem_full[b], acc_phase, abort_flag)) {
                pair_abort(abort_flag, peer_abort);
                break;
            }
            tc_fence_after();
            const TileInfo ti = decode_tile(tile, prefix, n_active, n_tiles);
            const int seg0 = t_seg0[ti.a];
            const int n_e = t_rows[ti.a];
            const int r0 = ti.m * kPairBM + row0_in_tile;
            uint16_t* out0 = args.out + static_cast<int64_t>(seg0 + r0) * args.out_ld + ti.n * out_cols_per_tile;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * kGemmBN);
            epilogue_cols_staged(args.swiglu, taddr, out0, args.out_ld, min(32, n_e - r0), 0,
                                 args.swiglu ? kGemmBN / 2 : kGemmBN, epi_stage + (warp - 2) * kEpiStageBytes);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tmem_empty0 + static_cast<uint32_t>(b) * 8u);
        }
    }

    // -- teardown -------------------------------------------------------------------
    // The peer may raise this CTA's abort flag at any time, so every thread acts
    // on one snapshot taken after the roles have finished.
    __syncthreads();
    if (threadIdx.x == 0) s_misc[2] = *abort_flag;
    if (warp == 1 && crank == 0) {
        // rank 0: every MMA it issued has completed (a no-op wait on the normal path)
        if (elect_one()) umma_commit_pair(smem_u32(drain_bar));
        __syncwarp();
        volatile int never = 0;
        mbar_wait(drain_bar, 0, &never);
    }
    __syncthreads();
    if (s_misc[2]) {
        // let this CTA's in-flight TMA copies land before its shared memory is released
        const unsigned long long t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 2000000ull) __nanosleep(1000);
    }
    tc_fence_before();
    cluster_sync_all();  // no remote arrival or MMA read of this CTA's memory is still pending
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace pdx
