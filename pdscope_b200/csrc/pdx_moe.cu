// libpdx_moe.so: the C ABI declared in include/pdx_moe.h.
//
// Unity build: the kernel files are included here so the whole library is
// one translation unit (one copy of the device error word, no -rdc).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <utility>

#include "combine.cu"
#include "ffn_decode.cu"
#include "ffn_gemm.cu"
#include "ffn_gemv.cu"
#include "ffn_stream.cu"
#include "pack.cu"
#include "ep.cu"
#include "ep_p2p.cu"
#include "route.cu"

namespace pdx {
namespace {

thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};
// Wall-time limit of the peer-exchange flag waits (k_ep_layout_p2p,
// k_ep_wait_back), read when those kernels are launched (or captured).
constexpr uint64_t kMaxFlagWaitNs = 60000000000ull;  // 60 s
std::atomic<uint64_t> g_flag_wait_ns{kWaitLimitNs};

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return status;
}

int ok() {
    t_last_error.clear();
    return PDX_OK;
}

#define PDX_CUDA_TRY(expr)                                                                   \
    do {                                                                                     \
        cudaError_t _e = (expr);                                                             \
        if (_e != cudaSuccess) return fail(PDX_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
    } while (0)

#define PDX_LAUNCHED()                                                                              \
    do {                                                                                            \
        g_launches.fetch_add(1, std::memory_order_relaxed);                                         \
        cudaError_t _e = cudaGetLastError();                                                        \
        if (_e != cudaSuccess) return fail(PDX_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(_e)); \
    } while (0)

// Launch with programmatic stream serialisation (PDL): the kernel may begin
// while its predecessor in the stream is still running; it synchronises with
// griddep_wait() before touching the predecessor's results.  The overlap pays
// for the short decode kernels; prefill-size launches (hundreds of µs each)
// clear g_pdl_enabled so an early-launched dependent (e.g. a 10^5-CTA row
// gather) never holds SM resources the next GEMM's CTA pairs are waiting for.
#ifndef PDX_PREFILL_PDL
#define PDX_PREFILL_PDL 0
#endif
thread_local bool g_pdl_enabled = true;
struct PdlScope {
    bool saved;
    explicit PdlScope(bool on) : saved(g_pdl_enabled) { g_pdl_enabled = on; }
    ~PdlScope() { g_pdl_enabled = saved; }
};
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl_enabled ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define PDX_PDL_TRY(expr)                                                                             \
    do {                                                                                              \
        g_launches.fetch_add(1, std::memory_order_relaxed);                                           \
        cudaError_t _e = (expr);                                                                      \
        if (_e != cudaSuccess) return fail(PDX_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(_e)); \
    } while (0)

// k_combine_norm with the values-per-thread instance the row length needs.
template <typename... Args>
cudaError_t launch_combine_norm(int64_t H, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
    if (H <= 8 * kCombineThreads)
        return launch_pdl(k_combine_norm<8>, grid, block, smem, stream, std::forward<Args>(args)...);
    if (H <= 16 * kCombineThreads)
        return launch_pdl(k_combine_norm<16>, grid, block, smem, stream, std::forward<Args>(args)...);
    return launch_pdl(k_combine_norm<kLnMaxPerThread>, grid, block, smem, stream, std::forward<Args>(args)...);
}

constexpr size_t kAlign = 256;
// SM count the launch plans assume (B200), so that a workspace query and the
// launch it sizes always agree; the plans only shape the work, not results.
constexpr int kPlanSMs = 148;
constexpr int kMaxExperts = 1024;
inline size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Row gather grid: one warp per row, at most 8 CTAs per SM resident at once.
inline dim3 gather_grid(int64_t rows) {
    return dim3(static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((rows + kGatherWarps - 1) / kGatherWarps,
                                                                             8 * kPlanSMs))));
}

// Bump allocator over the caller's workspace.
struct Carver {
    char* base;
    size_t cap;
    size_t used = 0;
    bool overflow = false;
    void* take(size_t bytes) {
        const size_t off = used;
        used = align_up(used + bytes);
        if (used > cap) overflow = true;
        return base ? base + off : nullptr;
    }
};

constexpr int kMaxDevices = 64;
int g_num_sms[kMaxDevices] = {0};
int g_pair_clusters[kMaxDevices] = {0};

int cur_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    return (dev >= 0 && dev < kMaxDevices) ? dev : 0;
}
bool g_attrs_set[kMaxDevices] = {false};
std::mutex g_dev_mutex;

int device_setup(int* sms_out) {
    int dev = 0;
    PDX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(PDX_ERR_UNSUPPORTED, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!g_attrs_set[dev]) {
        int sms = 0;
        PDX_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        int major = 0;
        PDX_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10) return fail(PDX_ERR_UNSUPPORTED, "pdx_moe is built for sm_100a; device %d is sm_%d", dev, major);
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_grouped_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kGemmSmemBytes)));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_pack_scan_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>((11 * kMaxExperts + 1 + kPackScanSmemInts) * 4)));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_router_logits_dmma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kDmmaSmemBytes)));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_grouped_gemm_pair, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kGemmPairSmemBytes)));
        {   // CTA pairs that can be resident at once (one CTA per SM)
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * (sms / 2));
            cfg.blockDim = dim3(kPairThreads);
            cfg.dynamicSmemBytes = kGemmPairSmemBytes;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, k_grouped_gemm_pair, &cfg) != cudaSuccess || clusters < 1) {
                cudaGetLastError();
                clusters = sms / 2;
            }
            g_pair_clusters[dev] = std::min(clusters, sms / 2);
        }
        const int gemv_smem = 128 * 1024;
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_gateup_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemv_smem));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_gateup_gemv<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemv_smem));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_down_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemv_smem));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_down_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemv_smem));
        const int ss = static_cast<int>(kStreamSmemBytes);
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_stream_gemm<16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_stream_gemm<16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_stream_gemm<32, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_stream_gemm<32, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_stream_gemm<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        PDX_CUDA_TRY(cudaFuncSetAttribute(k_stream_gemm<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        const int ds = static_cast<int>(kDecSmemBytes);
#define PDX_DEC_ATTR(D, NB, NT2) \
    PDX_CUDA_TRY(cudaFuncSetAttribute(k_decode_ffn<D, NB, NT2>, cudaFuncAttributeMaxDynamicSharedMemorySize, ds))
        PDX_DEC_ATTR(true, 16, 16); PDX_DEC_ATTR(true, 16, 32); PDX_DEC_ATTR(true, 16, 64);
        PDX_DEC_ATTR(true, 32, 16); PDX_DEC_ATTR(true, 32, 32); PDX_DEC_ATTR(true, 32, 64);
        PDX_DEC_ATTR(true, 64, 16); PDX_DEC_ATTR(true, 64, 32); PDX_DEC_ATTR(true, 64, 64);
        PDX_DEC_ATTR(false, 16, 16); PDX_DEC_ATTR(false, 32, 32); PDX_DEC_ATTR(false, 64, 64);
#undef PDX_DEC_ATTR
        g_num_sms[dev] = sms;
        g_attrs_set[dev] = true;
    }
    *sms_out = g_num_sms[dev];
    return PDX_OK;
}

// ---- TMA descriptors -------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int encode_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return fail(PDX_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(PDX_ERR_INVALID, "TMA base not 16-byte aligned");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGemmBK), box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PDX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return PDX_OK;
}

// ---- shape checks -----------------------------------------------------------------
constexpr int kMaxTopK = 32;
constexpr int64_t kTailMaxTokens = 64;     // fused route tail up to this many tokens
constexpr int64_t kPackSingleMax = 1024;   // single-CTA pack up to this many assignments (4 scatter rounds)
constexpr int64_t kStreamMaxRowsPerExpert = 48;  // auto mode: weight streaming up to this average

int check_route_shape(int64_t T, int64_t H, int64_t E, int32_t k) {
    if (T < 1) return fail(PDX_ERR_INVALID, "empty expert routing (T=%lld)", static_cast<long long>(T));
    if (E < 1 || k < 1 || k > E) return fail(PDX_ERR_INVALID, "invalid routing parameters (E=%lld, top_k=%d)",
                                             static_cast<long long>(E), k);
    if (E > kMaxExperts) return fail(PDX_ERR_UNSUPPORTED, "E=%lld > %d experts", static_cast<long long>(E), kMaxExperts);
    if (k > kMaxTopK) return fail(PDX_ERR_UNSUPPORTED, "top_k=%d > %d", k, kMaxTopK);
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "hidden size %lld must be a positive multiple of 8",
                                    static_cast<long long>(H));
    if (T * k >= (int64_t(1) << 31) || T * E >= (int64_t(1) << 40))
        return fail(PDX_ERR_UNSUPPORTED, "T=%lld too large", static_cast<long long>(T));
    return PDX_OK;
}

bool gemm_shape_ok(int64_t H, int64_t I) { return H % 256 == 0 && I % 128 == 0 && H >= 256 && I >= 128; }
bool is_gemm_mode(int mode) { return mode == PDX_FFN_GEMM || mode == PDX_FFN_GEMM_1CTA || mode == PDX_FFN_GEMM_PAIR; }
bool stream_shape_ok(int64_t H, int64_t I) { return H % 128 == 0 && I % 128 == 0 && H >= 128 && I >= 128; }

// Auto mode picks the path from the average rows per expert: the
// weight-streaming path reads each active expert's weights once per 16/32/64-row
// token tile, the token-tiled GEMM once per 128-row tile at full tensor-core
// tile efficiency.  Measured on one Qwen3-30B-A3B layer (E=128, k=8, CUDA-graph
// replay): streaming is ahead up to T = 512 (32 rows per expert: 265 vs 272 us),
// the GEMM from T = 1024 (64 rows per expert: 294 vs 309 us) on.
int resolve_mode(int32_t mode, int64_t rows, int64_t E, int64_t H, int64_t I) {
    if (mode != PDX_FFN_AUTO) return mode;
    const bool few_rows = rows <= kStreamMaxRowsPerExpert * std::max<int64_t>(E, 1);
    if (!few_rows && gemm_shape_ok(H, I)) return PDX_FFN_GEMM;
    if (stream_shape_ok(H, I)) return PDX_FFN_GEMV;
    if (gemm_shape_ok(H, I)) return PDX_FFN_GEMM;
    return PDX_FFN_SIMT;
}

int check_ffn_shape(int64_t H, int64_t I, int32_t mode) {
    if (H < 8 || I < 8 || H % 8 || I % 8)
        return fail(PDX_ERR_UNSUPPORTED, "H=%lld, I=%lld must be positive multiples of 8", static_cast<long long>(H),
                    static_cast<long long>(I));
    if (mode == PDX_FFN_SIMT) {
        if (I % 16 || H % 32)
            return fail(PDX_ERR_UNSUPPORTED, "SIMT path needs I %% 16 == 0 and H %% 32 == 0");
        if (H > 4096 || I > 4096)
            return fail(PDX_ERR_UNSUPPORTED, "SIMT path supports H, I <= 4096");
    } else if (mode == PDX_FFN_GEMV || mode == PDX_FFN_GEMV_STAGED) {
        if (!stream_shape_ok(H, I))
            return fail(PDX_ERR_UNSUPPORTED, "weight-streaming path needs H %% 128 == 0 and I %% 128 == 0");
    } else if (is_gemm_mode(mode)) {
        if (!gemm_shape_ok(H, I))
            return fail(PDX_ERR_UNSUPPORTED, "tcgen05 path needs H %% 256 == 0 and I %% 128 == 0");
    } else {
        return fail(PDX_ERR_INVALID, "unknown FFN mode %d", mode);
    }
    return PDX_OK;
}

int check_weights(const pdx_expert_weights* w, int64_t H, int64_t I) {
    if (!w || !w->gate || !w->up || !w->down) return fail(PDX_ERR_INVALID, "expert weights missing");
    if (w->num_slots < 1) return fail(PDX_ERR_INVALID, "num_slots must be >= 1");
    if (w->num_slots > 1 && (w->gate_stride % H || w->up_stride % H || w->down_stride % I ||
                             w->gate_stride < I * H || w->up_stride < I * H || w->down_stride < H * I))
        return fail(PDX_ERR_INVALID, "slot strides must be multiples of the row length and cover one expert");
    if ((reinterpret_cast<uintptr_t>(w->gate) | reinterpret_cast<uintptr_t>(w->up) |
         reinterpret_cast<uintptr_t>(w->down)) & 15u)
        return fail(PDX_ERR_INVALID, "expert weights must be 16-byte aligned");
    return PDX_OK;
}

ExpertSlab to_slab(const pdx_expert_weights* w) {
    ExpertSlab s;
    s.gate = static_cast<const uint16_t*>(w->gate);
    s.up = static_cast<const uint16_t*>(w->up);
    s.down = static_cast<const uint16_t*>(w->down);
    s.gate_stride = w->gate_stride;
    s.up_stride = w->up_stride;
    s.down_stride = w->down_stride;
    s.num_slots = w->num_slots;
    s.slot_of_expert = w->slot_of_expert;
    return s;
}

// ---- internal launchers ---------------------------------------------------------------
struct RouteBufs {
    uint16_t* logits;
    int64_t* selected;
    uint16_t* weights;
    double* partials;       // split-K router partials (T > kTailMaxTokens)
};

// Dynamic shared memory of k_topk_pack for N = T*k assignments.
size_t topk_pack_smem_bytes(int64_t E, int64_t N) {
    return block_pack_smem_ints(E, N, kTopkPackThreads / 32) * sizeof(int);
}

// Split-K of the tiled router (T > kTailMaxTokens only).  A 64 x 128 tile
// over all of K is ~2.7 * 10^5 FP64-tensor cycles at H = 2048 (~130 us on one
// SM), so a few hundred tokens (a handful of tiles) need many K splits to
// occupy the GPU, while large batches need few.  The split count is bounded by
// what three waves of units over two CTAs per SM can use (so the partial
// buffer stays small at prefill sizes) and by kMaxRouterSplits.
constexpr int kMaxRouterSplits = 32;
constexpr int kRouterSlots = 2 * kPlanSMs;
int64_t router_tiles(int64_t T, int64_t E) { return ((T + kDmT - 1) / kDmT) * ((E + kDmE - 1) / kDmE); }
int router_split_bound(int64_t T, int64_t E) {
    const int64_t tiles = std::max<int64_t>(1, router_tiles(T, E));
    return static_cast<int>(std::min<int64_t>(kMaxRouterSplits, (3 * kRouterSlots + tiles - 1) / tiles));
}
size_t route_partial_bytes(int64_t T, int64_t E) {
    const int s = router_split_bound(T, E);
    return T > kTailMaxTokens && s > 1 ? static_cast<size_t>(s) * T * E * sizeof(double) : 0;
}

// K splits per router tile: the count minimising the modelled time -- waves
// of units over the resident CTAs times the unit's share of a whole-K tile,
// plus the FP64 partials each extra split writes and k_topk_partials reads
// back; ties keep fewer splits.  Each split keeps >= 2 K chunks.
int router_splits(int64_t T, int64_t E, int64_t H) {
    const int64_t tiles = router_tiles(T, E);
    const double tile_us = static_cast<double>(H) * kDmT * kDmE / (64.0 * 1.9e3);  // FP64 FMA/clk/SM x clk/us
    const double partial_us_per_split = static_cast<double>(T) * E * 16.0 / 6.5e6;  // write + read at ~6.5 TB/s
    int best = 1;
    double best_t = 1e30;
    for (int s = 1; s <= router_split_bound(T, E); ++s) {
        if (s > 1 && H / s < 2 * kDmK) break;
        const int64_t units = tiles * s;
        const double t = static_cast<double>((units + kRouterSlots - 1) / kRouterSlots) * tile_us / s +
                         (s > 1 ? s * partial_us_per_split : 0.0);
        if (t < best_t - 1e-9) { best_t = t; best = s; }
    }
    return best;
}

// Routing: exact logits, then top-k (with fused_pack at decode sizes, top-k
// and the pack in one CTA).
int launch_route(const void* x, const void* gate, int64_t T, int64_t H, int64_t E, int32_t k, int32_t normalize,
                 const RouteBufs& b, const PackOut* fused_pack, cudaStream_t stream, unsigned int* zero_ptr = nullptr,
                 int64_t zero_words = 0) {
    if (T > kTailMaxTokens) {
        // prefill sizes: tiled FP64 logits, then one warp per token for top-k
        int sms = 0;
        int st = device_setup(&sms);
        if (st) return st;
        const int64_t tiles = router_tiles(T, E);
        const int splits = router_splits(T, E, H);
        const int k_per_split = static_cast<int>(((H + splits - 1) / splits + kDmK - 1) / kDmK * kDmK);
        k_router_logits_dmma<<<static_cast<unsigned>(tiles * splits), kDmThreads, kDmmaSmemBytes, stream>>>(
            static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(gate), static_cast<int>(T),
            static_cast<int>(H), static_cast<int>(E), splits, k_per_split, b.logits, b.partials);
        PDX_LAUNCHED();
        const int warps_per_cta = 8;
        const int grid = static_cast<int>((T + warps_per_cta - 1) / warps_per_cta);
        with_epl(E, [&](auto epl) {
            constexpr int EPL = decltype(epl)::value;
            if (splits > 1)
                k_topk_partials<EPL><<<grid, warps_per_cta * 32, 0, stream>>>(
                    b.partials, splits, static_cast<int>(T), static_cast<int>(E), k, normalize, b.logits, b.selected,
                    b.weights);
            else
                k_topk<EPL><<<grid, warps_per_cta * 32, 0, stream>>>(b.logits, static_cast<int>(T),
                                                                     static_cast<int>(E), k, normalize, b.selected,
                                                                     b.weights, nullptr, 0);
            return 0;
        });
        PDX_LAUNCHED();
        if (fused_pack) return fail(PDX_ERR_UNSUPPORTED, "fused pack is only available for T <= %lld",
                                    static_cast<long long>(kTailMaxTokens));
        return PDX_OK;
    }
    // decode sizes: logits on many CTAs, then top-k (with fused_pack: top-k and
    // the pack, one CTA), chained by programmatic dependent launch
    const int n_tb = static_cast<int>((T + kRouteTB - 1) / kRouteTB);
    const int n_eb = static_cast<int>((E + kRouteEB - 1) / kRouteEB);
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    const uint16_t* gb = static_cast<const uint16_t*>(gate);
    if (T <= kSmallRouteT && H <= static_cast<int64_t>(kSmallRouteMaxChunks) * kSmallRouteThreads * 8)
        PDX_PDL_TRY(launch_pdl(k_router_small, dim3(static_cast<unsigned>(E)), dim3(kSmallRouteThreads), 0, stream,
                               xb, gb, static_cast<int>(T), static_cast<int>(H), static_cast<int>(E), b.logits));
    else
        PDX_PDL_TRY(launch_pdl(k_router_logits, dim3(static_cast<unsigned>(n_tb * n_eb)), dim3(kRouteWarps * 32), 0,
                               stream, xb, gb, static_cast<int>(T), static_cast<int>(H), static_cast<int>(E),
                               b.logits));
    const int Ti = static_cast<int>(T), Ei = static_cast<int>(E);
    if (fused_pack && T > kSmallRouteT) {
        // Past a few tokens one CTA's issue slots bound the top-k (64 tokens on one
        // SM took ~14 us); spread it, one warp per token over T/4 CTAs, then pack
        // in one CTA.
        const int tk_warps = 4;
        const int tk_grid = static_cast<int>((T + tk_warps - 1) / tk_warps);
        PDX_PDL_TRY(with_epl(E, [&](auto epl) {
            return launch_pdl(k_topk<decltype(epl)::value>, dim3(tk_grid), dim3(tk_warps * 32), 0, stream,
                              static_cast<const uint16_t*>(b.logits), Ti, Ei, k, normalize, b.selected, b.weights,
                              zero_ptr, static_cast<int>(zero_words));
        }));
        const size_t smem = block_pack_smem_ints(E, T * k, kPackThreads / 32) * sizeof(int);
        PDX_PDL_TRY(launch_pdl(k_pack_single, dim3(1), dim3(kPackThreads), smem, stream,
                               static_cast<const int64_t*>(b.selected), static_cast<const uint16_t*>(b.weights), Ti,
                               k, Ei, *fused_pack));
        return PDX_OK;
    }
    if (fused_pack) {
        // up to 32 assignments one warp packs, so the CTA needs only a warp per token
        const bool small = T * k <= 32;
        const size_t smem = small ? (2 * E + 1) * sizeof(int) : topk_pack_smem_bytes(E, T * k);
        const unsigned threads = small ? static_cast<unsigned>(32 * T) : static_cast<unsigned>(kTopkPackThreads);
        PDX_PDL_TRY(with_epl(E, [&](auto epl) {
            return launch_pdl(k_topk_pack<decltype(epl)::value>, dim3(1), dim3(threads), smem, stream,
                              static_cast<const uint16_t*>(b.logits), Ti, Ei, k, normalize, b.selected, b.weights,
                              *fused_pack, zero_ptr, static_cast<int>(zero_words));
        }));
        return PDX_OK;
    }
    const int warps_per_cta = 8;
    const int grid = static_cast<int>((T + warps_per_cta - 1) / warps_per_cta);
    PDX_PDL_TRY(with_epl(E, [&](auto epl) {
        return launch_pdl(k_topk<decltype(epl)::value>, dim3(grid), dim3(warps_per_cta * 32), 0, stream,
                          static_cast<const uint16_t*>(b.logits), Ti, Ei, k, normalize, b.selected, b.weights,
                          static_cast<unsigned int*>(nullptr), 0);
    }));
    return PDX_OK;
}

// Flat entries per CTA of the multi-CTA pack: enough CTAs to cover the SMs
// once (a multiple of one scatter round), at most kPackChunk.  The
// allocation-free entry point keeps kPackChunk (its documented scratch bound).
int64_t pack_chunk_for(int64_t N) {
    const int64_t per = (N + kPlanSMs - 1) / kPlanSMs;
    return std::min<int64_t>(kPackChunk, std::max<int64_t>(kPackMinChunk, (per + kPackMinChunk - 1) / kPackMinChunk *
                                                                               kPackMinChunk));
}
size_t pack_chunks(int64_t N, int64_t chunk) { return static_cast<size_t>((N + chunk - 1) / chunk); }
size_t pack_chunks(int64_t N) { return pack_chunks(N, pack_chunk_for(N)); }

int launch_pack(const int64_t* selected, const uint16_t* weights, int64_t T, int32_t k, int64_t E, const PackOut& o,
                int* chunk_hist, cudaStream_t stream, int64_t chunk = 0) {
    const int64_t N = T * k;
    if (N <= kPackSingleMax) {
        const size_t smem = block_pack_smem_ints(E, N, kPackThreads / 32) * sizeof(int);
        k_pack_single<<<1, kPackThreads, smem, stream>>>(selected, weights, static_cast<int>(T), k,
                                                          static_cast<int>(E), o);
        PDX_LAUNCHED();
        return PDX_OK;
    }
    if (chunk <= 0) chunk = pack_chunk_for(N);
    const int chunks = static_cast<int>(pack_chunks(N, chunk));
    int sms = 0;
    if (int st = device_setup(&sms)) return st;   // k_pack_scan's shared-memory limit
    k_pack_hist<<<chunks, kPackThreads, E * sizeof(int), stream>>>(selected, static_cast<int>(T), k,
                                                                     static_cast<int>(E), static_cast<int>(chunk),
                                                                     chunk_hist);
    PDX_LAUNCHED();
    if (static_cast<int64_t>(chunks) * E <= kPackScanSmemInts) {
        // every CTA derives its own chunk base from the staged histograms
        const size_t smem = (static_cast<size_t>(chunks) * E + 11 * E + 1) * sizeof(int);
        k_pack_scan_scatter<<<chunks, kPackThreads, smem, stream>>>(selected, weights, static_cast<int>(T), k,
                                                                     static_cast<int>(E), static_cast<int>(chunk),
                                                                     chunks, chunk_hist, o);
        PDX_LAUNCHED();
        return PDX_OK;
    }
    k_pack_scan<<<1, kPackThreads, (2 * E + 1) * sizeof(int), stream>>>(chunk_hist, chunks, static_cast<int>(E),
                                                                         o);
    PDX_LAUNCHED();
    k_pack_scatter<<<chunks, kPackThreads, (E + 8 * E) * sizeof(int), stream>>>(
        selected, weights, static_cast<int>(T), k, static_cast<int>(E), static_cast<int>(chunk), chunk_hist, o);
    PDX_LAUNCHED();
    return PDX_OK;
}

// Split-K / token-tile plan of the weight-streaming path.  It depends only on
// (rows, E, H, I), so the workspace query and the launch agree.

struct StreamPlan {
    int nt;
    int s1, s2;
    int64_t tiles1, tiles2;
    size_t partial_bytes, ticket_bytes;
};

#ifndef PDX_SPLIT_UNITS_PER_SM
#define PDX_SPLIT_UNITS_PER_SM 1
#endif
// K splits per weight tile of the decode GEMMs: about PDX_SPLIT_UNITS_PER_SM
// work units (tiles x splits) per SM, each split >= 4 K blocks.  One unit per
// SM measured best at every decode batch (1..64 tokens at the Qwen3-30B-A3B
// shape): a split costs an extra FP32 partial round trip and a ticketed
// reduction, and one weight tile per SM already keeps HBM busy once about 30
// experts are active.
int plan_splits(int num_kb, int64_t est_tiles) {
    const int64_t want = (PDX_SPLIT_UNITS_PER_SM * kPlanSMs + est_tiles / 2) / std::max<int64_t>(est_tiles, 1);
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, std::max(1, num_kb / 4))));
}

StreamPlan plan_stream(int64_t rows, int64_t E, int64_t H, int64_t I) {
    StreamPlan p{};
    const int64_t est_active = std::max<int64_t>(1, std::min(E, rows));
    const int64_t avg = (rows + est_active - 1) / est_active;
    p.nt = avg <= 12 ? 16 : (avg <= 24 ? 32 : 64);
    const int64_t nb_bound = rows / p.nt + est_active;
    p.tiles1 = (I / 128) * nb_bound;
    p.tiles2 = (H / 128) * nb_bound;
    p.s1 = plan_splits(static_cast<int>(H / 64), (I / 128) * est_active);
    p.s2 = plan_splits(static_cast<int>(I / 64), (H / 128) * est_active);
    const int64_t c1 = p.s1 > 1 ? p.tiles1 * p.s1 * 2 * p.nt : 0;
    const int64_t c2 = p.s2 > 1 ? p.tiles2 * p.s2 * p.nt : 0;
    p.partial_bytes = static_cast<size_t>(std::max(c1, c2)) * 128 * 4;
    p.ticket_bytes = static_cast<size_t>(std::max(p.tiles1, p.tiles2)) * 4 * 4;  // per GEMM
    return p;
}

// Single-launch weight-streaming FFN (ffn_decode.cu).  DIRECT form: the whole
// token matrix x [T, H] is the gate/up N operand, so it needs the packed
// tokens and T <= 64, and its shared-memory tables bound the rows.  PACKED
// form: gate/up tiles over packed rows (gathered first when tokens are
// given).  Both bound the active experts by the shared-memory tables.
bool decode_direct_ok(int64_t T, int64_t rows, int64_t E, int64_t H, int64_t I, const int32_t* tokens) {
    return tokens != nullptr && T >= 1 && T <= kDecMaxT && rows <= kDecMaxRows &&
           std::min(E, rows) <= kDecMaxActive && stream_shape_ok(H, I);
}
bool decode_packed_ok(int64_t rows, int64_t E, int64_t H, int64_t I) {
    return std::min(E, rows) <= kDecMaxActive && stream_shape_ok(H, I);
}

struct DecodePlan {
    bool direct;
    int nb, nt2;          // gate/up token tile (DIRECT: T rounded up to 16), down token tile
    int s1, s2;           // K slices per tile of each projection
    int64_t tiles1, tiles2;
    size_t p1_bytes, p2_bytes;
    int64_t zero_words;   // tickets of both projections + per-expert h counters
};

// Depends only on (rows, E, H, I), the form and T, so the workspace query
// (which sizes for any T) and the launch agree; token tiles and split counts
// are plan_stream's.
DecodePlan plan_decode(int64_t T, int64_t rows, int64_t E, int64_t H, int64_t I, bool direct) {
    DecodePlan p{};
    p.direct = direct;
    const int64_t est = std::max<int64_t>(1, std::min(E, rows));
    const int64_t avg = (rows + est - 1) / est;
    const int nt = avg <= 12 ? 16 : (avg <= 24 ? 32 : 64);
    p.nb = direct ? (T <= 16 ? 16 : (T <= 32 ? 32 : 64)) : nt;
    p.nt2 = nt;
    const int64_t m1 = I / 128, m2 = H / 128;
    p.tiles1 = direct ? est * m1 : m1 * (rows / p.nb + est);
    p.tiles2 = m2 * (rows / p.nt2 + est);
    p.s1 = plan_splits(static_cast<int>(H / 64), m1 * est);
    p.s2 = plan_splits(static_cast<int>(I / 64), m2 * est);
    if (p.s1 > 1)
        p.p1_bytes = direct ? static_cast<size_t>(m1 * p.s1 * rows) * 256 * 4
                            : static_cast<size_t>(p.tiles1 * p.s1 * 2 * p.nb) * 128 * 4;
    p.p2_bytes = p.s2 > 1 ? static_cast<size_t>(p.tiles2 * p.s2 * p.nt2) * 128 * 4 : 0;
    p.zero_words = 4 * p.tiles1 + 4 * p.tiles2 + est;
    return p;
}

struct DecodeBufs {
    DecodePlan plan;
    uint16_t* h;
    uint16_t* xp;            // PACKED form: gathered token rows
    float* p1;
    float* p2;
    unsigned int* counters;  // zero_words words, cleared before every launch
};

DecodeBufs carve_decode(Carver& c, int64_t T, int64_t rows, int64_t E, int64_t H, int64_t I, bool direct) {
    DecodeBufs b{};
    b.plan = plan_decode(T, rows, E, H, I, direct);
    b.h = static_cast<uint16_t*>(c.take(static_cast<size_t>(rows) * I * 2));
    if (!direct) b.xp = static_cast<uint16_t*>(c.take(static_cast<size_t>(rows) * H * 2));
    b.p1 = static_cast<float*>(c.take(std::max<size_t>(b.plan.p1_bytes, 16)));
    b.p2 = static_cast<float*>(c.take(std::max<size_t>(b.plan.p2_bytes, 16)));
    b.counters = static_cast<unsigned int*>(c.take(static_cast<size_t>(b.plan.zero_words) * 4));
    return b;
}

size_t ffn_ws_bytes(int64_t rows, int64_t E, int64_t H, int64_t I, int mode) {
    if (mode == PDX_FFN_GEMV) {
        // any of the single-launch forms or the staged one may run
        Carver c1{nullptr, SIZE_MAX}, c2{nullptr, SIZE_MAX};
        carve_decode(c1, 1, rows, E, H, I, true);
        carve_decode(c2, 1, rows, E, H, I, false);
        return std::max(std::max(c1.used, c2.used), ffn_ws_bytes(rows, E, H, I, PDX_FFN_GEMV_STAGED));
    }
    if (mode == PDX_FFN_GEMV_STAGED) mode = PDX_FFN_GEMV;
    size_t b = align_up(static_cast<size_t>(rows) * I * 2);                        // h
    if (is_gemm_mode(mode) || mode == PDX_FFN_GEMV) b += align_up(static_cast<size_t>(rows) * H * 2);  // x rows
    if (mode == PDX_FFN_GEMV) {
        const StreamPlan p = plan_stream(rows, E, H, I);
        b += align_up(p.partial_bytes) + align_up(2 * p.ticket_bytes);
    }
    return b;
}

template <int NT>
int launch_stream_pair(const CUtensorMap& tm_g, const CUtensorMap& tm_u, const CUtensorMap& tm_x,
                       const CUtensorMap& tm_d, const CUtensorMap& tm_h, const StreamPlan& p, StreamArgs a1,
                       StreamArgs a2, int sms, cudaStream_t stream) {
    const int grid1 = static_cast<int>(std::min<int64_t>(sms, p.tiles1 * p.s1));
    PDX_PDL_TRY(launch_pdl(k_stream_gemm<NT, true>, dim3(grid1), dim3(kStreamThreads), kStreamSmemBytes, stream,
                           tm_g, tm_u, tm_x, a1));
    const int grid2 = static_cast<int>(std::min<int64_t>(sms, p.tiles2 * p.s2));
    PDX_PDL_TRY(launch_pdl(k_stream_gemm<NT, false>, dim3(grid2), dim3(kStreamThreads), kStreamSmemBytes, stream,
                           tm_d, tm_d, tm_h, a2));
    return PDX_OK;
}

template <bool DIRECT, int NB, int NT2>
int launch_decode_kernel(dim3 grid, const CUtensorMap& tm_g, const CUtensorMap& tm_u, const CUtensorMap& tm_x,
                         const CUtensorMap& tm_d, const CUtensorMap& tm_h, const DecodeArgs& a, cudaStream_t stream) {
    PDX_PDL_TRY(launch_pdl(k_decode_ffn<DIRECT, NB, NT2>, grid, dim3(kDecThreads), kDecSmemBytes, stream, tm_g, tm_u,
                           tm_x, tm_d, tm_h, a));
    return PDX_OK;
}

template <int NB>
int launch_decode_direct(int nt2, dim3 grid, const CUtensorMap& tm_g, const CUtensorMap& tm_u,
                         const CUtensorMap& tm_x, const CUtensorMap& tm_d, const CUtensorMap& tm_h,
                         const DecodeArgs& a, cudaStream_t stream) {
    if (nt2 == 16) return launch_decode_kernel<true, NB, 16>(grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
    if (nt2 == 32) return launch_decode_kernel<true, NB, 32>(grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
    return launch_decode_kernel<true, NB, 64>(grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
}

// The single-launch FFN.  `zeroed`: the kernel before it in the stream already
// cleared b.counters (the routing kernels of pdx_moe_layer do); otherwise the
// row gather (PACKED form with tokens) or a clearing kernel does it first.
int launch_decode_ffn(const void* x, int64_t T, const int32_t* tokens, const int32_t* offsets, const int32_t* active,
                      int64_t rows, const pdx_expert_weights* w, int64_t H, int64_t I, void* y, const DecodeBufs& b,
                      bool zeroed, cudaStream_t stream) {
    int sms = 0;
    int st = device_setup(&sms);
    if (st) return st;
    const DecodePlan& p = b.plan;
    const int zero_words = zeroed ? 0 : static_cast<int>(p.zero_words);
    const void* xb = x;   // phase-1 B operand
    if (!p.direct && tokens) {
        PDX_PDL_TRY(launch_pdl(k_gather_rows, gather_grid(rows), dim3(kGatherWarps * 32), 0, stream,
                               static_cast<const uint16_t*>(x), tokens, static_cast<int>(rows), static_cast<int>(H),
                               b.xp, b.counters, zero_words));
        xb = b.xp;
    } else if (zero_words > 0) {
        PDX_PDL_TRY(launch_pdl(k_zero_words, dim3(static_cast<unsigned>(std::min(64, (zero_words + 255) / 256))),
                               dim3(256), 0, stream, b.counters, zero_words));
    }
    const int64_t gs = w->num_slots > 1 ? w->gate_stride / H : 0;
    const int64_t us = w->num_slots > 1 ? w->up_stride / H : 0;
    const int64_t ds = w->num_slots > 1 ? w->down_stride / I : 0;
    if ((w->num_slots - 1) * std::max(gs, std::max(us, ds)) + H >= (int64_t(1) << 31))
        return fail(PDX_ERR_UNSUPPORTED, "expert slab too large for 32-bit TMA row coordinates");
    CUtensorMap tm_g, tm_u, tm_x, tm_d, tm_h;
    if ((st = encode_2d(&tm_g, w->gate, (w->num_slots - 1) * gs + I, H, 128))) return st;
    if ((st = encode_2d(&tm_u, w->up, (w->num_slots - 1) * us + I, H, 128))) return st;
    if ((st = encode_2d(&tm_d, w->down, (w->num_slots - 1) * ds + H, I, 128))) return st;
    if ((st = encode_2d(&tm_x, xb, p.direct ? T : rows, H, p.nb))) return st;
    if ((st = encode_2d(&tm_h, b.h, rows, I, p.nt2))) return st;
    DecodeArgs a{offsets, active, tokens, w->slot_of_expert, w->num_slots, gs, us, ds,
                 static_cast<int>(H), static_cast<int>(I), static_cast<int>(T), static_cast<int>(rows),
                 p.s1, p.s2, b.h, static_cast<uint16_t*>(y), b.p1, b.p2,
                 b.counters, b.counters + 4 * p.tiles1, b.counters + 4 * p.tiles1 + 4 * p.tiles2};
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>(sms, p.tiles1 * p.s1 + p.tiles2 * p.s2)));
    if (!p.direct) {
        if (p.nb == 16) return launch_decode_kernel<false, 16, 16>(grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
        if (p.nb == 32) return launch_decode_kernel<false, 32, 32>(grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
        return launch_decode_kernel<false, 64, 64>(grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
    }
    if (p.nb == 16) return launch_decode_direct<16>(p.nt2, grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
    if (p.nb == 32) return launch_decode_direct<32>(p.nt2, grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
    return launch_decode_direct<64>(p.nt2, grid, tm_g, tm_u, tm_x, tm_d, tm_h, a, stream);
}

int launch_ffn(const void* x, int64_t T, const int32_t* tokens, const int32_t* offsets, const int32_t* active,
               int64_t E, int64_t rows, const pdx_expert_weights* w, int64_t H, int64_t I, void* y, int mode,
               Carver& ws, cudaStream_t stream) {
    if (mode == PDX_FFN_GEMV) {
        const bool direct = decode_direct_ok(T, rows, E, H, I, tokens);
        if (direct || decode_packed_ok(rows, E, H, I)) {
            const DecodeBufs b = carve_decode(ws, T, rows, E, H, I, direct);
            if (ws.overflow)
                return fail(PDX_ERR_WORKSPACE, "FFN workspace too small (%zu > %zu bytes)", ws.used, ws.cap);
            return launch_decode_ffn(x, T, tokens, offsets, active, rows, w, H, I, y, b, false, stream);
        }
    }
    if (mode == PDX_FFN_GEMV_STAGED) mode = PDX_FFN_GEMV;
    int sms = 0;
    int st = device_setup(&sms);
    if (st) return st;
    uint16_t* h = static_cast<uint16_t*>(ws.take(static_cast<size_t>(rows) * I * 2));
    uint16_t* xp = (is_gemm_mode(mode) || mode == PDX_FFN_GEMV)
                       ? static_cast<uint16_t*>(ws.take(static_cast<size_t>(rows) * H * 2))
                       : nullptr;
    StreamPlan plan{};
    float* partials = nullptr;
    unsigned int* tickets = nullptr;
    if (mode == PDX_FFN_GEMV) {
        plan = plan_stream(rows, E, H, I);
        partials = static_cast<float*>(ws.take(std::max<size_t>(plan.partial_bytes, 16)));
        tickets = static_cast<unsigned int*>(ws.take(2 * plan.ticket_bytes));  // GEMM1 | GEMM2
    }
    if (ws.overflow) return fail(PDX_ERR_WORKSPACE, "FFN workspace too small (%zu > %zu bytes)", ws.used, ws.cap);
    const ExpertSlab slab = to_slab(w);
    const int64_t max_active = std::min<int64_t>(E, rows);
    if (mode == PDX_FFN_SIMT) {
        const bool small = rows <= 64;
        const int rb = small ? 4 : 16;
        const int rpw_down = small ? 1 : 4;
        if (I % rb || H % (8 * rpw_down))
            return fail(PDX_ERR_UNSUPPORTED, "GEMV tiling needs I %% %d == 0 and H %% %d == 0", rb, 8 * rpw_down);
        const int64_t items1 = max_active * (I / rb);
        const int64_t items2 = max_active * (H / (8 * rpw_down));
        const int grid1 = static_cast<int>(std::min<int64_t>(items1, static_cast<int64_t>(sms) * 4));
        const int grid2 = static_cast<int>(std::min<int64_t>(items2, static_cast<int64_t>(sms) * 4));
        const size_t smem1 = static_cast<size_t>(kTokChunk) * H * 2 + 2 * rb * kTokChunk * 4;
        const size_t smem2 = static_cast<size_t>(kTokChunk) * I * 2 + 8 * rpw_down * kTokChunk * 4;
        const uint16_t* xb = static_cast<const uint16_t*>(x);
        if (small)
            k_gateup_gemv<4><<<grid1, kGemvThreads, smem1, stream>>>(xb, tokens, offsets, active, slab,
                                                                      static_cast<int>(H), static_cast<int>(I), h);
        else
            k_gateup_gemv<16><<<grid1, kGemvThreads, smem1, stream>>>(xb, tokens, offsets, active, slab,
                                                                       static_cast<int>(H), static_cast<int>(I), h);
        PDX_LAUNCHED();
        if (small)
            k_down_gemv<1><<<grid2, kGemvThreads, smem2, stream>>>(h, offsets, active, slab, static_cast<int>(H),
                                                                    static_cast<int>(I), static_cast<uint16_t*>(y));
        else
            k_down_gemv<4><<<grid2, kGemvThreads, smem2, stream>>>(h, offsets, active, slab, static_cast<int>(H),
                                                                    static_cast<int>(I), static_cast<uint16_t*>(y));
        PDX_LAUNCHED();
        return PDX_OK;
    }
    // prefill sizes launch without programmatic overlap (see launch_pdl)
    PdlScope pdl_scope(!is_gemm_mode(mode) || PDX_PREFILL_PDL);
    // tcgen05 paths: gather the packed x rows once (and clear the split-K tickets);
    // with tokens == NULL the rows of x are already in packed order.
    const int zero_words = mode == PDX_FFN_GEMV ? static_cast<int>(2 * plan.ticket_bytes / 4) : 0;
    if (tokens) {
        PDX_PDL_TRY(launch_pdl(k_gather_rows, gather_grid(rows), dim3(kGatherWarps * 32), 0, stream,
                               static_cast<const uint16_t*>(x), tokens, static_cast<int>(rows), static_cast<int>(H),
                               xp, tickets, zero_words));
    } else {
        xp = static_cast<uint16_t*>(const_cast<void*>(x));
        if (zero_words > 0)
            PDX_PDL_TRY(launch_pdl(k_zero_words, dim3(std::min(64, (zero_words + 255) / 256)), dim3(256), 0, stream,
                                   tickets, zero_words));
    }
    const int64_t gs = w->num_slots > 1 ? w->gate_stride / H : 0;
    const int64_t us = w->num_slots > 1 ? w->up_stride / H : 0;
    const int64_t ds = w->num_slots > 1 ? w->down_stride / I : 0;
    if ((w->num_slots - 1) * std::max(gs, std::max(us, ds)) + H >= (int64_t(1) << 31))
        return fail(PDX_ERR_UNSUPPORTED, "expert slab too large for 32-bit TMA row coordinates");
    CUtensorMap tm_x, tm_g, tm_u, tm_h, tm_d;
    if ((st = encode_2d(&tm_g, w->gate, (w->num_slots - 1) * gs + I, H, 128))) return st;
    if ((st = encode_2d(&tm_u, w->up, (w->num_slots - 1) * us + I, H, 128))) return st;
    if (mode == PDX_FFN_GEMV) {
        if ((st = encode_2d(&tm_x, xp, rows, H, plan.nt))) return st;
        if ((st = encode_2d(&tm_h, h, rows, I, plan.nt))) return st;
        if ((st = encode_2d(&tm_d, w->down, (w->num_slots - 1) * ds + H, I, 128))) return st;
        StreamArgs a1{offsets, active, w->slot_of_expert, w->num_slots, gs, us, static_cast<int>(H),
                      static_cast<int>(I / 128), plan.s1, h, I, partials, tickets};
        StreamArgs a2{offsets, active, w->slot_of_expert, w->num_slots, ds, ds, static_cast<int>(I),
                      static_cast<int>(H / 128), plan.s2, static_cast<uint16_t*>(y), H, partials,
                      tickets + plan.ticket_bytes / 4};
        if (plan.nt == 16) return launch_stream_pair<16>(tm_g, tm_u, tm_x, tm_d, tm_h, plan, a1, a2, sms, stream);
        if (plan.nt == 32) return launch_stream_pair<32>(tm_g, tm_u, tm_x, tm_d, tm_h, plan, a1, a2, sms, stream);
        return launch_stream_pair<64>(tm_g, tm_u, tm_x, tm_d, tm_h, plan, a1, a2, sms, stream);
    }
    // prefill: token-tiled grouped GEMM on single CTAs (128 x 256 tiles); CTA-pair
    // 256 x 256 tiles on request (mode PDX_FFN_GEMM_PAIR).  The pair form moves a
    // third less L2->SM data per FLOP but measured slower on a 12,450-token Zipf
    // prefill (1172 vs 1031 us per layer): the GEMM is bound by the power-capped
    // tensor clock, not by L2 bandwidth.
    const bool pair = mode == PDX_FFN_GEMM_PAIR;
    if (pair) {
        if ((st = encode_2d(&tm_x, xp, rows, H, 128))) return st;
        if ((st = encode_2d(&tm_h, h, rows, I, 128))) return st;
        if ((st = encode_2d(&tm_d, w->down, (w->num_slots - 1) * ds + H, I, 128))) return st;
        const int64_t pair_tiles_bound = rows / kPairBM + max_active;
        const int max_pairs = g_pair_clusters[cur_device()];
        GemmArgs a1{offsets, active, w->slot_of_expert, w->num_slots, gs, us, static_cast<int>(H),
                    static_cast<int>(I), 1, h, I};
        const int pairs1 = static_cast<int>(std::min<int64_t>(max_pairs, pair_tiles_bound * (I / (kGemmBN / 2))));
        PDX_PDL_TRY(launch_pdl(k_grouped_gemm_pair, dim3(2 * pairs1), dim3(kPairThreads), kGemmPairSmemBytes,
                               stream, tm_x, tm_g, tm_u, a1));
        GemmArgs a2{offsets, active, w->slot_of_expert, w->num_slots, ds, ds, static_cast<int>(I),
                    static_cast<int>(H), 0, static_cast<uint16_t*>(y), H};
        const int pairs2 = static_cast<int>(std::min<int64_t>(max_pairs, pair_tiles_bound * (H / kGemmBN)));
        PDX_PDL_TRY(launch_pdl(k_grouped_gemm_pair, dim3(2 * pairs2), dim3(kPairThreads), kGemmPairSmemBytes,
                               stream, tm_h, tm_d, tm_d, a2));
        return PDX_OK;
    }
    if ((st = encode_2d(&tm_x, xp, rows, H, kGemmBM))) return st;
    if ((st = encode_2d(&tm_h, h, rows, I, kGemmBM))) return st;
    if ((st = encode_2d(&tm_d, w->down, (w->num_slots - 1) * ds + H, I, kGemmBN))) return st;
    const int64_t m_tiles_bound = rows / kGemmBM + max_active;
    GemmArgs a1{offsets, active, w->slot_of_expert, w->num_slots, gs, us, static_cast<int>(H),
                static_cast<int>(I), 1, h, I};
    const int grid1 = static_cast<int>(std::min<int64_t>(sms, m_tiles_bound * (I / (kGemmBN / 2))));
    PDX_PDL_TRY(launch_pdl(k_grouped_gemm, dim3(grid1), dim3(kGemmThreads), kGemmSmemBytes, stream, tm_x, tm_g,
                           tm_u, a1));
    GemmArgs a2{offsets, active, w->slot_of_expert, w->num_slots, ds, ds, static_cast<int>(I),
                static_cast<int>(H), 0, static_cast<uint16_t*>(y), H};
    const int grid2 = static_cast<int>(std::min<int64_t>(sms, m_tiles_bound * (H / kGemmBN)));
    PDX_PDL_TRY(launch_pdl(k_grouped_gemm, dim3(grid2), dim3(kGemmThreads), kGemmSmemBytes, stream, tm_h, tm_d,
                           tm_d, a2));
    return PDX_OK;
}

// one expert owning rows [0, n): offsets = {0, n}, active = {1, 0}, tokens = 0..n-1
__global__ void k_single_expert_setup(int n, int32_t* offsets, int32_t* active, int32_t* tokens) {
    const int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
    if (i == 0) {
        offsets[0] = 0;
        offsets[1] = n;
        active[0] = 1;
        active[1] = 0;
    }
    if (i < n) tokens[i] = i;
}

struct PackBufs {
    PackOut o;
    int* chunk_hist;
};

PackBufs carve_pack(Carver& c, int64_t T, int32_t k, int64_t E, int32_t* counts_out) {
    const int64_t N = T * k;
    PackBufs p;
    p.o.counts = counts_out ? counts_out : static_cast<int32_t*>(c.take(E * 4));
    p.o.offsets = static_cast<int32_t*>(c.take((E + 1) * 4));
    p.o.tokens = static_cast<int32_t*>(c.take(N * 4));
    p.o.positions = static_cast<int32_t*>(c.take(N * 4));
    p.o.packed_w = static_cast<uint16_t*>(c.take(N * 2));
    p.o.inverse = static_cast<int32_t*>(c.take(N * 4));
    p.o.active = static_cast<int32_t*>(c.take((E + 1) * 4));
    p.chunk_hist = static_cast<int*>(c.take(pack_chunks(N) * E * 4));
    return p;
}

}  // namespace
}  // namespace pdx

using namespace pdx;

int check_norm_shape(int64_t H) {
    if (H < 8 || H % 8 || H > 8 * kLnThreads * (kLnMaxPerThread / 8))
        return fail(PDX_ERR_UNSUPPORTED, "layer norm needs H a multiple of 8 and <= %d",
                    8 * kLnThreads * (kLnMaxPerThread / 8));
    return PDX_OK;
}

extern "C" {

const char* pdx_last_error(void) { return t_last_error.c_str(); }

int pdx_abi_version(void) { return PDX_ABI_VERSION; }

uint64_t pdx_launch_count(void) { return g_launches.load(); }

size_t pdx_route_workspace_bytes(int64_t T, int64_t E) {
    T = std::max<int64_t>(T, 1);
    return align_up(static_cast<size_t>(T) * std::max<int64_t>(E, 0) * 2) +
           align_up(route_partial_bytes(T, std::max<int64_t>(E, 0)));
}

int pdx_route_topk(const void* x, const void* gate, int64_t T, int64_t H, int64_t E, int32_t top_k, int32_t normalize,
                   void* logits_out, int64_t* selected_out, void* weights_out, void* workspace,
                   size_t workspace_bytes, pdx_stream_t stream) {
    int st = check_route_shape(T, H, E, top_k);
    if (st) return st;
    if (!x || !gate || !selected_out || !weights_out) return fail(PDX_ERR_INVALID, "null routing argument");
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)))
        return fail(PDX_ERR_WORKSPACE, "workspace must be non-null and 256-byte aligned");
    Carver c{static_cast<char*>(workspace), workspace_bytes};
    RouteBufs b;
    b.logits = logits_out ? static_cast<uint16_t*>(logits_out) : static_cast<uint16_t*>(c.take(T * E * 2));
    b.partials = static_cast<double*>(c.take(route_partial_bytes(T, E)));
    b.selected = selected_out;
    b.weights = static_cast<uint16_t*>(weights_out);
    if (c.overflow) return fail(PDX_ERR_WORKSPACE, "route workspace too small");
    st = launch_route(x, gate, T, H, E, top_k, normalize, b, nullptr, stream);
    return st ? st : ok();
}

int pdx_topk_from_logits(const void* logits, int64_t T, int64_t E, int32_t top_k, int32_t normalize,
                         int64_t* selected_out, void* weights_out, pdx_stream_t stream) {
    int st = check_route_shape(T, 8, E, top_k);
    if (st) return st;
    if (!logits || !selected_out || !weights_out) return fail(PDX_ERR_INVALID, "null routing argument");
    const int warps_per_cta = 8;
    const int grid = static_cast<int>((T + warps_per_cta - 1) / warps_per_cta);
    with_epl(E, [&](auto epl) {
        k_topk<decltype(epl)::value><<<grid, warps_per_cta * 32, 0, stream>>>(
            static_cast<const uint16_t*>(logits), static_cast<int>(T), static_cast<int>(E), top_k, normalize,
            selected_out, static_cast<uint16_t*>(weights_out), nullptr, 0);
        return 0;
    });
    PDX_LAUNCHED();
    return ok();
}

size_t pdx_pack_workspace_bytes(int64_t T, int32_t top_k, int64_t E) {
    const int64_t N = std::max<int64_t>(T, 0) * std::max<int32_t>(top_k, 0);
    return align_up(pack_chunks(N) * std::max<int64_t>(E, 0) * 4) + kAlign;
}

int pdx_pack(const int64_t* selected, const void* weights, int64_t T, int32_t top_k, int64_t E, int32_t* counts,
             int32_t* offsets, int32_t* tokens, int32_t* positions, void* packed_w, int32_t* inverse,
             int32_t* active, void* workspace, size_t workspace_bytes, pdx_stream_t stream) {
    int st = check_route_shape(T, 8, E, top_k);
    if (st) return st;
    if (!selected || !weights || !counts || !offsets || !tokens || !positions || !packed_w || !inverse || !active)
        return fail(PDX_ERR_INVALID, "null packing argument");
    if (workspace_bytes < pdx_pack_workspace_bytes(T, top_k, E) || !workspace)
        return fail(PDX_ERR_WORKSPACE, "pack workspace too small");
    PackOut o{counts, offsets, tokens, positions, static_cast<uint16_t*>(packed_w), inverse, active};
    st = launch_pack(selected, static_cast<const uint16_t*>(weights), T, top_k, E, o, static_cast<int*>(workspace),
                     stream);
    return st ? st : ok();
}

int pdx_gather_rows(const void* x, const int32_t* tokens, int64_t rows, int64_t H, void* out, pdx_stream_t stream) {
    if (!x || !tokens || !out || rows < 0) return fail(PDX_ERR_INVALID, "null gather argument");
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    if (rows == 0) return ok();
    k_gather_rows<<<gather_grid(rows), kGatherWarps * 32, 0, stream>>>(
        static_cast<const uint16_t*>(x), tokens, static_cast<int>(rows), static_cast<int>(H),
        static_cast<uint16_t*>(out), nullptr, 0);
    PDX_LAUNCHED();
    return ok();
}

size_t pdx_ffn_workspace_bytes(int64_t rows, int64_t E, int64_t H, int64_t I, int32_t mode) {
    rows = std::max<int64_t>(rows, 1);
    E = std::max<int64_t>(E, 1);
    const int m = resolve_mode(mode, rows, E, H, I);
    return ffn_ws_bytes(rows, E, H, I, m) + kAlign;
}

int pdx_moe_ffn_grouped(const void* x, int64_t T, const int32_t* tokens, const int32_t* offsets,
                        const int32_t* active, int64_t E, int64_t rows, const pdx_expert_weights* weights, int64_t H,
                        int64_t I, void* y_out, int32_t mode, void* workspace, size_t workspace_bytes,
                        pdx_stream_t stream) {
    if (!x || !offsets || !active || !y_out) return fail(PDX_ERR_INVALID, "null FFN argument");
    if (T < 1 || rows < 1 || E < 1) return fail(PDX_ERR_INVALID, "empty FFN batch");
    const int m = resolve_mode(mode, rows, E, H, I);
    int st = check_ffn_shape(H, I, m);
    if (st) return st;
    if ((st = check_weights(weights, H, I))) return st;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)))
        return fail(PDX_ERR_WORKSPACE, "workspace must be non-null and 256-byte aligned");
    Carver c{static_cast<char*>(workspace), workspace_bytes};
    st = launch_ffn(x, T, tokens, offsets, active, E, rows, weights, H, I, y_out, m, c, stream);
    return st ? st : ok();
}

size_t pdx_expert_ffn_workspace_bytes(int64_t n, int64_t H, int64_t I) {
    const int64_t nn = std::max<int64_t>(n, 1);
    const int m = resolve_mode(PDX_FFN_AUTO, nn, 1, H, I);
    return align_up(8) * 2 + align_up(nn * 4) + ffn_ws_bytes(nn, 1, H, I, m) + kAlign;
}

int pdx_expert_ffn(const void* x, int64_t n, const void* gate, const void* up, const void* down, int64_t H, int64_t I,
                   void* y_out, void* workspace, size_t workspace_bytes, pdx_stream_t stream) {
    if (!x || !gate || !up || !down || !y_out) return fail(PDX_ERR_INVALID, "null expert argument");
    if (n < 1) return fail(PDX_ERR_INVALID, "expert input must have at least one row");
    const int m = resolve_mode(PDX_FFN_AUTO, n, 1, H, I);
    int st = check_ffn_shape(H, I, m);
    if (st) return st;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) ||
        workspace_bytes < pdx_expert_ffn_workspace_bytes(n, H, I))
        return fail(PDX_ERR_WORKSPACE, "expert FFN workspace too small");
    pdx_expert_weights w{gate, up, down, 0, 0, 0, 1, nullptr};
    if ((st = check_weights(&w, H, I))) return st;
    Carver c{static_cast<char*>(workspace), workspace_bytes};
    int32_t* offsets = static_cast<int32_t*>(c.take(8));
    int32_t* active = static_cast<int32_t*>(c.take(8));
    int32_t* tokens = static_cast<int32_t*>(c.take(n * 4));
    k_single_expert_setup<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(static_cast<int>(n), offsets,
                                                                                      active, tokens);
    PDX_LAUNCHED();
    st = launch_ffn(x, n, tokens, offsets, active, 1, n, &w, H, I, y_out, m, c, stream);
    return st ? st : ok();
}

int pdx_combine_layernorm(const void* y, const void* weights, const int32_t* inverse, int64_t T, int32_t top_k,
                          int64_t H, const void* residual, float eps, void* out, pdx_stream_t stream) {
    if (!y || !weights || !inverse || !residual || !out) return fail(PDX_ERR_INVALID, "null combine argument");
    if (T < 1 || top_k < 1) return fail(PDX_ERR_INVALID, "empty combine");
    if (top_k > kMaxTopK) return fail(PDX_ERR_UNSUPPORTED, "top_k > %d", kMaxTopK);
    int st = check_norm_shape(H);
    if (st) return st;
    if (!(eps > 0.f)) return fail(PDX_ERR_INVALID, "eps must be positive");
    PDX_PDL_TRY(launch_combine_norm(H, dim3(static_cast<unsigned>(T)), dim3(kCombineThreads), 0, stream,
                           static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(weights), inverse,
                           static_cast<int>(T), static_cast<int>(top_k), static_cast<int>(H),
                           static_cast<int>(T * top_k), static_cast<const uint16_t*>(residual), eps,
                           static_cast<uint16_t*>(out)));
    return ok();
}

int pdx_ep_combine_layernorm(const void* y, int64_t y_rows, const void* weights, const int32_t* inv_ep, int64_t T,
                             int32_t top_k, int64_t H, const void* residual, float eps, void* out,
                             pdx_stream_t stream) {
    if (!y || !weights || !inv_ep || !residual || !out) return fail(PDX_ERR_INVALID, "null combine argument");
    if (T < 1 || top_k < 1 || y_rows < 1) return fail(PDX_ERR_INVALID, "empty combine");
    if (top_k > kMaxTopK) return fail(PDX_ERR_UNSUPPORTED, "top_k > %d", kMaxTopK);
    int st = check_norm_shape(H);
    if (st) return st;
    if (!(eps > 0.f)) return fail(PDX_ERR_INVALID, "eps must be positive");
    PDX_PDL_TRY(launch_combine_norm(H, dim3(static_cast<unsigned>(T)), dim3(kCombineThreads), 0, stream,
                           static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(weights), inv_ep,
                           static_cast<int>(T), static_cast<int>(top_k), static_cast<int>(H),
                           static_cast<int>(y_rows), static_cast<const uint16_t*>(residual), eps,
                           static_cast<uint16_t*>(out)));
    return ok();
}

int pdx_combine(const void* y, const void* weights, const int32_t* inverse, int64_t T, int32_t top_k, int64_t H,
                const void* residual, void* out, pdx_stream_t stream) {
    if (!y || !weights || !inverse || !out) return fail(PDX_ERR_INVALID, "null combine argument");
    if (T < 1 || top_k < 1) return fail(PDX_ERR_INVALID, "empty combine");
    if (top_k > kMaxTopK) return fail(PDX_ERR_UNSUPPORTED, "top_k > %d", kMaxTopK);
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    k_combine<<<static_cast<unsigned>(T), kCombineThreads, 0, stream>>>(
        static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(weights), inverse, static_cast<int>(T), top_k,
        static_cast<int>(H), static_cast<int>(T * top_k), static_cast<const uint16_t*>(residual),
        static_cast<uint16_t*>(out));
    PDX_LAUNCHED();
    return ok();
}

int pdx_residual_layernorm(const void* y, const void* residual, int64_t T, int64_t H, float eps, void* out,
                           pdx_stream_t stream) {
    if (!y || !residual || !out) return fail(PDX_ERR_INVALID, "null layer-norm argument");
    if (T < 1) return fail(PDX_ERR_INVALID, "empty layer-norm batch");
    int st = check_norm_shape(H);
    if (st) return st;
    if (!(eps > 0.f)) return fail(PDX_ERR_INVALID, "eps must be positive");
    PDX_PDL_TRY(launch_pdl(k_residual_layernorm, dim3(static_cast<unsigned>(T)), dim3(kLnThreads), 0, stream,
                           static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(residual),
                           static_cast<int>(T), static_cast<int>(H), eps, static_cast<uint16_t*>(out)));
    return ok();
}

size_t pdx_layer_workspace_bytes(int64_t T, int64_t H, int64_t E, int32_t top_k, int64_t I, int32_t mode) {
    mode &= ~PDX_LAYER_OUT_NORM;
    T = std::max<int64_t>(T, 1);
    E = std::max<int64_t>(E, 1);
    top_k = std::max<int32_t>(top_k, 1);
    const int64_t N = T * top_k;
    Carver c{nullptr, SIZE_MAX};
    c.take(T * E * 2);           // logits
    c.take(route_partial_bytes(T, E));
    c.take(N * 8);               // selected
    c.take(N * 2);               // weights
    carve_pack(c, T, top_k, E, nullptr);
    c.take(N * H * 2);           // y
    const int m = resolve_mode(mode, T * top_k, E, H, I);
    return c.used + ffn_ws_bytes(N, E, H, I, m) + kAlign;
}

int pdx_moe_layer(const void* x, const void* gate, int64_t T, int64_t H, int64_t E, int32_t top_k, int32_t normalize,
                  const pdx_expert_weights* weights, int64_t I, const void* residual, void* out, void* logits_out,
                  int64_t* selected_out, void* weights_out, int32_t* counts_out, int32_t mode, void* workspace,
                  size_t workspace_bytes, pdx_stream_t stream) {
    int st = check_route_shape(T, H, E, top_k);
    if (st) return st;
    if (!x || !gate || !out) return fail(PDX_ERR_INVALID, "null layer argument");
    const bool out_norm = (mode & PDX_LAYER_OUT_NORM) != 0;
    mode &= ~PDX_LAYER_OUT_NORM;
    if (out_norm) {
        if (!residual) return fail(PDX_ERR_INVALID, "PDX_LAYER_OUT_NORM needs a residual");
        if ((st = check_norm_shape(H))) return st;
    }
    const int m = resolve_mode(mode, T * top_k, E, H, I);
    if ((st = check_ffn_shape(H, I, m))) return st;
    if ((st = check_weights(weights, H, I))) return st;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)))
        return fail(PDX_ERR_WORKSPACE, "workspace must be non-null and 256-byte aligned");
    const int64_t N = T * top_k;
    Carver c{static_cast<char*>(workspace), workspace_bytes};
    RouteBufs rb;
    rb.logits = logits_out ? static_cast<uint16_t*>(logits_out) : static_cast<uint16_t*>(c.take(T * E * 2));
    rb.partials = static_cast<double*>(c.take(route_partial_bytes(T, E)));
    rb.selected = selected_out ? selected_out : static_cast<int64_t*>(c.take(N * 8));
    rb.weights = weights_out ? static_cast<uint16_t*>(weights_out) : static_cast<uint16_t*>(c.take(N * 2));
    PackBufs pb = carve_pack(c, T, top_k, E, counts_out);
    uint16_t* y = static_cast<uint16_t*>(c.take(N * H * 2));
    // decode batches: both projections in one launch straight from x
    const bool one_launch = m == PDX_FFN_GEMV && decode_direct_ok(T, N, E, H, I, pb.o.tokens);
    DecodeBufs db{};
    if (one_launch) db = carve_decode(c, T, N, E, H, I, true);
    if (c.overflow) return fail(PDX_ERR_WORKSPACE, "layer workspace too small (%zu > %zu bytes)", c.used, c.cap);
    // the routing kernel also packs when the pack's shared memory fits the default 48 KiB
    // (and then clears the single-launch FFN's tickets and counters)
    const bool fused = T <= kTailMaxTokens && topk_pack_smem_bytes(E, N) <= 48 * 1024;
    const bool zeroed = fused && one_launch;
    if ((st = launch_route(x, gate, T, H, E, top_k, normalize, rb, fused ? &pb.o : nullptr, stream,
                           zeroed ? db.counters : nullptr, zeroed ? db.plan.zero_words : 0)))
        return st;
    if (!fused && (st = launch_pack(rb.selected, rb.weights, T, top_k, E, pb.o, pb.chunk_hist, stream))) return st;
    if (one_launch)
        st = launch_decode_ffn(x, T, pb.o.tokens, pb.o.offsets, pb.o.active, N, weights, H, I, y, db, zeroed, stream);
    else
        st = launch_ffn(x, T, pb.o.tokens, pb.o.offsets, pb.o.active, E, N, weights, H, I, y, m, c, stream);
    if (st) return st;
    if (out_norm)
        PDX_PDL_TRY(launch_combine_norm(H, dim3(static_cast<unsigned>(T)), dim3(kCombineThreads), 0, stream,
                               static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(rb.weights),
                               static_cast<const int32_t*>(pb.o.inverse), static_cast<int>(T),
                               static_cast<int>(top_k), static_cast<int>(H), static_cast<int>(N),
                               static_cast<const uint16_t*>(residual), PDX_LAYER_NORM_EPS,
                               static_cast<uint16_t*>(out)));
    else
        PDX_PDL_TRY(launch_pdl(k_combine, dim3(static_cast<unsigned>(T)), dim3(kCombineThreads), 0, stream,
                               static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(rb.weights),
                               static_cast<const int32_t*>(pb.o.inverse), static_cast<int>(T),
                               static_cast<int>(top_k), static_cast<int>(H), static_cast<int>(N),
                               static_cast<const uint16_t*>(residual), static_cast<uint16_t*>(out)));
    return ok();
}

int pdx_ep_dispatch(const void* x, const int32_t* tokens, const int32_t* positions, const int32_t* offsets, int64_t T,
                    int32_t top_k, int64_t H, int64_t E, int32_t ranks, int64_t capacity, void* send_rows,
                    int32_t* inv_ep, pdx_stream_t stream) {
    if (!x || !tokens || !positions || !offsets || !send_rows || !inv_ep) return fail(PDX_ERR_INVALID, "null EP argument");
    if (T < 1 || top_k < 1 || ranks < 1 || E % ranks || capacity < 1)
        return fail(PDX_ERR_INVALID, "EP dispatch needs T, top_k >= 1, E divisible by ranks, capacity >= 1");
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    if (static_cast<int64_t>(ranks) * capacity >= (int64_t(1) << 31)) return fail(PDX_ERR_UNSUPPORTED, "capacity too large");
    const int64_t rows = T * top_k;
    PDX_PDL_TRY(launch_pdl(k_ep_dispatch, dim3(static_cast<unsigned>(rows)), dim3(256), 0, stream,
                           static_cast<const uint16_t*>(x), tokens, positions, offsets, static_cast<int>(rows),
                           static_cast<int>(H), static_cast<int>(E), static_cast<int>(E / ranks), capacity,
                           static_cast<uint16_t*>(send_rows), inv_ep));
    return ok();
}

int pdx_ep_layout(const int32_t* recv_counts, int32_t ranks, int64_t local_experts, int64_t capacity,
                  int64_t rows_cap, int32_t* offsets_l, int32_t* active_l, int32_t* perm, pdx_stream_t stream) {
    if (!recv_counts || !offsets_l || !active_l || !perm) return fail(PDX_ERR_INVALID, "null EP argument");
    if (ranks < 1 || ranks > 32 || local_experts < 1 || capacity < 0) return fail(PDX_ERR_INVALID, "invalid EP layout");
    if (ranks * local_experts > kEpMaxExperts) return fail(PDX_ERR_UNSUPPORTED, "more than %d experts", kEpMaxExperts);
    if (rows_cap < 0 || rows_cap >= (int64_t(1) << 31)) return fail(PDX_ERR_UNSUPPORTED, "receive buffer too large");
    PDX_PDL_TRY(launch_pdl(k_ep_layout, dim3(1), dim3(1024), 0, stream, recv_counts, static_cast<int>(ranks),
                           static_cast<int>(local_experts), capacity, static_cast<int>(rows_cap), offsets_l,
                           active_l, perm));
    return ok();
}

int pdx_ep_regroup(const void* recv, const int32_t* perm, const int32_t* offsets_l, int64_t local_experts,
                   int64_t rows_cap, int64_t H, void* grouped, pdx_stream_t stream) {
    if (!recv || !perm || !offsets_l || !grouped) return fail(PDX_ERR_INVALID, "null EP argument");
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    if (rows_cap < 1) return ok();
    PDX_PDL_TRY(launch_pdl(k_ep_regroup, dim3(static_cast<unsigned>(rows_cap)), dim3(256), 0, stream,
                           static_cast<const uint16_t*>(recv), perm, offsets_l, static_cast<int>(local_experts),
                           static_cast<int>(rows_cap), static_cast<int>(H), static_cast<uint16_t*>(grouped)));
    return ok();
}

int pdx_ep_ungroup(const void* grouped, const int32_t* perm, const int32_t* offsets_l, int64_t local_experts,
                   int64_t rows_cap, int64_t H, void* recv_layout, pdx_stream_t stream) {
    if (!grouped || !perm || !offsets_l || !recv_layout) return fail(PDX_ERR_INVALID, "null EP argument");
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    if (rows_cap < 1) return ok();
    PDX_PDL_TRY(launch_pdl(k_ep_ungroup, dim3(static_cast<unsigned>(rows_cap)), dim3(256), 0, stream,
                           static_cast<const uint16_t*>(grouped), perm, offsets_l, static_cast<int>(local_experts),
                           static_cast<int>(rows_cap), static_cast<int>(H), static_cast<uint16_t*>(recv_layout)));
    return ok();
}

int pdx_ep_combine(const void* y, int64_t y_rows, const void* weights, const int32_t* inv_ep, int64_t T,
                   int32_t top_k, int64_t H, const void* residual, void* out, pdx_stream_t stream) {
    if (!y || !weights || !inv_ep || !out) return fail(PDX_ERR_INVALID, "null combine argument");
    if (T < 1 || top_k < 1 || y_rows < 1) return fail(PDX_ERR_INVALID, "empty combine");
    if (top_k > kMaxTopK) return fail(PDX_ERR_UNSUPPORTED, "top_k > %d", kMaxTopK);
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    PDX_PDL_TRY(launch_pdl(k_combine, dim3(static_cast<unsigned>(T)), dim3(kCombineThreads), 0, stream,
                           static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(weights), inv_ep,
                           static_cast<int>(T), static_cast<int>(top_k), static_cast<int>(H),
                           static_cast<int>(y_rows), static_cast<const uint16_t*>(residual),
                           static_cast<uint16_t*>(out)));
    return ok();
}

int pdx_p2p_alloc(size_t bytes, void** ptr_out) {
    if (!ptr_out || bytes == 0) return fail(PDX_ERR_INVALID, "invalid exchange allocation");
    *ptr_out = nullptr;
    PDX_CUDA_TRY(cudaMalloc(ptr_out, bytes));
    PDX_CUDA_TRY(cudaMemset(*ptr_out, 0, bytes));
    return ok();
}

int pdx_p2p_free(void* ptr) {
    if (ptr) PDX_CUDA_TRY(cudaFree(ptr));
    return ok();
}

int pdx_ipc_handle(void* ptr, void* handle_out) {
    if (!ptr || !handle_out) return fail(PDX_ERR_INVALID, "null IPC argument");
    cudaIpcMemHandle_t h;
    PDX_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr));
    std::memcpy(handle_out, &h, sizeof(h));
    return ok();
}

int pdx_ipc_open(const void* handle, void** ptr_out) {
    if (!handle || !ptr_out) return fail(PDX_ERR_INVALID, "null IPC argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    PDX_CUDA_TRY(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
    return ok();
}

int pdx_ipc_close(void* ptr) {
    if (ptr) PDX_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return ok();
}

static pdx::P2PLayer to_p2p(const pdx_p2p_layer* l) {
    pdx::P2PLayer o;
    o.recv = reinterpret_cast<const unsigned long long*>(l->recv);
    o.back = reinterpret_cast<const unsigned long long*>(l->back);
    o.cnt = reinterpret_cast<const unsigned long long*>(l->cnt);
    o.rflag = reinterpret_cast<const unsigned long long*>(l->rflag);
    o.bflag = reinterpret_cast<const unsigned long long*>(l->bflag);
    o.step = reinterpret_cast<unsigned long long*>(l->step);
    o.ticket = l->ticket;
    return o;
}

static int check_p2p(const pdx_p2p_layer* l, int32_t ranks, int32_t rank) {
    if (!l || !l->recv || !l->back || !l->cnt || !l->rflag || !l->bflag || !l->step || !l->ticket)
        return fail(PDX_ERR_INVALID, "incomplete exchange layer");
    if (ranks < 1 || ranks > 32 || rank < 0 || rank >= ranks) return fail(PDX_ERR_INVALID, "invalid rank");
    return PDX_OK;
}

int pdx_ep_dispatch_p2p(const void* x, const int32_t* tokens, const int32_t* positions, const int32_t* offsets,
                        int64_t T, int32_t top_k, int64_t H, int64_t E, int32_t ranks, int32_t rank, int64_t capacity,
                        const pdx_p2p_layer* layer, int32_t* inv_ep, pdx_stream_t stream) {
    int st = check_p2p(layer, ranks, rank);
    if (st) return st;
    if (!x || !tokens || !positions || !offsets || !inv_ep) return fail(PDX_ERR_INVALID, "null EP argument");
    if (T < 1 || top_k < 1 || E % ranks || capacity < 1 || E / ranks > kEpMaxExperts / ranks)
        return fail(PDX_ERR_INVALID, "invalid expert-parallel shape");
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    int sms = 0;
    if ((st = device_setup(&sms))) return st;
    const int64_t rows = T * top_k;
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 2 * sms)));
    pdx::k_ep_dispatch_p2p<<<grid, 256, 0, stream>>>(
        static_cast<const uint16_t*>(x), tokens, positions, offsets, static_cast<int>(T * top_k),
        static_cast<int>(H), static_cast<int>(E), static_cast<int>(E / ranks), ranks, rank, capacity,
        to_p2p(layer), inv_ep);
    PDX_LAUNCHED();
    return ok();
}

int pdx_ep_layout_p2p(int32_t ranks, int32_t rank, int64_t local_experts, int64_t capacity, int64_t rows_cap,
                      const pdx_p2p_layer* layer, int32_t* offsets_l, int32_t* active_l, int32_t* perm,
                      pdx_stream_t stream) {
    int st = check_p2p(layer, ranks, rank);
    if (st) return st;
    if (!offsets_l || !active_l || !perm) return fail(PDX_ERR_INVALID, "null EP layout argument");
    if (local_experts < 1 || ranks * local_experts > pdx::kEpMaxExperts || capacity < 1 || rows_cap < 1)
        return fail(PDX_ERR_UNSUPPORTED, "expert-parallel layout supports ranks*local_experts <= %d",
                    pdx::kEpMaxExperts);
    pdx::k_ep_layout_p2p<<<1, 1024, 0, stream>>>(ranks, static_cast<int>(local_experts), capacity,
                                                 static_cast<int>(rows_cap), to_p2p(layer), rank, offsets_l,
                                                 active_l, perm, g_flag_wait_ns.load());
    PDX_LAUNCHED();
    return ok();
}

int pdx_ep_return_p2p(const void* grouped, const int32_t* perm, const int32_t* offsets_l, int64_t local_experts,
                      int64_t rows_cap, int64_t H, int32_t ranks, int32_t rank, int64_t capacity,
                      const pdx_p2p_layer* layer, pdx_stream_t stream) {
    int st = check_p2p(layer, ranks, rank);
    if (st) return st;
    if (!grouped || !perm || !offsets_l || rows_cap < 1 || capacity < 1)
        return fail(PDX_ERR_INVALID, "invalid EP return argument");
    if (H < 8 || H % 8) return fail(PDX_ERR_UNSUPPORTED, "H must be a positive multiple of 8");
    int sms = 0;
    if ((st = device_setup(&sms))) return st;
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((rows_cap + 7) / 8, 2 * sms)));
    pdx::k_ep_return_p2p<<<grid, 256, 0, stream>>>(
        static_cast<const uint16_t*>(grouped), perm, offsets_l, static_cast<int>(local_experts),
        static_cast<int>(rows_cap), static_cast<int>(H), ranks, rank, capacity, to_p2p(layer));
    PDX_LAUNCHED();
    return ok();
}

int pdx_ep_wait_back(int32_t ranks, int32_t rank, const pdx_p2p_layer* layer, pdx_stream_t stream) {
    int st = check_p2p(layer, ranks, rank);
    if (st) return st;
    pdx::k_ep_wait_back<<<1, 32, 0, stream>>>(ranks, rank, to_p2p(layer), g_flag_wait_ns.load());
    PDX_LAUNCHED();
    return ok();
}

int pdx_set_flag_wait_limit_ns(uint64_t ns) {
    if (ns == 0) ns = kWaitLimitNs;
    if (ns > kMaxFlagWaitNs) return fail(PDX_ERR_INVALID, "flag wait limit above %llu ns",
                                         static_cast<unsigned long long>(kMaxFlagWaitNs));
    g_flag_wait_ns.store(ns);
    return ok();
}

int pdx_device_error(pdx_stream_t stream, uint32_t* code_out) {
    PDX_CUDA_TRY(cudaStreamSynchronize(stream));
    unsigned int code = 0;
    PDX_CUDA_TRY(cudaMemcpyFromSymbol(&code, g_device_error, sizeof(code)));
    if (code) {
        const unsigned int zero = 0;
        PDX_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
    }
    if (code_out) *code_out = code;
    if (code) return fail(PDX_ERR_DEVICE, "device error code %u", code);
    return ok();
}

}  // extern "C"

// Allocation-free packing (fixed device scratch); uses the helpers above.
#include "pack_static.cu"

// native host side of offload mode (calls the entry points above)
#include "offload_host.cu"
