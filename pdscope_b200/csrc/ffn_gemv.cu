// Decode-path grouped expert FFN: weight-streaming GEMV over active experts.
//
// Reference: expert_forward() -- expertbench/adapters/qwen.py:87-90, run once
// per routed expert by ExpertExecutor.gpu (expertbench/executor.py:454-488).
// With few tokens per expert the FFN is a weight stream: every BF16 weight is
// read once from HBM with 128-bit loads while the handful of token rows of
// that expert sit in shared memory.  Work items are (active expert, block of
// weight rows) pairs taken from the device-side active list, so no host sync
// is needed and idle experts cost nothing.
#include "pdx_common.cuh"

namespace pdx {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kTokChunk = 8;  // token rows staged per pass

struct ExpertSlab {
    const uint16_t* gate;
    const uint16_t* up;
    const uint16_t* down;
    int64_t gate_stride, up_stride, down_stride, num_slots;
    const int32_t* slot_of_expert;
};

__device__ __forceinline__ int64_t expert_slot(const ExpertSlab& w, int e) {
    const int64_t s = w.slot_of_expert ? static_cast<int64_t>(w.slot_of_expert[e]) : static_cast<int64_t>(e);
    if (s < 0 || s >= w.num_slots) {
        raise_error(PDX_DEVERR_BAD_SLOT);
        return -1;
    }
    return s;
}

__device__ __forceinline__ void fma8(const uint4& wv, const uint4& xv, float& acc) {
    const uint32_t a[4] = {wv.x, wv.y, wv.z, wv.w};
    const uint32_t b[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc = fmaf(__uint_as_float(a[i] << 16), __uint_as_float(b[i] << 16), acc);
        acc = fmaf(__uint_as_float(a[i] & 0xFFFF0000u), __uint_as_float(b[i] & 0xFFFF0000u), acc);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Dot products of one weight row (length K, BF16) with nt staged rows
// xs[t*K ...] (smem); lane-strided 16-byte chunks, FP32 accumulation.
// Returns the full sums in every lane.
template <int MAXC>
__device__ __forceinline__ void row_dots(const uint16_t* __restrict__ wrow, const uint16_t* xs, int K, int nt,
                                         float* out) {
    const int lane = static_cast<int>(lane_id());
    float acc[kTokChunk];
#pragma unroll
    for (int t = 0; t < kTokChunk; ++t) acc[t] = 0.f;
    for (int base = 0; base < K; base += MAXC * 256) {
        uint4 wv[MAXC];
#pragma unroll
        for (int j = 0; j < MAXC; ++j) {
            const int kk = base + j * 256 + lane * 8;
            wv[j] = kk < K ? __ldg(reinterpret_cast<const uint4*>(wrow + kk)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < MAXC; ++j) {
            const int kk = base + j * 256 + lane * 8;
            if (kk < K) {
#pragma unroll
                for (int t = 0; t < kTokChunk; ++t)
                    if (t < nt) fma8(wv[j], *reinterpret_cast<const uint4*>(xs + t * K + kk), acc[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kTokChunk; ++t)
        if (t < nt) out[t] = warp_sum(acc[t]);
}

// h[p, n] = bf16( bf16(silu(bf16(x_p . Wg[n]))) * bf16(x_p . Wu[n]) )
// RB gate rows + RB up rows per work item; RPW = 2*RB/8 rows per warp.
// dynamic smem: xs[kTokChunk][H] bf16 + res[2*RB][kTokChunk] f32.
template <int RB>
__global__ void __launch_bounds__(kGemvThreads) k_gateup_gemv(const uint16_t* __restrict__ x,
                                                              const int32_t* __restrict__ tokens,
                                                              const int32_t* __restrict__ offsets,
                                                              const int32_t* __restrict__ active, ExpertSlab w,
                                                              int H, int I, uint16_t* __restrict__ h_out) {
    constexpr int RPW = (2 * RB) / kGemvWarps;
    static_assert(RPW >= 1 && RPW * kGemvWarps == 2 * RB, "rows per warp");
    extern __shared__ __align__(16) unsigned char smem_gemv[];
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem_gemv);
    float* res = reinterpret_cast<float*>(smem_gemv + static_cast<size_t>(kTokChunk) * H * 2);
    const int warp = static_cast<int>(threadIdx.x >> 5);
    const int n_active = active[0];
    const int blocks_per_expert = I / RB;
    const int items = n_active * blocks_per_expert;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int e = active[1 + item / blocks_per_expert];
        const int n0 = (item % blocks_per_expert) * RB;
        const int64_t slot = expert_slot(w, e);
        if (slot < 0) continue;
        const int seg0 = offsets[e];
        const int seg1 = offsets[e + 1];
        for (int c0 = seg0; c0 < seg1; c0 += kTokChunk) {
            const int nt = min(kTokChunk, seg1 - c0);
            __syncthreads();  // previous pass done with xs/res
            const int vec_per_row = H / 8;
            for (int i = threadIdx.x; i < nt * vec_per_row; i += blockDim.x) {
                const int t = i / vec_per_row, v = i % vec_per_row;
                const int src_row = tokens ? tokens[c0 + t] : c0 + t;  // NULL: rows already in packed order
                reinterpret_cast<uint4*>(xs + t * H)[v] =
                    __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(src_row) * H) + v);
            }
            __syncthreads();
#pragma unroll 1
            for (int r = 0; r < RPW; ++r) {
                const int lr = warp * RPW + r;  // 0..2RB-1: first RB gate rows, then RB up rows
                const uint16_t* wrow = lr < RB ? w.gate + slot * w.gate_stride + static_cast<int64_t>(n0 + lr) * H
                                               : w.up + slot * w.up_stride + static_cast<int64_t>(n0 + lr - RB) * H;
                float dots[kTokChunk];
                row_dots<8>(wrow, xs, H, nt, dots);
                if (lane_id() == 0)
                    for (int t = 0; t < nt; ++t) res[lr * kTokChunk + t] = dots[t];
            }
            __syncthreads();
            for (int i = threadIdx.x; i < RB * nt; i += blockDim.x) {
                const int j = i / nt, t = i % nt;
                const float g = round_bf16(res[j * kTokChunk + t]);
                const float u = round_bf16(res[(RB + j) * kTokChunk + t]);
                const float s = round_bf16(__fdiv_rn(g, 1.0f + expf(-g)));
                h_out[static_cast<size_t>(c0 + t) * I + n0 + j] = f2bits(s * u);
            }
        }
    }
}

// y[p, n] = bf16( h_p . Wd[n] );  RD = 8 * RPW rows of Wd per work item.
// dynamic smem: hs[kTokChunk][I] bf16 + res[RD][kTokChunk] f32.
template <int RPW>
__global__ void __launch_bounds__(kGemvThreads) k_down_gemv(const uint16_t* __restrict__ h,
                                                            const int32_t* __restrict__ offsets,
                                                            const int32_t* __restrict__ active, ExpertSlab w, int H,
                                                            int I, uint16_t* __restrict__ y) {
    constexpr int RD = RPW * kGemvWarps;
    extern __shared__ __align__(16) unsigned char smem_gemv[];
    uint16_t* hs = reinterpret_cast<uint16_t*>(smem_gemv);
    float* res = reinterpret_cast<float*>(smem_gemv + static_cast<size_t>(kTokChunk) * I * 2);
    const int warp = static_cast<int>(threadIdx.x >> 5);
    const int n_active = active[0];
    const int blocks_per_expert = H / RD;
    const int items = n_active * blocks_per_expert;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int e = active[1 + item / blocks_per_expert];
        const int n0 = (item % blocks_per_expert) * RD;
        const int64_t slot = expert_slot(w, e);
        if (slot < 0) continue;
        const int seg0 = offsets[e];
        const int seg1 = offsets[e + 1];
        for (int c0 = seg0; c0 < seg1; c0 += kTokChunk) {
            const int nt = min(kTokChunk, seg1 - c0);
            __syncthreads();
            const int vec_per_row = I / 8;
            for (int i = threadIdx.x; i < nt * vec_per_row; i += blockDim.x) {
                const int t = i / vec_per_row, v = i % vec_per_row;
                reinterpret_cast<uint4*>(hs + t * I)[v] =
                    reinterpret_cast<const uint4*>(h + static_cast<size_t>(c0 + t) * I)[v];
            }
            __syncthreads();
#pragma unroll 1
            for (int r = 0; r < RPW; ++r) {
                const int lr = warp * RPW + r;
                const uint16_t* wrow = w.down + slot * w.down_stride + static_cast<int64_t>(n0 + lr) * I;
                float dots[kTokChunk];
                row_dots<4>(wrow, hs, I, nt, dots);
                if (lane_id() == 0)
                    for (int t = 0; t < nt; ++t) res[lr * kTokChunk + t] = dots[t];
            }
            __syncthreads();
            for (int i = threadIdx.x; i < RD * nt; i += blockDim.x) {
                const int t = i / RD, j = i % RD;
                y[static_cast<size_t>(c0 + t) * H + n0 + j] = f2bits(res[j * kTokChunk + t]);
            }
        }
    }
}

}  // namespace pdx
