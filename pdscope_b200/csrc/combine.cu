// Combine and row-gather kernels.
//
// Combine replaces the fused merge of expertbench/pdscope_runtime.py:454-464
//   output.index_add_(0, index, rows.to(bf16) * weight)
// (and the native finish_and_merge scatter, native/native_layer_dispatch.cpp:88)
// with a deterministic gather: every output row is owned by one CTA, which
// reads its k expert rows through the inverse permutation, forms the BF16
// product y*w exactly as the reference does, accumulates in FP32 in slot
// order and rounds once.  No atomics, so results do not depend on scheduling.
#include "pdx_common.cuh"

namespace pdx {

constexpr int kCombineThreads = 256;

__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        w[i] = static_cast<uint32_t>(f2bits(f[2 * i])) | (static_cast<uint32_t>(f2bits(f[2 * i + 1])) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Combine setup: the k (row, weight) pairs of token t into shared memory.
// Entries outside [0, y_rows) are flagged and contribute nothing.
__device__ __forceinline__ void combine_slots(const uint16_t* __restrict__ weights,
                                              const int32_t* __restrict__ inverse, int t, int k, int y_rows,
                                              int* s_row, float* s_w) {
    if (threadIdx.x < static_cast<unsigned>(k)) {
        int row = inverse[static_cast<size_t>(t) * k + threadIdx.x];
        float w = bits2f(weights[static_cast<size_t>(t) * k + threadIdx.x]);
        if (row < 0 || row >= y_rows) {
            raise_error(PDX_DEVERR_BAD_EXPERT);
            row = 0;
            w = 0.f;
        }
        s_row[threadIdx.x] = row;
        s_w[threadIdx.x] = w;
    }
    __syncthreads();
}

// acc[0..8) += sum_{s<k} bf16(y[row_s][c..c+8) * w_s), FP32, in slot order
// (the loads of up to 8 expert rows are issued before accumulating).
__device__ __forceinline__ void combine_chunk(const uint16_t* __restrict__ y, const int* s_row, const float* s_w,
                                              int k, int H, int c, float* acc) {
    for (int s0 = 0; s0 < k; s0 += 8) {
        uint4 rv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (s0 + j < k)
                rv[j] = __ldg(reinterpret_cast<const uint4*>(y + static_cast<size_t>(s_row[s0 + j]) * H + c));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (s0 + j < k) {
                float v[8];
                unpack8(rv[j], v);
                const float w = s_w[s0 + j];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] += round_bf16(v[i] * w);
            }
        }
    }
}

// out[t] = bf16( residual[t] + sum_{s<k} bf16(y[inverse[t*k+s]] * w[t*k+s]) )
// y has y_rows rows; inverse entries outside [0, y_rows) are flagged and skipped.
__global__ void __launch_bounds__(kCombineThreads) k_combine(const uint16_t* __restrict__ y,
                                                             const uint16_t* __restrict__ weights,
                                                             const int32_t* __restrict__ inverse, int T, int k,
                                                             int H, int y_rows, const uint16_t* __restrict__ residual,
                                                             uint16_t* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const int t = static_cast<int>(blockIdx.x);
    if (t >= T) return;
    __shared__ int s_row[32];
    __shared__ float s_w[32];
    combine_slots(weights, inverse, t, k, y_rows, s_row, s_w);
    for (int c = static_cast<int>(threadIdx.x) * 8; c < H; c += blockDim.x * 8) {
        float acc[8];
        if (residual) {
            unpack8(*reinterpret_cast<const uint4*>(residual + static_cast<size_t>(t) * H + c), acc);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        }
        combine_chunk(y, s_row, s_w, k, H, c, acc);
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + c) = pack8(acc);
    }
}

// out[p] = x[tokens[p]]  (inputs[flat_tokens], pdscope_runtime.py:333-336).
// One warp per packed row over a grid sized to the SMs (a CTA per row made
// the block scheduler the limit at prefill sizes: 99,600 rows took 127 us);
// each lane keeps up to 8 16-byte chunks of its row in flight.  CTA 0 also
// clears `zero_words` words (the split-K tickets of the FFN kernels that
// follow), so no memset node separates the kernels of the chain.
constexpr int kGatherWarps = 8;
__global__ void __launch_bounds__(kGatherWarps * 32) k_gather_rows(const uint16_t* __restrict__ x,
                                                                   const int32_t* __restrict__ tokens, int rows,
                                                                   int H, uint16_t* __restrict__ out,
                                                                   unsigned int* __restrict__ zero_ptr,
                                                                   int zero_words) {
    griddep_wait();
    griddep_launch();
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < zero_words; i += blockDim.x) zero_ptr[i] = 0u;
    const int lane = static_cast<int>(threadIdx.x & 31);
    const int chunks = H / 8;   // 16-byte chunks per row
    for (int p = static_cast<int>(blockIdx.x) * kGatherWarps + static_cast<int>(threadIdx.x >> 5); p < rows;
         p += static_cast<int>(gridDim.x) * kGatherWarps) {
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(__ldg(tokens + p)) * H);
        uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(p) * H);
        for (int c0 = 0; c0 < chunks; c0 += 8 * 32) {
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + j * 32 + lane;
                if (c < chunks) v[j] = __ldg(src + c);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + j * 32 + lane;
                if (c < chunks) dst[c] = v[j];
            }
        }
    }
}

// Clears n words (the split-K tickets) when the FFN reads rows already in
// packed order and no gather kernel runs.
__global__ void k_zero_words(unsigned int* __restrict__ p, int n) {
    griddep_wait();
    griddep_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = 0u;
}

// Next-layer activation of a synthetic multi-layer stack, as the reference's
// two-layer protocol forms it (benchmarks/pdscope_compare.py:609-705):
//   out[t] = bf16( layer_norm( float(y[t]) + float(residual[t]) ) )
// (no affine, population variance, eps; FP32 statistics).  y is the MoE layer
// output (BF16).  One CTA per token; up to kLnMaxPerThread values per thread
// stay in registers between the two reductions.
constexpr int kLnThreads = 256;
constexpr int kLnMaxPerThread = 32;  // H <= 8192

__device__ __forceinline__ float block_sum_ln(float v, float* red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
    __syncthreads();  // red[] free from a previous reduction
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) tot += red[w];  // fixed order
    return tot;
}

// Normalise the row held in v (this thread's chunks c = (tid + 256 j) * 8)
// and store it: population variance, FP32 statistics in a fixed order.
template <int VPT>
__device__ __forceinline__ void layernorm_store(float (&v)[VPT], float sum, int H, float eps, uint16_t* out_row,
                                                float* red) {
    const float mean = block_sum_ln(sum, red) / static_cast<float>(H);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < VPT / 8; ++j) {
        const int c = (static_cast<int>(threadIdx.x) + j * kLnThreads) * 8;
        if (c < H) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float d = v[j * 8 + i] - mean;
                q += d * d;
            }
        }
    }
    const float var = block_sum_ln(q, red) / static_cast<float>(H);
    const float inv = 1.0f / sqrtf(var + eps);
#pragma unroll
    for (int j = 0; j < VPT / 8; ++j) {
        const int c = (static_cast<int>(threadIdx.x) + j * kLnThreads) * 8;
        if (c < H) {
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (v[j * 8 + i] - mean) * inv;
            *reinterpret_cast<uint4*>(out_row + c) = pack8(o);
        }
    }
}

// out may alias y or residual: a CTA reads its whole row before writing it.
__global__ void __launch_bounds__(kLnThreads) k_residual_layernorm(const uint16_t* y, const uint16_t* residual,
                                                                   int T, int H, float eps, uint16_t* out) {
    griddep_wait();
    griddep_launch();
    const int t = static_cast<int>(blockIdx.x);
    if (t >= T) return;
    __shared__ float red[32];
    float v[kLnMaxPerThread];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kLnMaxPerThread / 8; ++j) {
        const int c = (static_cast<int>(threadIdx.x) + j * kLnThreads) * 8;
        if (c < H) {
            float a[8], b[8];
            unpack8(*reinterpret_cast<const uint4*>(y + static_cast<size_t>(t) * H + c), a);
            unpack8(*reinterpret_cast<const uint4*>(residual + static_cast<size_t>(t) * H + c), b);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[j * 8 + i] = a[i] + b[i];
                s += v[j * 8 + i];
            }
        }
    }
    layernorm_store<kLnMaxPerThread>(v, s, H, eps, out + static_cast<size_t>(t) * H, red);
}

// Combine and next-layer norm in one pass, bit-identical to k_combine (no
// residual) followed by k_residual_layernorm:
//   out[t] = bf16( layer_norm( bf16(sum_s bf16(y_s * w_s)) + residual[t] ) )
// residual must not alias y (the expert rows of other tokens); it may alias out.
// VPT = values per thread (8 per 2048 of H): only the registers the row needs,
// so more tokens are in flight per SM (each token's chain is load -> two block
// reductions -> store; at prefill sizes the kernel is bound by how many of
// those chains overlap).
template <int VPT>
__global__ void __launch_bounds__(kCombineThreads) k_combine_norm(const uint16_t* __restrict__ y,
                                                                  const uint16_t* __restrict__ weights,
                                                                  const int32_t* __restrict__ inverse, int T, int k,
                                                                  int H, int y_rows, const uint16_t* residual,
                                                                  float eps, uint16_t* out) {
    griddep_wait();
    griddep_launch();
    const int t = static_cast<int>(blockIdx.x);
    if (t >= T) return;
    __shared__ int s_row[32];
    __shared__ float s_w[32];
    __shared__ float red[32];
    combine_slots(weights, inverse, t, k, y_rows, s_row, s_w);
    float v[VPT];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < VPT / 8; ++j) {
        const int c = (static_cast<int>(threadIdx.x) + j * kLnThreads) * 8;
        if (c < H) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            combine_chunk(y, s_row, s_w, k, H, c, acc);
            float r[8];
            unpack8(*reinterpret_cast<const uint4*>(residual + static_cast<size_t>(t) * H + c), r);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[j * 8 + i] = round_bf16(acc[i]) + r[i];
                sum += v[j * 8 + i];
            }
        }
    }
    layernorm_store<VPT>(v, sum, H, eps, out + static_cast<size_t>(t) * H, red);
}

}  // namespace pdx
