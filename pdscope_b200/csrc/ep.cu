// Expert-parallel layout kernels (experts sharded over ranks).
//
// The reference is single-GPU; this is the B200 expert-parallel form of the
// same layer.  Expert e lives on rank e / EL (EL = E / ranks).  After the
// local route + pack, the packed rows bound for rank d are the contiguous
// range [offsets[d*EL], offsets[(d+1)*EL]), ordered by expert.
//
// A receiving rank gets one block per source rank s; inside block s the rows
// of local expert l follow one another.  k_ep_layout + k_ep_regroup make each
// local expert's rows from every source contiguous (source order s = 0..R-1,
// then the source's own order) -- each expert's weights are then streamed once
// per layer however many ranks sent it rows -- and k_ep_ungroup puts the FFN
// results back in the receive layout for the return exchange.
#include "pdx_common.cuh"
#include "routing.cuh"

namespace pdx {

constexpr int kEpMaxExperts = 1024;

// send[d*C + pos] = x[tokens[p]] for packed row p of destination d at position
// pos = p - offsets[d*EL]; inv_ep[positions[p]] = d*C + pos (the combine map).
__global__ void __launch_bounds__(256) k_ep_dispatch(const uint16_t* __restrict__ x,
                                                     const int32_t* __restrict__ tokens,
                                                     const int32_t* __restrict__ positions,
                                                     const int32_t* __restrict__ offsets, int rows, int H, int E,
                                                     int EL, int64_t capacity, uint16_t* __restrict__ send,
                                                     int32_t* __restrict__ inv_ep) {
    griddep_wait();
    griddep_launch();
    const int p = static_cast<int>(blockIdx.x);
    if (p >= rows) return;
    __shared__ int64_t s_dst;
    if (threadIdx.x == 0) {
        int lo = 0, hi = E - 1;  // expert of row p: largest e with offsets[e] <= p
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (offsets[mid] <= p) lo = mid; else hi = mid - 1;
        }
        const int d = lo / EL;
        const int64_t pos = p - offsets[d * EL];
        int64_t dst = static_cast<int64_t>(d) * capacity + pos;
        if (pos >= capacity) {  // cannot happen for capacity >= T*min(k, EL); flag and drop
            raise_error(PDX_DEVERR_BAD_EXPERT);
            dst = -1;
        }
        s_dst = dst;
        inv_ep[positions[p]] = static_cast<int32_t>(dst < 0 ? 0 : dst);
    }
    __syncthreads();
    const int64_t dst = s_dst;
    if (dst < 0) return;
    const size_t src = static_cast<size_t>(tokens[p]) * H;
    for (int c = static_cast<int>(threadIdx.x) * 8; c < H; c += blockDim.x * 8)
        *reinterpret_cast<uint4*>(send + dst * H + c) = __ldg(reinterpret_cast<const uint4*>(x + src + c));
}

// Layout of the regrouped rows from the counts s_cnt[s*EL + l] (shared
// memory), computed by the whole CTA:
//   s_blk[s*EL+l]  start of (s, l) inside the receive buffer (source block s at
//                  s*capacity, or blocks back to back when capacity == 0)
//   s_grp[s*EL+l]  start of (s, l) inside the regrouped rows (expert-major, then source)
//   s_off[l]       start of local expert l's regrouped rows (s_off[EL] = total)
//   active_l       active_l[0] = #experts with rows, then their ids ascending
// With `clamp`, a source whose counts overflow its block of `capacity` rows
// has the excess counts zeroed and the error word raised.  One thread per
// source for the per-source prefixes, one per expert for the per-expert sums,
// one warp for the prefix over experts.  smem s_src[R], s_tot[EL].
__device__ void ep_layout_block(int* s_cnt, int R, int EL, int64_t capacity, bool clamp, int* s_blk, int* s_grp,
                                int* s_off, int* s_src, int* s_tot, int32_t* active_l) {
    const int tid = static_cast<int>(threadIdx.x);
    if (clamp && tid < R) {
        int64_t run = 0;
        for (int l = 0; l < EL; ++l) {
            int c = s_cnt[tid * EL + l];
            if (c < 0 || run + c > capacity) {
                raise_error(PDX_DEVERR_BAD_EXPERT);
                c = 0;
            }
            s_cnt[tid * EL + l] = c;
            run += c;
        }
    }
    __syncthreads();
    if (tid < R) {
        int t = 0;
        for (int l = 0; l < EL; ++l) t += s_cnt[tid * EL + l];
        s_src[tid] = t;
    }
    for (int l = tid; l < EL; l += blockDim.x) {
        int t = 0;
        for (int s = 0; s < R; ++s) t += s_cnt[s * EL + l];
        s_tot[l] = t;
    }
    __syncthreads();
    if (tid < R) {
        int64_t run = capacity > 0 ? static_cast<int64_t>(tid) * capacity : 0;
        if (capacity == 0)
            for (int s = 0; s < tid; ++s) run += s_src[s];
        for (int l = 0; l < EL; ++l) {
            s_blk[tid * EL + l] = static_cast<int>(run);
            run += s_cnt[tid * EL + l];
        }
    }
    if (tid < 32) warp_exclusive_scan(s_tot, EL, s_off, active_l, nullptr);
    __syncthreads();
    for (int l = tid; l < EL; l += blockDim.x) {
        int g = s_off[l];
        for (int s = 0; s < R; ++s) {
            s_grp[s * EL + l] = g;
            g += s_cnt[s * EL + l];
        }
    }
    __syncthreads();
}

// perm[g] = receive-buffer row of regrouped row g, for g < rows_cap: one
// thread per regrouped row, its (source, expert) pair found by bisection over
// the pairs in regrouped order (s_grp is ascending in l-major, s-minor order).
__device__ void ep_layout_perm(const int* s_blk, const int* s_grp, const int* s_off, int R, int EL, int rows_cap,
                               int32_t* __restrict__ perm) {
    const int total = min(s_off[EL], rows_cap);
    const int n = R * EL;
    for (int g = static_cast<int>(threadIdx.x); g < total; g += blockDim.x) {
        int lo = 0, hi = n - 1;   // largest pair index q (q = l*R + s) with s_grp[pair] <= g
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            const int l = mid / R, s = mid % R;
            if (s_grp[s * EL + l] <= g) lo = mid; else hi = mid - 1;
        }
        // the last pair starting at or before g is the one holding g: pairs
        // between it and g's pair would start after g
        const int l = lo / R, s = lo % R;
        perm[g] = s_blk[s * EL + l] + (g - s_grp[s * EL + l]);
    }
}

// Layout of the regrouped rows from recv_counts[s*EL + l]:
//   offsets_l[l]  start of local expert l's rows (offsets_l[EL] = total)
//   active_l      active_l[0] = #experts with rows, then their ids
//   perm[g]       receive-buffer row of regrouped row g (g < total)
// capacity > 0: source block s starts at s*capacity; capacity == 0: blocks
// are back to back.  One CTA (R*EL <= 1024 pairs); entries of perm at or past
// rows_cap are never written.
__global__ void __launch_bounds__(1024) k_ep_layout(const int32_t* __restrict__ recv_counts, int R, int EL,
                                                    int64_t capacity, int rows_cap, int32_t* __restrict__ offsets_l,
                                                    int32_t* __restrict__ active_l, int32_t* __restrict__ perm) {
    griddep_wait();
    griddep_launch();
    __shared__ int s_cnt[kEpMaxExperts];   // [s][l]
    __shared__ int s_blk[kEpMaxExperts];   // start of (s, l) inside the receive buffer
    __shared__ int s_grp[kEpMaxExperts];   // start of (s, l) inside the regrouped rows
    __shared__ int s_off[kEpMaxExperts + 1];
    __shared__ int s_src[32], s_tot[kEpMaxExperts];
    const int n = R * EL;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s_cnt[i] = recv_counts[i];
    __syncthreads();
    ep_layout_block(s_cnt, R, EL, capacity, false, s_blk, s_grp, s_off, s_src, s_tot, active_l);
    for (int i = threadIdx.x; i <= EL; i += blockDim.x) offsets_l[i] = s_off[i];
    ep_layout_perm(s_blk, s_grp, s_off, R, EL, rows_cap, perm);
}

// xg[g] = recv[perm[g]] for g < offsets_l[EL] (device-side bound).
__global__ void __launch_bounds__(256) k_ep_regroup(const uint16_t* __restrict__ recv,
                                                    const int32_t* __restrict__ perm,
                                                    const int32_t* __restrict__ offsets_l, int EL, int rows_cap,
                                                    int H, uint16_t* __restrict__ xg) {
    griddep_wait();
    griddep_launch();
    const int g = static_cast<int>(blockIdx.x);
    if (g >= rows_cap || g >= offsets_l[EL]) return;
    const int src = perm[g];
    if (src < 0 || src >= rows_cap) {
        raise_error(PDX_DEVERR_BAD_EXPERT);
        return;
    }
    for (int c = static_cast<int>(threadIdx.x) * 8; c < H; c += blockDim.x * 8)
        *reinterpret_cast<uint4*>(xg + static_cast<size_t>(g) * H + c) =
            __ldg(reinterpret_cast<const uint4*>(recv + static_cast<size_t>(src) * H + c));
}

// y_recv[perm[g]] = yg[g] for g < offsets_l[EL].
__global__ void __launch_bounds__(256) k_ep_ungroup(const uint16_t* __restrict__ yg,
                                                    const int32_t* __restrict__ perm,
                                                    const int32_t* __restrict__ offsets_l, int EL, int rows_cap,
                                                    int H, uint16_t* __restrict__ y_recv) {
    griddep_wait();
    griddep_launch();
    const int g = static_cast<int>(blockIdx.x);
    if (g >= rows_cap || g >= offsets_l[EL]) return;
    const int dst = perm[g];
    if (dst < 0 || dst >= rows_cap) {
        raise_error(PDX_DEVERR_BAD_EXPERT);
        return;
    }
    for (int c = static_cast<int>(threadIdx.x) * 8; c < H; c += blockDim.x * 8)
        *reinterpret_cast<uint4*>(y_recv + static_cast<size_t>(dst) * H + c) =
            __ldg(reinterpret_cast<const uint4*>(yg + static_cast<size_t>(g) * H + c));
}

}  // namespace pdx
