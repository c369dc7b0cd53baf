// Expert-parallel exchange over NVLink peer memory (no collective library).
//
// Each rank's exchange region is mapped into every other rank (CUDA IPC), so
// the dispatch kernel stores the packed rows straight into the destination
// rank's receive block and the return kernel stores the FFN rows straight into
// the source rank's return block; a flag per (layer, source) published with a
// system-scope release after the stores tells the receiver a block is
// complete.  Per layer and rank:
//   recv [R][C][H]  rows from source s at block s        (written by rank s)
//   back [R][C][H]  results from rank d at block d       (written by rank d)
//   cnt  [R][EL]    rows per local expert from source s  (written by rank s)
//   rflag[R], bflag[R]  step number of the last complete block of each source
// One buffer per layer: a rank can only reach layer l of step n+1 after every
// rank has finished step n, so no block is rewritten while being read.  The
// step number of the layer is a local counter, advanced by the last kernel of
// the layer (k_ep_wait_back), so the graph of a decode step replays unchanged.
// Waits are bounded (2 s unless pdx_set_flag_wait_limit_ns sets another
// limit); on a timeout the error word is raised and the layout is left empty,
// so nothing downstream reads or writes outside its buffers.  Everything is
// plain st/ld over NVLink: no TMA, no cluster or multicast operation.
#include "pdx_common.cuh"

namespace pdx {

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Pointer table of one layer, one entry per rank (this rank's own entry is
// its local address).
struct P2PLayer {
    const unsigned long long* recv;   // [R] -> uint16_t[R*C*H]
    const unsigned long long* back;   // [R] -> uint16_t[R*C*H]
    const unsigned long long* cnt;    // [R] -> int32_t[R*EL]
    const unsigned long long* rflag;  // [R] -> uint64_t[R]
    const unsigned long long* bflag;  // [R] -> uint64_t[R]
    unsigned long long* step;         // local: completed steps of this layer
    unsigned int* ticket;             // local: [2] last-CTA tickets (dispatch, return)
};

// Bounded wait until every flag[s] (s < R) reaches `want`; one CTA.  Returns
// false (and raises the error word) after `limit_ns` of wall time.
__device__ bool wait_flags(const unsigned long long* flags, int R, unsigned long long want,
                           unsigned long long limit_ns) {
    __shared__ int s_bad;
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < R) {
        const unsigned long long t0 = global_timer_ns();
        while (ld_acquire_sys(flags + threadIdx.x) < want) {
            if (global_timer_ns() - t0 > limit_ns) {
                raise_error(PDX_DEVERR_WAIT_TIMEOUT);
                s_bad = 1;
                break;
            }
            __nanosleep(200);
        }
    }
    __syncthreads();
    return s_bad == 0;
}

// Dispatch: packed row p (expert e, destination d = e / EL, position pos in the
// block for d) -> recv block `me` of rank d; inv_ep[positions[p]] = d*C + pos.
// One warp per row, grid-stride; the last CTA publishes the per-expert counts
// and then the flags of all ranks.
__global__ void __launch_bounds__(256) k_ep_dispatch_p2p(const uint16_t* __restrict__ x,
                                                         const int32_t* __restrict__ tokens,
                                                         const int32_t* __restrict__ positions,
                                                         const int32_t* __restrict__ offsets, int rows, int H, int E,
                                                         int EL, int R, int me, int64_t C, P2PLayer lay,
                                                         int32_t* __restrict__ inv_ep) {
    griddep_wait();
    const unsigned long long step = *lay.step + 1ull;
    const int warps = static_cast<int>(blockDim.x >> 5);
    const int lane = static_cast<int>(threadIdx.x & 31);
    for (int p = static_cast<int>(blockIdx.x) * warps + static_cast<int>(threadIdx.x >> 5); p < rows;
         p += static_cast<int>(gridDim.x) * warps) {
        int64_t dst = -1;
        int d = 0;
        if (lane == 0) {
            int lo = 0, hi = E - 1;  // expert of row p: largest e with offsets[e] <= p
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (offsets[mid] <= p) lo = mid; else hi = mid - 1;
            }
            d = lo / EL;
            const int64_t pos = p - offsets[d * EL];
            dst = static_cast<int64_t>(d) * C + pos;
            if (pos >= C) {
                raise_error(PDX_DEVERR_BAD_EXPERT);
                dst = -1;
            }
            inv_ep[positions[p]] = static_cast<int32_t>(dst < 0 ? 0 : dst);
        }
        dst = __shfl_sync(0xffffffffu, dst, 0);
        d = __shfl_sync(0xffffffffu, d, 0);
        if (dst < 0) continue;
        const int64_t pos = dst - static_cast<int64_t>(d) * C;
        uint16_t* out = reinterpret_cast<uint16_t*>(lay.recv[d]) + (static_cast<int64_t>(me) * C + pos) * H;
        const uint16_t* src = x + static_cast<size_t>(tokens[p]) * H;
        for (int c = lane * 8; c < H; c += 32 * 8)
            *reinterpret_cast<uint4*>(out + c) = __ldg(reinterpret_cast<const uint4*>(src + c));
    }
    // completion: every CTA's stores are visible system-wide before the last
    // CTA publishes
    __threadfence_system();
    __syncthreads();
    __shared__ unsigned int s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(&lay.ticket[0], 1u) == gridDim.x - 1 ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();
    for (int i = threadIdx.x; i < R * EL; i += blockDim.x) {
        const int d = i / EL, l = i % EL;
        const int e = d * EL + l;
        reinterpret_cast<int32_t*>(lay.cnt[d])[me * EL + l] = offsets[e + 1] - offsets[e];
    }
    __threadfence_system();
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < R)
        st_release_sys(reinterpret_cast<unsigned long long*>(lay.rflag[threadIdx.x]) + me, step);
    if (threadIdx.x == 0) lay.ticket[0] = 0u;
}

// Waits for every source's block of this layer, then lays the received rows
// out by local expert exactly as k_ep_layout (block s at s*C).  One CTA.
__global__ void __launch_bounds__(1024) k_ep_layout_p2p(int R, int EL, int64_t C, int rows_cap, P2PLayer lay, int me,
                                                        int32_t* __restrict__ offsets_l,
                                                        int32_t* __restrict__ active_l, int32_t* __restrict__ perm,
                                                        unsigned long long limit_ns) {
    griddep_wait();
    const unsigned long long step = *lay.step + 1ull;
    const bool ok = wait_flags(reinterpret_cast<const unsigned long long*>(lay.rflag[me]), R, step, limit_ns);
    __shared__ int s_cnt[kEpMaxExperts];
    __shared__ int s_blk[kEpMaxExperts];
    __shared__ int s_grp[kEpMaxExperts];
    __shared__ int s_off[kEpMaxExperts + 1];
    __shared__ int s_src[32], s_tot[kEpMaxExperts];
    const int n = R * EL;
    const int32_t* cnt = reinterpret_cast<const int32_t*>(lay.cnt[me]);
    for (int i = threadIdx.x; i < n; i += blockDim.x) s_cnt[i] = ok ? __ldcg(cnt + i) : 0;
    __syncthreads();
    // a source's counts must fit its block: clamp (and flag) anything else
    ep_layout_block(s_cnt, R, EL, C, true, s_blk, s_grp, s_off, s_src, s_tot, active_l);
    for (int i = threadIdx.x; i <= EL; i += blockDim.x) offsets_l[i] = s_off[i];
    ep_layout_perm(s_blk, s_grp, s_off, R, EL, rows_cap, perm);
}

// Return: regrouped FFN row g (receive position perm[g] = s*C + pos) -> back
// block `me` of rank s at pos; one warp per row, grid-stride.  The last CTA
// publishes the flags of all ranks (also those this rank returned nothing to).
__global__ void __launch_bounds__(256) k_ep_return_p2p(const uint16_t* __restrict__ yg,
                                                       const int32_t* __restrict__ perm,
                                                       const int32_t* __restrict__ offsets_l, int EL, int rows_cap,
                                                       int H, int R, int me, int64_t C, P2PLayer lay) {
    griddep_wait();
    const unsigned long long step = *lay.step + 1ull;
    const int warps = static_cast<int>(blockDim.x >> 5);
    const int lane = static_cast<int>(threadIdx.x & 31);
    const int total = min(rows_cap, offsets_l[EL]);
    for (int g = static_cast<int>(blockIdx.x) * warps + static_cast<int>(threadIdx.x >> 5); g < total;
         g += static_cast<int>(gridDim.x) * warps) {
        const int p = perm[g];
        if (p < 0 || p >= rows_cap) {
            if (lane == 0) raise_error(PDX_DEVERR_BAD_EXPERT);
            continue;
        }
        const int s = static_cast<int>(p / C);
        const int64_t pos = p - static_cast<int64_t>(s) * C;
        uint16_t* dst = reinterpret_cast<uint16_t*>(lay.back[s]) + (static_cast<int64_t>(me) * C + pos) * H;
        for (int c = lane * 8; c < H; c += 32 * 8)
            *reinterpret_cast<uint4*>(dst + c) =
                __ldg(reinterpret_cast<const uint4*>(yg + static_cast<size_t>(g) * H + c));
    }
    __threadfence_system();
    __syncthreads();
    __shared__ unsigned int s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(&lay.ticket[1], 1u) == gridDim.x - 1 ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();
    if (static_cast<int>(threadIdx.x) < R)
        st_release_sys(reinterpret_cast<unsigned long long*>(lay.bflag[threadIdx.x]) + me, step);
    if (threadIdx.x == 0) lay.ticket[1] = 0u;
}

// Waits for every rank's returned block of this layer, then closes the layer
// (advances its step counter).  One CTA; the combine that follows reads the
// back blocks.
__global__ void __launch_bounds__(32) k_ep_wait_back(int R, int me, P2PLayer lay, unsigned long long limit_ns) {
    griddep_wait();
    const unsigned long long step = *lay.step + 1ull;
    wait_flags(reinterpret_cast<const unsigned long long*>(lay.bflag[me]), R, step, limit_ns);
    __syncthreads();
    if (threadIdx.x == 0) *lay.step = step;
}

}  // namespace pdx
