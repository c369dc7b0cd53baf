/*
 * pdx_moe.h -- C ABI of the B200 (sm_100a) MoE expert-execution library.
 *
 * One shared library, libpdx_moe.so, implements the per-layer MoE expert path
 * of PDScope (nezha-Anonymous/PDScope): top-k gate softmax with
 * renormalisation, ragged token->expert packing, the grouped SwiGLU expert FFN
 * and the fused weighted combine.  Each entry point below names the reference
 * interface it replaces (paths inside the reference project).
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are caller-owned DEVICE pointers (BF16 passed as
 *     void*, raw IEEE bfloat16 bits), dense row-major, on the current device.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) and never synchronises the host, except pdx_device_error.
 *   - Nothing allocates device memory.  Scratch comes from a caller-provided
 *     workspace whose minimum size the matching *_workspace_bytes query
 *     returns; it must be 256-byte aligned.
 *   - The return value is a pdx_status; on failure pdx_last_error() returns a
 *     thread-local message.  PDX_ERR_INVALID corresponds to the reference's
 *     ValueError (contract violations), the others to RuntimeError.
 */
#ifndef PDX_MOE_H
#define PDX_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *pdx_stream_t; /* identical to cudaStream_t */

typedef enum pdx_status {
    PDX_OK = 0,
    PDX_ERR_INVALID = 1,     /* bad shape/argument: reference raises ValueError */
    PDX_ERR_UNSUPPORTED = 2, /* valid, but outside the shapes these kernels cover */
    PDX_ERR_WORKSPACE = 3,   /* workspace NULL, misaligned or too small */
    PDX_ERR_CUDA = 4,        /* a CUDA runtime call failed */
    PDX_ERR_DEVICE = 5       /* a kernel raised the device error word */
} pdx_status;

/* Device error codes (read back by pdx_device_error). */
#define PDX_DEVERR_NONE 0u
#define PDX_DEVERR_WAIT_TIMEOUT 1u  /* a bounded mbarrier wait expired */
#define PDX_DEVERR_BAD_EXPERT 2u    /* routed expert id outside [0, E) */
#define PDX_DEVERR_BAD_SLOT 3u      /* slot_of_expert[e] outside [0, num_slots) */

/* Thread-local description of the last failure ("" after success). */
const char *pdx_last_error(void);

/* ABI version of this header (bumped on any signature change). */
#define PDX_ABI_VERSION 1
int pdx_abi_version(void);

/*
 * Expert weight placement.  Expert e lives in slot s = slot_of_expert[e]
 * (identity when slot_of_expert is NULL); its three projections are
 *   gate = (bf16*)gate + s*gate_stride  [I, H]   (gate_proj.weight)
 *   up   = (bf16*)up   + s*up_stride    [I, H]   (up_proj.weight)
 *   down = (bf16*)down + s*down_stride  [H, I]   (down_proj.weight)
 * Strides are in elements.  The reference's ExpertExecutor cache slab
 * (expertbench/executor.py:219-227, 323-331: equal slots holding gate|up|down
 * back to back) is described without copying by gate = slab,
 * up = slab + I*H, down = slab + 2*I*H and all strides = 3*I*H.
 * gate_stride must be a multiple of H and down_stride a multiple of I.
 */
typedef struct pdx_expert_weights {
    const void *gate;
    const void *up;
    const void *down;
    int64_t gate_stride;
    int64_t up_stride;
    int64_t down_stride;
    int64_t num_slots;
    const int32_t *slot_of_expert; /* device int32[E] or NULL */
} pdx_expert_weights;

/* ---------------------------------------------------------------------------
 * a1. Routing.  Replaces route() -- expertbench/adapters/qwen.py:140-152:
 *   logits = F.linear(x, gate)                       (BF16, [T,E])
 *   p = softmax(logits.float()); w, ids = topk(p, k) (ties as on CUDA)
 *   if normalize: w /= w.sum(-1);  weights = w.to(bf16)
 * Logits are the exact dot products rounded once to BF16 (FP64 accumulation).
 * logits_out may be NULL (then the workspace holds them).
 */
size_t pdx_route_workspace_bytes(int64_t T, int64_t E);
int pdx_route_topk(const void *x, const void *gate, int64_t T, int64_t H, int64_t E,
                   int32_t top_k, int32_t normalize, void *logits_out,
                   int64_t *selected_out, void *weights_out, void *workspace,
                   size_t workspace_bytes, pdx_stream_t stream);

/* Softmax + top-k + renormalisation of given BF16 logits [T,E]
 * (qwen.py:148-152 alone). */
int pdx_topk_from_logits(const void *logits, int64_t T, int64_t E, int32_t top_k,
                         int32_t normalize, int64_t *selected_out, void *weights_out,
                         pdx_stream_t stream);

/* ---------------------------------------------------------------------------
 * a2/a3. Packing.  Replaces compact_expert_groups() --
 * expertbench/pdscope_runtime.py:16-39 (and expert_groups(), qwen.py:155-174,
 * which yields the same order).  Stable counting sort of the T*k assignments
 * taken in slot-major order (flat index f = s*T + t):
 *   counts[E]       assignments per expert            (bincount, :26)
 *   offsets[E+1]    exclusive prefix of counts
 *   tokens[T*k]     packed row p -> token t           (order % T, :29)
 *   positions[T*k]  packed row p -> t*k + s           (:29)
 *   packed_w[T*k]   BF16 weights in packed order      (:31)
 *   inverse[T*k]    t*k + s -> packed row p
 *   active[E+1]     active[0] = #experts with count>0, active[1..] = their ids
 *                   ascending
 * Ids outside [0,E) set PDX_DEVERR_BAD_EXPERT (reference: ValueError, :27).
 */
size_t pdx_pack_workspace_bytes(int64_t T, int32_t top_k, int64_t E);
int pdx_pack(const int64_t *selected, const void *weights, int64_t T, int32_t top_k,
             int64_t E, int32_t *counts, int32_t *offsets, int32_t *tokens,
             int32_t *positions, void *packed_w, int32_t *inverse, int32_t *active,
             void *workspace, size_t workspace_bytes, pdx_stream_t stream);

/* Allocation-free packing.  No counterpart in the reference: PDScope always
 * packs with torch allocations.  Same contract and outputs as pdx_pack, for
 * callers that cannot allocate device memory where they pack (a plugin inside
 * a host process whose allocator owns the device's memory, an FFI caller with
 * no device allocator, a latency-critical path that cannot afford
 * cudaMalloc's device-wide synchronisation).  Its scratch is a fixed
 * file-scope device array of PDX_PACK_STATIC_MAX_HIST_INTS ints (256 KiB, held
 * by every GPU that loads the library until exit); sizes needing more,
 * ceil(T*top_k/4096)*E > PDX_PACK_STATIC_MAX_HIST_INTS (possible only when
 * T*top_k > 8192), return PDX_ERR_UNSUPPORTED.  All calls share that array: calls whose kernels
 * overlap on the GPU race.  The first call on a device resolves the array's
 * device address (cudaGetSymbolAddress) with that device current; make it
 * before any stream capture.  The address is kept for the life of the
 * process's primary context on that device (not across cudaDeviceReset). */
#define PDX_PACK_STATIC_MAX_HIST_INTS 65536
int pdx_pack_static(const int64_t *selected, const void *weights, int64_t T, int32_t top_k,
                    int64_t E, int32_t *counts, int32_t *offsets, int32_t *tokens,
                    int32_t *positions, void *packed_w, int32_t *inverse, int32_t *active,
                    pdx_stream_t stream);

/* a4. Row gather x[tokens[p]] -> out[p]  (inputs[flat_tokens],
 * pdscope_runtime.py:333-336). */
int pdx_gather_rows(const void *x, const int32_t *tokens, int64_t rows, int64_t H,
                    void *out, pdx_stream_t stream);

/* ---------------------------------------------------------------------------
 * a5. Grouped expert FFN.  Replaces the per-expert ExpertExecutor.gpu ->
 * expert_forward loop (expertbench/executor.py:454-488, qwen.py:87-90):
 *   y[p] = F.linear(silu(F.linear(x[tok], Wg)) * F.linear(x[tok], Wu), Wd)
 * for every packed row p of every active expert, UNWEIGHTED, in packed order,
 * with the reference's BF16 roundings (after each linear, after silu, after
 * the product).  `x` is the [T,H] token matrix; rows are gathered through
 * `tokens` (tokens == NULL: x already holds the `rows` rows in packed order).
 * mode: 0 = auto (the decode path up to 48 rows per expert on average, else
 * the prefill path); 1 = decode path (weights streamed by TMA as the
 * tcgen05 M operand, tokens as N, split-K for few experts; with `tokens`
 * given and T <= 64 one launch computes both projections straight from x,
 * otherwise a row gather and one launch per projection); 2 = prefill path
 * (tcgen05 grouped GEMM tiled over tokens, 128 x 256 tiles on single CTAs);
 * 3 = SIMT weight-streaming GEMV (an independent implementation kept for
 * cross-checks and for shapes the tcgen05 paths do not tile); 4 = the prefill
 * path (same as 2); 5 = the prefill path on CTA pairs (tcgen05 cta_group::2,
 * 256 x 256 tiles); 6 = the decode path always as row gather + one launch
 * per projection (a cross-check of the single-launch form).
 */
#define PDX_FFN_AUTO 0
#define PDX_FFN_GEMV 1
#define PDX_FFN_GEMM 2
#define PDX_FFN_SIMT 3
#define PDX_FFN_GEMM_1CTA 4
#define PDX_FFN_GEMM_PAIR 5
#define PDX_FFN_GEMV_STAGED 6
size_t pdx_ffn_workspace_bytes(int64_t rows, int64_t E, int64_t H, int64_t I, int32_t mode);
int pdx_moe_ffn_grouped(const void *x, int64_t T, const int32_t *tokens,
                        const int32_t *offsets, const int32_t *active, int64_t E,
                        int64_t rows, const pdx_expert_weights *weights, int64_t H,
                        int64_t I, void *y_out, int32_t mode, void *workspace,
                        size_t workspace_bytes, pdx_stream_t stream);

/* Single expert, the ExpertExecutor.gpu_backend plug-in
 * (expertbench/executor.py:178, 476-477): y[n,H] = expert_forward(x[n,H]). */
size_t pdx_expert_ffn_workspace_bytes(int64_t n, int64_t H, int64_t I);
int pdx_expert_ffn(const void *x, int64_t n, const void *gate, const void *up,
                   const void *down, int64_t H, int64_t I, void *y_out, void *workspace,
                   size_t workspace_bytes, pdx_stream_t stream);

/* ---------------------------------------------------------------------------
 * a7. Combine.  Replaces the fused merge
 *   output.index_add_(0, index, rows.to(bf16) * weight)
 * (expertbench/pdscope_runtime.py:454-464; native finish_and_merge,
 * native/native_layer_dispatch.cpp:73-90).  Deterministic gather form:
 *   out[t] = bf16( residual[t] + sum_s bf16(y[inverse[t*k+s]] * w[t*k+s]) )
 * accumulated in FP32 over s = 0..k-1.  residual may be NULL (zeros, as the
 * reference's torch.zeros_like output); `weights` is the [T,k] routing weight
 * matrix.
 */
int pdx_combine(const void *y, const void *weights, const int32_t *inverse, int64_t T,
                int32_t top_k, int64_t H, const void *residual, void *out,
                pdx_stream_t stream);

/* Next-layer activation of a multi-layer stack, as the reference's two-layer
 * protocol forms it (benchmarks/pdscope_compare.py:609-705, `x =
 * F.layer_norm(out.float() + x.float(), (H,)).to(bf16)`): out[t] =
 * bf16(layer_norm(float(y[t]) + float(residual[t]))) -- no affine, population
 * variance, FP32 statistics.  y, residual, out: [T,H] BF16; H a multiple of 8,
 * <= 8192; out may alias y or residual.  Not part of the reference's MoE path;
 * it keeps a synthetic stack's activations at unit scale. */
int pdx_residual_layernorm(const void *y, const void *residual, int64_t T, int64_t H, float eps, void *out,
                           pdx_stream_t stream);

/* Combine and next-layer norm in one pass (bit-identical to pdx_combine with
 * residual = NULL followed by pdx_residual_layernorm): out[t] =
 * bf16(layer_norm(bf16(sum_s bf16(y_s * w_s)) + residual[t])).  residual must
 * not alias y; it may alias out. */
int pdx_combine_layernorm(const void *y, const void *weights, const int32_t *inverse, int64_t T, int32_t top_k,
                          int64_t H, const void *residual, float eps, void *out, pdx_stream_t stream);

/* OR into pdx_moe_layer's mode: out = layer_norm(MoE(x) + residual) with
 * eps PDX_LAYER_NORM_EPS (the fused combine above); residual is required. */
#define PDX_LAYER_OUT_NORM 0x100
#define PDX_LAYER_NORM_EPS 1e-5f

/* ---- Offload mode: experts in pinned host memory, copy-engine pipeline ------
 * The native host side of the reference's demand/prefetch pipeline
 * (ExpertExecutor.load/finish_load, expertbench/executor.py:333-390; the
 * demand loop and next-layer prefetch of PDScopeCudaRuntime.forward,
 * expertbench/pdscope_runtime.py:284-399).  Expert (l, e) is the
 * 3*inter*hidden BF16 slot [gate_proj | up_proj | down_proj] at
 * host_experts + (l*experts + e) * 3*inter*hidden.  Per layer a fixed list of
 * experts (the hot table's first hot_per_layer rows, then an optional static
 * tier) keeps device slots; every other expert is copied on demand into an
 * LRU ring of cache_slots slots; the experts the next layer's gate picks on
 * the current activation are prefetched behind the demand copies.  The
 * caller provides the device pool (pdx_offload_pool_bytes) and workspace
 * (pdx_offload_workspace_bytes); create() allocates only host-side objects
 * (a copy stream, events, pinned staging).  One handle per device; calls on
 * one handle must be serialised. */
typedef struct pdx_offload pdx_offload;
typedef struct {
    int32_t layers, experts, hidden, inter, top_k, normalize;
    const void *const *gates;      /* [layers] device BF16 [experts, hidden] */
    const void *host_experts;      /* pinned host BF16, layout above */
    const int32_t *fixed_count;    /* [layers] experts with fixed slots per layer */
    const int32_t *fixed_experts;  /* per layer, fixed_count[l] expert ids, concatenated */
    int32_t hot_per_layer;         /* the first this-many fixed experts of a layer count as hot */
    int32_t chunk;                 /* demand experts per FFN launch */
    int32_t prefetch;              /* 1: prefetch the next layer's predicted experts */
    int64_t cache_slots;           /* LRU ring slots */
    int64_t max_tokens;            /* largest T of a forward call */
} pdx_offload_config;
typedef struct {
    int64_t h2d_bytes, demand_copies, prefetch_copies, prefetch_used, prefetch_wasted;
    int64_t cache_hits, hot_hits, warm_hits, expert_uses, layers;
} pdx_offload_stats;
size_t pdx_offload_pool_bytes(const pdx_offload_config *cfg);
size_t pdx_offload_workspace_bytes(const pdx_offload_config *cfg);
int pdx_offload_create(const pdx_offload_config *cfg, void *pool, void *workspace, size_t workspace_bytes,
                       pdx_offload **out);
/* out = residual + MoE_layer(x) (residual may be NULL), or with norm != 0
 * layer_norm(MoE_layer(x) + residual).  Synchronises `stream` once (the
 * routing counts), as the reference's grouping does. */
int pdx_offload_forward_layer(pdx_offload *h, int32_t layer, const void *x, int64_t T, const void *residual,
                              int32_t norm, void *out, pdx_stream_t stream);
int pdx_offload_get_stats(const pdx_offload *h, pdx_offload_stats *out);
void pdx_offload_destroy(pdx_offload *h);

/* Trace of the last pdx_offload_forward_layer call: what the reference's
 * per-layer row records (PDScopeCudaRuntime.forward's return value,
 * expertbench/pdscope_runtime.py:492-512 -- token counts, the placement of
 * every routed expert, the demand copies, the prefetch ledger), produced by
 * the native engine itself.  Optional outputs (NULL = skipped):
 * counts_out [2*experts] (routed counts of this layer, then the predicted
 * counts of the next layer, zeros on the last layer), placement_out [experts]
 * (PDX_PLACE_*), prefetch_out [experts] (the first prefetch_issued entries:
 * next-layer experts whose copies this layer issued, in issue order),
 * demand_out [experts] (the first `demand` entries, in copy order). */
#define PDX_PLACE_NONE 0     /* not routed in this layer */
#define PDX_PLACE_HOT 1      /* hot-table slot */
#define PDX_PLACE_WARM 2     /* static cache tier slot */
#define PDX_PLACE_CACHE 3    /* cache-ring hit whose copy had completed at reveal */
#define PDX_PLACE_LOADING 4  /* cache-ring hit whose copy was still in flight at reveal */
#define PDX_PLACE_DEMAND 5   /* copied on demand by this layer */
typedef struct {
    int32_t layer, routed_experts, hot, warm, cache_ready, cache_loading, demand, demand_chunks;
    int32_t prefetch_issued, prefetch_used, prefetch_skipped;
    int64_t tokens, h2d_bytes;
} pdx_offload_trace;
int pdx_offload_last_trace(const pdx_offload *h, pdx_offload_trace *out, int32_t *counts_out,
                           int32_t *placement_out, int32_t *prefetch_out, int32_t *demand_out);
/* Device-to-device copy of the last call's selected ids [T, top_k] int64
 * (which = 0) or of the next-layer prediction's (which = 1), so a caller can
 * fingerprint the routing as the reference's row does (selected_sha256).
 * T must be the last call's token count. */
int pdx_offload_copy_selected(const pdx_offload *h, int32_t which, int64_t T, int64_t *selected_out,
                              pdx_stream_t stream);

/* ---------------------------------------------------------------------------
 * Whole layer: route -> pack -> grouped FFN -> combine, all on `stream`, no
 * host synchronisation (PDScopeCudaRuntime.forward's GPU work,
 * expertbench/pdscope_runtime.py:208-512, with every expert resident).
 * Optional outputs (NULL = kept in the workspace): logits [T,E] BF16,
 * selected [T,k] int64, weights [T,k] BF16, counts [E] int32.
 */
size_t pdx_layer_workspace_bytes(int64_t T, int64_t H, int64_t E, int32_t top_k,
                                 int64_t I, int32_t mode);
int pdx_moe_layer(const void *x, const void *gate, int64_t T, int64_t H, int64_t E,
                  int32_t top_k, int32_t normalize, const pdx_expert_weights *weights,
                  int64_t I, const void *residual, void *out, void *logits_out,
                  int64_t *selected_out, void *weights_out, int32_t *counts_out,
                  int32_t mode, void *workspace, size_t workspace_bytes,
                  pdx_stream_t stream);

/* ---------------------------------------------------------------------------
 * Expert parallelism.  No counterpart in the reference (single-GPU); these
 * lay the same layer out over `ranks` GPUs with expert e on rank e / EL,
 * EL = E / ranks; the exchange itself is NCCL all-to-all (see
 * pdscope_b200/expert_parallel.py).
 *
 * pdx_ep_dispatch: after route + pack, copy each packed row p (expert e,
 * destination d = e / EL, position pos = p - offsets[d*EL]) from x[tokens[p]]
 * to send_rows[d*capacity + pos] and set inv_ep[positions[p]] = d*capacity +
 * pos.  capacity must be >= T*min(top_k, EL) (the most rows one rank can send
 * to another).
 */
int pdx_ep_dispatch(const void *x, const int32_t *tokens, const int32_t *positions,
                    const int32_t *offsets, int64_t T, int32_t top_k, int64_t H, int64_t E,
                    int32_t ranks, int64_t capacity, void *send_rows, int32_t *inv_ep,
                    pdx_stream_t stream);

/* pdx_ep_layout: from recv_counts[s*EL + l] (rows received from rank s for
 * local expert l) build the regrouped layout in which each local expert's
 * rows from every source are contiguous (sources in rank order):
 * offsets_l[EL+1] (offsets_l[EL] = rows received), active_l[EL+1] (format of
 * pdx_pack's active) and perm[g] = receive-buffer row of regrouped row g.
 * capacity > 0: source block s starts at s*capacity in the receive buffer;
 * capacity == 0: blocks are back to back.  rows_cap = rows of the receive
 * buffer (and of perm); nothing is written past it. */
int pdx_ep_layout(const int32_t *recv_counts, int32_t ranks, int64_t local_experts,
                  int64_t capacity, int64_t rows_cap, int32_t *offsets_l, int32_t *active_l,
                  int32_t *perm, pdx_stream_t stream);

/* pdx_ep_regroup: grouped[g] = recv[perm[g]]; pdx_ep_ungroup:
 * recv_layout[perm[g]] = grouped[g]; both for g < offsets_l[EL] (read on the
 * device), rows_cap = rows of the receive buffer.  Between them,
 * pdx_moe_ffn_grouped runs on `grouped` with tokens = NULL, offsets_l,
 * active_l and the rank's EL local experts. */
int pdx_ep_regroup(const void *recv, const int32_t *perm, const int32_t *offsets_l,
                   int64_t local_experts, int64_t rows_cap, int64_t H, void *grouped,
                   pdx_stream_t stream);
int pdx_ep_ungroup(const void *grouped, const int32_t *perm, const int32_t *offsets_l,
                   int64_t local_experts, int64_t rows_cap, int64_t H, void *recv_layout,
                   pdx_stream_t stream);

/* pdx_ep_combine: pdx_combine over y[y_rows, H] addressed through inv_ep. */
int pdx_ep_combine(const void *y, int64_t y_rows, const void *weights, const int32_t *inv_ep,
                   int64_t T, int32_t top_k, int64_t H, const void *residual, void *out,
                   pdx_stream_t stream);
/* pdx_ep_combine with the next-layer norm fused (as pdx_combine_layernorm):
 * out[t] = bf16(layer_norm(bf16(sum_s bf16(y[inv_ep[t*k+s]] * w)) + residual[t])). */
int pdx_ep_combine_layernorm(const void *y, int64_t y_rows, const void *weights, const int32_t *inv_ep, int64_t T,
                             int32_t top_k, int64_t H, const void *residual, float eps, void *out,
                             pdx_stream_t stream);

/* ---- Expert-parallel exchange over NVLink peer memory ----------------------
 * The padded (decode) exchange without a collective library: each rank's
 * exchange region is mapped into the other ranks (CUDA IPC).  Per layer and
 * rank the region holds recv [R][C][H] and back [R][C][H] BF16 blocks, cnt
 * [R][EL] int32 and rflag/bflag [R] uint64; a pdx_p2p_layer gives, per rank
 * (index = rank), the addresses of that rank's recv/back/cnt/rflag/bflag of
 * this layer as mapped in the calling process, plus this rank's step counter
 * and two ticket words (zero-initialised).  Sequence per layer:
 *   pdx_ep_dispatch_p2p -> pdx_ep_layout_p2p -> pdx_ep_regroup (local recv) ->
 *   pdx_moe_ffn_grouped -> pdx_ep_return_p2p -> pdx_ep_wait_back ->
 *   pdx_ep_combine / pdx_combine_layernorm (local back, y_rows = R*C).
 * The two wait steps spin (bounded, 2 s) on flags written by the other ranks:
 * every rank must run the same sequence, one rank per GPU. */
typedef struct {
    const uint64_t *recv, *back, *cnt, *rflag, *bflag; /* device arrays [R] of addresses */
    uint64_t *step;                                     /* device, this rank */
    uint32_t *ticket;                                   /* device [2], this rank */
} pdx_p2p_layer;
int pdx_p2p_alloc(size_t bytes, void **ptr_out);   /* cudaMalloc + zero fill (exchange regions only) */
int pdx_p2p_free(void *ptr);
int pdx_ipc_handle(void *ptr, void *handle_out);   /* 64-byte cudaIpcMemHandle_t */
int pdx_ipc_open(const void *handle, void **ptr_out);
int pdx_ipc_close(void *ptr);
int pdx_ep_dispatch_p2p(const void *x, const int32_t *tokens, const int32_t *positions, const int32_t *offsets,
                        int64_t T, int32_t top_k, int64_t H, int64_t E, int32_t ranks, int32_t rank, int64_t capacity,
                        const pdx_p2p_layer *layer, int32_t *inv_ep, pdx_stream_t stream);
int pdx_ep_layout_p2p(int32_t ranks, int32_t rank, int64_t local_experts, int64_t capacity, int64_t rows_cap,
                      const pdx_p2p_layer *layer, int32_t *offsets_l, int32_t *active_l, int32_t *perm,
                      pdx_stream_t stream);
int pdx_ep_return_p2p(const void *grouped, const int32_t *perm, const int32_t *offsets_l, int64_t local_experts,
                      int64_t rows_cap, int64_t H, int32_t ranks, int32_t rank, int64_t capacity,
                      const pdx_p2p_layer *layer, pdx_stream_t stream);
int pdx_ep_wait_back(int32_t ranks, int32_t rank, const pdx_p2p_layer *layer, pdx_stream_t stream);

/* Wall-time limit of the two flag waits above, in ns (0 = the default 2 s;
 * at most 60 s), for launches made after the call (a captured graph keeps the
 * limit it was captured with).  A wait that runs out raises
 * PDX_DEVERR_WAIT_TIMEOUT, leaves the layout empty and returns.  No
 * counterpart in the reference, which has no multi-GPU path; the analogue
 * there is the run guard's deadline (benchmarks/pdscope_compare.py:153-161). */
int pdx_set_flag_wait_limit_ns(uint64_t ns);

/* Synchronise `stream`, then read and clear this device's error word.
 * *code_out receives a PDX_DEVERR_* value; returns PDX_ERR_DEVICE if nonzero. */
int pdx_device_error(pdx_stream_t stream, uint32_t *code_out);

/* Number of kernels this library has launched in this process (all devices);
 * used by benchmarks to report their own launch count. */
uint64_t pdx_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* PDX_MOE_H */
