// Offload mode, host side in C++: the per-layer orchestration of the
// copy-engine expert pipeline (the native successor of the reference's
// per-layer Python loop, expertbench/pdscope_runtime.py:284-399, and of
// native/native_layer_dispatch.cpp).
//
// Experts live in pinned host memory; per layer a fixed set (hot table + an
// optional static tier) keeps device slots, the rest are demand-copied into an
// LRU cache ring on a copy stream.  One layer:
//   1. route + pack with this layer's gate, and with the next layer's gate on
//      the same activation (gate-fallback predictor, pdscope_runtime.py:245-249);
//      both expert-count vectors come back in one pinned copy + one sync;
//   2. fixed / ring-resident experts go straight to the grouped FFN; misses are
//      copied (one cudaMemcpyAsync per 9 MiB expert slot) in chunks, one event
//      per chunk; the next layer's predicted experts are queued behind them;
//   3. one grouped FFN launch over the ready experts, then one per demand chunk
//      after its event; one combine (optionally fused with the next-layer norm).
// A ring slot is overwritten only after the compute event of its last reader,
// and never while the current layer holds it.  Copy-stream and compute-stream
// events come from separate rings, so a recycled event always marks a later
// point of the same stream (waiting on it is conservative, never early).
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

namespace pdx {

struct OffloadEngine {
    pdx_offload_config cfg{};
    std::vector<const void*> gates;
    int64_t per = 0;                    // elements per expert slot
    int64_t n_fixed = 0, n_ring = 0;
    uint16_t* pool = nullptr;           // device: [n_fixed + n_ring][per]
    std::vector<int32_t> fixed_slot;    // [L*E] slot or -1
    std::vector<uint8_t> is_warm;       // [L*E]
    // cache ring (LRU as an intrusive list: head = least recently used)
    std::vector<int64_t> ring_key, ring_prev, ring_next;
    std::vector<int32_t> ring_ready, ring_last;  // event indices or -1
    std::vector<uint8_t> ring_prefetched;
    std::vector<int32_t> where;         // [L*E] ring index or -1
    int64_t lru_head = -1, lru_tail = -1;
    // events
    static constexpr int kEvents = 256;
    cudaEvent_t copy_ev[kEvents] = {}, comp_ev[kEvents] = {};
    int copy_next = 0, comp_next = 0;
    cudaStream_t copy_stream = nullptr;
    // pinned host staging
    int32_t* h_counts = nullptr;        // [2][E]
    int32_t* h_table = nullptr;         // [L][E]
    int32_t* h_active = nullptr;        // [max_launch][E+1]
    int max_launch = 0;
    // device scratch carved from the caller's workspace
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int32_t* d_table = nullptr;         // [L][E]
    int32_t* d_active = nullptr;        // [max_launch][E+1]
    pdx_offload_stats st{};
    // trace of the last forward_layer call
    pdx_offload_trace trace{};
    std::vector<int32_t> tr_counts;     // [2][E] routed counts of this layer and predicted next-layer counts
    std::vector<int32_t> tr_place;      // [E] PDX_PLACE_*
    std::vector<int32_t> tr_prefetch;   // next-layer experts whose copies this layer issued, in issue order
    std::vector<int32_t> tr_demand;     // demand-copied experts in copy order

    void lru_unlink(int64_t i) {
        const int64_t p = ring_prev[i], n = ring_next[i];
        if (p >= 0) ring_next[p] = n; else lru_head = n;
        if (n >= 0) ring_prev[n] = p; else lru_tail = p;
        ring_prev[i] = ring_next[i] = -1;
    }
    void lru_push_back(int64_t i) {
        ring_prev[i] = lru_tail;
        ring_next[i] = -1;
        if (lru_tail >= 0) ring_next[lru_tail] = i; else lru_head = i;
        lru_tail = i;
    }
    void touch(int64_t i) { lru_unlink(i); lru_push_back(i); }
};

struct OffloadBufs {  // per-call device buffers carved from the workspace
    uint16_t* logits[2];
    int64_t* sel[2];
    uint16_t* w[2];
    int32_t* counts;  // [2][E]
    int32_t* offsets[2];
    int32_t* tokens[2];
    int32_t* positions[2];
    uint16_t* packed_w[2];
    int32_t* inverse[2];
    int32_t* active[2];
    uint16_t* rows;
    void* op_ws;
    size_t op_ws_bytes;
};

size_t offload_op_ws_bytes(const pdx_offload_config& c, int64_t T) {
    const int64_t n = T * c.top_k;
    size_t b = pdx_route_workspace_bytes(T, c.experts);
    b = std::max(b, pdx_pack_workspace_bytes(T, c.top_k, c.experts));
    b = std::max(b, pdx_ffn_workspace_bytes(n, c.experts, c.hidden, c.inter, PDX_FFN_AUTO));
    return b;
}

// Carves the buffers of one call with T tokens (T <= max_tokens); with base
// == nullptr it only measures.
OffloadBufs carve_offload(const pdx_offload_config& c, int64_t T, void* base, size_t cap, size_t* used) {
    Carver cv{static_cast<char*>(base), base ? cap : SIZE_MAX};
    const int64_t E = c.experts, n = T * c.top_k;
    OffloadBufs b{};
    for (int r = 0; r < 2; ++r) {
        b.logits[r] = static_cast<uint16_t*>(cv.take(T * E * 2));
        b.sel[r] = static_cast<int64_t*>(cv.take(n * 8));
        b.w[r] = static_cast<uint16_t*>(cv.take(n * 2));
        b.offsets[r] = static_cast<int32_t*>(cv.take((E + 1) * 4));
        b.tokens[r] = static_cast<int32_t*>(cv.take(n * 4));
        b.positions[r] = static_cast<int32_t*>(cv.take(n * 4));
        b.packed_w[r] = static_cast<uint16_t*>(cv.take(n * 2));
        b.inverse[r] = static_cast<int32_t*>(cv.take(n * 4));
        b.active[r] = static_cast<int32_t*>(cv.take((E + 1) * 4));
    }
    b.counts = static_cast<int32_t*>(cv.take(2 * E * 4));
    b.rows = static_cast<uint16_t*>(cv.take(n * c.hidden * 2));
    b.op_ws_bytes = offload_op_ws_bytes(c, T);
    b.op_ws = cv.take(b.op_ws_bytes);
    if (used) *used = cv.used;
    return b;
}

int offload_max_launch(const pdx_offload_config& c) { return 1 + (c.experts + c.chunk - 1) / c.chunk; }

size_t offload_ws_bytes(const pdx_offload_config& c) {
    size_t used = 0;
    carve_offload(c, std::max<int64_t>(c.max_tokens, 1), nullptr, 0, &used);
    const size_t tables = align_up(static_cast<size_t>(c.layers) * c.experts * 4) +
                          align_up(static_cast<size_t>(offload_max_launch(c)) * (c.experts + 1) * 4);
    return align_up(used) + tables + kAlign;
}

int64_t offload_fixed_total(const pdx_offload_config& c) {
    int64_t t = 0;
    for (int32_t l = 0; l < c.layers; ++l) t += c.fixed_count[l];
    return t;
}

int check_offload_config(const pdx_offload_config* c) {
    if (!c) return fail(PDX_ERR_INVALID, "null offload config");
    if (c->layers < 1 || c->experts < 1 || c->hidden < 8 || c->inter < 8 || c->top_k < 1 || c->top_k > c->experts)
        return fail(PDX_ERR_INVALID, "invalid offload shape");
    if (!c->gates || !c->host_experts || !c->fixed_count) return fail(PDX_ERR_INVALID, "null offload argument");
    for (int32_t l = 0; l < c->layers; ++l)
        if (c->fixed_count[l] < 0 || c->fixed_count[l] > c->experts)
            return fail(PDX_ERR_INVALID, "fixed expert count of layer %d out of range", l);
    if (offload_fixed_total(*c) > 0 && !c->fixed_experts) return fail(PDX_ERR_INVALID, "null fixed expert list");
    if (c->cache_slots < 1 || c->chunk < 1 || c->max_tokens < 1) return fail(PDX_ERR_INVALID, "invalid offload sizes");
    return PDX_OK;
}

}  // namespace pdx

using pdx::OffloadEngine;

extern "C" {

size_t pdx_offload_pool_bytes(const pdx_offload_config* c) {
    if (pdx::check_offload_config(c)) return 0;
    const int64_t per = 3 * static_cast<int64_t>(c->hidden) * c->inter;
    return static_cast<size_t>(pdx::offload_fixed_total(*c) + c->cache_slots) * per * 2;
}

size_t pdx_offload_workspace_bytes(const pdx_offload_config* c) {
    return pdx::check_offload_config(c) ? 0 : pdx::offload_ws_bytes(*c);
}

void pdx_offload_destroy(pdx_offload* h) {
    OffloadEngine* e = reinterpret_cast<OffloadEngine*>(h);
    if (!e) return;
    if (e->copy_stream) cudaStreamSynchronize(e->copy_stream);
    for (int i = 0; i < OffloadEngine::kEvents; ++i) {
        if (e->copy_ev[i]) cudaEventDestroy(e->copy_ev[i]);
        if (e->comp_ev[i]) cudaEventDestroy(e->comp_ev[i]);
    }
    if (e->copy_stream) cudaStreamDestroy(e->copy_stream);
    if (e->h_counts) cudaFreeHost(e->h_counts);
    if (e->h_table) cudaFreeHost(e->h_table);
    if (e->h_active) cudaFreeHost(e->h_active);
    delete e;
}

int pdx_offload_create(const pdx_offload_config* c, void* pool, void* workspace, size_t workspace_bytes,
                       pdx_offload** out) {
    using namespace pdx;
    int st = check_offload_config(c);
    if (st) return st;
    if (!out || !pool || !workspace) return fail(PDX_ERR_INVALID, "null offload buffer");
    if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) || workspace_bytes < offload_ws_bytes(*c))
        return fail(PDX_ERR_WORKSPACE, "offload workspace too small or misaligned");
    *out = nullptr;
    OffloadEngine* e = new (std::nothrow) OffloadEngine();
    if (!e) return fail(PDX_ERR_CUDA, "out of host memory");
    e->cfg = *c;
    const int64_t L = c->layers, E = c->experts;
    e->gates.assign(c->gates, c->gates + L);
    e->per = 3 * static_cast<int64_t>(c->hidden) * c->inter;
    e->n_fixed = offload_fixed_total(*c);
    e->n_ring = c->cache_slots;
    e->pool = static_cast<uint16_t*>(pool);
    e->fixed_slot.assign(L * E, -1);
    e->is_warm.assign(L * E, 0);
    int64_t s = 0, off = 0;
    for (int64_t l = 0; l < L; ++l) {
        for (int32_t j = 0; j < c->fixed_count[l]; ++j) {
            const int32_t ex = c->fixed_experts[off + j];
            if (ex < 0 || ex >= E || e->fixed_slot[l * E + ex] >= 0) {
                pdx_offload_destroy(reinterpret_cast<pdx_offload*>(e));
                return fail(PDX_ERR_INVALID, "fixed expert list of layer %lld is invalid", static_cast<long long>(l));
            }
            e->fixed_slot[l * E + ex] = static_cast<int32_t>(s++);
            e->is_warm[l * E + ex] = j >= c->hot_per_layer ? 1 : 0;
        }
        off += c->fixed_count[l];
    }
    const int64_t R = e->n_ring;
    e->ring_key.assign(R, -1);
    e->ring_prev.assign(R, -1);
    e->ring_next.assign(R, -1);
    e->ring_ready.assign(R, -1);
    e->ring_last.assign(R, -1);
    e->ring_prefetched.assign(R, 0);
    e->where.assign(L * E, -1);
    for (int64_t i = 0; i < R; ++i) e->lru_push_back(i);
    e->max_launch = offload_max_launch(*c);
    auto bail = [&](const char* what, cudaError_t err) {
        pdx_offload_destroy(reinterpret_cast<pdx_offload*>(e));
        return fail(PDX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
    };
    cudaError_t err;
    if ((err = cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking)) != cudaSuccess)
        return bail("copy stream", err);
    for (int i = 0; i < OffloadEngine::kEvents; ++i) {
        if ((err = cudaEventCreateWithFlags(&e->copy_ev[i], cudaEventDisableTiming)) != cudaSuccess)
            return bail("event", err);
        if ((err = cudaEventCreateWithFlags(&e->comp_ev[i], cudaEventDisableTiming)) != cudaSuccess)
            return bail("event", err);
    }
    if ((err = cudaHostAlloc(reinterpret_cast<void**>(&e->h_counts), 2 * E * 4, cudaHostAllocDefault)) != cudaSuccess ||
        (err = cudaHostAlloc(reinterpret_cast<void**>(&e->h_table), L * E * 4, cudaHostAllocDefault)) != cudaSuccess ||
        (err = cudaHostAlloc(reinterpret_cast<void**>(&e->h_active), e->max_launch * (E + 1) * 4,
                             cudaHostAllocDefault)) != cudaSuccess)
        return bail("pinned staging", err);
    std::memset(e->h_table, 0, L * E * 4);
    // device tables at the end of the workspace
    size_t used = 0;
    carve_offload(*c, c->max_tokens, nullptr, 0, &used);
    char* wsb = static_cast<char*>(workspace);
    e->ws = workspace;
    e->ws_bytes = align_up(used);
    e->d_table = reinterpret_cast<int32_t*>(wsb + e->ws_bytes);
    e->d_active = reinterpret_cast<int32_t*>(wsb + e->ws_bytes + align_up(static_cast<size_t>(L) * E * 4));
    // fixed experts into their slots (once, synchronous)
    const uint16_t* host = static_cast<const uint16_t*>(c->host_experts);
    for (int64_t l = 0; l < L; ++l)
        for (int64_t ex = 0; ex < E; ++ex) {
            const int32_t fs = e->fixed_slot[l * E + ex];
            if (fs < 0) continue;
            if ((err = cudaMemcpyAsync(e->pool + fs * e->per, host + (l * E + ex) * e->per, e->per * 2,
                                       cudaMemcpyHostToDevice, e->copy_stream)) != cudaSuccess)
                return bail("fixed expert copy", err);
        }
    if ((err = cudaMemsetAsync(e->d_table, 0, L * E * 4, e->copy_stream)) != cudaSuccess) return bail("memset", err);
    if ((err = cudaStreamSynchronize(e->copy_stream)) != cudaSuccess) return bail("fixed expert copy", err);
    *out = reinterpret_cast<pdx_offload*>(e);
    return ok();
}

int pdx_offload_get_stats(const pdx_offload* h, pdx_offload_stats* out) {
    const OffloadEngine* e = reinterpret_cast<const OffloadEngine*>(h);
    if (!e || !out) return fail(PDX_ERR_INVALID, "null offload handle");
    *out = e->st;
    return ok();
}

int pdx_offload_forward_layer(pdx_offload* h, int32_t layer, const void* x, int64_t T, const void* residual,
                              int32_t norm, void* out, pdx_stream_t stream) {
    using namespace pdx;
    OffloadEngine* e = reinterpret_cast<OffloadEngine*>(h);
    if (!e || !x || !out) return fail(PDX_ERR_INVALID, "null offload argument");
    const pdx_offload_config& c = e->cfg;
    if (layer < 0 || layer >= c.layers) return fail(PDX_ERR_INVALID, "layer %d out of range", layer);
    if (T < 1 || T > c.max_tokens) return fail(PDX_ERR_INVALID, "T=%lld outside [1, max_tokens]", static_cast<long long>(T));
    if (norm && !residual) return fail(PDX_ERR_INVALID, "the next-layer norm needs a residual");
    const int64_t E = c.experts, H = c.hidden, I = c.inter, k = c.top_k, n = T * k;
    OffloadBufs b = carve_offload(c, T, e->ws, e->ws_bytes, nullptr);
    const bool predict = c.prefetch && layer + 1 < c.layers;
    int st;
    // 1. routing of this layer (and the next layer's gate on the same activation)
    for (int r = 0; r < (predict ? 2 : 1); ++r) {
        if ((st = pdx_route_topk(x, e->gates[layer + r], T, H, E, static_cast<int32_t>(k), c.normalize, b.logits[r],
                                 b.sel[r], b.w[r], b.op_ws, b.op_ws_bytes, stream)))
            return st;
        if ((st = pdx_pack(b.sel[r], b.w[r], T, static_cast<int32_t>(k), E, b.counts + r * E, b.offsets[r],
                           b.tokens[r], b.positions[r], b.packed_w[r], b.inverse[r], b.active[r], b.op_ws,
                           b.op_ws_bytes, stream)))
            return st;
    }
    PDX_CUDA_TRY(cudaMemcpyAsync(e->h_counts, b.counts, (predict ? 2 : 1) * E * 4, cudaMemcpyDeviceToHost, stream));
    PDX_CUDA_TRY(cudaStreamSynchronize(stream));  // the per-layer grouping sync
    e->st.layers += 1;
    // trace of this layer (read back by pdx_offload_last_trace)
    pdx_offload_trace tr{};
    tr.layer = layer;
    tr.tokens = T;
    const pdx_offload_stats st0 = e->st;
    e->tr_counts.assign(2 * E, 0);
    std::copy(e->h_counts, e->h_counts + E, e->tr_counts.begin());
    if (predict) std::copy(e->h_counts + E, e->h_counts + 2 * E, e->tr_counts.begin() + E);
    e->tr_place.assign(E, PDX_PLACE_NONE);
    e->tr_prefetch.clear();
    e->tr_demand.clear();
    e->trace = tr;  // a layer that fails below leaves this partial trace

    // 2. placement
    const int64_t base = static_cast<int64_t>(layer) * E;
    int32_t* table = e->h_table + base;
    std::vector<int32_t> ready, demand;
    std::vector<int64_t> pinned;
    std::vector<int32_t> waits;
    auto is_pinned = [&](int64_t i) { return std::find(pinned.begin(), pinned.end(), i) != pinned.end(); };
    for (int64_t ex = 0; ex < E; ++ex) {
        if (e->h_counts[ex] <= 0) continue;
        e->st.expert_uses += 1;
        const int32_t fs = e->fixed_slot[base + ex];
        tr.routed_experts += 1;
        if (fs >= 0) {
            table[ex] = fs;
            ready.push_back(static_cast<int32_t>(ex));
            if (e->is_warm[base + ex]) e->st.warm_hits += 1; else e->st.hot_hits += 1;
            e->tr_place[ex] = e->is_warm[base + ex] ? PDX_PLACE_WARM : PDX_PLACE_HOT;
            continue;
        }
        const int32_t ri = e->where[base + ex];
        if (ri >= 0) {
            e->st.cache_hits += 1;
            if (e->ring_prefetched[ri]) {
                e->st.prefetch_used += 1;
                e->ring_prefetched[ri] = 0;
            }
            e->touch(ri);
            pinned.push_back(ri);
            table[ex] = static_cast<int32_t>(e->n_fixed + ri);
            ready.push_back(static_cast<int32_t>(ex));
            bool loading = false;
            if (e->ring_ready[ri] >= 0) {
                waits.push_back(e->ring_ready[ri]);
                const cudaError_t q = cudaEventQuery(e->copy_ev[e->ring_ready[ri]]);
                if (q == cudaErrorNotReady) {
                    loading = true;
                    cudaGetLastError();  // a pending copy is a status, not an error
                } else if (q != cudaSuccess) {
                    return fail(PDX_ERR_CUDA, "copy event: %s", cudaGetErrorString(q));
                }
            }
            e->tr_place[ex] = loading ? PDX_PLACE_LOADING : PDX_PLACE_CACHE;
            continue;
        }
        demand.push_back(static_cast<int32_t>(ex));
        e->tr_place[ex] = PDX_PLACE_DEMAND;
    }
    e->tr_demand.assign(demand.begin(), demand.end());
    const uint16_t* host = static_cast<const uint16_t*>(c.host_experts);
    // acquire the least recently used ring slot outside `pinned` for key
    auto copy_in = [&](int64_t key, bool prefetched, int64_t* slot_out) -> int {
        int64_t i = e->lru_head;
        while (i >= 0 && is_pinned(i)) i = e->ring_next[i];
        if (i < 0) return fail(PDX_ERR_UNSUPPORTED, "every cache slot is held by the current layer; enlarge the ring");
        if (e->ring_key[i] >= 0) {
            e->where[e->ring_key[i]] = -1;
            if (e->ring_prefetched[i]) e->st.prefetch_wasted += 1;
        }
        if (e->ring_last[i] >= 0) PDX_CUDA_TRY(cudaStreamWaitEvent(e->copy_stream, e->comp_ev[e->ring_last[i]], 0));
        e->ring_key[i] = key;
        e->ring_ready[i] = -1;
        e->ring_last[i] = -1;
        e->ring_prefetched[i] = prefetched ? 1 : 0;
        e->where[key] = static_cast<int32_t>(i);
        e->touch(i);
        PDX_CUDA_TRY(cudaMemcpyAsync(e->pool + (e->n_fixed + i) * e->per, host + key * e->per, e->per * 2,
                                     cudaMemcpyHostToDevice, e->copy_stream));
        e->st.h2d_bytes += e->per * 2;
        if (prefetched) e->st.prefetch_copies += 1; else e->st.demand_copies += 1;
        *slot_out = i;
        return PDX_OK;
    };
    // Records a copy-stream event after the copies into `idxs` and makes it
    // their ready event.  Also called on an error path, so that no slot whose
    // copy was issued is left without one (a later hit waits on it).
    auto mark_ready = [&](const std::vector<int64_t>& idxs, int* ev_out) -> int {
        const int ev = e->copy_next;
        e->copy_next = (e->copy_next + 1) % OffloadEngine::kEvents;
        PDX_CUDA_TRY(cudaEventRecord(e->copy_ev[ev], e->copy_stream));
        for (int64_t i : idxs) e->ring_ready[i] = ev;
        if (ev_out) *ev_out = ev;
        return PDX_OK;
    };
    std::vector<std::vector<int32_t>> chunks;
    std::vector<int> chunk_ev;
    for (size_t c0 = 0; c0 < demand.size(); c0 += c.chunk) {
        std::vector<int32_t> part(demand.begin() + c0, demand.begin() + std::min(demand.size(), c0 + c.chunk));
        std::vector<int64_t> idxs;
        for (int32_t ex : part) {
            int64_t slot;
            if ((st = copy_in(base + ex, false, &slot))) {
                if (!idxs.empty()) mark_ready(idxs, nullptr);
                return st;
            }
            pinned.push_back(slot);
            idxs.push_back(slot);
            table[ex] = static_cast<int32_t>(e->n_fixed + slot);
        }
        int ev = 0;
        if ((st = mark_ready(idxs, &ev))) return st;
        chunks.push_back(part);
        chunk_ev.push_back(ev);
    }
    // 3. the next layer's predicted experts, queued behind the demand copies
    if (predict) {
        const int64_t nbase = base + E;
        std::vector<int64_t> issued;
        for (int64_t ex = 0; ex < E; ++ex) {
            if (e->h_counts[E + ex] <= 0) continue;
            if (e->fixed_slot[nbase + ex] >= 0 || e->where[nbase + ex] >= 0) continue;
            if (static_cast<int64_t>(pinned.size() + issued.size()) >= e->n_ring) {
                for (int64_t rest = ex; rest < E; ++rest)   // the reference's prefetch_capacity_skipped
                    if (e->h_counts[E + rest] > 0 && e->fixed_slot[nbase + rest] < 0 && e->where[nbase + rest] < 0)
                        tr.prefetch_skipped += 1;
                break;
            }
            int64_t slot;
            const size_t before = pinned.size();
            pinned.insert(pinned.end(), issued.begin(), issued.end());
            st = copy_in(nbase + ex, true, &slot);
            pinned.resize(before);
            if (st) {
                if (!issued.empty()) mark_ready(issued, nullptr);
                return st;
            }
            issued.push_back(slot);
            e->tr_prefetch.push_back(static_cast<int32_t>(ex));
        }
        if (!issued.empty() && (st = mark_ready(issued, nullptr))) return st;
    }
    // 4. tables and active lists, then the FFN launches
    const int launches = 1 + static_cast<int>(chunks.size());
    auto fill = [&](int row, const std::vector<int32_t>& lst) {
        int32_t* a = e->h_active + row * (E + 1);
        a[0] = static_cast<int32_t>(lst.size());
        std::copy(lst.begin(), lst.end(), a + 1);
    };
    fill(0, ready);
    for (size_t i = 0; i < chunks.size(); ++i) fill(1 + static_cast<int>(i), chunks[i]);
    PDX_CUDA_TRY(cudaMemcpyAsync(e->d_table + base, table, E * 4, cudaMemcpyHostToDevice, stream));
    PDX_CUDA_TRY(cudaMemcpyAsync(e->d_active, e->h_active, launches * (E + 1) * 4, cudaMemcpyHostToDevice, stream));
    for (int ev : waits) PDX_CUDA_TRY(cudaStreamWaitEvent(stream, e->copy_ev[ev], 0));
    pdx_expert_weights wt{};
    wt.gate = e->pool;
    wt.up = e->pool + I * H;
    wt.down = e->pool + 2 * I * H;
    wt.gate_stride = wt.up_stride = wt.down_stride = e->per;
    wt.num_slots = e->n_fixed + e->n_ring;
    wt.slot_of_expert = e->d_table + base;
    for (int li = 0; li < launches; ++li) {
        if (li == 0 && ready.empty()) continue;
        if (li > 0) PDX_CUDA_TRY(cudaStreamWaitEvent(stream, e->copy_ev[chunk_ev[li - 1]], 0));
        if ((st = pdx_moe_ffn_grouped(x, T, b.tokens[0], b.offsets[0], e->d_active + li * (E + 1), E, n, &wt, H, I,
                                      b.rows, PDX_FFN_AUTO, b.op_ws, b.op_ws_bytes, stream)))
            return st;
    }
    if (norm)
        st = pdx_combine_layernorm(b.rows, b.w[0], b.inverse[0], T, static_cast<int32_t>(k), H, residual,
                                   PDX_LAYER_NORM_EPS, out, stream);
    else
        st = pdx_combine(b.rows, b.w[0], b.inverse[0], T, static_cast<int32_t>(k), H, residual, out, stream);
    if (st) return st;
    const int done = e->comp_next;
    e->comp_next = (e->comp_next + 1) % OffloadEngine::kEvents;
    PDX_CUDA_TRY(cudaEventRecord(e->comp_ev[done], stream));
    for (int64_t i : pinned) e->ring_last[i] = done;
    for (int32_t ex = 0; ex < E; ++ex) {
        tr.hot += e->tr_place[ex] == PDX_PLACE_HOT;
        tr.warm += e->tr_place[ex] == PDX_PLACE_WARM;
        tr.cache_ready += e->tr_place[ex] == PDX_PLACE_CACHE;
        tr.cache_loading += e->tr_place[ex] == PDX_PLACE_LOADING;
    }
    tr.demand = static_cast<int32_t>(demand.size());
    tr.demand_chunks = static_cast<int32_t>(chunks.size());
    tr.prefetch_issued = static_cast<int32_t>(e->tr_prefetch.size());
    tr.prefetch_used = static_cast<int32_t>(e->st.prefetch_used - st0.prefetch_used);
    tr.h2d_bytes = e->st.h2d_bytes - st0.h2d_bytes;
    e->trace = tr;
    return ok();
}

int pdx_offload_last_trace(const pdx_offload* h, pdx_offload_trace* out, int32_t* counts_out, int32_t* placement_out,
                           int32_t* prefetch_out, int32_t* demand_out) {
    const OffloadEngine* e = reinterpret_cast<const OffloadEngine*>(h);
    if (!e || !out) return pdx::fail(PDX_ERR_INVALID, "null offload trace argument");
    if (e->tr_place.empty()) return pdx::fail(PDX_ERR_INVALID, "no layer has run on this offload handle");
    *out = e->trace;
    if (counts_out) std::copy(e->tr_counts.begin(), e->tr_counts.end(), counts_out);
    if (placement_out) std::copy(e->tr_place.begin(), e->tr_place.end(), placement_out);
    if (prefetch_out) std::copy(e->tr_prefetch.begin(), e->tr_prefetch.end(), prefetch_out);
    if (demand_out) std::copy(e->tr_demand.begin(), e->tr_demand.end(), demand_out);
    return pdx::ok();
}

int pdx_offload_copy_selected(const pdx_offload* h, int32_t which, int64_t T, int64_t* selected_out,
                              pdx_stream_t stream) {
    using namespace pdx;
    const OffloadEngine* e = reinterpret_cast<const OffloadEngine*>(h);
    if (!e || !selected_out || (which != 0 && which != 1)) return fail(PDX_ERR_INVALID, "invalid selected copy");
    if (e->tr_place.empty() || T != e->trace.tokens)
        return fail(PDX_ERR_INVALID, "T must be the token count of the last forward_layer call");
    if (which == 1 && e->trace.layer + 1 >= e->cfg.layers)
        return fail(PDX_ERR_INVALID, "the last layer has no next-layer prediction");
    OffloadBufs b = carve_offload(e->cfg, T, e->ws, e->ws_bytes, nullptr);
    PDX_CUDA_TRY(cudaMemcpyAsync(selected_out, b.sel[which], T * e->cfg.top_k * 8, cudaMemcpyDeviceToDevice, stream));
    return ok();
}

}  // extern "C"
