// pdx_pack_static: the packing entry point without a caller workspace.
//
// Some callers of this library cannot allocate device memory at the point
// where they pack a layer's routing: a plugin living inside a host process
// whose own allocator has reserved the device's memory and forbids outside
// allocations, a foreign-language caller (C, Go, Java via FFI) that has no
// device allocator of its own, or a latency-critical path where cudaMalloc's
// implicit device-wide synchronisation is not acceptable.  For them this entry
// point keeps its scratch -- the per-chunk expert histograms of the multi-CTA
// counting sort -- in a fixed file-scope device array instead of a workspace.
//
// The array belongs to the library image, so every GPU that loads the library
// holds it (kPackStaticHistInts ints = 256 KiB) until the process exits.
// Every call shares it: two calls whose kernels overlap on the GPU (different
// streams, no ordering) race on it.  Each call overwrites every histogram
// entry it later reads, so nothing in the array has to start at zero and the
// previous call's leftovers are harmless.
#include "routing.cuh"

namespace pdx {

constexpr int kPackStaticHistInts = PDX_PACK_STATIC_MAX_HIST_INTS;

static __device__ __align__(256) int g_pack_static_hist[kPackStaticHistInts];

namespace {

// Device address of g_pack_static_hist, resolved once per device.  In host
// code the array's name is only a stand-in for the symbol, never a pointer a
// kernel may use, so the address comes from cudaGetSymbolAddress with the
// device current.  The cached address lives as long as the process's primary
// context of that device: after cudaDeviceReset (or any teardown of that
// context) the library must not be called on the device again.
int* g_pack_static_ptr[kMaxDevices] = {nullptr};
std::mutex g_pack_static_mutex;

int pack_static_scratch(int** out) {
    int dev = 0;
    PDX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(PDX_ERR_UNSUPPORTED, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_pack_static_mutex);
    if (!g_pack_static_ptr[dev]) {
        void* p = nullptr;
        PDX_CUDA_TRY(cudaGetSymbolAddress(&p, g_pack_static_hist));
        g_pack_static_ptr[dev] = static_cast<int*>(p);
    }
    *out = g_pack_static_ptr[dev];
    return PDX_OK;
}

}  // namespace
}  // namespace pdx

extern "C" int pdx_pack_static(const int64_t* selected, const void* weights, int64_t T, int32_t top_k, int64_t E,
                               int32_t* counts, int32_t* offsets, int32_t* tokens, int32_t* positions,
                               void* packed_w, int32_t* inverse, int32_t* active, pdx_stream_t stream) {
    using namespace pdx;
    int st = check_route_shape(T, 8, E, top_k);
    if (st) return st;
    if (!selected || !weights || !counts || !offsets || !tokens || !positions || !packed_w || !inverse || !active)
        return fail(PDX_ERR_INVALID, "null packing argument");
    const int64_t N = T * top_k;
    const int64_t need = static_cast<int64_t>(pack_chunks(N, kPackChunk)) * E;
    if (N > kPackSingleMax && need > kPackStaticHistInts)
        return fail(PDX_ERR_UNSUPPORTED,
                    "pdx_pack_static: ceil(T*top_k/%d)*E = %lld histogram entries exceeds the fixed %d "
                    "(use pdx_pack with a workspace)",
                    kPackChunk, static_cast<long long>(need), kPackStaticHistInts);
    int* scratch = nullptr;
    if ((st = pack_static_scratch(&scratch))) return st;
    PackOut o{counts, offsets, tokens, positions, static_cast<uint16_t*>(packed_w), inverse, active};
    st = launch_pack(selected, static_cast<const uint16_t*>(weights), T, top_k, E, o, scratch, stream, kPackChunk);
    return st ? st : ok();
}
