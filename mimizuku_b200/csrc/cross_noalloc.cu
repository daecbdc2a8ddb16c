// mmz_cross_attn_noalloc: the decoder cross-attention of mmz_cross_attn for callers that cannot allocate device
// memory. Some hosts hand a library no allocator and forbid cudaMalloc after start-up: a process embedded in an
// application that owns a fixed device-memory budget, or a real-time loop that cannot take cudaMalloc's implicit
// device synchronisation. Such a caller cannot provide the scratch buffer mmz_cross_attn asks for, so this entry point
// brings its own: a file-scope device array of fixed size, which every GPU that loads the library holds until the
// process exits.
//
// Limit: 640 (sequence, head) items per call, i.e. batch x heads <= 640 (32 sequences of Whisper large-v3, 20 heads),
// 7.9 MB of scratch. Larger calls are rejected with an error.
//
// The array is shared by every call on a device and keeps the last call's contents; nothing in it needs to start at
// zero (every value a call reads was written earlier in the same call). Calls that overlap on the GPU (other streams,
// other threads) race on the array and must be serialised by the caller. mmz_init resolves the array's device address
// (cudaGetSymbolAddress, with that device current) and caches it per device, so the entry point itself only reads the
// cached pointer; a device reset (cudaDeviceReset) invalidates it, and mmz_init must be called again on that device
// before the next call. Without a prior mmz_init the first call resolves the address itself.
#include <mutex>

#include "../../include/mimizuku_b200.h"
#include "common.cuh"
#include "launch.h"

namespace mmz {

constexpr int NOALLOC_MAX_ITEMS = 640;
constexpr size_t NOALLOC_ITEM_BYTES = (size_t)TENC * 4 + 24 * 8 + 24 * HD * 4;  // S, stat and part of one item
constexpr size_t NOALLOC_BYTES = NOALLOC_MAX_ITEMS * NOALLOC_ITEM_BYTES;

static __device__ __align__(256) unsigned char g_cross_scratch[NOALLOC_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[64];  // device address of g_cross_scratch, per device

static int current_dev() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    return dev;
}

// Resolves the array's device address on the current device and caches it (called by mmz_init, with the device
// current; again after a device reset). In host code the symbol g_cross_scratch is only a host-side stand-in; the
// kernels must be given this address.
int noalloc_resolve() {
    const int dev = current_dev();
    if (dev < 0) return fail("cross_attn_noalloc: no CUDA device");
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_cross_scratch);
    if (e != cudaSuccess || !p)
        return failf("cross_attn_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    g_noalloc_addr[dev] = p;
    return 0;
}

// the cached address of the current device (resolved here if mmz_init was not called on it)
static int noalloc_scratch(void** out) {
    const int dev = current_dev();
    if (dev < 0) return fail("cross_attn_noalloc: no CUDA device");
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        *out = g_noalloc_addr[dev];
    }
    if (*out) return 0;
    if (noalloc_resolve()) return -1;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    *out = g_noalloc_addr[dev];
    return 0;
}

}  // namespace mmz

using namespace mmz;

extern "C" int mmz_cross_attn_noalloc(const void* q, const void* kv, void* out, void* align, const int* aslot,
                                      const int* ctr, const int* done, int batch, int layer, int nl, int d, int na,
                                      int max_t, void* stream) {
    if (batch < 1 || d < HD || d % HD) return fail("cross_attn_noalloc: bad shape");
    const long items = (long)batch * (d / HD);
    const size_t need = cross_attn_scratch_bytes(batch, d);
    if (items > NOALLOC_MAX_ITEMS || need > NOALLOC_BYTES)
        return failf("cross_attn_noalloc: batch x heads = %ld exceeds the static scratch (%d items, %zu bytes); use "
                     "mmz_cross_attn with a caller-provided scratch buffer",
                     items, NOALLOC_MAX_ITEMS, NOALLOC_BYTES);
    void* scratch = nullptr;
    if (noalloc_scratch(&scratch)) return -1;
    return launch_cross_attn(q, kv, out, align, aslot, ctr, done, batch, layer, nl, d, na, max_t, scratch, need,
                             (cudaStream_t)stream);
}
