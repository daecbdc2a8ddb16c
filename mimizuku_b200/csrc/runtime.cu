// Per-device runtime state of the library: the status word every bounded wait reports into, kernel attributes,
// the calling thread's last error, and tensor-map encoding through the driver entry point.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"
#include "launch.h"

namespace mmz {

__device__ unsigned g_status[4];

static thread_local std::string t_err;

int fail(const char* msg) {
    t_err = msg ? msg : "error";
    return -1;
}

int failf(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return fail(buf);
}

const char* last_error() { return t_err.c_str(); }

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return failf("%s: launch failed: %s", what, cudaGetErrorString(e));
    return 0;
}

int check_pdl(cudaError_t e, const char* what) {
    if (e != cudaSuccess) return failf("%s: launch failed: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

static std::mutex g_mu;
static DevCtx g_ctx[64];

// Fills c for device dev (current): device checks, the status word's device address, kernel attributes. Called with
// g_mu held; c.ok is set only at the end, so a context that was ok stays usable while it is refreshed.
static void init_ctx(DevCtx& c, int dev) {
    c.inited = true;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
        c.ok = false;
        c.err = "cudaGetDeviceProperties failed";
        return;
    }
    if (prop.major != 10 || prop.minor != 0) {
        c.ok = false;
        c.err = "the mimizuku_b200 kernels are built for sm_100a (B200) only";
        return;
    }
    c.sms = prop.multiProcessorCount;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) {
        c.ok = false;
        c.err = "cudaGetSymbolAddress(status) failed";
        return;
    }
    c.status = (unsigned*)p;
    if (const char* s = getenv("MMZ_WAIT_LIMIT_MS")) c.limit_ns = (unsigned long long)atoll(s) * 1000000ull;
    init_dec_attn_attrs(c);
    init_enc_attn_attrs();
    init_dec_linear_attrs();
    init_logits_argmax_attrs();
    init_gemm_attrs(c);
    init_gemv_attrs();
    init_align_attrs();
    cudaGetLastError();
    c.ok = true;
    c.err = "";
}

static int current_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    return dev;
}

DevCtx& dev_ctx() {
    const int dev = current_device();
    if (dev < 0) {
        static DevCtx bad;
        bad.ok = false;
        bad.err = "no CUDA device";
        return bad;
    }
    DevCtx& c = g_ctx[dev];
    if (c.inited) return c;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!c.inited) init_ctx(c, dev);
    return c;
}

DevCtx& dev_ctx_refresh() {
    const int dev = current_device();
    if (dev < 0) return dev_ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    init_ctx(g_ctx[dev], dev);
    return g_ctx[dev];
}

// cuTensorMapEncodeTiled through the runtime's driver entry point
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

static int make_tmap(CUtensorMap* map, int rank, const void* base, const uint64_t* dims, const uint64_t* strides,
                     const uint32_t* box, int swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -1;
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), (const cuuint64_t*)dims,
                    (const cuuint64_t*)strides, (const cuuint32_t*)box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                    : swizzle == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                    : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -1;
}

// Failure-detection self-test: a barrier nothing ever arrives on. Warp 0 waits with the suspending bounded wait, warp
// 1 with the spinning one; the first to give up reports (ST_TIMEOUT, K_SELFTEST, 1 or 2) and makes the other stop.
// The kernel then returns normally and the context stays usable.
__global__ void wait_selftest_kernel(unsigned* status, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        abort = 0;
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x < 32) mbar_wait(&bar, 0, &abort, limit_ns, status, K_SELFTEST, 1);
    else mbar_wait_spin(&bar, 0, &abort, limit_ns, status, K_SELFTEST, 2);
}

int launch_wait_selftest(int limit_ms, cudaStream_t st) {
    if (limit_ms < 1 || limit_ms > 10000) return fail("wait_selftest: 1 <= limit_ms <= 10000");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    wait_selftest_kernel<<<1, 64, 0, st>>>(dc.status, (unsigned long long)limit_ms * 1000000ull);
    return check_launch("wait_selftest");
}

int make_tmap_2d(CUtensorMap* map, const void* base, const uint64_t dims[2], const uint64_t strides[1],
                 const uint32_t box[2], int swizzle) {
    return make_tmap(map, 2, base, dims, strides, box, swizzle);
}

int make_tmap_3d(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                 const uint32_t box[3], int swizzle) {
    return make_tmap(map, 3, base, dims, strides, box, swizzle);
}

}  // namespace mmz
