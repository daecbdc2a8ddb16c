// The decoder's linear layers at m <= 8 sequences, bit-identical to the reference's gemv kernels
// (kernels/whisper.cu:501-567, used by src/gpu.rs:211-228 instead of cuBLAS up to 8 rows): y[m][n] = rh(x[m] . W[n] +
// bias[n]). The sums are the reference's - the output of column n comes from the 32 lanes of one warp, lane l
// accumulating the 8-element groups k = 256 i + 8 l .. + 7 in increasing i with one fused multiply-add per element,
// then the xor butterfly over offsets 16, 8, 4, 2, 1, then the bias added in fp32 before the single rounding - and
// everything else is this library's:
//   - a persistent grid (one 8-warp CTA per SM); warp w of CTA b takes the 4-column items w * grid + b, + 8 * grid, ...
//     so that items spread over the SMs first;
//   - each warp streams its items' weight rows through its own ring of stages in shared memory, filled by bulk copies
//     that lane 0 issues ahead of the arithmetic, the first ones before the wait for the kernel before (the weights do
//     not depend on it). A stage holds the item's 4 rows over a K chunk (a multiple of 256, so each lane's groups keep
//     their order); the chunk is as long as the shared memory allows with two stages per warp, so that a whole row
//     block is one contiguous copy where it fits (k = 1280: 10 KB per copy, 160 KB in flight per SM). Larger copies
//     were measured faster than more of smaller ones (512-value chunks in 4 stages: the logits at 33.3 us against
//     22.8 us with whole rows);
//   - x (m rows of k) is staged once per CTA by bulk copies after that wait;
//   - the products pair two sequences in one fp32x2 fused multiply-add (each half rounded on its own, so the sums are
//     the scalar ones);
//   - the reduction over the lanes halves the values at each butterfly level (a lane keeps half, its partner the
//     other half) instead of reducing every value on every lane: the same tree of additions, 31 shuffles for the 32
//     sums of a warp instead of 160.
// A CTA whose shared memory would not hold x and two stages of 256-value chunks takes the register-streaming form of
// gemv_row.cuh.
#include "common.cuh"
#include "gemv_row.cuh"
#include "launch.h"

namespace mmz {
namespace gq {
constexpr int WARPS = 8;
constexpr int COLS = 4;          // columns (weight rows) per item
constexpr int HEAD = 1024;       // barriers and the abort flag
constexpr int SMEM_MAX = 227 * 1024;
constexpr int MAX_STAGES = 8;
// the ring's K chunk and stage count for m rows of k: the longest chunk that two stages per warp allow next to x (no
// longer than k rounded up to 256), then as many stages as fit, up to 8; kc = 0 when not even 256 fits
struct Plan {
    int kc = 0, stages = 0;
    size_t smem = 0;
};
inline Plan plan(int m, int k) {
    Plan p;
    const long budget = (long)SMEM_MAX - HEAD - (long)m * k * 2;
    const long per_kc = (long)WARPS * COLS * 2;  // bytes of one value of chunk over a stage of every warp
    if (budget < 2 * per_kc * 256) return p;
    const int kr = (k + 255) / 256 * 256;
    long kc = budget / (2 * per_kc) / 256 * 256;
    if (kc > kr) kc = kr;
    long st = budget / (per_kc * kc);
    if (st > MAX_STAGES) st = MAX_STAGES;
    p.kc = (int)kc;
    p.stages = (int)st;
    p.smem = HEAD + (size_t)per_kc * kc * st + (size_t)m * k * 2;
    return p;
}
}  // namespace gq

// kc: the K chunk of a stage (a multiple of 256), stages: ring stages per warp (Plan)
template <int MR>
__global__ void __launch_bounds__(256, 1) gemv_ring_kernel(const h16* __restrict__ x, int ldx,
                                                           const h16* __restrict__ W, h16* __restrict__ y, int ldy,
                                                           int M, int N, int K, const h16* __restrict__ bias, int kc,
                                                           int stages, int gelu, unsigned* status,
                                                           unsigned long long limit_ns) {
    using namespace gq;
    extern __shared__ __align__(1024) unsigned char sm[];
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);  // [WARPS][stages]
    uint64_t* xbar = full + WARPS * stages;
    volatile int* abort = reinterpret_cast<volatile int*>(xbar + 1);
    const int stage = COLS * kc;  // values per stage
    h16* ring = reinterpret_cast<h16*>(sm + HEAD);
    h16* xs = ring + WARPS * stages * stage;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = (N + COLS - 1) / COLS, nch = (K + kc - 1) / kc;
    const int nw = gridDim.x * WARPS, gw = warp * gridDim.x + blockIdx.x;
    const int my_items = gw < items ? (items - 1 - gw) / nw + 1 : 0;
    const int nunits = my_items * nch;
    if (threadIdx.x == 0) {
        for (int i = 0; i <= WARPS * stages; i++) mbar_init(full + i, 1);
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    uint64_t* myfull = full + warp * stages;
    h16* myring = ring + warp * stages * stage;
    // lane 0: unit v = (item v / nch of this warp, chunk v % nch) into stage v % stages, the rows at a pitch of the
    // chunk's length (so that a single-chunk item is one contiguous copy)
    auto issue = [&](int v) {
        const int n0 = (gw + (v / nch) * nw) * COLS, k0 = (v % nch) * kc;
        const int rows = min(COLS, N - n0), len = min(kc, K - k0);
        uint64_t* bar = myfull + v % stages;
        h16* dst = myring + (v % stages) * stage;
        mbar_expect_tx(bar, (uint32_t)(rows * len * 2));
        if (nch == 1)
            bulk_g2s(dst, W + (long)n0 * K, (uint32_t)(rows * len * 2), bar);
        else
            for (int r = 0; r < rows; r++)
                bulk_g2s(dst + r * len, W + (long)(n0 + r) * K + k0, (uint32_t)(len * 2), bar);
    };
    if (lane == 0)
        for (int v = 0; v < min(stages, nunits); v++) issue(v);
    griddep_wait();  // x comes from the kernel before
    if (threadIdx.x == 0) {
        mbar_expect_tx(xbar, (uint32_t)(M * K * 2));
        for (int m = 0; m < M; m++) bulk_g2s(xs + m * K, x + (long)m * ldx, (uint32_t)(K * 2), xbar);
    }
    griddep_launch_dependents();
    int v = 0;  // units consumed
    // every decision to leave is taken by the whole warp (the loop below shuffles across all its lanes)
    bool ok = __all_sync(0xffffffff, mbar_wait(xbar, 0, abort, limit_ns, status, K_GEMV, 0));
    for (int t = 0; ok && t < my_items; t++) {
        float acc[COLS][MR];
#pragma unroll
        for (int c = 0; c < COLS; c++)
#pragma unroll
            for (int m = 0; m < MR; m++) acc[c][m] = 0.f;
        for (int ch = 0; ch < nch; ch++, v++) {
            if (!__all_sync(0xffffffff,
                            mbar_wait(myfull + v % stages, (v / stages) & 1, abort, limit_ns, status, K_GEMV, 1))) {
                ok = false;
                break;
            }
            const int k0 = ch * kc, len = min(kc, K - k0);
            const h16* st = myring + (v % stages) * stage;
#pragma unroll 1
            for (int kl = 8 * lane; kl < len; kl += 256) {  // this lane's groups of the chunk, in order
                float w[COLS][8];
#pragma unroll
                for (int c = 0; c < COLS; c++) halves8(*reinterpret_cast<const uint4*>(st + c * len + kl), w[c]);
                const h16* xk = xs + k0 + kl;
                gemv_group<MR, COLS>(
                    w, [&](int m) { return *reinterpret_cast<const uint4*>(xk + m * K); }, M, acc);
            }
            __syncwarp();
            if (lane == 0 && v + stages < nunits) {
                fence_proxy_async_smem();  // this warp's reads of the stage come before the copy that refills it
                issue(v + stages);
            }
        }
        if (!ok) break;
        gemv_store<MR, COLS>(acc, lane, (gw + t * nw) * COLS, y, ldy, M, N, bias, gelu != 0);
    }
    if (!ok) {
        // copies this warp issued and has not consumed land before it leaves; bounded, whatever the abort flag says
        const int issued = min(nunits, v + stages);
        for (int u = v; u < issued; u++) {
            const uint64_t t0 = globaltimer();
            while (!mbar_test_wait(myfull + u % stages, (u / stages) & 1) && globaltimer() - t0 < limit_ns) {
            }
        }
        if (threadIdx.x == 0) {
            const uint64_t t0 = globaltimer();
            while (!mbar_test_wait(xbar, 0) && globaltimer() - t0 < limit_ns) {
            }
        }
    }
}

// the register form; GB groups of loads in flight per lane, MINB CTAs per SM
template <int MR, int GB, int MINB>
__global__ void __launch_bounds__(256, MINB) gemv_kernel(const h16* __restrict__ x, int ldx,
                                                         const h16* __restrict__ W, h16* __restrict__ y, int ldy, int M,
                                                         int N, int K, const h16* __restrict__ bias, int gelu) {
    gemv_rows<MR, GB>(x, ldx, W, y, ldy, M, N, K, bias, gelu != 0);
}

template <int GB, int MINB>
static cudaError_t launch_rows(const h16* X, int ldx, const h16* W, h16* Y, int ldy, int m, int n, int k,
                               const h16* B, int gelu, cudaStream_t st) {
    const dim3 grid((n + gv::WARPS * gv::COLS - 1) / (gv::WARPS * gv::COLS));
    if (m == 1) return launch_pdl(gemv_kernel<1, GB, MINB>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B, gelu);
    if (m == 2) return launch_pdl(gemv_kernel<2, GB, MINB>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B, gelu);
    if (m <= 4) return launch_pdl(gemv_kernel<4, GB, MINB>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B, gelu);
    return launch_pdl(gemv_kernel<8, GB, MINB>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B, gelu);
}

void init_gemv_attrs() {
    cudaFuncSetAttribute(gemv_ring_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gq::SMEM_MAX);
    cudaFuncSetAttribute(gemv_ring_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gq::SMEM_MAX);
    cudaFuncSetAttribute(gemv_ring_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gq::SMEM_MAX);
    cudaFuncSetAttribute(gemv_ring_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gq::SMEM_MAX);
}

int launch_gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
                bool gelu, cudaStream_t st) {
    if (m < 1 || m > 8 || n < 1 || k < 8 || k % 8 || ldx < k || ldy < n)
        return fail("gemv: 1 <= m <= 8, k a multiple of 8, ldx >= k, ldy >= n");
    if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ((long)ldx * 2) % 16)
        return fail("gemv: x and w 16-byte aligned, x rows a multiple of 16 bytes");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    auto X = (const h16*)x;
    auto W = (const h16*)w;
    auto Y = (h16*)y;
    auto B = (const h16*)bias;
    const int g = gelu ? 1 : 0;
    cudaError_t e;
    // a test hook: MMZ_TEST_GEMV_ROWS=1 takes the register form with 5 groups in flight and one CTA per SM
    const char* t = getenv("MMZ_TEST_GEMV_ROWS");
    const bool rows_form = t && t[0] == '1';
    // Short rows over a long vocabulary (the tiny models' logits, k <= 512) stream best in the register form with
    // two CTAs per SM (measured: 9.3 us against 14.1 us in the ring at 51865 x 384, m = 1); everything else goes
    // through the ring where it fits (every large-model shape: up to 3.6x the register form at m = 8).
    if (k <= 512 && n >= 8192 && !rows_form) return check_pdl(launch_rows<2, 2>(X, ldx, W, Y, ldy, m, n, k, B, g, st), "gemv");
    const gq::Plan pl = gq::plan(m, k);
    if (pl.kc > 0 && !rows_form) {
        const int items = (n + gq::COLS - 1) / gq::COLS;
        const dim3 grid(items < dc.sms ? items : dc.sms);
        const int kc = pl.kc, ns = pl.stages;
        if (m == 1) e = launch_pdl(gemv_ring_kernel<1>, grid, dim3(256), pl.smem, st, X, ldx, W, Y, ldy, m, n, k, B, kc, ns, g, dc.status, dc.limit_ns);
        else if (m == 2) e = launch_pdl(gemv_ring_kernel<2>, grid, dim3(256), pl.smem, st, X, ldx, W, Y, ldy, m, n, k, B, kc, ns, g, dc.status, dc.limit_ns);
        else if (m <= 4) e = launch_pdl(gemv_ring_kernel<4>, grid, dim3(256), pl.smem, st, X, ldx, W, Y, ldy, m, n, k, B, kc, ns, g, dc.status, dc.limit_ns);
        else e = launch_pdl(gemv_ring_kernel<8>, grid, dim3(256), pl.smem, st, X, ldx, W, Y, ldy, m, n, k, B, kc, ns, g, dc.status, dc.limit_ns);
        return check_pdl(e, "gemv");
    }
    return check_pdl(launch_rows<gv::GB, 1>(X, ldx, W, Y, ldy, m, n, k, B, g, st), "gemv");
}

}  // namespace mmz
