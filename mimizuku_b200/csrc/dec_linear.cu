// Decoder linear layers for sm_100a: y[m][n] = rh(x[m][:] . W[n][:] + b[n]) for the batch of decoding sequences
// (m <= 32), optionally followed by GELU (fc1), replacing the cuBLAS GEMMs of the reference's decoder step
// (src/gpu.rs:208-247 lin / lin_onto_bias, src/model.rs:664-714) and the separate gelu_inplace kernel.
//
// At m <= 32 the product is a stream over W (2 bytes per weight, 2 x 32 flops per weight): memory-bound, so the design
// is about keeping W moving, with the 5th-generation tensor cores doing the arithmetic:
//   * W rows are the MMA's M side: a CTA owns 128 rows of W and computes the 128 x 32 tile of y^T in TMEM
//     (tcgen05.mma kind::f16, M128 N32 K16, A = W tile, B = x tile, both K-major with 128-byte swizzle)
//   * K is split across the CTAs of a thread-block cluster (up to 16), each streaming its share of the 64-wide K chunks
//     through a 4-stage TMA ring (a 16 KB W tile and the 4 KB x tile per stage); launched as a programmatic
//     dependent, a CTA issues its first W tiles before it waits for the kernel before (which x comes from)
//   * the cluster's partial tiles meet in shared memory: every rank sends rank q its partials of the rows q owns with
//     one bulk shared::cluster copy completing on q's mbarrier; q sums the slices in split order (deterministic),
//     adds the bias, rounds to fp16 (GELU for fc1) and stores its rows of y
// Warp 0 lane 0 issues the copies, warp 1 lane 0 the MMAs; the four warps read TMEM in the epilogue. Every wait is
// bounded.
#include "common.cuh"
#include "launch.h"

namespace mmz {
namespace lin {

constexpr int BN = 128;       // W rows per CTA (MMA M)
constexpr int BM = 32;        // batch rows (MMA N)
constexpr int BK = 64;        // K per chunk (one 128-byte swizzle atom)
constexpr int NS = 4;         // ring stages
constexpr int WT = BN * BK * 2;  // 16 KB
constexpr int XT = BM * BK * 2;  // 4 KB
constexpr uint32_t IDESC = idesc_f16_f32(BN, BM, false);

constexpr int RP = BM + 1;    // padded partial row: conflict-free stores by row and reads by row

// this CTA's partial tile, [owner rank][row of its slice][batch row], lives in the W ring once every MMA that read the
// ring has completed: 97 KB of shared memory, so two CTAs fit an SM
static_assert(BN * RP * 4 <= NS * WT, "the partial tile fits in the W ring");
struct Smem {
    uint8_t w[NS][WT];
    uint8_t x[NS][XT];
    float recv[BN * RP];       // [source rank][row of this rank's slice][batch row]
    uint64_t full[NS], empty[NS], done, got;
    uint32_t tmem;
    int abort;
};

__device__ __forceinline__ float gelu_ref(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

}  // namespace lin

using namespace lin;

// grid (S, tiles), cluster (S, 1, 1), block 128, dynamic shared memory sizeof(Smem)
__global__ void __launch_bounds__(128) dec_linear_splitk_kernel(const __grid_constant__ CUtensorMap wmap,
                                                         const __grid_constant__ CUtensorMap xmap,
                                                         const h16* __restrict__ bias, h16* __restrict__ y, int ldy,
                                                         int m, int n, int k, int gelu, unsigned* status,
                                                         unsigned long long limit_ns) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    const int S = gridDim.x, r = blockIdx.x, tile = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = k / BK, c0 = (int)((long)r * nch / S), c1 = (int)((long)(r + 1) * nch / S);
    volatile int* abort = &s.abort;
    const int R = BN / S;
    const uint32_t slice_bytes = (uint32_t)(R * RP * 4);  // a multiple of 16 for every S in {1, 2, 4, 8, 16}
    int issued = 0;
    auto issue_w = [&](int i) {  // one stage: the byte count of both copies, then the W tile
        const int st = i % NS, c = c0 + i;
        mbar_expect_tx(&s.full[st], WT + XT);
        tma_load_2d(s.w[st], &wmap, c * BK, tile * BN, &s.full[st]);
    };
    auto issue_x = [&](int i) {
        const int st = i % NS, c = c0 + i;
        tma_load_2d(s.x[st], &xmap, c * BK, 0, &s.full[st]);
    };
    griddep_launch_dependents();  // the next kernel may be scheduled as soon as every CTA here runs
    if (threadIdx.x == 0) {
        // the weight copies go out first: W does not depend on the kernel before, so with a programmatic dependent
        // launch they overlap its tail
        s.abort = 0;
        for (int i = 0; i < NS; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.done, 1);
        mbar_init(&s.got, 1);
        fence_mbar_init();
        prefetch_tmap(&wmap);
        prefetch_tmap(&xmap);
        for (; issued < NS && issued < c1 - c0; issued++) issue_w(issued);
        mbar_expect_tx(&s.got, slice_bytes * S);  // the partials of this rank's rows, one slice from every rank
    }
    griddep_wait();  // x comes from the kernel before
    if (threadIdx.x == 0)
        for (int i = 0; i < issued; i++) issue_x(i);
    // the other ranks may send into this CTA's receive buffer once its barriers exist
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    if (warp == 0) {
        tmem_alloc(&s.tmem, 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tacc = s.tmem;
    bool ok = true;
    if (threadIdx.x == 0) {
        // ------------------------------------------------------------ producer
        for (int i = issued; i < c1 - c0; i++) {
            const int st = i % NS;
            if (!mbar_wait(&s.empty[st], ((i / NS) - 1) & 1, abort, limit_ns, status, K_LIN, 1)) break;
            issue_w(i);
            issue_x(i);
            issued = i + 1;
        }
        if (*abort)
            for (int i = issued > NS ? issued - NS : 0; i < issued; i++)
                mbar_wait(&s.full[i % NS], (i / NS) & 1, nullptr, limit_ns, nullptr, 0, 0);
    } else if (threadIdx.x == 32) {
        // ------------------------------------------------------------ MMA issuer
        // descriptors formed once and advanced by constants (a stage, a K step only move the start address field)
        const uint64_t wd0 = sdesc_sw128(smem_u32(s.w[0]), 16, 1024), xd0 = sdesc_sw128(smem_u32(s.x[0]), 16, 1024);
        constexpr uint64_t WSTAGE = WT >> 4, XSTAGE = XT >> 4, KSTEP = 32 >> 4;
        for (int c = c0; c < c1; c++) {
            const int i = c - c0, st = i % NS;
            if (!mbar_wait_spin(&s.full[st], (i / NS) & 1, abort, limit_ns, status, K_LIN, 2)) break;
            tc_fence_after();
            const uint64_t wd = wd0 + st * WSTAGE, xd = xd0 + st * XSTAGE;
#pragma unroll
            for (int kk = 0; kk < BK / 16; kk++)
                umma_f16_ss(tacc, wd + kk * KSTEP, xd + kk * KSTEP, IDESC, (c > c0 || kk > 0) ? 1u : 0u);
            umma_commit(&s.empty[st]);
        }
        umma_commit(&s.done);  // completes when every MMA above has finished (at once if there were none)
    }
    // ---------------------------------------------------------------- epilogue
    // each thread holds one W row's 32 partial sums; rank q of the cluster owns rows [q R, q R + R) of the tile: every
    // rank sends q its partials of them with one bulk shared::cluster copy that completes on q's `got` barrier, and q
    // sums the S slices in split order
    ok = __syncthreads_and(mbar_wait_spin(&s.done, 0, abort, limit_ns, status, K_LIN, 3) && !*abort);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every rank's `got` barrier is initialised
    if (ok) {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tacc + ((uint32_t)(warp * 32) << 16), v);  // lane = W row, column = batch row
        const int row = warp * 32 + lane;
        float* dst = reinterpret_cast<float*>(s.w[0]) + row * RP;  // [row / R][row % R][j] = [row][j]
#pragma unroll
        for (int j = 0; j < BM; j++) dst[j] = c1 > c0 ? __uint_as_float(v[j]) : 0.f;
        fence_proxy_async_smem();  // the bulk copies read these stores through the async proxy
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && ok)
        for (int q = 0; q < S; q++)
            bulk_s2s_cluster(dsmem_addr(&s.recv[r * R * RP], q), smem_u32(reinterpret_cast<float*>(s.w[0]) + q * R * RP), slice_bytes,
                             dsmem_addr(&s.got, q));
    // waits even after an earlier failure, so that no copy into this CTA is still in flight when it leaves
    ok = __syncthreads_and(mbar_wait_cluster(&s.got, 0, nullptr, limit_ns, status, K_LIN, 4) && ok);
    if (ok) {
        for (int i = threadIdx.x; i < R * BM; i += 128) {
            const int rl = i % R, j = i / R;
            float acc = 0.f;
            for (int q = 0; q < S; q++) acc += s.recv[(q * R + rl) * RP + j];
            const int col = tile * BN + r * R + rl;
            if (j < m && col < n) {
                float o = rh(acc + (bias ? f(bias[col]) : 0.f));
                if (gelu) o = gelu_ref(o);
                y[(long)j * ldy + col] = h(o);
            }
        }
    }
    // the receivers have their slices, so the copies out of this CTA's send buffer are done once all ranks are here
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tacc, 32);
    }
}

int launch_dec_linear(const void* x, int ldx, const void* w, const void* bias, void* y, int ldy, int m, int n, int k,
                      bool gelu, cudaStream_t st) {
    if (m < 1 || m > BM || n < 1 || k < BK || k % BK) return fail("dec_linear: m <= 32, k a multiple of 64");
    if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ((ldx * 2) & 15) || ldx < k)
        return fail("dec_linear: x, W 16-byte aligned, ldx >= k with 16-byte row pitch");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    CUtensorMap wm, xm;
    const uint64_t wd[2] = {(uint64_t)k, (uint64_t)n}, ws[1] = {(uint64_t)k * 2};
    const uint32_t wb[2] = {BK, BN};
    const uint64_t xd[2] = {(uint64_t)k, (uint64_t)m}, xs[1] = {(uint64_t)ldx * 2};
    const uint32_t xb[2] = {BK, BM};
    if (make_tmap_2d(&wm, w, wd, ws, wb, 128) || make_tmap_2d(&xm, x, xd, xs, xb, 128))
        return fail("dec_linear: cuTensorMapEncodeTiled failed");
    // split K over a cluster of S CTAs (a power of two up to 16, at least one chunk each) so that the launch has up to
    // two CTAs per SM: at m <= 32 the product is a stream over W, and more CTAs keep more of it in flight
    const int tiles = (n + BN - 1) / BN, nch = k / BK;
    int S = 1;
    while (S < 16 && S * 2 <= nch && tiles * S * 2 <= 2 * dc.sms) S *= 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, tiles, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.dynamicSmemBytes = sizeof(Smem);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // a programmatic dependent of the kernel before
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, dec_linear_splitk_kernel, wm, xm, (const h16*)bias, (h16*)y, ldy, m, n, k,
                                       gelu ? 1 : 0, dc.status, dc.limit_ns);
    if (e != cudaSuccess) return failf("dec_linear: launch failed: %s", cudaGetErrorString(e));
    return 0;
}

void init_dec_linear_attrs() {
    cudaFuncSetAttribute(dec_linear_splitk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem));
    cudaFuncSetAttribute(dec_linear_splitk_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

}  // namespace mmz
