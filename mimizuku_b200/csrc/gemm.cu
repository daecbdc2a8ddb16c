// The encoder's linear layers and the cross-K/V projection on the 5th-generation tensor cores, for sm_100a:
// C = rh(A B^T + bias) (src/gpu.rs:208-236 lin, src/model.rs:551-623), with the work around them folded into the
// epilogue: the exact-erf GELU of the convolutions and of fc1 (gelu_inplace, kernels/whisper.cu:107-112, applied to the
// rounded value as the separate kernel does), or the store of the cross k/v into the decoder's head-contiguous
// [layer][k|v][head][1500][64] layout (model.rs:614-623 and fill_bias_heads, whisper.cu:99-104: there a bias image
// written first and a strided-batched GEMM accumulated onto it).
//
// A persistent CTA per SM takes every gridDim-th tile of 128 rows x BN columns (BN 256, or 128 where that balances
// the tiles over the SMs better):
//   warp 0      TMA producer: A (activations, [M][lda]) and B (weights, [N][K]) tiles of 64 K through a 4- or
//               6-stage ring (128-byte swizzle); the weight tiles of the first stages are issued before the wait for
//               the kernel before (the weights do not depend on it), the activation tiles after it
//   warp 1      MMA issuer: M128 N(BN) K16 products into one of two TMEM accumulators, so that one tile's epilogue
//               overlaps the next tile's products; descriptors formed once and advanced by constants
//   warps 2-9   epilogue: two warps per TMEM lane quarter, each half of a tile's columns; thread = row, 32 columns
//               at a time from TMEM, + bias (fp32), rounded to fp16, GELU, 16-byte stores
// Every wait is bounded; a CTA that gives up reports into the status word, lets its copies land, waits for its MMAs
// and frees its TMEM.
#include "common.cuh"
#include "launch.h"

namespace mmz {
namespace gm {

constexpr int BM = 128;        // rows per tile (MMA M)
constexpr int BK = 64;         // K per stage (one 128-byte swizzle atom)
constexpr int NTHREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int EPW = 8;         // epilogue warps: two per TMEM lane quarter, each half of a tile's columns
constexpr int AT = BM * BK * 2;  // 16 KB

template <int BN>
struct Cfg {
    static constexpr int NS = BN == 256 ? 4 : 6;  // 48 KB or 32 KB per stage
    static constexpr int BT = BN * BK * 2;
    static constexpr uint32_t IDESC = idesc_f16_f32(BM, BN, false);
};

template <int BN>
struct Smem {
    uint8_t a[Cfg<BN>::NS][AT];
    uint8_t b[Cfg<BN>::NS][Cfg<BN>::BT];
    float bias[2][BN];  // the columns of the tile being written (two tiles in flight)
    uint64_t full[Cfg<BN>::NS], empty[Cfg<BN>::NS], accf[2], acce[2], fin;
    uint32_t tmem;
    int abort;
};

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

}  // namespace gm

using namespace gm;

// grid min(SMs, tiles), block NTHREADS, dynamic shared memory sizeof(Smem<BN>) + 1024 (alignment slack).
// mode 0: C[m][n] at c + m ldc + n; 1: the same after GELU; 2: head blocks, C[m][n] at c + (n / 64) blk + m 64 + n % 64
template <int BN>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_bias_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                     const h16* __restrict__ bias, h16* __restrict__ c, long ldc, int M, int N, int K, int mode,
                     long blk, unsigned* status, unsigned long long limit_ns) {
    using C = Cfg<BN>;
    constexpr int NS = C::NS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    Smem<BN>& s = *reinterpret_cast<Smem<BN>*>(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (M + BM - 1) / BM, T = mt * (N / BN), G = gridDim.x, cta = blockIdx.x;
    const int my = cta < T ? (T - cta + G - 1) / G : 0;  // tiles of this CTA: cta, cta + G, ...
    const int nch = K / BK, nq = my * nch;
    volatile int* abort = &s.abort;
    auto tile_m0 = [&](int i) { return ((cta + i * G) % mt) * BM; };  // rows fastest: concurrent tiles share weights
    auto tile_n0 = [&](int i) { return ((cta + i * G) / mt) * BN; };
    int issued = 0;  // producer: stages issued (weights and activations)
    if (warp == 0 && lane == 0) {
        s.abort = 0;
        for (int i = 0; i < NS; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&s.accf[a], 1);
            mbar_init(&s.acce[a], EPW);  // one arrival per epilogue warp
        }
        mbar_init(&s.fin, 1);
        fence_mbar_init();
        prefetch_tmap(&amap);
        prefetch_tmap(&bmap);
        // the weights do not depend on the kernel before: the first stages' weight tiles go out before the wait
        for (int q = 0; q < NS && q < nq; q++) {
            mbar_expect_tx(&s.full[q], AT + C::BT);
            tma_load_2d(s.b[q], &bmap, (q % nch) * BK, tile_n0(q / nch), &s.full[q]);
        }
    }
    if (warp == 1) {
        tmem_alloc(&s.tmem, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_wait();  // the activations come from the kernel before
    const uint32_t tb = s.tmem;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            for (int q = 0; q < NS && q < nq; q++) tma_load_2d(s.a[q], &amap, (q % nch) * BK, tile_m0(q / nch), &s.full[q]);
            issued = NS < nq ? NS : nq;
            for (int q = issued; q < nq; q++) {
                const int st = q % NS, i = q / nch, kc = q % nch;
                if (!mbar_wait_spin(&s.empty[st], ((q / NS) - 1) & 1, abort, limit_ns, status, K_GEMM, 1)) break;
                mbar_expect_tx(&s.full[st], AT + C::BT);
                tma_load_2d(s.b[st], &bmap, kc * BK, tile_n0(i), &s.full[st]);
                tma_load_2d(s.a[st], &amap, kc * BK, tile_m0(i), &s.full[st]);
                issued = q + 1;
            }
            if (*abort)  // let every issued copy land before the shared memory is released
                for (int q = issued > NS ? issued - NS : 0; q < issued; q++)
                    mbar_wait(&s.full[q % NS], (q / NS) & 1, nullptr, limit_ns, nullptr, 0, 0);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint64_t ad0 = sdesc_sw128(smem_u32(s.a[0]), 16, 1024), bd0 = sdesc_sw128(smem_u32(s.b[0]), 16, 1024);
            constexpr uint64_t ASTAGE = AT >> 4, BSTAGE = C::BT >> 4, KSTEP = 32 >> 4;
            bool ok = true;
            for (int i = 0; ok && i < my; i++) {
                const int a = i & 1;
                if (i >= 2 && !mbar_wait_spin(&s.acce[a], ((i >> 1) - 1) & 1, abort, limit_ns, status, K_GEMM, 2)) break;
                tc_fence_after();
                for (int kc = 0; kc < nch; kc++) {
                    const int q = i * nch + kc, st = q % NS;
                    if (!mbar_wait_spin(&s.full[st], (q / NS) & 1, abort, limit_ns, status, K_GEMM, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = ad0 + st * ASTAGE, bd = bd0 + st * BSTAGE;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        umma_f16_ss(tb + a * BN, ad + kk * KSTEP, bd + kk * KSTEP, C::IDESC, (kc > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&s.empty[st]);
                }
                if (ok) umma_commit(&s.accf[a]);
            }
        }
        if (lane == 0) umma_commit(&s.fin);  // completes once every MMA issued above has finished
    } else {
        // ---------------------------------------------------------------- epilogue (warps 2-9)
        const int qd = warp & 3;                 // the TMEM lane quarter this warp may read
        const int half = (warp - 2) >> 2;        // which half of the tile's columns
        const int ep = threadIdx.x - 64;         // 0 .. 255
        const uint32_t tl = tb + ((uint32_t)(qd * 32) << 16);
        for (int i = 0; i < my; i++) {
            const int a = i & 1, m0 = tile_m0(i), n0 = tile_n0(i);
            for (int j = ep; j < BN; j += 32 * EPW) s.bias[a][j] = bias ? f(bias[n0 + j]) : 0.f;
            asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight epilogue warps: the tile's bias is in place
            if (!__all_sync(0xffffffff, mbar_wait_spin(&s.accf[a], (i >> 1) & 1, abort, limit_ns, status, K_GEMM, 4)))
                continue;
            tc_fence_after();
            const int row = m0 + qd * 32 + lane;
#pragma unroll 1
            for (int ch = half * (BN / 64); ch < (half + 1) * (BN / 64); ch++) {
                uint32_t v[32];
                tmem_ld32(tl + a * BN + ch * 32, v);
                if (ch == (half + 1) * (BN / 64) - 1) {  // the accumulator may take the tile after next
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.acce[a]);
                }
                if (row < M) {
                    uint32_t pk[16];
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const int cc = ch * 32 + 2 * e;
                        h16 h0 = h(__uint_as_float(v[2 * e]) + s.bias[a][cc]);
                        h16 h1 = h(__uint_as_float(v[2 * e + 1]) + s.bias[a][cc + 1]);
                        if (mode == 1) {
                            h0 = h(gelu_erf(f(h0)));
                            h1 = h(gelu_erf(f(h1)));
                        }
                        __half2 p2 = __halves2half2(h0, h1);
                        pk[e] = *reinterpret_cast<uint32_t*>(&p2);
                    }
                    const int n = n0 + ch * 32;
                    uint4* dst = reinterpret_cast<uint4*>(mode == 2 ? c + (n / 64) * blk + (long)row * 64 + (n % 64)
                                                                    : c + (long)row * ldc + n);
#pragma unroll
                    for (int u = 0; u < 4; u++) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
                }
            }
        }
    }
    // teardown: every role is done with TMEM; the MMA pipe must drain before the MMA warp releases it
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        mbar_wait(&s.fin, 0, nullptr, limit_ns, status, K_GEMM, 5);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tb, 2 * BN);
    }
}

// the fraction of SM slots busy over the waves of T tiles on `sms` persistent CTAs
static double balance(long T, int sms) {
    const long waves = (T + sms - 1) / sms;
    return (double)T / (double)(waves * sms);
}

int launch_gemm_bias(const void* a, int lda, const void* w, const void* bias, void* c, long ldc, int M, int N, int K,
                     int mode, long blk, cudaStream_t st) {
    if (M < 1 || N < 128 || N % 128 || K < BK || K % BK || mode < 0 || mode > 2)
        return fail("gemm_bias: N a multiple of 128, K a multiple of 64");
    if (((uintptr_t)a & 15) || ((uintptr_t)w & 15) || ((uintptr_t)c & 15) || ((lda * 2) & 15) || lda < K ||
        (mode != 2 && (ldc < N || (ldc * 2) & 15)) || (mode == 2 && (N % 64 || blk < (long)M * 64 || (blk * 2) & 15)))
        return fail("gemm_bias: 16-byte aligned operands and row pitches");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    const long mt = (M + BM - 1) / BM;
    // 256-column tiles unless 128 balances the tiles over the SMs clearly better
    const bool wide = N % 256 == 0 && balance(mt * (N / 256), dc.sms) + 0.05 >= balance(mt * (N / 128), dc.sms);
    const int bn = wide ? 256 : 128;
    CUtensorMap am, bm;
    const uint64_t ad[2] = {(uint64_t)K, (uint64_t)M}, as[1] = {(uint64_t)lda * 2};
    const uint32_t ab[2] = {BK, BM};
    const uint64_t bd[2] = {(uint64_t)K, (uint64_t)N}, bs[1] = {(uint64_t)K * 2};
    const uint32_t bb[2] = {BK, (uint32_t)bn};
    if (make_tmap_2d(&am, a, ad, as, ab, true) || make_tmap_2d(&bm, w, bd, bs, bb, true))
        return fail("gemm_bias: cuTensorMapEncodeTiled failed");
    const long T = mt * (N / bn);
    const int grid = (int)(T < dc.sms ? T : dc.sms);
    if (wide)
        return check_pdl(launch_pdl(gemm_bias_kernel<256>, dim3(grid), dim3(NTHREADS), sizeof(Smem<256>) + 1024, st,
                                    am, bm, (const h16*)bias, (h16*)c, ldc, M, N, K, mode, blk, dc.status, dc.limit_ns),
                         "gemm_bias");
    return check_pdl(launch_pdl(gemm_bias_kernel<128>, dim3(grid), dim3(NTHREADS), sizeof(Smem<128>) + 1024, st, am, bm,
                                (const h16*)bias, (h16*)c, ldc, M, N, K, mode, blk, dc.status, dc.limit_ns),
                     "gemm_bias");
}

void init_gemm_attrs() {
    cudaFuncSetAttribute(gemm_bias_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem<256>) + 1024);
    cudaFuncSetAttribute(gemm_bias_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem<128>) + 1024);
}

}  // namespace mmz
