// The encoder's linear layers and the cross-K/V projection on the 5th-generation tensor cores, for sm_100a:
// C = rh(A B^T + bias) (src/gpu.rs:208-236 lin, src/model.rs:551-623), with the work around them folded into the
// epilogue: the exact-erf GELU of the convolutions and of fc1 (gelu_inplace, kernels/whisper.cu:107-112, applied to the
// rounded value as the separate kernel does), or the store of the cross k/v into the decoder's head-contiguous
// [layer][k|v][head][1500][64] layout (model.rs:614-623 and fill_bias_heads, whisper.cu:99-104: there a bias image
// written first and a strided-batched GEMM accumulated onto it).
//
// Two persistent kernels. Where N is a multiple of 256 and M > 128, gemm_pair_kernel (below): tiles of 256 x 256 on a
// pair of CTAs (cta_group::2), 32 KB of operands per SM per 64-wide K step, TMA stores from the epilogue. Otherwise
// gemm_bias_kernel: a CTA per SM takes every gridDim-th tile of 128 rows x BN columns (BN 256, or 128 where that
// balances the tiles over the SMs better):
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

// ============================================================================ a pair of CTAs per tile (cta_group::2)
//
// The same product on tiles of 256 rows x 256 columns, each computed by a cluster of two CTAs on two SMs as one
// M256 N256 K16 MMA stream: CTA r of the pair loads its 128 rows of A and its 128 rows of the weight tile (half of
// B), and the even CTA issues the MMAs, which read both CTAs' shared memory and leave each CTA its 128 rows x 256
// columns of the accumulator in its own TMEM. Per SM, 32 KB of operands per 64-wide K step feed 4 x 1 MFLOP of MMA
// (48 KB in the single-CTA kernel above, which ran the encoder's qkv projection at 1134 TFLOP/s against this kernel's
// 1314). The epilogue stages each 32 x 64 output box in shared memory (128-byte
// swizzle) and stores it with TMA: with thread-per-row 16-byte stores instead (as in the single-CTA kernel) this
// kernel took 54.5 against 32.4 us on the 24000 x 1280 x 384 convolution, where the epilogue is the larger part.
//   warp 0 (each CTA)  TMA producer for its own halves; every copy counts its bytes on the even CTA's `full` barrier,
//                      whose phase the even CTA's producer opens with the expected bytes of both CTAs
//   warp 1 (even CTA)  MMA issuer; each stage's completion is committed to both CTAs' `empty` barriers, each tile's to
//                      both CTAs' `accf` barriers; TMEM is allocated and released by warp 1 of both CTAs
//   warps 2-9          epilogue in each CTA on its own TMEM rows (as above); the accumulator is released by arrivals
//                      of both CTAs' epilogue warps on the even CTA's `acce` barrier
// Each CTA fetches its own operand halves: no copy lands in both CTAs.
namespace gp {
constexpr int BMC = 128;                // rows per CTA (the pair's MMA has M = 256)
constexpr int BN = 256;                 // tile columns (MMA N)
constexpr int NS = 5;                   // 32 KB per stage
constexpr int PEPW = 8;                 // epilogue warps: two per TMEM lane quarter, each 128 of the tile's columns
constexpr int PTHREADS = 64 + 32 * PEPW;
constexpr int BT = BN / 2 * BK * 2;     // this CTA's half of the weight tile: 16 KB
constexpr int OT = 32 * 64 * 2;         // an epilogue warp's output box: 32 rows x 64 columns, 128-byte swizzle
constexpr uint32_t IDESC = idesc_f16_f32(2 * BMC, BN, false);
struct PairSmem {
    uint8_t a[NS][AT];
    uint8_t b[NS][BT];
    uint8_t out[PEPW][OT];
    float bias[2][BN];
    uint64_t full[NS], empty[NS], accf[2], acce[2], fin;
    uint32_t tmem;
    int abort;
};
}  // namespace gp

// The pairs' tiles: 256 rows x 256 columns, rows fastest (pairs working at once share weight tiles); pair p takes
// tiles p, p + G, ... (G pairs).
// grid 2 x (pairs), cluster (2, 1, 1), block PTHREADS, dynamic shared memory sizeof(gp::PairSmem) + 1024.
// bmap: the weights with a box of 128 rows (half of a tile's columns); cmap: the output with a box of 32 x 64.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gp::PTHREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                     const __grid_constant__ CUtensorMap cmap, const h16* __restrict__ bias, int M, int N, int K,
                     int mode, unsigned* status, unsigned long long limit_ns) {
    using namespace gp;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    PairSmem& s = *reinterpret_cast<PairSmem*>(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();  // 0: the CTA that issues the MMAs
    const bool lead = rank == 0;
    const int mt = (M + 2 * BMC - 1) / (2 * BMC), T = mt * (N / BN), G = gridDim.x / 2, pid = blockIdx.x / 2;
    const int my = pid < T ? (T - pid + G - 1) / G : 0;  // tiles of this pair: pid, pid + G, ...
    const int nch = K / BK, nq = my * nch;
    auto tile_m0 = [&](int i) { return ((pid + i * G) % mt) * 2 * BMC; };  // the pair's first row
    auto tile_n0 = [&](int i) { return ((pid + i * G) / mt) * BN; };
    volatile int* abort = &s.abort;
    if (warp == 0 && lane == 0) {
        s.abort = 0;
        for (int i = 0; i < NS; i++) {
            mbar_init(&s.full[i], 1);  // the even CTA's producer (expected bytes of both CTAs)
            mbar_init(&s.empty[i], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&s.accf[a], 1);
            mbar_init(&s.acce[a], 2 * PEPW);  // both CTAs' epilogue warps (used in the even CTA)
        }
        mbar_init(&s.fin, 1);
        fence_mbar_init();
        prefetch_tmap(&amap);
        prefetch_tmap(&bmap);
        prefetch_tmap(&cmap);
    }
    if (warp == 1) {
        tmem_alloc_pair(&s.tmem, 2 * BN);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before either touches the other's
    tc_fence_after();
    const uint32_t tb = s.tmem;
    int issued = 0;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer (each CTA, its own halves)
        // the work item is formed once per tile; per stage only the K offset and the ring slot move
        const uint32_t full0 = dsmem_addr(&s.full[0], 0);
        struct Cursor {
            int i, kc, brow, arow;
        };
        auto start = [&](Cursor& c, int i) {
            c.i = i;
            c.kc = 0;
            c.brow = tile_n0(i) + (int)rank * (BN / 2);
            c.arow = tile_m0(i) + (int)rank * BMC;
        };
        auto next = [&](Cursor& c) {
            if (++c.kc == nch) start(c, c.i + 1);
        };
        const int pro = NS < nq ? NS : nq;
        if (lane == 0) {  // the weights do not depend on the kernel before: the first stages' go out before the wait
            Cursor c;
            start(c, 0);
            for (int q = 0; q < pro; q++, next(c)) {
                if (lead) mbar_expect_tx(&s.full[q], 2 * (AT + BT));
                tma_load_2d_pair(s.b[q], &bmap, c.kc * BK, c.brow, full0 + 8 * q);
            }
        }
        griddep_wait();  // the activations come from the kernel before
        if (lane == 0) {
            Cursor c;
            start(c, 0);
            for (int q = 0; q < pro; q++, next(c)) tma_load_2d_pair(s.a[q], &amap, c.kc * BK, c.arow, full0 + 8 * q);
            issued = pro;
            int st = pro % NS, ph = pro / NS;  // ring slot and its use count
            for (int q = pro; q < nq; q++, next(c)) {
                if (!mbar_wait_spin(&s.empty[st], (ph - 1) & 1, abort, limit_ns, status, K_GEMM, 11)) break;
                if (lead) mbar_expect_tx(&s.full[st], 2 * (AT + BT));
                tma_load_2d_pair(s.b[st], &bmap, c.kc * BK, c.brow, full0 + 8 * st);
                tma_load_2d_pair(s.a[st], &amap, c.kc * BK, c.arow, full0 + 8 * st);
                issued = q + 1;
                if (++st == NS) {
                    st = 0;
                    ph++;
                }
            }
            // let the copies counted on this CTA's barriers land before shared memory is released (the odd CTA's land
            // on the even CTA's barriers, which the even CTA waits for here; the pair leaves together)
            if (*abort && lead)
                for (int q = issued > NS ? issued - NS : 0; q < issued; q++)
                    mbar_wait(&s.full[q % NS], (q / NS) & 1, nullptr, limit_ns, nullptr, 0, 0);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (even CTA)
        if (lead && lane == 0) {
            const uint64_t ad0 = sdesc_sw128(smem_u32(s.a[0]), 16, 1024), bd0 = sdesc_sw128(smem_u32(s.b[0]), 16, 1024);
            constexpr uint64_t ASTAGE = AT >> 4, BSTAGE = BT >> 4, KSTEP = 32 >> 4;
            const uint32_t empty0[2] = {dsmem_addr(&s.empty[0], 0), dsmem_addr(&s.empty[0], 1)};
            const uint32_t accf0[2] = {dsmem_addr(&s.accf[0], 0), dsmem_addr(&s.accf[0], 1)};
            bool ok = true;
            int st = 0, ph = 0;  // ring slot and its use count
            for (int i = 0; ok && i < my; i++) {
                const int a = i & 1;
                if (i >= 2 && !mbar_wait_cluster(&s.acce[a], ((i >> 1) - 1) & 1, abort, limit_ns, status, K_GEMM, 12))
                    break;
                tc_fence_after();
                for (int kc = 0; kc < nch; kc++) {
                    if (!mbar_wait_spin(&s.full[st], ph & 1, abort, limit_ns, status, K_GEMM, 13)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = ad0 + st * ASTAGE, bd = bd0 + st * BSTAGE;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        umma_f16_ss_pair(tb + a * BN, ad + kk * KSTEP, bd + kk * KSTEP, IDESC, (kc > 0 || kk > 0) ? 1u : 0u);
                    umma_commit_pair(empty0[0] + 8 * st);
                    umma_commit_pair(empty0[1] + 8 * st);
                    if (++st == NS) {
                        st = 0;
                        ph++;
                    }
                }
                if (ok) {
                    umma_commit_pair(accf0[0] + 8 * a);
                    umma_commit_pair(accf0[1] + 8 * a);
                }
            }
            umma_commit_pair(dsmem_addr(&s.fin, 0));  // both CTAs: every MMA issued above has finished
            umma_commit_pair(dsmem_addr(&s.fin, 1));
        }
    } else {
        // ---------------------------------------------------------------- epilogue (warps 2-9, each CTA)
        // a warp reads its 32 rows x 128 columns of the accumulator at once, releases it, and writes them as two
        // 32 x 64 boxes through its shared-memory box (128-byte swizzle: conflict-free row writes) and TMA stores
        const int qd = warp & 3;                 // the TMEM lane quarter this warp may read
        const int half = (warp - 2) >> 2;        // which half of the tile's columns
        const int ep = threadIdx.x - 64;         // 0 .. 255
        const uint32_t tl = tb + ((uint32_t)(qd * 32) << 16);
        const uint32_t acce0 = dsmem_addr(&s.acce[0], 0);
        uint8_t* box = s.out[warp - 2];
        for (int i = 0; i < my; i++) {
            const int a = i & 1, n0 = tile_n0(i);
            s.bias[a][ep] = bias ? f(bias[n0 + ep]) : 0.f;
            asm volatile("bar.sync 1, %0;" ::"n"(32 * PEPW) : "memory");  // the epilogue warps: the tile's bias is in place
            if (!__all_sync(0xffffffff, mbar_wait_spin(&s.accf[a], (i >> 1) & 1, abort, limit_ns, status, K_GEMM, 14)))
                continue;
            tc_fence_after();
            uint32_t v[128];
            tmem_ld128(tl + a * BN + half * 128, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {  // the accumulator may take the tile after next
                if (lead) mbar_arrive(&s.acce[a]);
                else mbar_arrive_remote(acce0 + 8 * a);
            }
            const int row0 = tile_m0(i) + (int)rank * BMC + qd * 32;
            if (row0 >= M) continue;  // this warp's rows are all past the end (the box would start out of range)
            const float2* bz = reinterpret_cast<const float2*>(&s.bias[a][half * 128]);
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {
                if (lane == 0) bulk_wait_read<0>();  // the box's previous store has read it
                __syncwarp();
#pragma unroll
                for (int u = 0; u < 8; u++) {  // 16-byte chunk u of this thread's row: columns hb 64 + 8u ..
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int k = hb * 64 + u * 8 + 2 * e;
                        __half2 hv = __float22half2_rn(
                            fadd2(make_float2(__uint_as_float(v[k]), __uint_as_float(v[k + 1])), bz[k >> 1]));
                        if (mode == 1) {
                            float2 g = __half22float2(hv);
                            hv = __float22half2_rn(make_float2(gelu_erf(g.x), gelu_erf(g.y)));
                        }
                        pk[e] = *reinterpret_cast<uint32_t*>(&hv);
                    }
                    *reinterpret_cast<uint4*>(box + lane * 128 + ((u ^ (lane & 7)) << 4)) =
                        make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                fence_proxy_async_smem();  // the box's writes are visible to the tensor copy
                __syncwarp();
                if (lane == 0) {
                    const int n = n0 + half * 128 + hb * 64;
                    if (mode == 2) tma_store_3d(&cmap, 0, row0, n / 64, box);
                    else tma_store_2d(&cmap, n, row0, box);
                    bulk_commit();
                }
            }
        }
        if (lane == 0) bulk_wait_all();
    }
    // teardown: every MMA into either CTA's TMEM has finished before the pair releases it, and neither CTA leaves
    // while the other may still signal its barriers
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        mbar_wait(&s.fin, 0, nullptr, limit_ns, status, K_GEMM, 15);
        __syncwarp();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tb, 2 * BN);
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
    if (make_tmap_2d(&am, a, ad, as, ab, 128) || make_tmap_2d(&bm, w, bd, bs, bb, 128))
        return fail("gemm_bias: cuTensorMapEncodeTiled failed");
    // pairs of CTAs on 256 x 256 tiles where the shape has them (MMZ_TEST_GEMM_1SM=1 keeps one CTA per tile, a test
    // hook); each pair's CTAs load 128-row halves of the weight tile
    const char* one = getenv("MMZ_TEST_GEMM_1SM");
    if (dc.gemm_pairs > 0 && N % 256 == 0 && M > BM && !(one && one[0] == '1')) {
        CUtensorMap cm;
        const uint32_t hb1[2] = {BK, 128};
        int e = make_tmap_2d(&bm, w, bd, bs, hb1, 128);
        if (mode == 2) {  // [N / 64 blocks][M rows][64]
            const uint64_t cd[3] = {64, (uint64_t)M, (uint64_t)(N / 64)}, cs[2] = {128, (uint64_t)blk * 2};
            const uint32_t cb[3] = {64, 32, 1};
            e = e || make_tmap_3d(&cm, c, cd, cs, cb, 128);
        } else {
            const uint64_t cd[2] = {(uint64_t)N, (uint64_t)M}, cs[1] = {(uint64_t)ldc * 2};
            const uint32_t cb[2] = {64, 32};
            e = e || make_tmap_2d(&cm, c, cd, cs, cb, 128);
        }
        if (e) return fail("gemm_bias: cuTensorMapEncodeTiled failed");
        const long T2 = ((M + 255) / 256) * (long)(N / 256);
        const int pairs = (int)(T2 < dc.gemm_pairs ? T2 : dc.gemm_pairs);
        return check_pdl(launch_pdl(gemm_pair_kernel, dim3(2 * pairs), dim3(gp::PTHREADS), sizeof(gp::PairSmem) + 1024,
                                    st, am, bm, cm, (const h16*)bias, M, N, K, mode, dc.status, dc.limit_ns),
                         "gemm_bias");
    }
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

void init_gemm_attrs(DevCtx& c) {
    cudaFuncSetAttribute(gemm_bias_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem<256>) + 1024);
    cudaFuncSetAttribute(gemm_bias_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem<128>) + 1024);
    c.gemm_pairs = 0;
    if (cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             sizeof(gp::PairSmem) + 1024) != cudaSuccess)
        return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (c.sms / 2));
    cfg.blockDim = dim3(gp::PTHREADS);
    cfg.dynamicSmemBytes = sizeof(gp::PairSmem) + 1024;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg) == cudaSuccess) c.gemm_pairs = n;
}

}  // namespace mmz
