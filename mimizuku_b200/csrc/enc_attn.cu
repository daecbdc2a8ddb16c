// Encoder self-attention for sm_100a: O = softmax(0.125 Q K^T) V per (clip, head) over the 1500 encoder positions,
// head size 64, fp16 in, fp32 accumulation (replaces enc_flash, kernels/whisper.cu:168-299 of the reference).
//
// One CTA computes a 128-query tile of one (clip, head) with the 5th-generation tensor cores, 10 warps:
//   warp 0      TMA producers: lane 0 copies Q once and the K tiles of 128 keys through a 3-stage ring, lane 1 the V
//               tiles through a 2-stage ring (128-byte swizzle, read straight out of the interleaved [clip][1500][3d]
//               qkv buffer with a 3-D tensor map that zero-fills the rows past 1500 of each clip); a stage is refilled
//               as soon as the product that read it is done
//   warp 1      MMA issuer (one thread): S = Q K^T (M128 N128 K64) into TMEM, then O += P V (M128 N64 K128) with P
//               read from TMEM and V as an MN-major shared-memory operand; completion is signalled with
//               tcgen05.commit
//   warps 2-9   softmax: a warp owns 16 query rows (TMEM lanes) and loads their scores with the 16x256b shape, so
//               thread t holds rows t / 4 and t / 4 + 8 of them, two keys of every 8-key block: the 4 threads of a
//               row are lanes of one warp and agree on its maximum through two shuffles. Each loads its 64 scores
//               from TMEM into registers (which frees S for the next QK product at once), keeps its share of the
//               two row sums, writes its 32 packed probabilities (fp16) into TMEM with the matching 16x128b shape
//               for the P.V product and rescales its columns of the two O rows when a maximum moves
// TMEM holds S (columns 0-127), O (128-191) and P (192-255): 256 columns, so two CTAs share an SM and the softmax
// warps of one overlap the MMAs and copies of the other (16 softmax warps per SM).
//
// Numerics follow the reference kernel: fp32 scores scaled by 0.125 after the product (:252), online softmax with
// the running maximum, P rounded to fp16 for P.V while the row sum uses the unrounded p (:269-277), O / l rounded to
// fp16 (:297). exp is taken as 2^(s * 0.125 * log2 e - m) (ex2.approx, a quarter of them by a polynomial on the FMA
// pipe); key tiles are 128 wide instead of 64, so P's rounding points differ from the reference's by the choice of
// running maximum only.
//
// Every mbarrier wait is bounded; a CTA that times out reports into the status word, lets its copies land, waits
// for its MMAs, frees its TMEM and exits.
#include "common.cuh"
#include "launch.h"

namespace mmz {
namespace enc {

constexpr int BM = 128;                      // queries per CTA
constexpr int BN = 128;                      // keys per tile
constexpr int NKT = (TENC + BN - 1) / BN;    // 12 key tiles (the last holds 92 keys)
constexpr int NQT = (TENC + BM - 1) / BM;    // 12 query tiles
constexpr int LAST_VALID = TENC - (NKT - 1) * BN;  // 92 keys in the last tile
static_assert(LAST_VALID > 64, "the first key half of the last tile is whole");
constexpr unsigned POLY_PAIRS = 0x8888u;      // pairs c (of 16) whose exponentials run on the FMA pipe: c % 4 == 3
constexpr int KST = 3;                       // K ring stages
constexpr int VST = 2;                       // V ring stages
constexpr int TILE = BN * HD * 2;            // 16384 bytes: 128 rows x 128 bytes
constexpr int TMEM_COLS = 256;
constexpr int NTHREADS = 320;
constexpr uint32_t IDESC_QK = idesc_f16_f32(128, 128, false);
constexpr uint32_t IDESC_PV = idesc_f16_f32(128, 64, true);
constexpr uint32_t SBO = 1024;               // 8 rows x 128 bytes

struct Smem {
    uint8_t q[TILE];
    uint8_t k[KST][TILE];
    uint8_t v[VST][TILE];
    uint64_t bar_q, bar_kf[KST], bar_ke[KST], bar_vf[VST], bar_ve[VST];
    uint64_t bar_sf, bar_sfree, bar_pf, bar_od, bar_fin;
    uint32_t tmem;
    int abort;
};

}  // namespace enc

using namespace enc;

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// grid (12 query tiles, heads, clips), block NTHREADS (320), dynamic shared memory sizeof(Smem)
__global__ void __launch_bounds__(NTHREADS, 2)
    enc_flash_kernel(const __grid_constant__ CUtensorMap qkv_map, h16* __restrict__ out, int d, unsigned* status,
                     unsigned long long limit_ns) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    const int qt = blockIdx.x, hh = blockIdx.y, g = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (smem_u32(smem_raw) & 1023) {  // the swizzled tiles need a 1024-byte aligned base
        if (threadIdx.x == 0) report(status, ST_MISALIGNED, K_ENC, 0);
        return;
    }
    volatile int* abort = &s.abort;
    griddep_wait();  // launched as a programmatic dependent of the qkv projection
    if (threadIdx.x == 0) {
        s.abort = 0;
        mbar_init(&s.bar_q, 1);
        for (int i = 0; i < KST; i++) {
            mbar_init(&s.bar_kf[i], 1);
            mbar_init(&s.bar_ke[i], 1);
        }
        for (int i = 0; i < VST; i++) {
            mbar_init(&s.bar_vf[i], 1);
            mbar_init(&s.bar_ve[i], 1);
        }
        mbar_init(&s.bar_sf, 1);
        mbar_init(&s.bar_sfree, 8);  // one arrival per softmax warp
        mbar_init(&s.bar_pf, 8);
        mbar_init(&s.bar_od, 1);
        mbar_init(&s.bar_fin, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&s.tmem, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = s.tmem;
    const uint32_t tS = tbase, tO = tbase + 128, tP = tbase + 192;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producers: lane 0 Q and K, lane 1 V
        // (two queues, so a K tile is fetched as soon as its stage is free of the QK product that read it, without
        // waiting behind V)
        if (lane < 2) {
            if (lane == 0) {
                prefetch_tmap(&qkv_map);
                mbar_expect_tx(&s.bar_q, TILE);
                tma_load_3d(s.q, &qkv_map, hh * HD, qt * BM, g, &s.bar_q);
            }
            const int nst = lane == 0 ? KST : VST;
            uint64_t* full = lane == 0 ? s.bar_kf : s.bar_vf;
            uint64_t* empty = lane == 0 ? s.bar_ke : s.bar_ve;
            uint8_t* dst = lane == 0 ? &s.k[0][0] : &s.v[0][0];
            const int col = (lane == 0 ? d : 2 * d) + hh * HD;
            int issued = 0;
            for (int j = 0; j < NKT; j++) {
                const int st = j % nst, n = j / nst;
                if (n > 0 && !mbar_wait(&empty[st], (n - 1) & 1, abort, limit_ns, status, K_ENC, 10 + lane)) break;
                mbar_expect_tx(&full[st], TILE);
                tma_load_3d(dst + st * TILE, &qkv_map, col, j * BN, g, &full[st]);
                issued = j + 1;
            }
            if (*abort) {  // let every issued copy land before the shared memory is released
                if (lane == 0) mbar_wait(&s.bar_q, 0, nullptr, limit_ns, nullptr, 0, 0);
                for (int j = issued > nst ? issued - nst : 0; j < issued; j++)
                    mbar_wait(&full[j % nst], (j / nst) & 1, nullptr, limit_ns, nullptr, 0, 0);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            // Shared-memory descriptors are formed once; a K step, a ring stage or a V row block only advances the
            // start-address field (16-byte units; every address of the CTA's shared memory fits its 14 bits). This
            // keeps each MMA's issue to a few instructions: recomputing the descriptor per MMA cost the issuing
            // thread ~50 cycles of dependent integer work per MMA.
            const uint64_t qd = sdesc_sw128(smem_u32(s.q), 16, SBO);
            const uint64_t kd0 = sdesc_sw128(smem_u32(s.k[0]), 16, SBO);
            const uint64_t vd0 = sdesc_sw128(smem_u32(s.v[0]), TILE, SBO);
            constexpr uint64_t STAGE = TILE >> 4, KSTEP = 32 >> 4, VSTEP = (16 * 128) >> 4;
            bool ok = mbar_wait_spin(&s.bar_q, 0, abort, limit_ns, status, K_ENC, 20) &&
                      mbar_wait_spin(&s.bar_kf[0], 0, abort, limit_ns, status, K_ENC, 21);
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++)
                    umma_f16_ss(tS, qd + kk * KSTEP, kd0 + kk * KSTEP, IDESC_QK, kk > 0);
                umma_commit(&s.bar_sf);
                umma_commit(&s.bar_ke[0]);
            }
            for (int j = 0; ok && j < NKT; j++) {
                if (j + 1 < NKT) {
                    const int st1 = (j + 1) % KST;
                    ok = mbar_wait_spin(&s.bar_sfree, j & 1, abort, limit_ns, status, K_ENC, 22) &&
                         mbar_wait_spin(&s.bar_kf[st1], ((j + 1) / KST) & 1, abort, limit_ns, status, K_ENC, 23);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t kd = kd0 + st1 * STAGE;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; kk++)
                        umma_f16_ss(tS, qd + kk * KSTEP, kd + kk * KSTEP, IDESC_QK, kk > 0);
                    umma_commit(&s.bar_sf);
                    umma_commit(&s.bar_ke[st1]);
                }
                const int sv = j % VST;
                ok = mbar_wait_spin(&s.bar_pf, j & 1, abort, limit_ns, status, K_ENC, 24) &&
                     mbar_wait_spin(&s.bar_vf[sv], (j / VST) & 1, abort, limit_ns, status, K_ENC, 25);
                if (!ok) break;
                tc_fence_after();
                const uint64_t vd = vd0 + sv * STAGE;
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++)
                    umma_f16_ts(tO, tP + kk * 8, vd + kk * VSTEP, IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&s.bar_od);
                umma_commit(&s.bar_ve[sv]);
            }
            umma_commit(&s.bar_fin);  // completes once every MMA issued above has finished
        }
    } else {
        // ---------------------------------------------------------------- softmax (warps 2..9)
        // A warp owns 16 query rows (TMEM lanes) of its lane quarter and reads them with the 16x256b shape: thread t
        // holds rows t / 4 and t / 4 + 8 of those 16, two columns of every 8-column block, so the 4 threads sharing a
        // row are lanes of one warp and meet through shuffles.
        const int quarter = warp & 3;        // a warp may only touch TMEM lanes 32 * (warp % 4) .. + 31
        const int sub16 = (warp - 2) >> 2;   // which 16 lanes of the quarter
        const int q4 = lane & 3, rl = lane >> 2;
        const int row0 = quarter * 32 + sub16 * 16 + rl;  // and row0 + 8
        const uint32_t tl = tbase + ((uint32_t)(quarter * 32 + sub16 * 16) << 16);
        const float sl2 = 0.125f * 1.4426950408889634f;  // 0.125 * log2(e)
        const float2 sl2_2 = make_float2(sl2, sl2);
        float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
        bool ok = true;
        for (int j = 0; j < NKT; j++) {
            ok = __all_sync(0xffffffff, mbar_wait_spin(&s.bar_sf, j & 1, abort, limit_ns, status, K_ENC, 30));
            if (!ok) break;
            tc_fence_after();
            uint32_t raw[64];  // block b: [4b, 4b + 1] row0, [4b + 2, 4b + 3] row0 + 8, keys 8b + 2 q4 + {0, 1}
            tmem_ld_16x256b_x16(tl + (tS - tbase), raw);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.bar_sfree);  // the warp's scores are in registers: the next QK may start
            float* sv = reinterpret_cast<float*>(raw);
            if (j == NKT - 1) {  // keys past 1500 (zero-filled K rows)
#pragma unroll
                for (int b = 0; b < 16; b++)
#pragma unroll
                    for (int e = 0; e < 2; e++)
                        if (8 * b + 2 * q4 + e >= LAST_VALID) sv[4 * b + e] = sv[4 * b + 2 + e] = -INFINITY;
            }
            // the row maxima: this thread's 32 scores of each row, then the row's 4 threads
            float mx[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float a0 = fmaxf(sv[2 * h], sv[2 * h + 1]), a1 = fmaxf(sv[4 + 2 * h], sv[5 + 2 * h]);
#pragma unroll
                for (int b = 2; b < 16; b += 2) {
                    a0 = fmax3(a0, sv[4 * b + 2 * h], sv[4 * b + 2 * h + 1]);
                    a1 = fmax3(a1, sv[4 * b + 4 + 2 * h], sv[4 * b + 5 + 2 * h]);
                }
                mx[h] = fmaxf(a0, a1);
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2)) * sl2;
            }
            // the running maximum only moves when the tile's exceeds it by more than 8 (log2 units): the
            // probabilities then stay below 2^8 (exact in fp16), and the O row is rescaled far less often
            float corr[2];
            float2 nmn2[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float mn = mx[h] > m[h] + 8.f ? mx[h] : m[h];
                corr[h] = mn == m[h] ? 1.f : ex2_approx(m[h] - mn);
                m[h] = mn;
                nmn2[h] = make_float2(-mn, -mn);
            }
            // exponentials (a quarter of the blocks on the FMA pipe), packed P in the 16x128b mapping: register 2b
            // row0, 2b + 1 row0 + 8, column 4b + q4 = keys 8b + 2 q4, 8b + 2 q4 + 1; stored in two halves
            float2 rs[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {
                uint32_t pk[16];
#pragma unroll
                for (int bb = 0; bb < 8; bb++)
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int b = hb * 8 + bb;
                        const float2 x = ffma2(make_float2(sv[4 * b + 2 * h], sv[4 * b + 2 * h + 1]), sl2_2, nmn2[h]);
                        float2 e;
                        if ((b & 3) == 3) {
                            e = exp2_poly2(x);
                        } else {
                            e.x = ex2_approx(x.x);
                            e.y = ex2_approx(x.y);
                        }
                        rs[h] = fadd2(rs[h], e);
                        pk[2 * bb + h] = pack_h2(e.x, e.y);
                    }
                if (hb == 0 && j > 0) {
                    // P.V of the previous tile must be complete: it reads the P columns and accumulates into O
                    ok = __all_sync(0xffffffff,
                                    mbar_wait_spin(&s.bar_od, (j - 1) & 1, abort, limit_ns, status, K_ENC, 31));
                    if (!ok) break;
                    tc_fence_after();
                }
                tmem_st_16x128b_x8(tl + (tP - tbase) + hb * 32, pk);
            }
            if (!ok) break;
#pragma unroll
            for (int h = 0; h < 2; h++) l[h] = l[h] * corr[h] + (rs[h].x + rs[h].y);
            // the running max moved: rescale the two O rows before the next P.V
            if (j > 0 && __any_sync(0xffffffff, corr[0] != 1.f || corr[1] != 1.f)) {
                uint32_t r[32];
                tmem_ld_16x256b_x8(tl + (tO - tbase), r);
#pragma unroll
                for (int b = 0; b < 8; b++)
#pragma unroll
                    for (int e = 0; e < 4; e++) r[4 * b + e] = __float_as_uint(__uint_as_float(r[4 * b + e]) * corr[e >> 1]);
                tmem_st_16x256b_x8(tl + (tO - tbase), r);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.bar_pf);
        }
        if (ok) ok = __all_sync(0xffffffff, mbar_wait_spin(&s.bar_od, (NKT - 1) & 1, abort, limit_ns, status, K_ENC, 32));
        if (ok) {
            // the row sums are the row's 4 threads' shares
            float lt[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                lt[h] = l[h] + __shfl_xor_sync(0xffffffff, l[h], 1);
                lt[h] += __shfl_xor_sync(0xffffffff, lt[h], 2);
            }
            tc_fence_after();
            uint32_t r[32];
            tmem_ld_16x256b_x8(tl + (tO - tbase), r);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int qrow = qt * BM + row0 + 8 * h;
                if (qrow < TENC) {
                    uint32_t* dst = reinterpret_cast<uint32_t*>(out + ((long)g * TENC + qrow) * d + hh * HD + 2 * q4);
#pragma unroll
                    for (int b = 0; b < 8; b++)
                        dst[4 * b] = pack_h2(__uint_as_float(r[4 * b + 2 * h]) / lt[h],
                                             __uint_as_float(r[4 * b + 2 * h + 1]) / lt[h]);
                }
            }
        }
    }
    // teardown: every role is done with TMEM; the MMA pipe must drain before warp 0 releases it
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        mbar_wait(&s.bar_fin, 0, nullptr, limit_ns, status, K_ENC, 40);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

int launch_enc_flash(const void* qkv, void* out, int groups, int d, cudaStream_t st) {
    if (groups < 1 || d < HD || d % HD) return fail("enc_flash: d must be a multiple of 64 and groups >= 1");
    if (((uintptr_t)qkv & 15) || ((uintptr_t)out & 15)) return fail("enc_flash: qkv and out must be 16-byte aligned");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    CUtensorMap map;
    const uint64_t dims[3] = {(uint64_t)3 * d, (uint64_t)TENC, (uint64_t)groups};
    const uint64_t strides[2] = {(uint64_t)3 * d * 2, (uint64_t)TENC * 3 * d * 2};
    const uint32_t box[3] = {HD, BM, 1};
    if (make_tmap_3d(&map, qkv, dims, strides, box, 128)) return fail("enc_flash: cuTensorMapEncodeTiled failed");
    dim3 grid(NQT, d / HD, groups);
    return check_pdl(launch_pdl(enc_flash_kernel, grid, dim3(NTHREADS), sizeof(Smem), st, map, (h16*)out, d, dc.status,
                                dc.limit_ns),
                     "enc_flash");
}

void init_enc_attn_attrs() {
    cudaFuncSetAttribute(enc_flash_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem));
}

}  // namespace mmz
