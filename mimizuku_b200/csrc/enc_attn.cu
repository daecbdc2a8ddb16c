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
//   warps 2-9   softmax: query row i of the tile (TMEM lane i) is shared by two threads, one per half of the 128
//               keys of a tile (warps 2-5: keys 0-63, warps 6-9: keys 64-127). Each loads its 64 scores from TMEM
//               into registers (which frees S for the next QK product at once), exchanges its row maximum with its
//               partner through shared memory, keeps its share of the row sum, writes its 64 probabilities (fp16)
//               into TMEM for the P.V product and rescales its 32 columns of the O row when the maximum moves
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
    float xmax[2][2][BM];                    // [tile parity][key half][row]: the partners' row maxima, then sums
    uint64_t bar_q, bar_kf[KST], bar_ke[KST], bar_vf[VST], bar_ve[VST];
    uint64_t bar_sf, bar_sfree, bar_pf, bar_od, bar_fin;
    uint64_t bar_x[4];                       // per lane quarter: the two threads of a row have exchanged a value
    uint32_t tmem;
    int abort;
};

}  // namespace enc

using namespace enc;

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// grid (12 query tiles, heads, clips), block 384, dynamic shared memory sizeof(Smem)
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
        for (int i = 0; i < 4; i++) mbar_init(&s.bar_x[i], 2);  // the two warps of a lane quarter
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
            const uint32_t qa = smem_u32(s.q);
            bool ok = mbar_wait_spin(&s.bar_q, 0, abort, limit_ns, status, K_ENC, 20) &&
                      mbar_wait_spin(&s.bar_kf[0], 0, abort, limit_ns, status, K_ENC, 21);
            if (ok) {
                tc_fence_after();
                const uint32_t ka = smem_u32(s.k[0]);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++)
                    umma_f16_ss(tS, sdesc_sw128(qa + kk * 32, 16, SBO), sdesc_sw128(ka + kk * 32, 16, SBO), IDESC_QK,
                                kk > 0);
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
                    const uint32_t ka = smem_u32(s.k[st1]);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; kk++)
                        umma_f16_ss(tS, sdesc_sw128(qa + kk * 32, 16, SBO), sdesc_sw128(ka + kk * 32, 16, SBO),
                                    IDESC_QK, kk > 0);
                    umma_commit(&s.bar_sf);
                    umma_commit(&s.bar_ke[st1]);
                }
                const int sv = j % VST;
                ok = mbar_wait_spin(&s.bar_pf, j & 1, abort, limit_ns, status, K_ENC, 24) &&
                     mbar_wait_spin(&s.bar_vf[sv], (j / VST) & 1, abort, limit_ns, status, K_ENC, 25);
                if (!ok) break;
                tc_fence_after();
                const uint32_t va = smem_u32(s.v[sv]);
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++)
                    umma_f16_ts(tO, tP + kk * 8, sdesc_sw128(va + kk * 16 * 128, TILE, SBO), IDESC_PV,
                                (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&s.bar_od);
                umma_commit(&s.bar_ve[sv]);
            }
            umma_commit(&s.bar_fin);  // completes once every MMA issued above has finished
        }
    } else {
        // ---------------------------------------------------------------- softmax (warps 2..9, two threads per row)
        const int quarter = warp & 3;        // a warp may only touch TMEM lanes 32 * (warp % 4) .. + 31
        const int hf = (warp - 2) >> 2;      // key half of the tile
        const int row = quarter * 32 + lane;
        const uint32_t loff = (uint32_t)(quarter * 32) << 16;
        const uint32_t tSh = tS + loff + hf * 64, tPh = tP + loff + hf * 32, tOh = tO + loff + hf * 32;
        const float sl2 = 0.125f * 1.4426950408889634f;  // 0.125 * log2(e)
        const float2 sl2_2 = make_float2(sl2, sl2);
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < NKT; j++) {
            const bool last = j == NKT - 1 && hf == 1;  // keys 92.. of the last tile are past 1500
            ok = __all_sync(0xffffffff, mbar_wait_spin(&s.bar_sf, j & 1, abort, limit_ns, status, K_ENC, 30));
            if (!ok) break;
            tc_fence_after();
            uint32_t raw[64];
            tmem_ld64(tSh, raw);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.bar_sfree);  // the warp's scores are in registers: the next QK may start
            float* sv = reinterpret_cast<float*>(raw);
            if (last) {
#pragma unroll
                for (int c = LAST_VALID - 64; c < 64; c++) sv[c] = -INFINITY;
            }
            // the maximum of this thread's 64 scores, four chains
            float a0 = fmaxf(sv[0], sv[1]), a1 = fmaxf(sv[2], sv[3]), a2 = fmaxf(sv[4], sv[5]), a3 = fmaxf(sv[6], sv[7]);
#pragma unroll
            for (int c = 8; c < 64; c += 8) {
                a0 = fmax3(a0, sv[c], sv[c + 1]);
                a1 = fmax3(a1, sv[c + 2], sv[c + 3]);
                a2 = fmax3(a2, sv[c + 4], sv[c + 5]);
                a3 = fmax3(a3, sv[c + 6], sv[c + 7]);
            }
            float tmax = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
            // exchange with the partner thread of this row (the other key half)
            s.xmax[j & 1][hf][row] = tmax;
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.bar_x[quarter]);
            ok = __all_sync(0xffffffff, mbar_wait_spin(&s.bar_x[quarter], j & 1, abort, limit_ns, status, K_ENC, 33));
            if (!ok) break;
            tmax = fmaxf(tmax, s.xmax[j & 1][hf ^ 1][row]) * sl2;
            // the running maximum only moves when the tile's exceeds it by more than 8 (log2 units): the
            // probabilities then stay below 2^8 (exact in fp16), and the O row is rescaled far less often
            const float mn = tmax > m + 8.f ? tmax : m;
            const float corr = mn == m ? 1.f : ex2_approx(m - mn);
            m = mn;
            const float2 nmn2 = make_float2(-mn, -mn);
            float2 rs2 = make_float2(0.f, 0.f), rs2b = make_float2(0.f, 0.f);
            // exponentials (a quarter of the pairs on the FMA pipe), P into TMEM in two halves
#pragma unroll
            for (int h2 = 0; h2 < 2; h2++) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const int cc = h2 * 16 + c;
                    const float2 x = ffma2(make_float2(sv[2 * cc], sv[2 * cc + 1]), sl2_2, nmn2);
                    float2 e;
                    if ((POLY_PAIRS >> c) & 1) {
                        e = exp2_poly2(x);
                    } else {
                        e.x = ex2_approx(x.x);
                        e.y = ex2_approx(x.y);
                    }
                    if (c & 1) rs2b = fadd2(rs2b, e);
                    else rs2 = fadd2(rs2, e);
                    pk[c] = pack_h2(e.x, e.y);
                }
                if (h2 == 0 && j > 0) {
                    // P.V of the previous tile must be complete: it reads the P columns and accumulates into O
                    ok = __all_sync(0xffffffff, mbar_wait_spin(&s.bar_od, (j - 1) & 1, abort, limit_ns, status, K_ENC, 31));
                    if (!ok) break;
                    tc_fence_after();
                }
                tmem_st16(tPh + h2 * 16, pk);
            }
            if (!ok) break;
            l = l * corr + ((rs2.x + rs2.y) + (rs2b.x + rs2b.y));
            // the running max moved: rescale this thread's 32 columns of the O row before the next P.V
            if (j > 0 && __any_sync(0xffffffff, corr != 1.f)) {
                uint32_t r[32];
                tmem_ld32(tOh, r);
#pragma unroll
                for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
                tmem_st32(tOh, r);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.bar_pf);
        }
        if (ok) ok = __all_sync(0xffffffff, mbar_wait_spin(&s.bar_od, (NKT - 1) & 1, abort, limit_ns, status, K_ENC, 32));
        if (ok) {
            // the row sum is the two halves' shares
            s.xmax[NKT & 1][hf][row] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.bar_x[quarter]);
            ok = __all_sync(0xffffffff, mbar_wait_spin(&s.bar_x[quarter], NKT & 1, abort, limit_ns, status, K_ENC, 34));
        }
        if (ok) {
            const float lt = l + s.xmax[NKT & 1][hf ^ 1][row];
            tc_fence_after();
            const int qrow = qt * BM + row;
            uint32_t r[32];
            tmem_ld32(tOh, r);
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 16; i++) o[i] = pack_h2(__uint_as_float(r[2 * i]) / lt, __uint_as_float(r[2 * i + 1]) / lt);
            if (qrow < TENC) {
                uint4* dst = reinterpret_cast<uint4*>(out + ((long)g * TENC + qrow) * d + hh * HD + hf * 32);
#pragma unroll
                for (int i = 0; i < 4; i++) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
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
    if (make_tmap_3d(&map, qkv, dims, strides, box, true)) return fail("enc_flash: cuTensorMapEncodeTiled failed");
    dim3 grid(NQT, d / HD, groups);
    return check_pdl(launch_pdl(enc_flash_kernel, grid, dim3(NTHREADS), sizeof(Smem), st, map, (h16*)out, d, dc.status,
                                dc.limit_ns),
                     "enc_flash");
}

void init_enc_attn_attrs() {
    cudaFuncSetAttribute(enc_flash_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem));
}

}  // namespace mmz
