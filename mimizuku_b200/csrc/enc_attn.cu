// Encoder self-attention for sm_100a: O = softmax(0.125 Q K^T) V per (clip, head) over the 1500 encoder positions,
// head size 64, fp16 in, fp32 accumulation (replaces enc_flash, kernels/whisper.cu:168-299 of the reference).
//
// One CTA computes a 128-query tile of one (clip, head) with the 5th-generation tensor cores:
//   warp 0      TMA producers: Q once, then K and V tiles of 128 keys through 2-stage rings (128-byte swizzle, read
//               straight out of the interleaved [clip][1500][3d] qkv buffer with a 3-D tensor map, which zero-fills
//               the rows past 1500 of each clip); a K stage is refilled as soon as its QK product is done
//   warp 1      MMA issuer (one thread): S = Q K^T (M128 N128 K64) into TMEM, then O += P V (M128 N64 K128) with P
//               from shared memory and V as an MN-major operand; completion is signalled with tcgen05.commit
//   warps 2-5   softmax: thread i owns query row i of the tile (TMEM lane i), reads its 128 scores from TMEM,
//               keeps the running max and sum, rescales its O row in TMEM when the max moves, and writes P (fp16) into
//               a K-major 128-byte-swizzled tile for the next MMA; at the end O / l -> fp16 -> global
// TMEM holds S (128 columns) and O (64 columns); 256 columns are allocated so two CTAs share an SM, and the softmax
// of one CTA overlaps the MMAs and copies of the other.
//
// Numerics follow the reference kernel: fp32 scores scaled by 0.125 after the product (:252), online softmax with
// the running maximum, P rounded to fp16 for P.V while the row sum uses the unrounded p (:269-277), O / l rounded to
// fp16 (:297). exp is taken as 2^(s * 0.125 * log2 e - m) (ex2.approx); key tiles are 128 wide instead of 64, so P's
// rounding points differ from the reference's by the choice of running maximum only.
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
constexpr int NSTAGE = 2;
constexpr int TILE = BN * HD * 2;            // 16384 bytes: 128 rows x 128 bytes
constexpr int TMEM_COLS = 256;
constexpr uint32_t IDESC_QK = idesc_f16_f32(128, 128, false);
constexpr uint32_t IDESC_PV = idesc_f16_f32(128, 64, true);
constexpr uint32_t SBO = 1024;               // 8 rows x 128 bytes

struct Smem {
    uint8_t q[TILE];
    uint8_t k[NSTAGE][TILE];
    uint8_t v[NSTAGE][TILE];
    uint8_t p[2][TILE];                      // P [128 rows][128 keys] as two K-major atoms of 64 keys
    uint64_t bar_q, bar_kf[NSTAGE], bar_vf[NSTAGE], bar_ke[NSTAGE], bar_ve[NSTAGE];
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

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// grid (12 query tiles, heads, clips), block 192, dynamic shared memory sizeof(Smem)
__global__ void __launch_bounds__(192, 2)
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
    if (threadIdx.x == 0) {
        s.abort = 0;
        mbar_init(&s.bar_q, 1);
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&s.bar_kf[i], 1);
            mbar_init(&s.bar_vf[i], 1);
            mbar_init(&s.bar_ke[i], 1);
            mbar_init(&s.bar_ve[i], 1);
        }
        mbar_init(&s.bar_sf, 1);
        mbar_init(&s.bar_sfree, 128);
        mbar_init(&s.bar_pf, 128);
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
    const uint32_t tS = tbase, tO = tbase + 128;

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
            uint64_t* full = lane == 0 ? s.bar_kf : s.bar_vf;
            uint64_t* empty = lane == 0 ? s.bar_ke : s.bar_ve;
            uint8_t(*dst)[TILE] = lane == 0 ? s.k : s.v;
            const int col = (lane == 0 ? d : 2 * d) + hh * HD;
            int issued = 0;
            for (int j = 0; j < NKT; j++) {
                const int st = j % NSTAGE, n = j / NSTAGE;
                if (n > 0 && !mbar_wait(&empty[st], (n - 1) & 1, abort, limit_ns, status, K_ENC, 10 + lane)) break;
                mbar_expect_tx(&full[st], TILE);
                tma_load_3d(dst[st], &qkv_map, col, j * BN, g, &full[st]);
                issued = j + 1;
            }
            if (*abort) {  // let every issued copy land before the shared memory is released
                if (lane == 0) mbar_wait(&s.bar_q, 0, nullptr, limit_ns, nullptr, 0, 0);
                for (int j = issued > NSTAGE ? issued - NSTAGE : 0; j < issued; j++)
                    mbar_wait(&full[j % NSTAGE], (j / NSTAGE) & 1, nullptr, limit_ns, nullptr, 0, 0);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t qa = smem_u32(s.q);
            bool ok = mbar_wait(&s.bar_q, 0, abort, limit_ns, status, K_ENC, 20) &&
                      mbar_wait(&s.bar_kf[0], 0, abort, limit_ns, status, K_ENC, 21);
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
                const int st = j % NSTAGE;
                if (j + 1 < NKT) {
                    const int st1 = (j + 1) % NSTAGE;
                    ok = mbar_wait(&s.bar_sfree, j & 1, abort, limit_ns, status, K_ENC, 22) &&
                         mbar_wait(&s.bar_kf[st1], ((j + 1) / NSTAGE) & 1, abort, limit_ns, status, K_ENC, 23);
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
                ok = mbar_wait(&s.bar_pf, j & 1, abort, limit_ns, status, K_ENC, 24) &&
                     mbar_wait(&s.bar_vf[st], (j / NSTAGE) & 1, abort, limit_ns, status, K_ENC, 25);
                if (!ok) break;
                tc_fence_after();
                const uint32_t va = smem_u32(s.v[st]);
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++) {
                    const uint32_t pa = smem_u32(s.p[kk >> 2]) + (kk & 3) * 32;
                    umma_f16_ss(tO, sdesc_sw128(pa, 16, SBO), sdesc_sw128(va + kk * 16 * 128, TILE, SBO), IDESC_PV,
                                (j > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&s.bar_od);
                umma_commit(&s.bar_ve[st]);
            }
            umma_commit(&s.bar_fin);  // completes once every MMA issued above has finished
        }
    } else {
        // ---------------------------------------------------------------- softmax (warps 2..5, thread = query row)
        const int quarter = warp & 3;  // a warp may only touch TMEM lanes 32 * (warp % 4) .. + 31
        const int row = quarter * 32 + lane;
        const uint32_t loff = (uint32_t)(quarter * 32) << 16;
        const float sl2 = 0.125f * 1.4426950408889634f;  // 0.125 * log2(e)
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        const uint32_t pbase = smem_u32(s.p[0]);
        for (int j = 0; j < NKT; j++) {
            ok = __all_sync(0xffffffff, mbar_wait(&s.bar_sf, j & 1, abort, limit_ns, status, K_ENC, 30));
            if (!ok) break;
            tc_fence_after();
            uint32_t raw[BN];
            tmem_ld128(tS + loff, raw);
            tc_fence_before();
            mbar_arrive(&s.bar_sfree);
            float* sv = reinterpret_cast<float*>(raw);
            if (j == NKT - 1) {  // keys past 1500 (zero-filled by the copy) take no weight
#pragma unroll
                for (int c = LAST_VALID; c < BN; c++) sv[c] = -INFINITY;
            }
            float tmax = fmaxf(sv[0], sv[1]);
#pragma unroll
            for (int c = 2; c < BN; c += 2) tmax = fmax3(tmax, sv[c], sv[c + 1]);
            const float mn = fmaxf(m, tmax * sl2);
            const float corr = ex2_approx(m - mn);
            m = mn;
            // exponentials of one pair of columns: a quarter of them on the FMA pipe (exp2_poly2), the rest on MUFU
            const float2 sl2_2 = make_float2(sl2, sl2), nmn2 = make_float2(-mn, -mn);
            float2 rs2 = make_float2(0.f, 0.f);
            auto pexp = [&](int c) -> uint32_t {
                const float2 x = ffma2(make_float2(sv[2 * c], sv[2 * c + 1]), sl2_2, nmn2);
                float2 e;
                if ((c & 3) == 3) {
                    e = exp2_poly2(x);
                } else {
                    e.x = ex2_approx(x.x);
                    e.y = ex2_approx(x.y);
                }
                rs2 = fadd2(rs2, e);
                return pack_h2(e.x, e.y);
            };
            // P row into the 128-byte swizzled K-major tile: 16-byte chunk c of a 128-byte row lands at c ^ (row % 8)
            auto pstore = [&](int c16, uint32_t a, uint32_t b, uint32_t c, uint32_t d4) {
                const uint32_t addr = pbase + (c16 >> 3) * TILE + row * 128 + (((c16 & 7) ^ (row & 7)) << 4);
                st_shared_v4(addr, a, b, c, d4);
            };
            // the first half of P is held in registers while the previous P.V may still read the P buffer
            uint32_t pk[BN / 4];
#pragma unroll
            for (int c = 0; c < BN / 4; c++) pk[c] = pexp(c);
            if (j > 0) {
                // P.V of the previous tile must be complete: it reads the P buffer and accumulates into O
                ok = __all_sync(0xffffffff, mbar_wait(&s.bar_od, (j - 1) & 1, abort, limit_ns, status, K_ENC, 31));
                if (!ok) break;
                tc_fence_after();
            }
#pragma unroll
            for (int c16 = 0; c16 < BN / 16; c16++) pstore(c16, pk[4 * c16], pk[4 * c16 + 1], pk[4 * c16 + 2], pk[4 * c16 + 3]);
            // the second half streams straight into the tile
#pragma unroll
            for (int c16 = BN / 16; c16 < BN / 8; c16++) {
                const uint32_t a = pexp(4 * c16), b = pexp(4 * c16 + 1), c = pexp(4 * c16 + 2), d4 = pexp(4 * c16 + 3);
                pstore(c16, a, b, c, d4);
            }
            l = l * corr + (rs2.x + rs2.y);
            // the running max moved: rescale this row of O before the next P.V accumulates into it
            if (j > 0 && __any_sync(0xffffffff, corr != 1.f)) {
#pragma unroll
                for (int c2 = 0; c2 < HD / 32; c2++) {
                    uint32_t r[32];
                    tmem_ld32(tO + loff + c2 * 32, r);
#pragma unroll
                    for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
                    tmem_st32(tO + loff + c2 * 32, r);
                }
                tmem_wait_st();
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&s.bar_pf);
        }
        if (ok) ok = __all_sync(0xffffffff, mbar_wait(&s.bar_od, (NKT - 1) & 1, abort, limit_ns, status, K_ENC, 32));
        if (ok) {
            tc_fence_after();
            const int qrow = qt * BM + row;
#pragma unroll
            for (int c2 = 0; c2 < HD / 32; c2++) {
                uint32_t r[32];
                tmem_ld32(tO + loff + c2 * 32, r);
                uint32_t o[16];
#pragma unroll
                for (int i = 0; i < 16; i++) o[i] = pack_h2(__uint_as_float(r[2 * i]) / l, __uint_as_float(r[2 * i + 1]) / l);
                if (qrow < TENC) {
                    uint4* dst = reinterpret_cast<uint4*>(out + ((long)g * TENC + qrow) * d + hh * HD + c2 * 32);
#pragma unroll
                    for (int i = 0; i < 4; i++) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
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
    if (make_tmap_3d(&map, qkv, dims, strides, box, true)) return fail("enc_flash: cuTensorMapEncodeTiled failed");
    dim3 grid(NQT, d / HD, groups);
    enc_flash_kernel<<<grid, 192, sizeof(Smem), st>>>(map, (h16*)out, d, dc.status, dc.limit_ns);
    return check_launch("enc_flash");
}

void init_enc_attn_attrs() {
    cudaFuncSetAttribute(enc_flash_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem));
}

}  // namespace mmz
