// The decoder step's logits fused with the greedy token choice, for sm_100a: for the m <= 32 sequences of the batch,
// logits = rh(x . emb^T) over the vocabulary (src/model.rs:714-716, the cuBLAS product onto a [b][V] buffer), then
// argmax_tok's choice of token p + 1 (kernels/whisper.cu:451-493) and, optionally, advance (:495) - without writing
// the [b][V] logits to memory (they may still be written, for inspection).
//
// The product streams the 51866 x 1280 embedding (133 MB) once: a persistent CTA per SM takes every gridDim-th tile of
// 128 vocabulary rows; its 4 warps of epilogue turn a finished tile into per-sequence candidates while the MMA warp
// already accumulates the next tile into the other half of its TMEM:
//   warp 4      TMA producer: the embedding tiles (64-wide K chunks, 128-byte swizzle) through an 8-stage ring, the
//               first stages issued before the wait for the kernel before (the embedding does not depend on it); x
//               (32 x K, rows past m zero-filled) once into shared memory after that wait
//   warp 5      MMA issuer: D[128 vocab rows][32 sequences] (M128 N32 K16, A = embedding tile, B = x) into one of two
//               TMEM accumulators, descriptors formed once and advanced by constants
//   warps 0-3   epilogue: thread = vocabulary row; its 32 fp32 sums are rounded to fp16 (the values argmax_tok reads
//               from the logits buffer), each kept sequence's value packed with its id into a 64-bit key (value order
//               above, lower id below: the largest key is argmax_tok's choice, ties to the lower id); a transpose
//               butterfly over the warp leaves lane b the warp's best key of sequence b; the four warps' bests meet in
//               shared memory and one 64-bit atomicMax per sequence and tile goes to the scratch word of sequence b.
// The last CTA to finish (a counter in the scratch) writes the chosen tokens and done flags exactly as argmax_tok does,
// advances ctr[0] if asked, and leaves the scratch zeroed for the next launch.
//
// The MMA order per tile (K chunks in order, four K16 products each, one accumulator) is that of this library's
// dec_linear kernel when it does not split K (every Whisper vocabulary: more than 128 x SM-count rows), so there the
// logits and therefore the tokens equal those of dec_linear followed by argmax_tok.
// Every wait is bounded; a CTA that gives up still counts itself in, so that the scratch is reset.
#include "common.cuh"
#include "launch.h"

namespace mmz {
namespace lga {

constexpr int BN = 128;                // vocabulary rows per tile (MMA M)
constexpr int BM = 32;                 // sequences (MMA N)
constexpr int BK = 64;                 // K per chunk (one 128-byte swizzle atom)
constexpr int NS = 8;                  // embedding ring stages
constexpr int KMAX = 1280;             // x stays in shared memory: K <= 1280 (every Whisper width)
constexpr int NCHMAX = KMAX / BK;
constexpr int WT = BN * BK * 2;        // 16 KB
constexpr int XT = BM * BK * 2;        // 4 KB
constexpr int NTHREADS = 192;          // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int TMA_WARP = 4, MMA_WARP = 5;
constexpr uint32_t IDESC = idesc_f16_f32(BN, BM, false);

struct Smem {
    uint8_t w[NS][WT];
    uint8_t x[NCHMAX][XT];
    unsigned long long red[2][4][BM];  // the epilogue warps' best keys per sequence (two tiles in flight)
    uint64_t full[NS], empty[NS], xfull, accf[2], acce[2], fin;
    uint32_t tmem;
    int abort, skip, p;
};

// argmax_tok's order as one unsigned comparison: the fp32 value of the fp16 logit in the high word (monotone map, -0
// equal to +0), 0xffffffff - id in the low word (equal values: the lower id is larger). 0 means no candidate; a NaN is
// never a candidate (argmax_tok's comparisons are false for it).
__device__ __forceinline__ unsigned long long arg_key(float v, int id) {
    if (v != v) return 0ull;
    if (v == 0.f) v = 0.f;
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xffffffffu - (uint32_t)id);
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) { return a > b ? a : b; }

}  // namespace lga

using namespace lga;

// scratch: best[32] (64-bit keys) and the CTA counter; zero before the first launch, zero again after every launch
struct LgaScratch {
    unsigned long long best[BM];
    unsigned int count;
};

// grid min(SMs, tiles), block NTHREADS, dynamic shared memory sizeof(Smem) + 1024 (alignment slack)
__global__ void __launch_bounds__(NTHREADS, 1)
    logits_argmax_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, int V,
                         int k, int m, const unsigned char* __restrict__ sup, int* tok, int* done, int* ctr, int maxT,
                         int prompt_len, int eos, int bs1, int bs2, h16* __restrict__ logits, int advance,
                         LgaScratch* scr, unsigned* status, unsigned long long limit_ns) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    Smem& s = *reinterpret_cast<Smem*>(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int tiles = (V + BN - 1) / BN, nch = k / BK;
    const int my_tiles = cta < tiles ? (tiles - cta + G - 1) / G : 0;
    const int nq = my_tiles * nch;  // embedding chunks this CTA streams
    volatile int* abort = &s.abort;
    int issued = 0;
    auto issue_w = [&](int q) {
        const int st = q % NS, i = q / nch, c = q % nch;
        mbar_expect_tx(&s.full[st], WT);
        tma_load_2d(s.w[st], &wmap, c * BK, (cta + i * G) * BN, &s.full[st]);
    };
    if (warp == TMA_WARP && lane == 0) {
        s.abort = 0;
        for (int i = 0; i < NS; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.xfull, 1);
        for (int a = 0; a < 2; a++) {
            mbar_init(&s.accf[a], 1);
            mbar_init(&s.acce[a], 4);  // one arrival per epilogue warp
        }
        mbar_init(&s.fin, 1);
        fence_mbar_init();
        prefetch_tmap(&wmap);
        prefetch_tmap(&xmap);
        // the embedding does not depend on the kernel before: its first stages go out before the dependency wait
        for (; issued < NS && issued < nq; issued++) issue_w(issued);
    }
    if (warp == MMA_WARP) {
        tmem_alloc(&s.tmem, 64);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_wait();  // x, tok, done and ctr come from earlier kernels
    if (threadIdx.x == 0) {
        const int p = ctr[0];
        s.p = p;
        s.skip = (p + 1 < prompt_len || p + 1 >= maxT) ? 1 : 0;  // argmax_tok chooses nothing at this position
    }
    __syncthreads();
    const uint32_t tacc = s.tmem;
    const int p = s.p;
    const bool skip = s.skip != 0;

    if (warp == TMA_WARP) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            if (!skip) {
                mbar_expect_tx(&s.xfull, nch * XT);
                for (int c = 0; c < nch; c++) tma_load_2d(s.x[c], &xmap, c * BK, 0, &s.xfull);
                for (int q = issued; q < nq; q++) {
                    const int st = q % NS;
                    if (!mbar_wait(&s.empty[st], ((q / NS) - 1) & 1, abort, limit_ns, status, K_LOGITS, 1)) break;
                    issue_w(q);
                    issued = q + 1;
                }
            }
            if (skip || *abort) {  // let every issued copy land before the shared memory is released
                for (int q = issued > NS ? issued - NS : 0; q < issued; q++)
                    mbar_wait(&s.full[q % NS], (q / NS) & 1, nullptr, limit_ns, nullptr, 0, 0);
                if (!skip) mbar_wait(&s.xfull, 0, nullptr, limit_ns, nullptr, 0, 0);
            }
        }
    } else if (warp == MMA_WARP) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && !skip) {
            const uint64_t wd0 = sdesc_sw128(smem_u32(s.w[0]), 16, 1024);
            const uint64_t xd0 = sdesc_sw128(smem_u32(s.x[0]), 16, 1024);
            constexpr uint64_t WSTAGE = WT >> 4, XSTAGE = XT >> 4, KSTEP = 32 >> 4;
            bool ok = mbar_wait_spin(&s.xfull, 0, abort, limit_ns, status, K_LOGITS, 2);
            for (int i = 0; ok && i < my_tiles; i++) {
                const int a = i & 1;
                if (i >= 2 && !mbar_wait_spin(&s.acce[a], ((i >> 1) - 1) & 1, abort, limit_ns, status, K_LOGITS, 3)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int c = 0; c < nch; c++) {
                    const int q = i * nch + c, st = q % NS;
                    if (!mbar_wait_spin(&s.full[st], (q / NS) & 1, abort, limit_ns, status, K_LOGITS, 4)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t wd = wd0 + st * WSTAGE, xd = xd0 + c * XSTAGE;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        umma_f16_ss(tacc + 32 * a, wd + kk * KSTEP, xd + kk * KSTEP, IDESC, (c > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&s.empty[st]);
                }
                if (!ok) break;
                umma_commit(&s.accf[a]);
            }
        }
        if (lane == 0) umma_commit(&s.fin);  // completes once every MMA issued above has finished
    } else if (!skip) {
        // ---------------------------------------------------------------- epilogue (warps 0-3)
        const bool first = p + 1 == prompt_len;
        const uint32_t tl = tacc + ((uint32_t)(warp * 32) << 16);
        // every warp reaches the named barrier of every tile, also after a wait gave up (with no candidates), so
        // that none is left waiting there
        for (int i = 0; i < my_tiles; i++) {
            const int a = i & 1;
            const bool okw =
                __all_sync(0xffffffff, mbar_wait_spin(&s.accf[a], (i >> 1) & 1, abort, limit_ns, status, K_LOGITS, 5));
            unsigned long long key[32];
            if (okw) {
                tc_fence_after();
                uint32_t acc[32];
                tmem_ld32(tl + 32 * a, acc);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.acce[a]);  // the accumulator may take the tile after next
                const int id = (cta + i * G) * BN + warp * 32 + lane;
                const bool cand = id < V && !sup[id] && !(first && (id == bs1 || id == bs2));
#pragma unroll
                for (int b = 0; b < 32; b++) {
                    const h16 hv = h(__uint_as_float(acc[b]));
                    key[b] = (cand && b < m) ? arg_key(f(hv), id) : 0ull;
                    if (logits && b < m && id < V) logits[(long)b * V + id] = hv;
                }
            } else {
#pragma unroll
                for (int b = 0; b < 32; b++) key[b] = 0ull;
            }
            // transpose butterfly: after the step of width w a lane keeps the sequences whose index has the lane's
            // bit w, so at the end lane b holds the warp's best key of sequence b
#pragma unroll
            for (int w = 16; w >= 1; w >>= 1) {
                const bool up = (lane & w) != 0;
#pragma unroll
                for (int j = 0; j < w; j++) {
                    const unsigned long long send = up ? key[j] : key[j + w];
                    const unsigned long long keep = up ? key[j + w] : key[j];
                    key[j] = umax64(keep, __shfl_xor_sync(0xffffffff, send, w));
                }
            }
            s.red[a][warp][lane] = key[0];
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
            if (warp == 0) {
                const unsigned long long best =
                    umax64(umax64(s.red[a][0][lane], s.red[a][1][lane]), umax64(s.red[a][2][lane], s.red[a][3][lane]));
                if (lane < m && best != 0ull) atomicMax(&scr->best[lane], best);
            }
        }
    }
    __syncthreads();
    // the CTA counts itself in; the last one chooses the tokens and resets the scratch
    if (warp == 0) {
        unsigned last = 0;
        if (lane == 0) {
            __threadfence();
            last = atomicAdd(&scr->count, 1u) == (unsigned)(G - 1) ? 1u : 0u;
            __threadfence();
        }
        last = __shfl_sync(0xffffffff, last, 0);
        if (last) {
            const unsigned long long best = atomicExch(&scr->best[lane], 0ull);
            if (!skip && lane < m) {
                const int t = (done[lane] || best == 0ull) ? eos : (int)(0xffffffffu - (uint32_t)best);
                tok[lane * maxT + p + 1] = t;
                if (t == eos) done[lane] = 1;
            }
            __syncwarp();
            if (lane == 0) {
                atomicExch(&scr->count, 0u);
                if (advance) ctr[0] = p + 1;
            }
        }
    }
    // teardown: the MMA pipe must drain before the MMA warp releases TMEM
    if (warp == MMA_WARP) {
        mbar_wait(&s.fin, 0, nullptr, limit_ns, status, K_LOGITS, 6);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tacc, 64);
    }
}

size_t logits_argmax_scratch_bytes() { return (sizeof(LgaScratch) + 15) & ~(size_t)15; }

int launch_logits_argmax(const void* x, int ldx, const void* emb, int V, int k, int m, const unsigned char* sup,
                         int* tok, int* done, int* ctr, int maxT, int prompt_len, int eos, int bs1, int bs2,
                         void* logits, bool advance, void* scratch, size_t scratch_bytes, cudaStream_t st) {
    if (m < 1 || m > BM || V < 1 || k < BK || k > KMAX || k % BK)
        return fail("logits_argmax: 1 <= m <= 32, k a multiple of 64 up to 1280");
    if (((uintptr_t)x & 15) || ((uintptr_t)emb & 15) || ((ldx * 2) & 15) || ldx < k)
        return fail("logits_argmax: x and emb 16-byte aligned, ldx >= k with a 16-byte row pitch");
    if (!scratch || ((uintptr_t)scratch & 15) || scratch_bytes < logits_argmax_scratch_bytes())
        return fail("logits_argmax: scratch too small or not 16-byte aligned");
    if (!sup || !tok || !done || !ctr) return fail("logits_argmax: null pointer");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    CUtensorMap wm, xm;
    const uint64_t wd[2] = {(uint64_t)k, (uint64_t)V}, ws[1] = {(uint64_t)k * 2};
    const uint32_t wb[2] = {BK, BN};
    const uint64_t xd[2] = {(uint64_t)k, (uint64_t)m}, xs[1] = {(uint64_t)ldx * 2};
    const uint32_t xb[2] = {BK, BM};
    if (make_tmap_2d(&wm, emb, wd, ws, wb, 128) || make_tmap_2d(&xm, x, xd, xs, xb, 128))
        return fail("logits_argmax: cuTensorMapEncodeTiled failed");
    const int tiles = (V + BN - 1) / BN;
    const int grid = tiles < dc.sms ? tiles : dc.sms;
    return check_pdl(launch_pdl(logits_argmax_kernel, dim3(grid), dim3(NTHREADS), sizeof(Smem) + 1024, st, wm, xm, V,
                                k, m, sup, tok, done, ctr, maxT, prompt_len, eos, bs1, bs2, (h16*)logits,
                                advance ? 1 : 0, (LgaScratch*)scratch, dc.status, dc.limit_ns),
                     "logits_argmax");
}

void init_logits_argmax_attrs() {
    cudaFuncSetAttribute(logits_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(Smem) + 1024);
}

}  // namespace mmz
