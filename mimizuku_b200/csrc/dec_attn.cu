// Decoder-step attention for sm_100a: causal self-attention over the KV cache (with the cache write of the current
// position folded in) and cross-attention over the 1500 encoder positions, which also records the alignment-head
// probabilities. Both are memory-bound:
//   self-attention   one CTA per (sequence, head) streams its K then V rows through an 8-deep ring of TMA tensor
//                    copies; one key per thread for the scores (the reference's warp butterfly restated as a tree),
//                    the reference's thread mapping for the softmax and P.V, so every sum runs in the reference's order
//   cross-attention  split-KV over 8 slices of 192 positions per (sequence, head), as two streaming kernels with
//                    every 16-byte load of a thread in flight at once and a small combine, chained by programmatic
//                    dependent launches
//
// Both read the position from device memory (ctr[0]) and skip finished sequences (done[b]), so one captured CUDA graph
// serves every decoding step, as the reference engine requires (kernels/whisper.cu:7-8).
//
// Rounding follows the reference kernels point for point: q * 0.125 -> fp16, scores -> fp16, probabilities -> fp16,
// outputs -> fp16 (kernels/whisper.cu:327, 335, 344, 352 for self-attention; 373, 388, 419, 440, 448 for
// cross-attention). The cross-attention reproduces the reference's association where that costs nothing: softmax
// statistics per 64-position chunk combined over the 24 chunks in order (kernels/whisper.cu:394-401, 414-417), P.V
// partials summed per chunk and then over chunks in order (:421-438, :447).
#include "common.cuh"
#include "launch.h"

namespace mmz {

// ============================================================================ cross-attention

constexpr int XCH = 64;                       // reference chunk (kernels/whisper.cu:360)
constexpr int XNCH = (TENC + XCH - 1) / XCH;  // 24 chunks
constexpr int XCPC = 3;                       // reference chunks per CTA (1: 66, 2: 51.1, 3: 49.3, 4: 51.0 us per layer)
constexpr int XCL = XNCH / XCPC;              // CTAs per (sequence, head)
constexpr int XPER = XCPC * XCH;              // positions per CTA
static_assert(XNCH % XCPC == 0 && XCPC <= 4, "whole chunks per CTA, one warp per chunk for the statistics");

// kv: [b][layer][k | v][head][1500][64] (kernels/whisper.cu:362-364)
__device__ __forceinline__ long xkv_off(int b, int layer, int kv, int hh, int nl, int nh) {
    return ((((long)b * nl + layer) * 2 + kv) * nh + hh) * (long)TENC * HD;
}

// ============================================================================ self-attention

constexpr int STILE = 32;   // cache rows per tensor copy
constexpr int SSTAGE = 8;   // copies in flight per CTA
constexpr int SMAXL = 512;  // longest context (max_t)

struct SelfSmem {
    h16 ring[SSTAGE][STILE * HD];  // 8 x 4 KB: K tiles (128-byte swizzle), then V tiles (plain), streamed through
    float q[HD];
    float sc[SMAXL];               // scores, then probabilities
    float wmax[4], wsum[4];        // per-warp partials of the block max and the block sum
    float red[HD];
    uint64_t full[SSTAGE];
    int abort;
    int nissued;                   // tiles issued so far (the highest index + 1)
};

__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
    return v;
}

// copies 64 halves (one head's slice of a row) with 8 threads, 16 bytes each
__device__ __forceinline__ void row_copy8(h16* dst, const h16* src, int t8) {
    reinterpret_cast<uint4*>(dst)[t8] = reinterpret_cast<const uint4*>(src)[t8];
}

// One key's score by one thread, bit for bit the reference's warp computation (kernels/whisper.cu:331-336): lane l's
// product q[2l] k[2l] + q[2l+1] k[2l+1] (contracted as fma(q[2l], k[2l], q[2l+1] k[2l+1])) and the xor-butterfly
// over 16, 8, 4, 2, 1, after which every lane holds the same sum, whose association is this tree:
// v1[i] = a[i] + a[i+16], v2[i] = v1[i] + v1[i+8], v3[i] = v2[i] + v2[i+4], (v3[0] + v3[2]) + (v3[1] + v3[3]).
// k: the key's 64 halves as eight 16-byte chunks (chunk c holds lanes 4c .. 4c + 3).
__device__ __forceinline__ float self_score(const float* __restrict__ q, const uint4 (&k)[8]) {
    float a[32];
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const __half2* h2 = reinterpret_cast<const __half2*>(&k[c]);
        const float4 qa = reinterpret_cast<const float4*>(q)[2 * c];
        const float4 qb = reinterpret_cast<const float4*>(q)[2 * c + 1];
        const float qq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float2 k2 = __half22float2(h2[e]);
            a[4 * c + e] = __fmaf_rn(qq[2 * e], k2.x, __fmul_rn(qq[2 * e + 1], k2.y));
        }
    }
    float v1[16], v2[8], v3[4];
#pragma unroll
    for (int i = 0; i < 16; i++) v1[i] = __fadd_rn(a[i], a[i + 16]);
#pragma unroll
    for (int i = 0; i < 8; i++) v2[i] = __fadd_rn(v1[i], v1[i + 8]);
#pragma unroll
    for (int i = 0; i < 4; i++) v3[i] = __fadd_rn(v2[i], v2[i + 4]);
    return __fadd_rn(__fadd_rn(v3[0], v3[2]), __fadd_rn(v3[1], v3[3]));
}

// grid (heads, B), block 128: one CTA per (sequence, head) (kernels/whisper.cu:321-353). The L = ctr[0] + 1 cached
// rows stream through an 8-deep ring of 32-row tensor copies (kmap: 128-byte swizzle, vmap: plain; 2-D maps over this
// layer's caches [B * maxT rows][d], box 64 x 32): the K tiles, then the V tiles.
//   scores   warp w takes the K tiles w, w + 4, ...: one key per lane, the whole 64-term product and the reference's
//            butterfly association in registers (self_score); the warp refills the stage it read by itself
//   softmax  the reference's block max and block sum (thread t sums the positions t, t + 128, ... in order)
//   P.V      thread (half, column) runs through the positions of its parity in order (:346-349), with each tile's
//            16 probabilities and values loaded before the chain of fused multiply-adds
// ctr[0], done and the cache rows before ctr[0] are read before the wait for the kernel before (they come from earlier
// decoding steps), so the first copies overlap that kernel's tail; row ctr[0] comes from qkv after the wait.
// 640 CTAs of 35 KB fit on the GPU at once, so the whole launch is one wave.
__global__ void __launch_bounds__(128)
    self_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                     const h16* __restrict__ qkv, h16* __restrict__ kc, h16* __restrict__ vc, h16* __restrict__ out,
                     const int* __restrict__ ctr, const int* __restrict__ done, int maxT, int d, unsigned* status,
                     unsigned long long limit_ns) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    SelfSmem& s = *reinterpret_cast<SelfSmem*>(smem_raw);
    const int hh = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    const int w = t >> 5, lane = t & 31;
    if (smem_u32(smem_raw) & 1023) {  // the swizzled K tiles need a 1024-byte aligned ring
        if (t == 0) report(status, ST_MISALIGNED, K_SELF, 0);
        return;
    }
    const int p = ctr[0], L = p + 1;
    const bool live = done[b] == 0;
    const int ntile = (L + STILE - 1) / STILE, total = 2 * ntile;
    auto issue = [&](int i) {  // tile i: K rows [32 i, 32 i + 32) for i < ntile, else V rows of tile i - ntile
        const int st = i % SSTAGE;
        const int row0 = b * maxT + (i < ntile ? i : i - ntile) * STILE;
        mbar_expect_tx(&s.full[st], STILE * HD * 2);
        tma_load_2d(s.ring[st], i < ntile ? &kmap : &vmap, hh * HD, row0, &s.full[st]);
        atomicMax(&s.nissued, i + 1);
    };
    if (t == 0 && live) {
        s.abort = 0;
        s.nissued = 0;
        for (int i = 0; i < SSTAGE; i++) mbar_init(&s.full[i], 1);
        fence_mbar_init();
        for (int i = 0; i < SSTAGE && i < total; i++) issue(i);
    }
    griddep_wait();  // launched as a programmatic dependent of the qkv projection
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    const long qrow = (long)b * 3 * d;
    const long crow = ((long)b * maxT + p) * d + hh * HD;
    if (t < 8) {  // the cache row of position p, for every sequence (kernels/whisper.cu:310-317)
        row_copy8(kc + crow, qkv + qrow + d + hh * HD, t);
        row_copy8(vc + crow, qkv + qrow + 2 * d + hh * HD, t);
    }
    if (!live) return;
    if (t < HD) s.q[t] = rh(f(qkv[qrow + hh * HD + t]) * 0.125f);  // :327
    __syncthreads();

    // ---------------------------------------------------------------- scores (:329-337)
    float kmax = -INFINITY;  // this lane's largest score (the block max is exact in any order)
    for (int i = w; i < ntile; i += 4) {
        const int st = i % SSTAGE;
        if (!__all_sync(0xffffffff, mbar_wait_spin(&s.full[st], (i / SSTAGE) & 1, &s.abort, limit_ns, status,
                                                    K_SELF, 1)))
            break;
        const int j = i * STILE + lane;
        if (j < L) {
            uint4 k[8];
            if (j == p) {  // the current position's key comes from qkv (its cache row is written above)
                const uint4* src = reinterpret_cast<const uint4*>(qkv + qrow + d + hh * HD);
#pragma unroll
                for (int c = 0; c < 8; c++) k[c] = src[c];
            } else {
                const unsigned char* row = reinterpret_cast<const unsigned char*>(s.ring[st]) + lane * 128;
#pragma unroll
                for (int c = 0; c < 8; c++) k[c] = *reinterpret_cast<const uint4*>(row + ((c ^ (lane & 7)) << 4));
            }
            const float sj = rh(self_score(s.q, k));  // :335
            s.sc[j] = sj;
            kmax = fmaxf(kmax, sj);
        }
        __syncwarp();
        if (lane == 0 && i + SSTAGE < total) issue(i + SSTAGE);  // only this warp read the stage
    }
    kmax = warp_max(kmax);
    if (lane == 0) s.wmax[w] = kmax;
    __syncthreads();

    // ---------------------------------------------------------------- softmax (:338-344, block_max / block_sum :22-46)
    // (the block max is the max of the warps' maxima of their scores; the sum keeps the reference's order: thread t
    // over positions t, t + 128, ..., then the warp butterfly and (w0 + w2) + (w1 + w3))
    const float m = fmaxf(fmaxf(s.wmax[0], s.wmax[1]), fmaxf(s.wmax[2], s.wmax[3]));
    float ex[SMAXL / 128];
    float e = 0.f;
#pragma unroll
    for (int u = 0; u < SMAXL / 128; u++) {
        const int j = t + 128 * u;
        ex[u] = j < L ? expf(s.sc[j] - m) : 0.f;
        if (j < L) e += ex[u];
    }
    e = warp_sum(e);
    if (lane == 0) s.wsum[w] = e;
    __syncthreads();
    const float sum = (s.wsum[0] + s.wsum[2]) + (s.wsum[1] + s.wsum[3]);
#pragma unroll
    for (int u = 0; u < SMAXL / 128; u++)
        if (t + 128 * u < L) s.sc[t + 128 * u] = rh(ex[u] / sum);
    __syncthreads();

    // ---------------------------------------------------------------- P.V (:345-352)
    const int col = t & (HD - 1), half = t >> 6;
    float acc = 0.f;
    for (int v = 0; v < ntile; v++) {
        const int i = ntile + v, st = i % SSTAGE, j0 = v * STILE;
        mbar_wait_spin(&s.full[st], (i / SSTAGE) & 1, &s.abort, limit_ns, status, K_SELF, 2);
        h16* tile = s.ring[st];
        if (p >= j0 && p < j0 + STILE) {  // the current position's values come from qkv
            if (t < 8) row_copy8(tile + (p - j0) * HD, qkv + qrow + 2 * d + hh * HD, t);
            __syncthreads();
        }
        float pj[STILE / 2], vj[STILE / 2];
#pragma unroll
        for (int u = 0; u < STILE / 2; u++) {  // tiles start at even positions: this thread's parity is half
            pj[u] = s.sc[j0 + half + 2 * u];
            vj[u] = f(tile[(half + 2 * u) * HD + col]);
        }
#pragma unroll
        for (int u = 0; u < STILE / 2; u++)
            if (j0 + half + 2 * u < L) acc = __fmaf_rn(pj[u], vj[u], acc);
        if (i + SSTAGE < total) {  // the stage is refilled: everyone must be done with it
            __syncthreads();
            if (t == 0) {
                fence_proxy_async_smem();  // the stage may hold the row written above
                issue(i + SSTAGE);
            }
        }
    }
    // :350-352
    if (half == 1) s.red[col] = acc;
    __syncthreads();
    if (half == 0) out[(long)b * d + hh * HD + col] = h(acc + s.red[col]);
    if (t == 0 && s.abort) {  // a wait gave up: let the copies in flight land before the shared memory is released
        const int n = s.nissued;
        for (int i = n - SSTAGE > 0 ? n - SSTAGE : 0; i < n; i++)
            mbar_wait(&s.full[i % SSTAGE], (i / SSTAGE) & 1, nullptr, limit_ns, nullptr, 0, 0);
    }
}

// ============================================================================ cross-attention kernels

// Cross-attention as three kernels with no waiting between CTAs: each CTA of the first two owns 192 positions of one
// (sequence, head); the scores kernel keeps all its 16-byte K loads in flight from registers, the P.V kernel pulls
// its 24 KB V slice into shared memory with three bulk TMA copies (one per 64-position chunk) issued before it waits
// for the scores.
//   cross_scores_kernel   fp16-rounded scores and the three 64-position chunk statistics of its slice -> scratch
//   cross_pv_kernel       issues its V loads, waits for the scores kernel (programmatic dependent launch), forms
//                         the global maximum and sum from the 24 statistics in chunk order, the probabilities (and
//                         the alignment rows), its three per-chunk P.V partials -> scratch
//   cross_combine_kernel  waits for the P.V kernel the same way and sums the 24 partials in chunk order
// Scratch per launch: S [B][heads][1500] f32, stat [B][heads][24] float2, part [B][heads][24][64] f32.

struct XScratch {
    float* S;
    float2* stat;
    float* part;
};

__host__ __device__ inline size_t cross_scratch_bytes(int batch, int nh) {
    const size_t items = (size_t)batch * nh;
    return items * TENC * 4 + items * XNCH * 8 + items * XNCH * HD * 4;
}
__host__ __device__ inline XScratch cross_scratch(void* base, int batch, int nh) {
    const size_t items = (size_t)batch * nh;
    char* p = (char*)base;
    XScratch x;
    x.S = (float*)p;
    p += items * TENC * 4;
    x.stat = (float2*)p;
    p += items * XNCH * 8;
    x.part = (float*)p;
    return x;
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// grid (8, heads, B), block 128. Every thread's twelve 16-byte K loads are issued before any is used, and before the
// wait for the kernel before (the q projection): K comes from the encoder and done from earlier decoding steps.
__global__ void __launch_bounds__(128) cross_scores_kernel(const h16* __restrict__ q, const h16* __restrict__ kv,
                                                           XScratch xs, const int* __restrict__ done, int layer,
                                                           int nl, int d) {
    constexpr int PT = XPER / 16;  // positions per lane group of 8
    __shared__ float qs[HD];
    __shared__ float sc[XPER];
    griddep_launch_dependents();  // the P.V kernel may start its V copies as soon as every CTA here is resident
    const int b = blockIdx.z, hh = blockIdx.y, r = blockIdx.x, t = threadIdx.x;
    const int nh = d / HD, bh = b * nh + hh;
    if (done[b]) return;
    const int j0 = r * XPER, n = min(XPER, TENC - j0);
    const int grp = t >> 3, sub = t & 7;
    const h16* K = kv + xkv_off(b, layer, 0, hh, nl, nh) + (long)j0 * HD + sub * 8;
    uint4 u[PT];
#pragma unroll
    for (int i = 0; i < PT; i++) {
        const int jj = grp + 16 * i;
        u[i] = jj < n ? ldg_stream(K + jj * HD) : make_uint4(0, 0, 0, 0);
    }
    griddep_wait();  // q comes from the kernel before; K and done from the encoder and earlier steps
    if (t < HD) qs[t] = rh(f(q[(long)b * d + hh * HD + t]) * 0.125f);
    __syncthreads();
    // scores: a group of 8 lanes per position (kernels/whisper.cu:376-392)
#pragma unroll
    for (int i = 0; i < PT; i++) {
        const int jj = grp + 16 * i;
        const __half2* p2 = reinterpret_cast<const __half2*>(&u[i]);
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float2 v = __half22float2(p2[e]);
            a += qs[sub * 8 + 2 * e] * v.x + qs[sub * 8 + 2 * e + 1] * v.y;
        }
        for (int o = 4; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffff, a, o);
        if (sub == 0) {
            a = jj < n ? rh(a) : -INFINITY;
            sc[jj] = a;
            if (jj < n) xs.S[(long)bh * TENC + j0 + jj] = a;
        }
    }
    __syncthreads();
    // chunk statistics, warp c for chunk c (kernels/whisper.cu:394-401)
    const int w = t >> 5, lane = t & 31;
    if (w < XCPC) {
        float a = sc[w * XCH + lane], b2 = sc[w * XCH + lane + 32];
        float m = fmaxf(a, b2);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffff, m, o));
        float sm = (a == -INFINITY ? 0.f : expf(a - m)) + (b2 == -INFINITY ? 0.f : expf(b2 - m));
        for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffff, sm, o);
        if (lane == 0) xs.stat[(long)bh * XNCH + r * XCPC + w] = make_float2(m, sm);
    }
}

// grid (8, heads, B), block 128; launched as a programmatic dependent of cross_scores_kernel
__global__ void __launch_bounds__(128, 8) cross_pv_kernel(const h16* __restrict__ kv, XScratch xs,
                                                          h16* __restrict__ align, const int* __restrict__ aslot,
                                                          const int* __restrict__ ctr, const int* __restrict__ done,
                                                          int layer, int nl, int d, int na, int maxT, unsigned* status,
                                                          unsigned long long limit_ns) {
    __shared__ __align__(128) h16 vs[XPER * HD];  // this CTA's V slice (bulk copies issued before the wait), then
                                                  // the group partials
    __shared__ float p[XPER];
    __shared__ float2 gs[XNCH];
    __shared__ float2 gms;  // the global (max, sum)
    __shared__ uint64_t bar[XCPC];
    static_assert(XCPC * 16 * HD * 4 <= XPER * HD * 2, "the group partials fit in the V slice");
    static_assert(XNCH <= 32, "one lane per chunk");
    __shared__ int abort;
    griddep_launch_dependents();  // the combine kernel may be scheduled as soon as every CTA here is resident
    const int b = blockIdx.z, hh = blockIdx.y, r = blockIdx.x, t = threadIdx.x;
    const int nh = d / HD, bh = b * nh + hh;
    if (done[b]) return;
    const int j0 = r * XPER, n = min(XPER, TENC - j0);
    const int grp = t >> 3, sub = t & 7;
    if (t == 0) {  // V does not depend on the scores: its copies are in flight before the wait
        abort = 0;
        const h16* V = kv + xkv_off(b, layer, 1, hh, nl, nh) + (long)j0 * HD;
        for (int c = 0; c < XCPC; c++) mbar_init(&bar[c], 1);
        fence_mbar_init();
        for (int c = 0; c < XCPC; c++) {
            const int nc = min(XCH, n - c * XCH);
            mbar_expect_tx(&bar[c], nc * HD * 2);
            bulk_g2s(vs + c * XCH * HD, V + (long)c * XCH * HD, nc * HD * 2, &bar[c]);
        }
    }
    griddep_wait();
    if (t < XNCH) gs[t] = __ldcg(&xs.stat[(long)bh * XNCH + t]);
    for (int jj = t; jj < n; jj += 128) p[jj] = __ldcg(&xs.S[(long)bh * TENC + j0 + jj]);
    __syncthreads();
    // the global max and sum over the 24 chunks in order (kernels/whisper.cu:414-417), formed once by warp 0: lane c
    // takes chunk c's exponential, and the sum runs through the chunks in order as fused multiply-adds
    if (t < 32) {
        const float2 g2 = t < XNCH ? gs[t] : make_float2(-INFINITY, 0.f);
        float mx = g2.x;
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
        const float e = t < XNCH ? expf(g2.x - mx) : 0.f;
        float sm = 0.f;
        for (int c = 0; c < XNCH; c++)
            sm = __fmaf_rn(__shfl_sync(0xffffffff, g2.y, c), __shfl_sync(0xffffffff, e, c), sm);
        if (t == 0) gms = make_float2(mx, sm);
    }
    __syncthreads();
    const float m = gms.x, sum = gms.y;
    const int slot = aslot[layer * nh + hh];
    h16* arow = slot >= 0 ? align + (((long)b * maxT + ctr[0]) * na + slot) * TENC + j0 : nullptr;
    for (int jj = t; jj < n; jj += 128) {
        float pj = rh(expf(p[jj] - m) / sum);
        p[jj] = pj;
        if (arow) arow[jj] = h(pj);
    }
    __syncthreads();
    // P.V per chunk: 16 groups x 8 lanes, a lane owns 8 of the 64 columns (kernels/whisper.cu:421-438); the three
    // chunks' group sums then meet in the V slice's space (keeping shared memory at 26 KB: 8 CTAs per SM)
    float a[XCPC][8];
#pragma unroll
    for (int c = 0; c < XCPC; c++) {
        mbar_wait_spin(&bar[c], 0, &abort, limit_ns, status, K_CROSS, 4 + c);
        const int nc = min(XCH, n - c * XCH);
#pragma unroll
        for (int e = 0; e < 8; e++) a[c][e] = 0.f;
        for (int jj = grp; jj < nc; jj += 16) {
            const uint4 u = *reinterpret_cast<const uint4*>(vs + (c * XCH + jj) * HD + sub * 8);
            const __half2* p2 = reinterpret_cast<const __half2*>(&u);
            const float pj = p[c * XCH + jj];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float2 v = __half22float2(p2[e]);
                a[c][2 * e] += pj * v.x;
                a[c][2 * e + 1] += pj * v.y;
            }
        }
    }
    __syncthreads();  // V is no longer read
    float* red = reinterpret_cast<float*>(vs);  // [XCPC][16][HD]
#pragma unroll
    for (int c = 0; c < XCPC; c++)
#pragma unroll
        for (int e = 0; e < 8; e++) red[(c * 16 + grp) * HD + sub * 8 + e] = a[c][e];
    __syncthreads();
    for (int i = t; i < XCPC * HD; i += 128) {
        const int c = i / HD, col = i % HD;
        float acc = 0.f;
        for (int g = 0; g < 16; g++) acc += red[(c * 16 + g) * HD + col];
        xs.part[((long)bh * XNCH + r * XCPC + c) * HD + col] = acc;
    }
    if (t == 0 && abort)
        for (int c = 0; c < XCPC; c++) mbar_wait(&bar[c], 0, nullptr, limit_ns, nullptr, 0, 0);
}

// grid (heads, B), block 64; launched as a programmatic dependent of cross_pv_kernel: the 24 partials of a
// (sequence, head) summed in chunk order (kernels/whisper.cu:443-449)
__global__ void __launch_bounds__(64) cross_combine_kernel(const float* __restrict__ part, h16* __restrict__ out,
                                                           const int* __restrict__ done, int d) {
    const int hh = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    const int bh = b * (d / HD) + hh;
    griddep_wait();  // no early launch of the next kernel: back-to-back cross-attentions ran 50.1 us against 45.8
    if (done[b]) return;
    float acc = 0.f;
    for (int c = 0; c < XNCH; c++) acc += __ldcg(&part[((long)bh * XNCH + c) * HD + t]);
    out[(long)b * d + hh * HD + t] = h(acc);
}

// The three kernels above as one launch, for the decoding step at small batches, where the launches rather than the
// bytes set its time: grid (8, heads, B) in clusters of the 8 CTAs of a (sequence, head), each with the same 192
// positions as cross_scores_kernel and cross_pv_kernel. The scores stay in shared memory; each CTA sends its three
// chunk statistics to every CTA of the cluster (distributed shared memory) and, after a cluster barrier, forms the
// global max and sum from all 24 in chunk order, as cross_pv_kernel does from the scratch; the chunk partials of P.V go
// to CTA 0 of the cluster, which sums them in chunk order after a second barrier, as cross_combine_kernel does. Every
// value is formed by the same operations in the same order as in the three kernels, so the outputs and the alignment
// probabilities are theirs bit for bit. K and V come from the encoder and ctr / done from earlier steps: all copies are
// in flight before the wait for the kernel before (q comes from it). Every CTA of a cluster has the same sequence, so a
// finished one leaves as a whole cluster, before either barrier.
__global__ void __cluster_dims__(XCL, 1, 1) __launch_bounds__(128)
    cross_fused_kernel(const h16* __restrict__ q, const h16* __restrict__ kv, h16* __restrict__ out,
                       h16* __restrict__ align, const int* __restrict__ aslot, const int* __restrict__ ctr,
                       const int* __restrict__ done, int layer, int nl, int d, int na, int maxT, unsigned* status,
                       unsigned long long limit_ns) {
    constexpr int PT = XPER / 16;  // positions per lane group of 8
    __shared__ __align__(128) h16 vs[XPER * HD];  // this CTA's V slice, then the group partials
    __shared__ float qs[HD];
    __shared__ float sc[XPER];      // the rounded scores, then the probabilities
    __shared__ float2 gs[XNCH];     // the 24 chunk statistics of the (sequence, head), from every CTA of the cluster
    __shared__ float part[XNCH * HD];  // CTA 0: the 24 chunk partials of P.V
    __shared__ float2 gms;
    __shared__ uint64_t bar[XCPC];
    __shared__ int abort;
    static_assert(XCPC * 16 * HD * 4 <= XPER * HD * 2, "the group partials fit in the V slice");
    const int b = blockIdx.z, hh = blockIdx.y, t = threadIdx.x;
    const int r = (int)cluster_rank();
    const int nh = d / HD;
    if (done[b]) return;
    cluster_arrive_relaxed();  // waited for before the first store into another CTA's shared memory
    const int j0 = r * XPER, n = min(XPER, TENC - j0);
    const int grp = t >> 3, sub = t & 7;
    const h16* K = kv + xkv_off(b, layer, 0, hh, nl, nh) + (long)j0 * HD + sub * 8;
    uint4 u[PT];
#pragma unroll
    for (int i = 0; i < PT; i++) {
        const int jj = grp + 16 * i;
        u[i] = jj < n ? ldg_stream(K + jj * HD) : make_uint4(0, 0, 0, 0);
    }
    if (t == 0) {
        abort = 0;
        const h16* V = kv + xkv_off(b, layer, 1, hh, nl, nh) + (long)j0 * HD;
        for (int c = 0; c < XCPC; c++) mbar_init(&bar[c], 1);
        fence_mbar_init();
        for (int c = 0; c < XCPC; c++) {
            const int nc = min(XCH, n - c * XCH);
            mbar_expect_tx(&bar[c], nc * HD * 2);
            bulk_g2s(vs + c * XCH * HD, V + (long)c * XCH * HD, nc * HD * 2, &bar[c]);
        }
    }
    griddep_wait();  // q comes from the kernel before
    griddep_launch_dependents();
    if (t < HD) qs[t] = rh(f(q[(long)b * d + hh * HD + t]) * 0.125f);
    __syncthreads();
    // scores: a group of 8 lanes per position (kernels/whisper.cu:376-392)
#pragma unroll
    for (int i = 0; i < PT; i++) {
        const int jj = grp + 16 * i;
        const __half2* p2 = reinterpret_cast<const __half2*>(&u[i]);
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float2 v = __half22float2(p2[e]);
            a += qs[sub * 8 + 2 * e] * v.x + qs[sub * 8 + 2 * e + 1] * v.y;
        }
        for (int o = 4; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffff, a, o);
        if (sub == 0) sc[jj] = jj < n ? rh(a) : -INFINITY;
    }
    __syncthreads();
    cluster_wait();  // every CTA of the cluster has started: its shared memory may be written
    // chunk statistics, warp c for chunk c (kernels/whisper.cu:394-401), sent to every CTA of the cluster
    const int w = t >> 5, lane = t & 31;
    if (w < XCPC) {
        float a = sc[w * XCH + lane], b2 = sc[w * XCH + lane + 32];
        float m = fmaxf(a, b2);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffff, m, o));
        float sm = (a == -INFINITY ? 0.f : expf(a - m)) + (b2 == -INFINITY ? 0.f : expf(b2 - m));
        for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffff, sm, o);
        if (lane < XCL) st_dsmem_f32x2(dsmem_addr(&gs[r * XCPC + w], lane), make_float2(m, sm));
    }
    cluster_sync();  // every CTA holds the 24 statistics
    // the global max and sum over the 24 chunks in order (kernels/whisper.cu:414-417), as in cross_pv_kernel
    if (t < 32) {
        const float2 g2 = t < XNCH ? gs[t] : make_float2(-INFINITY, 0.f);
        float mx = g2.x;
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
        const float e = t < XNCH ? expf(g2.x - mx) : 0.f;
        float sm = 0.f;
        for (int c = 0; c < XNCH; c++)
            sm = __fmaf_rn(__shfl_sync(0xffffffff, g2.y, c), __shfl_sync(0xffffffff, e, c), sm);
        if (t == 0) gms = make_float2(mx, sm);
    }
    __syncthreads();
    const float m = gms.x, sum = gms.y;
    const int slot = aslot[layer * nh + hh];
    h16* arow = slot >= 0 ? align + (((long)b * maxT + ctr[0]) * na + slot) * TENC + j0 : nullptr;
    for (int jj = t; jj < n; jj += 128) {
        float pj = rh(expf(sc[jj] - m) / sum);
        sc[jj] = pj;
        if (arow) arow[jj] = h(pj);
    }
    __syncthreads();
    // P.V per chunk (kernels/whisper.cu:421-438), as in cross_pv_kernel
    float a[XCPC][8];
#pragma unroll
    for (int c = 0; c < XCPC; c++) {
        mbar_wait_spin(&bar[c], 0, &abort, limit_ns, status, K_CROSS, 8 + c);
        const int nc = min(XCH, n - c * XCH);
#pragma unroll
        for (int e = 0; e < 8; e++) a[c][e] = 0.f;
        for (int jj = grp; jj < nc; jj += 16) {
            const uint4 uv = *reinterpret_cast<const uint4*>(vs + (c * XCH + jj) * HD + sub * 8);
            const __half2* p2 = reinterpret_cast<const __half2*>(&uv);
            const float pj = sc[c * XCH + jj];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float2 v = __half22float2(p2[e]);
                a[c][2 * e] += pj * v.x;
                a[c][2 * e + 1] += pj * v.y;
            }
        }
    }
    __syncthreads();  // V is no longer read
    float* red = reinterpret_cast<float*>(vs);  // [XCPC][16][HD]
#pragma unroll
    for (int c = 0; c < XCPC; c++)
#pragma unroll
        for (int e = 0; e < 8; e++) red[(c * 16 + grp) * HD + sub * 8 + e] = a[c][e];
    __syncthreads();
    for (int i = t; i < XCPC * HD; i += 128) {
        const int c = i / HD, col = i % HD;
        float acc = 0.f;
        for (int g = 0; g < 16; g++) acc += red[(c * 16 + g) * HD + col];
        st_dsmem_f32(dsmem_addr(&part[(r * XCPC + c) * HD + col], 0), acc);
    }
    if (t == 0 && abort)
        for (int c = 0; c < XCPC; c++) mbar_wait(&bar[c], 0, nullptr, limit_ns, nullptr, 0, 0);
    cluster_sync();  // CTA 0 holds the 24 partials
    if (r == 0 && t < HD) {  // the partials summed in chunk order (kernels/whisper.cu:443-449)
        float acc = 0.f;
        for (int c = 0; c < XNCH; c++) acc += part[c * HD + t];
        out[(long)b * d + hh * HD + t] = h(acc);
    }
}

// kernels/whisper.cu:310-317 as its own launch (the engine folds it into self_attn_kernel): k and v of position p
// into the caches, 16-byte copies.
__global__ void kv_write_kernel(const h16* __restrict__ qkv, h16* __restrict__ kc, h16* __restrict__ vc,
                                const int* __restrict__ ctr, int maxT, int d) {
    const int b = blockIdx.x, p = ctr[0];
    const long dst = ((long)b * maxT + p) * d;
    for (int c = threadIdx.x; c < d / 8; c += blockDim.x) {
        reinterpret_cast<uint4*>(kc + dst)[c] = reinterpret_cast<const uint4*>(qkv + (long)b * 3 * d + d)[c];
        reinterpret_cast<uint4*>(vc + dst)[c] = reinterpret_cast<const uint4*>(qkv + (long)b * 3 * d + 2 * d)[c];
    }
}

// ============================================================================ launchers

int launch_cross_fused(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                       const int* done, int batch, int layer, int nl, int d, int na, int maxT, cudaStream_t st) {
    if (batch < 1 || batch > 65535 || d < HD || d % HD || layer < 0 || layer >= nl || maxT < 1 || na < 0)
        return fail("cross_fused: bad shape");
    if (((uintptr_t)kv & 15) || ((uintptr_t)q & 3)) return fail("cross_fused: kv must be 16-byte aligned");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    return check_pdl(launch_pdl(cross_fused_kernel, dim3(XCL, d / HD, batch), dim3(128), 0, st, (const h16*)q,
                                (const h16*)kv, (h16*)out, (h16*)align, aslot, ctr, done, layer, nl, d, na, maxT,
                                dc.status, dc.limit_ns),
                     "cross_fused");
}

size_t cross_attn_scratch_bytes(int batch, int d) { return cross_scratch_bytes(batch, d / HD); }

int launch_cross_attn(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                            const int* done, int batch, int layer, int nl, int d, int na, int maxT, void* scratch,
                            size_t scratch_bytes, cudaStream_t st) {
    if (batch < 1 || d < HD || d % HD || layer < 0 || layer >= nl || maxT < 1 || na < 0)
        return fail("cross_attn: bad shape");
    if (((uintptr_t)kv & 15) || ((uintptr_t)q & 3)) return fail("cross_attn: kv must be 16-byte aligned");
    if (!scratch || ((uintptr_t)scratch & 15) || scratch_bytes < cross_scratch_bytes(batch, d / HD))
        return fail("cross_attn: scratch missing, misaligned or smaller than mmz_cross_attn_scratch_bytes");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    XScratch xs = cross_scratch(scratch, batch, d / HD);
    dim3 grid(XCL, d / HD, batch);
    if (check_pdl(launch_pdl(cross_scores_kernel, grid, dim3(128), 0, st, (const h16*)q, (const h16*)kv, xs, done,
                             layer, nl, d),
                  "cross_scores"))
        return -1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, cross_pv_kernel, (const h16*)kv, xs, (h16*)align, aslot, ctr, done,
                                       layer, nl, d, na, maxT, dc.status, dc.limit_ns);
    if (e != cudaSuccess) return failf("cross_pv: launch failed: %s", cudaGetErrorString(e));
    cfg.gridDim = dim3(d / HD, batch, 1);
    cfg.blockDim = dim3(HD, 1, 1);
    e = cudaLaunchKernelEx(&cfg, cross_combine_kernel, (const float*)xs.part, (h16*)out, done, d);
    if (e != cudaSuccess) return failf("cross_combine: launch failed: %s", cudaGetErrorString(e));
    return 0;
}

int launch_self_attn(const void* qkv, void* kc, void* vc, void* out, const int* ctr, const int* done, int batch,
                     int maxT, int d, cudaStream_t st) {
    if (batch < 1 || d < HD || d % HD || maxT < 1 || maxT > SMAXL) return fail("self_attn: bad shape (maxT <= 512)");
    if (((uintptr_t)kc & 15) || ((uintptr_t)vc & 15) || ((uintptr_t)qkv & 15))
        return fail("self_attn: buffers must be 16-byte aligned");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    CUtensorMap km, vm;
    const uint64_t dims[2] = {(uint64_t)d, (uint64_t)batch * maxT};
    const uint64_t strides[1] = {(uint64_t)d * 2};
    const uint32_t box[2] = {HD, STILE};
    if (make_tmap_2d(&km, kc, dims, strides, box, 128) || make_tmap_2d(&vm, vc, dims, strides, box, 0))
        return fail("self_attn: cuTensorMapEncodeTiled failed");
    dim3 grid(d / HD, batch);
    return check_pdl(launch_pdl(self_attn_kernel, grid, dim3(128), sizeof(SelfSmem), st, km, vm, (const h16*)qkv,
                                (h16*)kc, (h16*)vc, (h16*)out, ctr, done, maxT, d, dc.status, dc.limit_ns),
                     "self_attn");
}

int launch_kv_write(const void* qkv, void* kc, void* vc, const int* ctr, int batch, int maxT, int d, cudaStream_t st) {
    if (batch < 1 || d % 8 || maxT < 1) return fail("kv_write: bad shape");
    kv_write_kernel<<<batch, 128, 0, st>>>((const h16*)qkv, (h16*)kc, (h16*)vc, ctr, maxT, d);
    return check_launch("kv_write");
}

void init_dec_attn_attrs(DevCtx&) {
    cudaFuncSetAttribute(self_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(SelfSmem));
}

}  // namespace mmz
