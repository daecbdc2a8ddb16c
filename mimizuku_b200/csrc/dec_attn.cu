// Decoder-step attention for sm_100a: causal self-attention over the KV cache (with the cache write of the current
// position folded in) and cross-attention over the 1500 encoder positions, which also records the alignment-head
// probabilities. Both are memory-bound split-KV kernels: a thread-block cluster covers one (sequence, head), each CTA
// pulls its slice of K and V into shared memory with one TMA transaction per operand, and the softmax statistics and
// partial outputs are exchanged through distributed shared memory, so a step needs one launch per attention and no
// global scratch.
//
// Both kernels read the position from device memory (ctr[0]) and skip finished sequences (done[b]), so one captured
// CUDA graph serves every decoding step, as the reference engine requires (kernels/whisper.cu:7-8).
//
// Rounding follows the reference kernels point for point: q * 0.125 -> fp16, scores -> fp16, probabilities -> fp16,
// outputs -> fp16 (kernels/whisper.cu:327, 335, 344, 352 for self-attention; 373, 388, 419, 440, 448 for
// cross-attention). Reductions reproduce the reference's association where that costs nothing: the cross-attention
// softmax statistics are formed per 64-position chunk and combined over the 24 chunks in order
// (kernels/whisper.cu:394-401, 414-417) and the P.V partials are summed per chunk and then over chunks in order
// (:421-438, :447); the self-attention exp-sum follows the 128-thread strided block sum of :342-343.
#include "common.cuh"
#include "launch.h"

namespace mmz {

// ============================================================================ cross-attention

constexpr int XCL = 8;            // CTAs per (sequence, head)
constexpr int XCH = 64;           // reference chunk (kernels/whisper.cu:360)
constexpr int XPER = 3 * XCH;     // positions per CTA: three reference chunks; 8 x 192 >= 1500
constexpr int XNCH = (TENC + XCH - 1) / XCH;  // 24 chunks

struct CrossSmem {
    h16 k[XPER * HD];             // 24576 B, TMA destination (16-byte aligned)
    h16 v[XPER * HD];
    float q[HD];
    float p[XPER];                // scores, then probabilities
    float2 cstat[4];              // this CTA's chunk statistics (max, sum of exp), read by the cluster
    float2 gstat[XNCH];
    float red[16][HD];
    float part[3][HD];            // this CTA's per-chunk P.V partials, read by rank 0
    uint64_t bar[2];
    int abort;
};

// kv: [b][layer][k | v][head][1500][64] (kernels/whisper.cu:362-364)
__device__ __forceinline__ long xkv_off(int b, int layer, int kv, int hh, int nl, int nh) {
    return ((((long)b * nl + layer) * 2 + kv) * nh + hh) * (long)TENC * HD;
}

__global__ void __cluster_dims__(XCL, 1, 1) __launch_bounds__(128)
    cross_attn_kernel(const h16* __restrict__ q, const h16* __restrict__ kv, h16* __restrict__ out,
                      h16* __restrict__ align, const int* __restrict__ aslot, const int* __restrict__ ctr,
                      const int* __restrict__ done, int layer, int nl, int d, int na, int maxT, unsigned* status,
                      unsigned long long limit_ns) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    CrossSmem& s = *reinterpret_cast<CrossSmem*>(smem_raw);
    const int b = blockIdx.z, hh = blockIdx.y, r = blockIdx.x, t = threadIdx.x;
    const int nh = d / HD;
    if (done[b]) return;  // the whole cluster shares b
    const int j0 = r * XPER, n = min(XPER, TENC - j0);
    const h16* K = kv + xkv_off(b, layer, 0, hh, nl, nh) + (long)j0 * HD;
    const h16* V = kv + xkv_off(b, layer, 1, hh, nl, nh) + (long)j0 * HD;
    if (t == 0) {
        s.abort = 0;
        mbar_init(&s.bar[0], 1);
        mbar_init(&s.bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (t == 0) {
        mbar_expect_tx(&s.bar[0], n * HD * 2);
        bulk_g2s(s.k, K, n * HD * 2, &s.bar[0]);
        mbar_expect_tx(&s.bar[1], n * HD * 2);
        bulk_g2s(s.v, V, n * HD * 2, &s.bar[1]);
    }
    if (t < HD) s.q[t] = rh(f(q[(long)b * d + hh * HD + t]) * 0.125f);
    __syncthreads();
    mbar_wait(&s.bar[0], 0, &s.abort, limit_ns, status, K_CROSS, 1);

    // scores: a group of 8 lanes per position, 16-byte loads (kernels/whisper.cu:376-392)
    const int grp = t >> 3, sub = t & 7;
    for (int jj = grp; jj < XPER; jj += 16) {
        float a = 0.f;
        if (jj < n) {
            uint4 u = *reinterpret_cast<const uint4*>(s.k + jj * HD + sub * 8);
            const __half2* p2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float2 v = __half22float2(p2[e]);
                a += s.q[sub * 8 + 2 * e] * v.x + s.q[sub * 8 + 2 * e + 1] * v.y;
            }
        }
        for (int o = 4; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffff, a, o);
        if (sub == 0) s.p[jj] = jj < n ? rh(a) : -INFINITY;
    }
    __syncthreads();
    // per-chunk (max, sum of exp): warp c takes chunk c (kernels/whisper.cu:394-401)
    const int w = t >> 5, lane = t & 31;
    if (w < 3) {
        float a = s.p[w * XCH + lane], b2 = s.p[w * XCH + lane + 32];
        float m = fmaxf(a, b2);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffff, m, o));
        float sm = (a == -INFINITY ? 0.f : expf(a - m)) + (b2 == -INFINITY ? 0.f : expf(b2 - m));
        for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffff, sm, o);
        if (lane == 0) s.cstat[w] = make_float2(m, sm);
    }
    cluster_sync();
    // the 24 chunk statistics in chunk order, then the global max and sum (kernels/whisper.cu:414-417)
    if (t < XNCH) s.gstat[t] = ld_dsmem_f32x2(dsmem_addr(&s.cstat[t % 3], t / 3));
    __syncthreads();
    float m = -INFINITY;
    for (int c = 0; c < XNCH; c++) m = fmaxf(m, s.gstat[c].x);
    float sum = 0.f;
    for (int c = 0; c < XNCH; c++) {
        float2 st = s.gstat[c];
        sum += st.y * expf(st.x - m);
    }
    const int slot = aslot[layer * nh + hh];
    h16* arow = slot >= 0 ? align + (((long)b * maxT + ctr[0]) * na + slot) * TENC + j0 : nullptr;
    for (int jj = t; jj < n; jj += 128) {
        float pj = rh(expf(s.p[jj] - m) / sum);
        s.p[jj] = pj;
        if (arow) arow[jj] = h(pj);
    }
    __syncthreads();
    mbar_wait(&s.bar[1], 0, &s.abort, limit_ns, status, K_CROSS, 2);
    // P.V per chunk: 16 groups x 8 lanes, a lane owns 8 of the 64 columns (kernels/whisper.cu:421-438)
    for (int c = 0; c < 3; c++) {
        const int nc = min(XCH, n - c * XCH);
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int jj = grp; jj < nc; jj += 16) {
            uint4 u = *reinterpret_cast<const uint4*>(s.v + (c * XCH + jj) * HD + sub * 8);
            const __half2* p2 = reinterpret_cast<const __half2*>(&u);
            float pj = s.p[c * XCH + jj];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                float2 v = __half22float2(p2[k]);
                a[2 * k] += pj * v.x;
                a[2 * k + 1] += pj * v.y;
            }
        }
#pragma unroll
        for (int k = 0; k < 8; k++) s.red[grp][sub * 8 + k] = a[k];
        __syncthreads();
        if (t < HD) {
            float acc = 0.f;
            for (int g = 0; g < 16; g++) acc += s.red[g][t];
            s.part[c][t] = acc;
        }
        __syncthreads();
    }
    cluster_sync();
    // sum of the 24 chunk partials in order (kernels/whisper.cu:443-449)
    if (r == 0 && t < HD) {
        float acc = 0.f;
        for (int c = 0; c < XNCH; c++) acc += ld_dsmem_f32(dsmem_addr(&s.part[c % 3][t], c / 3));
        out[(long)b * d + hh * HD + t] = h(acc);
    }
    cluster_sync();  // keeps every CTA's shared memory alive until rank 0 has read it
    if (t == 0 && s.abort) {  // a wait gave up: let the copies land before the shared memory is released
        mbar_wait(&s.bar[0], 0, nullptr, limit_ns, nullptr, 0, 0);
        mbar_wait(&s.bar[1], 0, nullptr, limit_ns, nullptr, 0, 0);
    }
}

// ============================================================================ self-attention

constexpr int SCL = 4;     // CTAs per (sequence, head)
constexpr int SPER = 128;  // positions per CTA: 4 x 128 >= 448 (the longest Whisper decoder context)

struct SelfSmem {
    h16 k[SPER * HD];  // 16384 B, TMA destination
    h16 v[SPER * HD];
    float q[HD];
    float sc[SPER];
    float e[SPER];     // exp(score - max), read by the cluster for the exp-sum
    float wred[4];
    float cmax;
    float pv[2][HD];   // this CTA's even / odd-position P.V partials
    uint64_t bar[2];
    int abort;
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

// grid (SCL, heads, B), cluster (SCL, 1, 1), block 128. CTA r owns cache positions [128 r, 128 r + 128).
// kmap / vmap: 2-D tensor maps over this layer's caches [B * maxT rows][d], box 64 x 128.
__global__ void __cluster_dims__(SCL, 1, 1) __launch_bounds__(128)
    self_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                     const h16* __restrict__ qkv, h16* __restrict__ kc, h16* __restrict__ vc, h16* __restrict__ out,
                     const int* __restrict__ ctr, const int* __restrict__ done, int maxT, int d, unsigned* status,
                     unsigned long long limit_ns) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    SelfSmem& s = *reinterpret_cast<SelfSmem*>(smem_raw);
    const int b = blockIdx.z, hh = blockIdx.y, r = blockIdx.x, t = threadIdx.x;
    const int w = t >> 5, lane = t & 31;
    const int p = ctr[0], L = p + 1;
    const int base = r * SPER, n = max(0, min(SPER, L - base));
    const bool owner = p >= base && p < base + SPER;
    const long qrow = (long)b * 3 * d;
    const long crow = ((long)b * maxT + p) * d + hh * HD;
    if (done[b]) {
        // the reference writes the cache row of every sequence (kernels/whisper.cu:310-317)
        if (owner && t < 8) {
            row_copy8(kc + crow, qkv + qrow + d + hh * HD, t);
            row_copy8(vc + crow, qkv + qrow + 2 * d + hh * HD, t);
        }
        return;  // the whole cluster shares b
    }
    if (t == 0) {
        s.abort = 0;
        mbar_init(&s.bar[0], 1);
        mbar_init(&s.bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (t == 0 && n > 0) {
        mbar_expect_tx(&s.bar[0], SPER * HD * 2);
        tma_load_2d(s.k, &kmap, hh * HD, b * maxT + base, &s.bar[0]);
        mbar_expect_tx(&s.bar[1], SPER * HD * 2);
        tma_load_2d(s.v, &vmap, hh * HD, b * maxT + base, &s.bar[1]);
    }
    if (t < HD) s.q[t] = rh(f(qkv[qrow + hh * HD + t]) * 0.125f);
    if (n > 0) {
        mbar_wait(&s.bar[0], 0, &s.abort, limit_ns, status, K_SELF, 1);
        if (owner && t < 8) {  // the current position comes from qkv: into shared memory and into the cache
            row_copy8(s.k + (p - base) * HD, qkv + qrow + d + hh * HD, t);
            row_copy8(kc + crow, qkv + qrow + d + hh * HD, t);
        }
    }
    __syncthreads();
    // scores: a warp per position, 2 elements per lane (kernels/whisper.cu:331-336)
    for (int i = w; i < n; i += 4) {
        float2 k2 = __half22float2(reinterpret_cast<const __half2*>(s.k + i * HD)[lane]);
        float a = s.q[2 * lane] * k2.x + s.q[2 * lane + 1] * k2.y;
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffff, a, o);
        if (lane == 0) s.sc[i] = rh(a);
    }
    __syncthreads();
    float mx = warp_max(t < n ? s.sc[t] : -INFINITY);
    if (lane == 0) s.wred[w] = mx;
    __syncthreads();
    if (t == 0) s.cmax = fmaxf(fmaxf(s.wred[0], s.wred[1]), fmaxf(s.wred[2], s.wred[3]));
    cluster_sync();
    float m = -INFINITY;
    for (int k = 0; k < SCL; k++) m = fmaxf(m, ld_dsmem_f32(dsmem_addr(&s.cmax, k)));
    if (t < n) s.e[t] = expf(s.sc[t] - m);
    cluster_sync();
    // thread t sums positions t, t + 128, ... as the reference's block does (kernels/whisper.cu:342), then the
    // reference's two-level warp reduction (block_sum, :22-33)
    float part = 0.f;
    for (int k = 0; k < SCL; k++)
        if (t + SPER * k < L) part += ld_dsmem_f32(dsmem_addr(&s.e[t], k));
    part = warp_sum(part);
    __syncthreads();
    if (lane == 0) s.wred[w] = part;
    __syncthreads();
    float tot = warp_sum(lane < 4 ? s.wred[lane] : 0.f);
    if (t < n) s.sc[t] = rh(expf(s.sc[t] - m) / tot);
    if (n > 0) {
        mbar_wait(&s.bar[1], 0, &s.abort, limit_ns, status, K_SELF, 2);
        if (owner && t < 8) {
            row_copy8(s.v + (p - base) * HD, qkv + qrow + 2 * d + hh * HD, t);
            row_copy8(vc + crow, qkv + qrow + 2 * d + hh * HD, t);
        }
    }
    __syncthreads();
    // P.V: thread (half, c) sums every other position (kernels/whisper.cu:346-352)
    {
        const int c = t & (HD - 1), half = t >> 6;
        float a = 0.f;
        for (int i = half; i < n; i += 2) a += s.sc[i] * f(s.v[i * HD + c]);
        s.pv[half][c] = a;
    }
    cluster_sync();
    if (r == 0 && t < HD) {
        float a0 = 0.f, a1 = 0.f;
        for (int k = 0; k < SCL; k++) {
            a0 += ld_dsmem_f32(dsmem_addr(&s.pv[0][t], k));
            a1 += ld_dsmem_f32(dsmem_addr(&s.pv[1][t], k));
        }
        out[(long)b * d + hh * HD + t] = h(a0 + a1);
    }
    cluster_sync();
    if (t == 0 && s.abort && n > 0) {
        mbar_wait(&s.bar[0], 0, nullptr, limit_ns, nullptr, 0, 0);
        mbar_wait(&s.bar[1], 0, nullptr, limit_ns, nullptr, 0, 0);
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

int launch_cross_attn(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                      const int* done, int batch, int layer, int nl, int d, int na, int maxT, cudaStream_t st) {
    if (batch < 1 || d < HD || d % HD || layer < 0 || layer >= nl || maxT < 1 || na < 0) return fail("cross_attn: bad shape");
    if (((uintptr_t)kv & 15) || ((uintptr_t)q & 3)) return fail("cross_attn: kv must be 16-byte aligned");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    dim3 grid(XCL, d / HD, batch);
    cross_attn_kernel<<<grid, 128, sizeof(CrossSmem), st>>>(
        (const h16*)q, (const h16*)kv, (h16*)out, (h16*)align, aslot, ctr, done, layer, nl, d, na, maxT, dc.status,
        dc.limit_ns);
    return check_launch("cross_attn");
}

int launch_self_attn(const void* qkv, void* kc, void* vc, void* out, const int* ctr, const int* done, int batch,
                     int maxT, int d, cudaStream_t st) {
    if (batch < 1 || d < HD || d % HD || maxT < 1 || maxT > SCL * SPER) return fail("self_attn: bad shape (maxT <= 512)");
    if (((uintptr_t)kc & 15) || ((uintptr_t)vc & 15) || ((uintptr_t)qkv & 15))
        return fail("self_attn: buffers must be 16-byte aligned");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    CUtensorMap km, vm;
    uint64_t dims[2] = {(uint64_t)d, (uint64_t)batch * maxT};
    uint64_t strides[1] = {(uint64_t)d * 2};
    uint32_t box[2] = {HD, SPER};
    if (make_tmap_2d(&km, kc, dims, strides, box, false) || make_tmap_2d(&vm, vc, dims, strides, box, false))
        return fail("self_attn: cuTensorMapEncodeTiled failed");
    dim3 grid(SCL, d / HD, batch);
    self_attn_kernel<<<grid, 128, sizeof(SelfSmem), st>>>(km, vm, (const h16*)qkv, (h16*)kc, (h16*)vc, (h16*)out, ctr,
                                                          done, maxT, d, dc.status, dc.limit_ns);
    return check_launch("self_attn");
}

int launch_kv_write(const void* qkv, void* kc, void* vc, const int* ctr, int batch, int maxT, int d, cudaStream_t st) {
    if (batch < 1 || d % 8 || maxT < 1) return fail("kv_write: bad shape");
    kv_write_kernel<<<batch, 128, 0, st>>>((const h16*)qkv, (h16*)kc, (h16*)vc, ctr, maxT, d);
    return check_launch("kv_write");
}

void init_dec_attn_attrs() {
    cudaFuncSetAttribute(cross_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(CrossSmem));
    cudaFuncSetAttribute(self_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(SelfSmem));
}

}  // namespace mmz
