// The engine's elementwise and token kernels around the attention path: the encoder stem helpers, the decoder
// embedding, the greedy token choice and the position counter, plus the harness's seeded weight initialiser.
// They compute what the reference engine's kernels of the same names compute (kernels/whisper.cu:92-139, 303-307,
// 451-495), with 16-byte accesses where the layout allows.
#include "common.cuh"
#include "launch.h"

namespace mmz {

static inline unsigned blocks(long n, int per) { return (unsigned)((n + per - 1) / per); }

// x[b] = h(tok_emb[tok[b, p]] + pos_emb[p]), p = ctr[0] (kernels/whisper.cu:303-307)
__global__ void embed_kernel(const int* __restrict__ tok, const int* __restrict__ ctr, const h16* __restrict__ emb,
                             const h16* __restrict__ pe, h16* __restrict__ x, int maxT, int d) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    const int b = blockIdx.x, p = ctr[0], t = tok[b * maxT + p];
    for (int c = threadIdx.x; c < d / 2; c += blockDim.x) {
        float2 e = __half22float2(reinterpret_cast<const __half2*>(emb + (long)t * d)[c]);
        float2 q = __half22float2(reinterpret_cast<const __half2*>(pe + (long)p * d)[c]);
        reinterpret_cast<__half2*>(x + (long)b * d)[c] = __floats2half2_rn(e.x + q.x, e.y + q.y);
    }
}

// Greedy choice of token p + 1 (kernels/whisper.cu:451-493): suppressed ids (sup[i] != 0, and bs1 / bs2 at the first
// generated position) are skipped, ties go to the lower id, prompt positions stay, finished rows and rows with every
// id suppressed get eos.
__device__ __forceinline__ void keep_best(float v, int i, float& best, int& bi) {
    if (v > best || (v == best && i < bi)) {
        best = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(1024) argmax_kernel(const h16* __restrict__ logits, int V, const unsigned char* sup,
                                                      int* tok, int* done, const int* ctr, int maxT, int prompt_len,
                                                      int eos, int bs1, int bs2) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    __shared__ float sv[32];
    __shared__ int si[32];
    const int b = blockIdx.x, p = ctr[0];
    if (p + 1 < prompt_len || p + 1 >= maxT) return;
    const bool first = p + 1 == prompt_len;
    const h16* lg = logits + (long)b * V;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    if ((V & 1) == 0) {
        // even V: every row starts 4-byte aligned, so ids are scanned in pairs, several loads in flight per thread;
        // each thread still visits its ids in increasing order, so ties keep the lower id
        const __half2* lg2 = reinterpret_cast<const __half2*>(lg);
        const unsigned short* sup2 = reinterpret_cast<const unsigned short*>(sup);
        const int n2 = V / 2;
#pragma unroll 4
        for (int j = threadIdx.x; j < n2; j += blockDim.x) {
            const float2 v = __half22float2(lg2[j]);
            const unsigned short sp = sup2[j];
            const int i = 2 * j;
            if (!(sp & 0xff) && !(first && (i == bs1 || i == bs2))) keep_best(v.x, i, best, bi);
            if (!(sp >> 8) && !(first && (i + 1 == bs1 || i + 1 == bs2))) keep_best(v.y, i + 1, best, bi);
        }
    } else {
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            if (sup[i] || (first && (i == bs1 || i == bs2))) continue;
            keep_best(f(lg[i]), i, best, bi);
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffff, best, o);
        const int oi = __shfl_xor_sync(0xffffffff, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        best = l < nw ? sv[l] : -INFINITY;
        bi = l < nw ? si[l] : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffff, best, o);
            const int oi = __shfl_xor_sync(0xffffffff, bi, o);
            if (ov > best || (ov == best && oi < bi)) {
                best = ov;
                bi = oi;
            }
        }
        if (l == 0) {
            const int t = (done[b] || bi == 0x7fffffff) ? eos : bi;
            tok[b * maxT + p + 1] = t;
            if (t == eos) done[b] = 1;
        }
    }
}

__global__ void advance_kernel(int* ctr) {
    griddep_wait();
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    ctr[0] += 1;
}

// conv1 as a GEMM operand: X[g, t, ci * 3 + k] = mel[g, ci, t + k - 1] (kernels/whisper.cu:121-129)
__global__ void im2col1_kernel(const h16* __restrict__ mel, h16* __restrict__ X, long n, int nm) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int j = (int)(i % (3 * nm));
    const long r = i / (3 * nm);
    const int t = (int)(r % NFR), g = (int)(r / NFR), ci = j / 3, tt = t + j % 3 - 1;
    X[i] = (tt >= 0 && tt < NFR) ? mel[((long)g * nm + ci) * NFR + tt] : h(0.f);
}

// conv2 (stride 2) as a GEMM operand: X[g, t, ci * 3 + k] = h1[g, 2t + k - 1, ci] (kernels/whisper.cu:131-139)
__global__ void im2col2_kernel(const h16* __restrict__ h1, h16* __restrict__ X, long n, int d) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int j = (int)(i % (3 * d));
    const long r = i / (3 * d);
    const int t = (int)(r % TENC), g = (int)(r / TENC), ci = j / 3, tt = 2 * t + j % 3 - 1;
    X[i] = (tt >= 0 && tt < NFR) ? h1[((long)g * NFR + tt) * d + ci] : h(0.f);
}

// The same two operands with wide accesses (the engine's path; the kernels above serve shapes these do not take):
//   im2col1_tile_kernel  a CTA takes 64 frames of one clip, stages mel[g][all channels][t0 - 1 .. t0 + 64] in shared
//                        memory (the transpose: channel-major in, frame-major out) and writes its 64 rows of 3 nm
//                        values with 16-byte stores; 3 nm a multiple of 8
//   im2col2_vec_kernel   a thread takes 8 channels of one output row: three 16-byte loads (input rows 2t - 1, 2t,
//                        2t + 1) and three 16-byte stores of the 24 interleaved values; d a multiple of 8
constexpr int I1T = 64;  // frames per CTA of im2col1_tile_kernel

// grid (ceil(NFR / 64), clips), block 256, dynamic shared memory nm x 66 halves
__global__ void __launch_bounds__(256) im2col1_tile_kernel(const h16* __restrict__ mel, h16* __restrict__ X, int nm) {
    extern __shared__ h16 tile[];  // [channel][I1T + 2]: frames t0 - 1 .. t0 + I1T
    constexpr int W = I1T + 2;
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const int g = blockIdx.y, t0 = blockIdx.x * I1T;
    for (int i = threadIdx.x; i < nm * W; i += blockDim.x) {
        const int ci = i / W, tt = t0 - 1 + i % W;
        tile[i] = (tt >= 0 && tt < NFR) ? mel[((long)g * nm + ci) * NFR + tt] : h(0.f);
    }
    __syncthreads();
    const int cpr = 3 * nm / 8;  // 16-byte chunks per output row
    for (int i = threadIdx.x; i < I1T * cpr; i += blockDim.x) {
        const int tr = i / cpr, c = i % cpr, t = t0 + tr;
        if (t >= NFR) break;  // i grows with tr: every later i is past the clip too
        __align__(16) h16 v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int j = c * 8 + e;  // X column: channel j / 3, tap j % 3
            v[e] = tile[(j / 3) * W + tr + j % 3];
        }
        *reinterpret_cast<uint4*>(X + ((long)g * NFR + t) * 3 * nm + c * 8) = *reinterpret_cast<const uint4*>(v);
    }
}

__global__ void im2col2_vec_kernel(const h16* __restrict__ h1, h16* __restrict__ X, long rows, int d) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const int c8 = d / 8;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * c8) return;
    const long r = i / c8;
    const int c = (int)(i % c8), t = (int)(r % TENC);
    const long g = r / TENC;
    uint4 in[3];
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const int tt = 2 * t + k - 1;
        in[k] = (tt >= 0 && tt < NFR) ? *reinterpret_cast<const uint4*>(h1 + (g * NFR + tt) * d + c * 8)
                                      : make_uint4(0, 0, 0, 0);
    }
    const h16* a = reinterpret_cast<const h16*>(in);
    __align__(16) h16 o[24];
#pragma unroll
    for (int e = 0; e < 8; e++)
#pragma unroll
        for (int k = 0; k < 3; k++) o[e * 3 + k] = a[k * 8 + e];
    uint4* dst = reinterpret_cast<uint4*>(X + r * 3 * d + c * 24);
#pragma unroll
    for (int u = 0; u < 3; u++) dst[u] = reinterpret_cast<const uint4*>(o)[u];
}

// exact (erf) GELU over half2 pairs (kernels/whisper.cu:106-113)
__device__ __forceinline__ float gelu(float v) { return gelu_erf(v); }
__global__ void gelu_kernel(__half2* x, long n2) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n2) return;
    const float2 v = __half22float2(x[i]);
    x[i] = __floats2half2_rn(gelu(v.x), gelu(v.y));
}
// the same, 8 values per 16-byte access (n a multiple of 8, x 16-byte aligned)
__global__ void gelu8_kernel(uint4* x, long n8) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    uint4 u = x[i];
    __half2* h2 = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float2 v = __half22float2(h2[e]);
        h2[e] = __floats2half2_rn(gelu(v.x), gelu(v.y));
    }
    x[i] = u;
}

// x[r, c] += pos[r % period, c] (kernels/whisper.cu:115-119)
// the same, 8 values per thread with 16-byte accesses (n a multiple of 8): each sum in f32, rounded once, as above
__global__ void add_pos_vec_kernel(h16* x, const h16* __restrict__ pos, long rows, int n, int period) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const int n8 = n / 8;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * n8) return;
    const long r = i / n8;
    const int c = (int)(i % n8);
    uint4* px = reinterpret_cast<uint4*>(x + r * n + c * 8);
    uint4 xv = *px;
    const uint4 pv = *reinterpret_cast<const uint4*>(pos + (r % period) * n + c * 8);
    __half2* xh = reinterpret_cast<__half2*>(&xv);
    const __half2* ph = reinterpret_cast<const __half2*>(&pv);
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float2 a = __half22float2(xh[e]), b = __half22float2(ph[e]);
        xh[e] = __float22half2_rn(make_float2(a.x + b.x, a.y + b.y));
    }
    *px = xv;
}

__global__ void add_pos_kernel(h16* x, const h16* __restrict__ pos, long rows, int n, int period) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * n) return;
    const long r = i / n;
    const int c = (int)(i % n);
    x[i] = h(f(x[i]) + f(pos[(r % period) * n + c]));
}

// rows of an output with row stride ld <- bias (kernels/whisper.cu:92-97), 8 halves per thread
__global__ void fill_bias_kernel(h16* y, const h16* __restrict__ bias, long rows, int n, long ld) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x, n8 = n / 8;
    if (i >= rows * n8) return;
    const long r = i / n8;
    const int c = (int)(i % n8);
    reinterpret_cast<uint4*>(y + r * ld)[c] = reinterpret_cast<const uint4*>(bias)[c];
}

// bias of the head-contiguous cross k/v buffer: y[blk, j, c] = bias[blk * 64 + c] (kernels/whisper.cu:99-104)
__global__ void fill_bias_heads_kernel(h16* y, const h16* __restrict__ bias, long n8) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    reinterpret_cast<uint4*>(y)[i] =
        reinterpret_cast<const uint4*>(bias)[(i / ((long)TENC * HD / 8)) * (HD / 8) + i % (HD / 8)];
}

// seeded N(mean, std) in fp16: splitmix64 of (seed, index) -> two uniforms -> Box-Muller
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
__global__ void fill_normal_kernel(h16* p, long n, unsigned long long seed, float mean, float std) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t r = splitmix64(seed * 0x2545f4914f6cdd1dull + (uint64_t)i);
    const float u1 = ((uint32_t)(r >> 40) + 0.5f) * (1.f / 16777216.f);
    const float u2 = (uint32_t)(r & 0xffffff) * (1.f / 16777216.f);
    const float z = sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
    p[i] = h(mean + std * z);
}

__global__ void f32_to_f16_kernel(const float* __restrict__ src, h16* __restrict__ dst, long n) {
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = h(src[i]);
}

int launch_embed(const int* tok, const int* ctr, const void* emb, const void* pe, void* x, int batch, int maxT, int d,
                 cudaStream_t st) {
    return check_pdl(launch_pdl(embed_kernel, dim3(batch), dim3(128), 0, st, tok, ctr, (const h16*)emb, (const h16*)pe,
                                (h16*)x, maxT, d),
                     "embed");
}

// Row softmax in place for the unfused encoder attention (kernels/whisper.cu:141-166, launched by src/model.rs:588):
// each fp16 row of n <= 2048 scores becomes rh(exp(s - max) / sum) with fp32 arithmetic inside. One warp per row,
// eight rows per CTA, 8-byte loads and stores (rows of a multiple of 4 values start 8-byte aligned); the maximum and
// the sum are warp shuffles, so no barrier is taken. The sum associates differently from the reference kernel's
// 256-thread tree, so a probability may differ from it in the last fp16 bit.
constexpr int SM_VEC = 16;  // 4-value vectors per lane: n <= 32 * 4 * 16 = 2048
__global__ void __launch_bounds__(256) softmax_rows_kernel(h16* __restrict__ s, long rows, int n) {
    griddep_wait();  // launched as a programmatic dependent of the scores product
    const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    h16* r = s + row * n;
    const int nv = n >> 2;  // whole vectors; n % 4 values follow
    float v[SM_VEC][4];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < SM_VEC; k++) {
        const int i = lane + 32 * k;
        if (i < nv) {
            const uint2 u = reinterpret_cast<const uint2*>(r)[i];
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            v[k][0] = a.x, v[k][1] = a.y, v[k][2] = b.x, v[k][3] = b.y;
        } else {
            v[k][0] = v[k][1] = v[k][2] = v[k][3] = -INFINITY;
        }
        m = fmaxf(m, fmaxf(fmaxf(v[k][0], v[k][1]), fmaxf(v[k][2], v[k][3])));
    }
    const int tail = n - 4 * nv;  // at most 3 values, taken by lanes 0..2
    float tv = lane < tail ? f(r[4 * nv + lane]) : -INFINITY;
    m = fmaxf(m, tv);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffff, m, o));
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < SM_VEC; k++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            v[k][e] = v[k][e] == -INFINITY ? 0.f : expf(v[k][e] - m);
            sum += v[k][e];
        }
    tv = tv == -INFINITY ? 0.f : expf(tv - m);
    sum += tv;
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, o);
    const float inv = 1.f / sum;
#pragma unroll
    for (int k = 0; k < SM_VEC; k++) {
        const int i = lane + 32 * k;
        if (i < nv) {
            const __half2 a = __floats2half2_rn(v[k][0] * inv, v[k][1] * inv);
            const __half2 b = __floats2half2_rn(v[k][2] * inv, v[k][3] * inv);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&a);
            u.y = *reinterpret_cast<const uint32_t*>(&b);
            reinterpret_cast<uint2*>(r)[i] = u;
        }
    }
    if (lane < tail) r[4 * nv + lane] = h(tv * inv);
}

int launch_softmax_rows(void* s, long rows, int n, cudaStream_t st) {
    if (rows < 1 || n < 1 || n > 32 * 4 * SM_VEC) return fail("softmax_rows: 1 <= n <= 2048");
    if (((uintptr_t)s & 7) || (n % 4 && rows > 1)) return fail("softmax_rows: rows must start 8-byte aligned");
    return check_pdl(launch_pdl(softmax_rows_kernel, dim3(blocks(rows, 8)), dim3(256), 0, st, (h16*)s, rows, n),
                     "softmax_rows");
}

int launch_argmax_tok(const void* logits, int V, const unsigned char* sup, int* tok, int* done, const int* ctr,
                      int batch, int maxT, int prompt_len, int eos, int bs1, int bs2, cudaStream_t st) {
    return check_pdl(launch_pdl(argmax_kernel, dim3(batch), dim3(1024), 0, st, (const h16*)logits, V, sup, tok, done,
                                ctr, maxT, prompt_len, eos, bs1, bs2),
                     "argmax_tok");
}

int launch_advance(int* ctr, cudaStream_t st) {
    return check_pdl(launch_pdl(advance_kernel, dim3(1), dim3(1), 0, st, ctr),
                     "advance");
}

int launch_im2col1(const void* mel, void* X, long n, int nm, cudaStream_t st) {
    const long row = 3L * nm * NFR;  // one clip's operand
    if (nm > 0 && (3 * nm) % 8 == 0 && n % row == 0 && ((uintptr_t)X & 15) == 0 && nm * (I1T + 2) * 2 <= 48 * 1024)
        return check_pdl(launch_pdl(im2col1_tile_kernel, dim3((NFR + I1T - 1) / I1T, (unsigned)(n / row)), dim3(256),
                                    (size_t)nm * (I1T + 2) * 2, st, (const h16*)mel, (h16*)X, nm),
                         "im2col1");
    return check_pdl(launch_pdl(im2col1_kernel, dim3(blocks(n, 256)), dim3(256), 0, st, (const h16*)mel, (h16*)X, n,
                                nm),
                     "im2col1");
}

int launch_im2col2(const void* h1, void* X, long n, int d, cudaStream_t st) {
    if (d > 0 && d % 8 == 0 && n % (3L * d) == 0 && ((uintptr_t)h1 & 15) == 0 && ((uintptr_t)X & 15) == 0)
        return check_pdl(launch_pdl(im2col2_vec_kernel, dim3(blocks(n / 3 / 8, 256)), dim3(256), 0, st,
                                    (const h16*)h1, (h16*)X, n / (3L * d), d),
                         "im2col2");
    return check_pdl(launch_pdl(im2col2_kernel, dim3(blocks(n, 256)), dim3(256), 0, st, (const h16*)h1, (h16*)X, n, d),
                     "im2col2");
}

int launch_gelu(void* x, long n, cudaStream_t st) {
    if (n % 8 == 0 && ((uintptr_t)x & 15) == 0)
        return check_pdl(launch_pdl(gelu8_kernel, dim3(blocks(n / 8, 256)), dim3(256), 0, st, (uint4*)x, n / 8),
                         "gelu");
    return check_pdl(launch_pdl(gelu_kernel, dim3(blocks(n / 2, 256)), dim3(256), 0, st, (__half2*)x, n / 2),
                     "gelu");
}

int launch_add_pos(void* x, const void* pos, long rows, int n, int period, cudaStream_t st) {
    if (n % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)pos & 15) == 0)
        return check_pdl(launch_pdl(add_pos_vec_kernel, dim3(blocks(rows * (n / 8), 256)), dim3(256), 0, st, (h16*)x,
                                    (const h16*)pos, rows, n, period),
                         "add_pos");
    return check_pdl(launch_pdl(add_pos_kernel, dim3(blocks(rows * n, 256)), dim3(256), 0, st, (h16*)x, (const h16*)pos,
                                rows, n, period),
                     "add_pos");
}

int launch_fill_bias(void* y, const void* bias, long rows, int n, long ld, cudaStream_t st) {
    return check_pdl(launch_pdl(fill_bias_kernel, dim3(blocks(rows * (n / 8), 256)), dim3(256), 0, st, (h16*)y,
                                (const h16*)bias, rows, n, ld),
                     "fill_bias");
}

int launch_fill_bias_heads(void* y, const void* bias, long n8, cudaStream_t st) {
    return check_pdl(launch_pdl(fill_bias_heads_kernel, dim3(blocks(n8, 256)), dim3(256), 0, st, (h16*)y,
                                (const h16*)bias, n8),
                     "fill_bias_heads");
}

int launch_fill_normal(void* p, long n, unsigned long long seed, float mean, float std, cudaStream_t st) {
    return check_pdl(launch_pdl(fill_normal_kernel, dim3(blocks(n, 256)), dim3(256), 0, st, (h16*)p, n, seed, mean,
                                std),
                     "fill_normal");
}

int launch_f32_to_f16(const float* src, void* dst, long n, cudaStream_t st) {
    return check_pdl(launch_pdl(f32_to_f16_kernel, dim3(blocks(n, 256)), dim3(256), 0, st, src, (h16*)dst, n),
                     "f32_to_f16");
}

}  // namespace mmz
