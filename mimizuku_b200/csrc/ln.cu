// Residual add fused with LayerNorm, and plain LayerNorm, for sm_100a (kernels/whisper.cu:48-82 of the reference).
//
// One 128-thread block per row (a warp per row from 1024 rows on, below) with the reference's thread mapping: thread t
// owns the half2 pairs t, t + 128, ...
// (:51, :54-57), but keeps them in registers, so x (and d) are read from HBM once and x = h(x + d) and the normalised
// row are written once; the reference block reads x again for each of its passes. Memory traffic per row is the
// algorithmic minimum (4 x dim x 2 bytes for add_layernorm).
//
// The statistics use the reference's own reduction tree (per-thread sums in pair order, a warp xor butterfly, then
// the butterfly over the four warp sums, :22-33), and mean = sum / dim, rstd = rsqrtf(var / dim + eps) and the output
// expression are the reference's (:52, :58, :61), so the results are bit-identical to the reference kernel's.
#include "common.cuh"
#include "launch.h"
#include "ln_row.cuh"

namespace mmz {

// KP = pairs per thread = ceil(n2 / 128); grid (rows), block 128
template <int KP, bool ADD>
__global__ void __launch_bounds__(128) ln_kernel(__half2* x, const __half2* dd, const __half2* w, const __half2* bias,
                                                 __half2* out, int n2, float eps) {
    ln_block_row<KP, ADD>(x, dd, w, bias, out, blockIdx.x, n2, eps);
}

// The same computation with one warp per row, for many rows (the encoder's 12 000): lane l plays the reference's
// threads l, l + 32, l + 64 and l + 96 (one per warp of the 128-thread block), keeps each one's sum in pair order,
// runs the per-warp butterfly on each, and adds the four warp sums as (w0 + w2) + (w1 + w3): the reference's
// arithmetic without a barrier or shared memory. Every load of the row is issued before the first store.
template <int KP, bool ADD>
__global__ void __launch_bounds__(128, 8) ln_warp_kernel(__half2* x, const __half2* dd, const __half2* w,
                                                      const __half2* bias, __half2* out, int rows, int n2,
                                                      float eps) {
    griddep_wait();  // launched as a programmatic dependent: x and d come from the kernel before
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    const long row = (long)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int l = threadIdx.x & 31;
    __half2* xr = x + row * n2;
    const __half2* dr = ADD ? dd + row * n2 : nullptr;
    __half2 hx[4][KP], hd[4][KP];
#pragma unroll
    for (int k = 0; k < KP; k++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = l + 32 * q + 128 * k;  // thread l + 32 q of the reference's block, its k-th pair
            hx[q][k] = i < n2 ? xr[i] : __float2half2_rn(0.f);
            if (ADD) hd[q][k] = i < n2 ? dr[i] : __float2half2_rn(0.f);
        }
    float2 v[4][KP];
    float s[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        s[q] = 0.f;
#pragma unroll
        for (int k = 0; k < KP; k++) {
            const int i = l + 32 * q + 128 * k;
            v[q][k] = make_float2(0.f, 0.f);
            if (i < n2) {
                float2 a = __half22float2(hx[q][k]);
                if (ADD) {
                    const float2 b = __half22float2(hd[q][k]);
                    const __half2 y = __floats2half2_rn(a.x + b.x, a.y + b.y);
                    xr[i] = y;
                    a = __half22float2(y);
                }
                v[q][k] = a;
                s[q] += a.x + a.y;
            }
        }
    }
#pragma unroll
    for (int q = 0; q < 4; q++) s[q] = xor_sum(s[q]);
    const float mean = ((s[0] + s[2]) + (s[1] + s[3])) / (2 * n2);
    float var[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        var[q] = 0.f;
#pragma unroll
        for (int k = 0; k < KP; k++)
            if (l + 32 * q + 128 * k < n2)
                var[q] += (v[q][k].x - mean) * (v[q][k].x - mean) + (v[q][k].y - mean) * (v[q][k].y - mean);
        var[q] = xor_sum(var[q]);
    }
    const float rstd = rsqrtf(((var[0] + var[2]) + (var[1] + var[3])) / (2 * n2) + eps);
    __half2* yr = out + row * n2;
#pragma unroll
    for (int k = 0; k < KP; k++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = l + 32 * q + 128 * k;
            if (i < n2) {
                const float2 wv = __half22float2(w[i]), bv = __half22float2(bias[i]);
                yr[i] = __floats2half2_rn((v[q][k].x - mean) * rstd * wv.x + bv.x,
                                          (v[q][k].y - mean) * rstd * wv.y + bv.y);
            }
        }
}

// The warp-per-row computation with 16-byte accesses (rows of a multiple of 8 values): lane l plays the reference's
// threads 4l .. 4l + 3, whose k-th pairs are the four consecutive pairs 128 k + 4 l .. + 3, so one 16-byte load brings
// them and each of the four still sums its own pairs in k order. The reference's per-warp butterfly over its 32 lanes
// (xor 16, 8, 4, 2, 1) becomes, for thread 4l + j of warp l / 8: xor 4, 2, 1 across lanes, then the two in-register
// steps (v[j] + v[j ^ 2]) and (u[j] + u[j ^ 1]); the four warps' sums are then added as (w0 + w2) + (w1 + w3). Every
// addition has the reference's operands (IEEE addition commutes), so the statistics are bit-identical; a quarter of
// the memory instructions of ln_warp_kernel.
template <int KP, bool ADD>
__global__ void __launch_bounds__(128, 8) ln_vec_kernel(__half2* x, const __half2* dd, const __half2* w,
                                                     const __half2* bias, __half2* out, int rows, int n2, float eps) {
    griddep_wait();  // launched as a programmatic dependent: x and d come from the kernel before
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    const long row = (long)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int l = threadIdx.x & 31;
    uint4* xr = reinterpret_cast<uint4*>(x + row * n2);
    const uint4* dr = ADD ? reinterpret_cast<const uint4*>(dd + row * n2) : nullptr;
    const int nv = n2 >> 2;  // 16-byte vectors in the row
    uint4 hx[KP], hd[KP];
#pragma unroll
    for (int k = 0; k < KP; k++) {
        const int i = l + 32 * k;
        hx[k] = i < nv ? xr[i] : make_uint4(0, 0, 0, 0);
        if (ADD) hd[k] = i < nv ? dr[i] : make_uint4(0, 0, 0, 0);
    }
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < KP; k++) {
        if (l + 32 * k < nv) {
            __half2* y2 = reinterpret_cast<__half2*>(&hx[k]);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float2 a = __half22float2(y2[j]);
                if (ADD) {
                    const float2 b = __half22float2(reinterpret_cast<const __half2*>(&hd[k])[j]);
                    y2[j] = __floats2half2_rn(a.x + b.x, a.y + b.y);
                    a = __half22float2(y2[j]);
                }
                s[j] += a.x + a.y;
            }
            if (ADD) xr[l + 32 * k] = hx[k];
        }
    }
    // block_sum: the reference warp's butterfly, then (w0 + w2) + (w1 + w3)
    auto block_sum = [&](float (&v)[4]) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            v[j] += __shfl_xor_sync(0xffffffff, v[j], 4);
            v[j] += __shfl_xor_sync(0xffffffff, v[j], 2);
            v[j] += __shfl_xor_sync(0xffffffff, v[j], 1);
        }
        const float ws = (v[0] + v[2]) + (v[1] + v[3]);
        const float w0 = __shfl_sync(0xffffffff, ws, 0), w1 = __shfl_sync(0xffffffff, ws, 8);
        const float w2 = __shfl_sync(0xffffffff, ws, 16), w3 = __shfl_sync(0xffffffff, ws, 24);
        return (w0 + w2) + (w1 + w3);
    };
    const float mean = block_sum(s) / (2 * n2);
    float var[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < KP; k++)
        if (l + 32 * k < nv) {
            const __half2* y2 = reinterpret_cast<const __half2*>(&hx[k]);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float2 v = __half22float2(y2[j]);
                var[j] += (v.x - mean) * (v.x - mean) + (v.y - mean) * (v.y - mean);
            }
        }
    const float rstd = rsqrtf(block_sum(var) / (2 * n2) + eps);
    uint4* yr = reinterpret_cast<uint4*>(out + row * n2);
    const uint4* wr = reinterpret_cast<const uint4*>(w);
    const uint4* br = reinterpret_cast<const uint4*>(bias);
#pragma unroll
    for (int k = 0; k < KP; k++) {
        const int i = l + 32 * k;
        if (i < nv) {
            const uint4 wq = wr[i], bq = br[i];
            const __half2* y2 = reinterpret_cast<const __half2*>(&hx[k]);
            uint4 o;
            __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float2 v = __half22float2(y2[j]);
                const float2 wv = __half22float2(reinterpret_cast<const __half2*>(&wq)[j]);
                const float2 bv = __half22float2(reinterpret_cast<const __half2*>(&bq)[j]);
                o2[j] = __floats2half2_rn((v.x - mean) * rstd * wv.x + bv.x, (v.y - mean) * rstd * wv.y + bv.y);
            }
            yr[i] = o;
        }
    }
}

constexpr int LN_WARP_ROWS = 1024;  // from this many rows on, a warp per row

template <bool ADD>
static int launch_ln(void* x, const void* d, const void* w, const void* b, void* out, int rows, int dim, float eps,
                     cudaStream_t st) {
    if (rows < 1 || dim < 2 || dim % 2 || dim > 2048) return fail("layernorm: dim must be even and <= 2048");
    const int n2 = dim / 2, kp = (n2 + 127) / 128;
    auto X = (__half2*)x;
    auto D = (const __half2*)d;
    auto W = (const __half2*)w;
    auto B = (const __half2*)b;
    auto Y = (__half2*)out;
    cudaError_t e = cudaSuccess;
    const bool warp_rows = rows >= LN_WARP_ROWS && kp <= 5;  // larger rows would not fit in registers
    // 16-byte rows: every row (and w, b) starts 16-byte aligned when dim is a multiple of 8 and the bases are
    const bool vec = warp_rows && dim % 8 == 0 &&
                     !(((uintptr_t)x | (uintptr_t)d | (uintptr_t)w | (uintptr_t)b | (uintptr_t)out) & 15);
    const dim3 wgrid((rows + 3) / 4);
    switch (kp) {
#define MMZ_LN(K)                                                                                                   \
    case K:                                                                                                         \
        e = vec         ? launch_pdl(ln_vec_kernel<K, ADD>, wgrid, dim3(128), 0, st, X, D, W, B, Y, rows, n2, eps)  \
            : warp_rows ? launch_pdl(ln_warp_kernel<K, ADD>, wgrid, dim3(128), 0, st, X, D, W, B, Y, rows, n2, eps) \
                        : launch_pdl(ln_kernel<K, ADD>, dim3(rows), dim3(128), 0, st, X, D, W, B, Y, n2, eps);      \
        break;
        MMZ_LN(1) MMZ_LN(2) MMZ_LN(3) MMZ_LN(4) MMZ_LN(5) MMZ_LN(6) MMZ_LN(7) MMZ_LN(8)
#undef MMZ_LN
        default: return fail("layernorm: dim too large");
    }
    return check_pdl(e, ADD ? "add_layernorm" : "layernorm");
}

int launch_layernorm(const void* x, const void* w, const void* b, void* out, int rows, int dim, float eps,
                     cudaStream_t st) {
    return launch_ln<false>(const_cast<void*>(x), nullptr, w, b, out, rows, dim, eps, st);
}

int launch_add_layernorm(void* x, const void* d, const void* w, const void* b, void* out, int rows, int dim, float eps,
                         cudaStream_t st) {
    return launch_ln<true>(x, d, w, b, out, rows, dim, eps, st);
}

}  // namespace mmz
