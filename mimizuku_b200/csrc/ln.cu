// Residual add fused with LayerNorm, and plain LayerNorm, for sm_100a (kernels/whisper.cu:48-82 of the reference).
//
// One warp owns a row and keeps it in registers: x (and d) are read from HBM once, x = h(x + d) is written once and
// the normalised row once, where the reference block re-reads x for each of its three passes. Memory traffic per
// row is therefore the algorithmic minimum (4 x dim x 2 bytes for add_layernorm).
//
// The statistics reproduce the reference's 128-thread block reduction bit for bit: lane l of the warp plays the
// reference threads l, l+32, l+64, l+96 (its four "virtual warps"), each virtual thread accumulates the half2 pairs
// t, t+128, ... in order (:51, :54-57), each virtual warp is reduced with the same xor butterfly (:24), and the four
// warp sums combine as (w0 + w2) + (w1 + w3), which is what the reference's second butterfly over part[0..3]
// computes (:29-31). mean = sum / dim, rstd = rsqrtf(var / dim + eps) and the output expression are the
// reference's own (:52, :58, :61).
#include "common.cuh"
#include "launch.h"

namespace mmz {

__device__ __forceinline__ float xor_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
    return v;
}

// KP = pairs per virtual thread = ceil(n2 / 128); rows of n2 half2 pairs; ADD: x = h(x + d) first.
// out may alias d (the reference engine normalises into the buffer it added from, model.rs:533, :607), so no
// pointer is declared __restrict__; every row is read completely before any of it is written.
template <int KP, bool ADD>
__global__ void __launch_bounds__(128) ln_kernel(__half2* x, const __half2* dd, const __half2* w, const __half2* bias,
                                                 __half2* out, int rows, int n2, float eps) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    __half2* xr = x + (long)row * n2;
    const __half2* dr = ADD ? dd + (long)row * n2 : nullptr;
    float2 v[4][KP];
    float s[4];
#pragma unroll
    for (int vw = 0; vw < 4; vw++) {
        s[vw] = 0.f;
#pragma unroll
        for (int k = 0; k < KP; k++) {
            const int i = 32 * vw + lane + 128 * k;
            v[vw][k] = make_float2(0.f, 0.f);
            if (i < n2) {
                float2 a = __half22float2(xr[i]);
                if (ADD) {
                    float2 b = __half22float2(dr[i]);
                    __half2 y = __floats2half2_rn(a.x + b.x, a.y + b.y);
                    xr[i] = y;
                    a = __half22float2(y);
                }
                v[vw][k] = a;
                s[vw] += a.x + a.y;
            }
        }
    }
#pragma unroll
    for (int vw = 0; vw < 4; vw++) s[vw] = xor_sum(s[vw]);
    const float mean = ((s[0] + s[2]) + (s[1] + s[3])) / (2 * n2);
#pragma unroll
    for (int vw = 0; vw < 4; vw++) {
        s[vw] = 0.f;
#pragma unroll
        for (int k = 0; k < KP; k++) {
            const int i = 32 * vw + lane + 128 * k;
            if (i < n2) {
                float2 a = v[vw][k];
                s[vw] += (a.x - mean) * (a.x - mean) + (a.y - mean) * (a.y - mean);
            }
        }
    }
#pragma unroll
    for (int vw = 0; vw < 4; vw++) s[vw] = xor_sum(s[vw]);
    const float rstd = rsqrtf(((s[0] + s[2]) + (s[1] + s[3])) / (2 * n2) + eps);
    __half2* yr = out + (long)row * n2;
#pragma unroll
    for (int vw = 0; vw < 4; vw++)
#pragma unroll
        for (int k = 0; k < KP; k++) {
            const int i = 32 * vw + lane + 128 * k;
            if (i < n2) {
                float2 a = v[vw][k], wv = __half22float2(w[i]), bv = __half22float2(bias[i]);
                yr[i] = __floats2half2_rn((a.x - mean) * rstd * wv.x + bv.x, (a.y - mean) * rstd * wv.y + bv.y);
            }
        }
}

template <bool ADD>
static int launch_ln(void* x, const void* d, const void* w, const void* b, void* out, int rows, int dim, float eps,
                     cudaStream_t st) {
    if (rows < 1 || dim < 2 || dim % 2 || dim > 2048) return fail("layernorm: dim must be even and <= 2048");
    const int n2 = dim / 2, kp = (n2 + 127) / 128;
    dim3 grid((rows + 3) / 4);
    auto X = (__half2*)x;
    auto D = (const __half2*)d;
    auto W = (const __half2*)w;
    auto B = (const __half2*)b;
    auto Y = (__half2*)out;
    switch (kp) {
#define MMZ_LN(K) \
    case K: ln_kernel<K, ADD><<<grid, 128, 0, st>>>(X, D, W, B, Y, rows, n2, eps); break;
        MMZ_LN(1) MMZ_LN(2) MMZ_LN(3) MMZ_LN(4) MMZ_LN(5) MMZ_LN(6) MMZ_LN(7) MMZ_LN(8)
#undef MMZ_LN
        default: return fail("layernorm: dim too large");
    }
    return check_launch(ADD ? "add_layernorm" : "layernorm");
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
