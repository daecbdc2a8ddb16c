// The 128-thread-block row of the layer norm, shared by ln.cu and the name-compatible image (dropin.cu): thread t owns
// the half2 pairs t, t + 128, ... of its row (kernels/whisper.cu:51, :54-57) and keeps them in registers, the
// statistics use the reference's reduction tree (per-thread sums in pair order, a warp xor butterfly, then the
// butterfly over the four warp sums, :22-33), and mean, rstd and the output expression are the reference's (:52, :58,
// :61): the results equal the reference kernel's bit for bit.
#pragma once
#include "common.cuh"

namespace mmz {

__device__ __forceinline__ float xor_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
    return v;
}

// block_sum of kernels/whisper.cu:22-33 for a 128-thread block: per-warp butterfly, then the butterfly over the
// four warp sums, which is (w0 + w2) + (w1 + w3) (the other lanes add zeros); `part` is not reused within a launch,
// so one barrier suffices
__device__ __forceinline__ float block_sum128(float v, float* part) {
    v = xor_sum(v);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
    __syncthreads();
    return (part[0] + part[2]) + (part[1] + part[3]);
}

// One row of n2 half2 pairs by a 128-thread block. KP = pairs per thread = ceil(n2 / 128); ADD: x = h(x + d) first.
// out may alias d (the reference engine normalises into the buffer it added from, model.rs:533, :607), so no
// pointer is declared __restrict__; a thread reads every element it will write before the first barrier.
template <int KP, bool ADD>
__device__ __forceinline__ void ln_block_row(__half2* x, const __half2* dd, const __half2* w, const __half2* bias,
                                             __half2* out, long row, int n2, float eps) {
    __shared__ float part[2][4];
    const int t = threadIdx.x;
    __half2 hw[KP], hb[KP];  // the parameters do not come from the kernel before: read them first
#pragma unroll
    for (int k = 0; k < KP; k++) {
        const int i = t + 128 * k;
        hw[k] = i < n2 ? w[i] : __float2half2_rn(0.f);
        hb[k] = i < n2 ? bias[i] : __float2half2_rn(0.f);
    }
    griddep_wait();  // launched as a programmatic dependent: x and d come from the kernel before
    griddep_launch_dependents();  // this kernel has waited: the next one may be scheduled (it waits for this one)
    __half2* xr = x + row * n2;
    const __half2* dr = ADD ? dd + row * n2 : nullptr;
    __half2 hx[KP], hd[KP];
#pragma unroll
    for (int k = 0; k < KP; k++) {
        const int i = t + 128 * k;
        hx[k] = i < n2 ? xr[i] : __float2half2_rn(0.f);
        if (ADD) hd[k] = i < n2 ? dr[i] : __float2half2_rn(0.f);
    }
    float2 v[KP];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < KP; k++) {
        const int i = t + 128 * k;
        v[k] = make_float2(0.f, 0.f);
        if (i < n2) {
            float2 a = __half22float2(hx[k]);
            if (ADD) {
                const float2 b = __half22float2(hd[k]);
                const __half2 y = __floats2half2_rn(a.x + b.x, a.y + b.y);
                xr[i] = y;
                a = __half22float2(y);
            }
            v[k] = a;
            s += a.x + a.y;
        }
    }
    const float mean = block_sum128(s, part[0]) / (2 * n2);
    float var = 0.f;
#pragma unroll
    for (int k = 0; k < KP; k++)
        if (t + 128 * k < n2) var += (v[k].x - mean) * (v[k].x - mean) + (v[k].y - mean) * (v[k].y - mean);
    const float rstd = rsqrtf(block_sum128(var, part[1]) / (2 * n2) + eps);
    __half2* yr = out + row * n2;
#pragma unroll
    for (int k = 0; k < KP; k++) {
        const int i = t + 128 * k;
        if (i < n2) {
            const float2 wv = __half22float2(hw[k]), bv = __half22float2(hb[k]);
            yr[i] = __floats2half2_rn((v[k].x - mean) * rstd * wv.x + bv.x, (v[k].y - mean) * rstd * wv.y + bv.y);
        }
    }
}

}  // namespace mmz
