// Token-timestamp cost on the GPU: the part of src/align.rs:6-43 that reduces the recorded alignment-head
// probabilities to the DTW cost matrix, for every clip of a batch at once, with the reference's arithmetic:
//   per head and column j: mean and standard deviation over the token rows (f32 sums in row order starting from -0.0,
//   rounded to fp16), z = rh(rh(w - mean) / sd) (0 where sd = 0);
//   per row: the width-7 median of z along the columns (reflect padding, f32 total order), summed over the heads in
//   order; cost = rh(sum / heads).
// The DTW itself (align.rs:44-106) is sequential per clip and stays on the host (times_from_cost), which now receives
// 4 bytes per (row, column) instead of the 2 x heads bytes of the raw probabilities.
//
// Every operation is an IEEE round-to-nearest intrinsic (no contraction, correctly rounded division and square root),
// so the cost matrix is bit-identical to the host restatement.
#include "common.cuh"
#include "launch.h"

namespace mmz {

constexpr int AL_THREADS = 128;
constexpr int AL_HALO = 3;                          // width 7
constexpr int AL_COLS = AL_THREADS - 2 * AL_HALO;   // 122 output columns per CTA
constexpr int AL_ROWS = 32;                         // token rows per chunk
constexpr int AL_MAXH = 16;                         // alignment heads

__device__ __forceinline__ int total_key(float x) {  // f32 total order as signed integer order
    const int k = __float_as_int(x);
    return k ^ (int)(((unsigned)(k >> 31)) >> 1);
}
__device__ __forceinline__ float key_value(int k) {  // the key map is its own inverse
    return __int_as_float(k ^ (int)(((unsigned)(k >> 31)) >> 1));
}
__device__ __forceinline__ void cx(int& a, int& b) {
    const int lo = min(a, b), hi = max(a, b);
    a = lo;
    b = hi;
}
// median of 7 keys: a 16-comparator sorting network (checked on every 0-1 input)
__device__ __forceinline__ int median7(int a0, int a1, int a2, int a3, int a4, int a5, int a6) {
    cx(a0, a6); cx(a2, a3); cx(a4, a5);
    cx(a0, a2); cx(a1, a4); cx(a3, a6);
    cx(a0, a1); cx(a2, a5); cx(a3, a4);
    cx(a1, a2); cx(a4, a6);
    cx(a2, a3); cx(a4, a5);
    cx(a1, a2); cx(a3, a4); cx(a5, a6);
    return a3;
}

// grid (ceil(1500 / 122), clips), block 128. align [clips][max_t][na][1500] fp16: token row i of clip s is position
// np + i; rows[s] token rows (at most max_t - np are read) and cols[s] frame columns (at most 1500) per clip.
// cost [clips][max_t][1500] f32, row i at index i.
__global__ void __launch_bounds__(AL_THREADS) align_cost_kernel(const h16* __restrict__ align,
                                                                const int* __restrict__ rows_of,
                                                                const int* __restrict__ cols_of, int np, int mt,
                                                                int na, float* __restrict__ cost) {
    __shared__ float mean_s[AL_MAXH][AL_THREADS], sd_s[AL_MAXH][AL_THREADS];
    __shared__ float zt[AL_ROWS][AL_THREADS];
    griddep_wait();  // launched as a programmatic dependent of the previous kernel
    const int s = blockIdx.y, t = threadIdx.x;
    const int rows = min(rows_of[s], mt - np), cols = min(cols_of[s], TENC);
    const int j0 = blockIdx.x * AL_COLS;
    if (rows <= 0 || cols <= 0 || j0 >= cols) return;
    // the column whose z-scores this thread computes: output column j0 + t - 3, reflected at the clip's edges
    int jz = j0 + t - AL_HALO;
    if (jz < 0) jz = -jz;
    else if (jz >= cols) jz = 2 * (cols - 1) - jz;
    const bool zcol = jz >= 0 && jz < cols;  // false only for halo columns no output of a short clip reads
    if (!zcol) jz = 0;
    const h16* base = align + ((size_t)s * mt + np) * na * TENC + jz;  // (row i, head a) at base[(i * na + a) * 1500]
    const float frows = (float)rows;
    for (int a = 0; a < na; a++) {
        float sum = -0.0f;  // Rust's f32 Sum starts from -0.0
        for (int i = 0; i < rows; i++) sum = __fadd_rn(sum, f(base[((size_t)i * na + a) * TENC]));
        const float mean_f = __fdiv_rn(sum, frows);
        float vs = -0.0f;
        for (int i = 0; i < rows; i++) {
            const float d = __fsub_rn(f(base[((size_t)i * na + a) * TENC]), mean_f);
            vs = __fadd_rn(vs, __fmul_rn(d, d));
        }
        mean_s[a][t] = rh(mean_f);
        sd_s[a][t] = rh(__fsqrt_rn(__fdiv_rn(vs, frows)));
    }
    const bool out_col = t >= AL_HALO && t < AL_HALO + AL_COLS && j0 + t - AL_HALO < cols;
    for (int i0 = 0; i0 < rows; i0 += AL_ROWS) {
        const int nr = min(AL_ROWS, rows - i0);
        float acc[AL_ROWS];
#pragma unroll
        for (int r = 0; r < AL_ROWS; r++) acc[r] = 0.f;
        for (int a = 0; a < na; a++) {
            const float mean = mean_s[a][t], sd = sd_s[a][t];
            for (int r = 0; r < nr; r++) {
                const float w = f(base[((size_t)(i0 + r) * na + a) * TENC]);
                zt[r][t] = sd > 0.f ? rh(__fdiv_rn(rh(__fsub_rn(w, mean)), sd)) : 0.f;
            }
            __syncthreads();
            if (out_col) {
#pragma unroll
                for (int r = 0; r < AL_ROWS; r++) {
                    if (r < nr) {
                        const float* z = &zt[r][t - AL_HALO];
                        const float v = cols > AL_HALO ? key_value(median7(total_key(z[0]), total_key(z[1]),
                                                                           total_key(z[2]), total_key(z[3]),
                                                                           total_key(z[4]), total_key(z[5]),
                                                                           total_key(z[6])))
                                                       : z[AL_HALO];
                        acc[r] = __fadd_rn(acc[r], v);
                    }
                }
            }
            __syncthreads();
        }
        if (out_col) {
            float* dst = cost + ((size_t)s * mt + i0) * TENC + j0 + t - AL_HALO;
#pragma unroll
            for (int r = 0; r < AL_ROWS; r++)
                if (r < nr) dst[(size_t)r * TENC] = rh(__fdiv_rn(acc[r], (float)na));
        }
    }
}

int launch_align_cost(const void* align, const int* rows, const int* cols, int n, int np, int mt, int na, void* cost,
                      cudaStream_t st) {
    if (n < 1 || np < 0 || mt < 1 || np >= mt || na < 1 || na > AL_MAXH)
        return fail("align_cost: bad shape (1 <= heads <= 16, 0 <= np < max_t)");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    dim3 grid((TENC + AL_COLS - 1) / AL_COLS, n);
    return check_pdl(launch_pdl(align_cost_kernel, grid, dim3(AL_THREADS), 0, st, (const h16*)align, rows, cols, np, mt,
                                na, (float*)cost),
                     "align_cost");
}

}  // namespace mmz
