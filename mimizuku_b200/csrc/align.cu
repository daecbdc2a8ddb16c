// Token-timestamp cost on the GPU: the part of src/align.rs:6-43 that reduces the recorded alignment-head
// probabilities to the DTW cost matrix, for every clip of a batch at once, with the reference's arithmetic:
//   per head and column j: mean and standard deviation over the token rows (f32 sums in row order starting from -0.0,
//   rounded to fp16), z = rh(rh(w - mean) / sd) (0 where sd = 0);
//   per row: the width-7 median of z along the columns (reflect padding, f32 total order), summed over the heads in
//   order; cost = rh(sum / heads).
// Then the DTW over -cost and the start time of each token row (align.rs:44-106), one CTA per clip: the cost table is
// filled along anti-diagonals (thread t owns row t + 1 and is t steps behind the thread above it, one block barrier
// per step), the moves are kept as 2-bit codes in shared memory (at most 512 rows x 94 words), and one thread walks
// the path back and forth as the reference does. Only the times (4 bytes per token) go back to the host.
//
// Every operation is an IEEE round-to-nearest intrinsic (no contraction, correctly rounded division and square root),
// so the cost matrix and the times are bit-identical to the host restatement.
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

constexpr int DT_THREADS = 512;            // token rows per clip at most
constexpr int DT_WPR = (TENC + 15) / 16;   // trace words per row: 16 two-bit moves each

__device__ __forceinline__ float pick4(const float4& v, int k) {
    return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// grid (clips), block 512, dynamic shared memory dtw_smem_bytes(mt). cost [clips][mt][1500] f32 as align_cost writes
// it; times [clips][mt]: entry i < rows[s] the start time of token row i, 0 past them (all 0 when cols[s] = 0).
__global__ void __launch_bounds__(DT_THREADS, 1) dtw_times_kernel(const float* __restrict__ cost,
                                                                  const int* __restrict__ rows_of,
                                                                  const int* __restrict__ cols_of, int mt,
                                                                  float* __restrict__ times) {
    extern __shared__ uint32_t tr[];                // [rows][DT_WPR] moves, then the path
    __shared__ float edge[2][DT_THREADS / 32];      // the last lane's cost per warp, by step parity
    griddep_wait();  // launched as a programmatic dependent of align_cost_kernel
    const int s = blockIdx.x, t = threadIdx.x, lane = t & 31, w = t >> 5;
    const int rows = min(rows_of[s], mt), cols = min(cols_of[s], TENC);
    float* out = times + (size_t)s * mt;
    if (rows <= 0 || cols <= 0) {  // align.rs:45-47 (no rows: nothing is timed)
        for (int i = t; i < mt; i += DT_THREADS) out[i] = 0.f;
        return;
    }
    // align.rs:66-85: cost[i][j] = -x[i-1][j-1] + min(diag, up, left), ties to the later of (diag, up, left);
    // row 0 is inf past column 0, column 0 inf past row 0, cost[0][0] = 0
    const bool live = t < rows;
    const float4* crow = reinterpret_cast<const float4*>(cost + ((size_t)s * mt + t) * TENC);
    float4 cv = make_float4(0.f, 0.f, 0.f, 0.f), nv = live ? __ldg(crow) : cv;
    float left = INFINITY, diag = t == 0 ? 0.f : INFINITY, cur = INFINITY;
    uint32_t bits = 0;
    const int steps = rows + cols - 1;
    for (int step = 0; step < steps; step++) {
        const int j = step - t + 1;  // the column of row t + 1 at this step
        float up = __shfl_up_sync(0xffffffff, cur, 1);
        if (lane == 0) up = w > 0 ? edge[(step + 1) & 1][w - 1] : INFINITY;
        if (live && j >= 1 && j <= cols) {
            const int k = (j - 1) & 3;
            if (k == 0) {
                cv = nv;
                if (j + 3 < cols) nv = __ldg(crow + ((j - 1) >> 2) + 1);
            }
            float c;
            uint32_t mv;
            if (diag < up && diag < left) {
                c = diag;
                mv = 0;
            } else if (up < diag && up < left) {
                c = up;
                mv = 1;
            } else {
                c = left;
                mv = 2;
            }
            // (float)((double)a + (double)b) of two floats is their correctly rounded f32 sum
            cur = __fadd_rn(-pick4(cv, k), c);
            left = cur;
            diag = up;
            bits |= mv << (2 * ((j - 1) & 15));
            if (((j - 1) & 15) == 15 || j == cols) {
                tr[t * DT_WPR + ((j - 1) >> 4)] = bits;
                bits = 0;
            }
        }
        if (lane == 31) edge[step & 1][w] = cur;
        __syncthreads();
    }
    if (t != 0) return;
    // align.rs:86-106: the path from (rows, cols) back to (0, 0); row 0 moves left, column 0 moves up
    short* ptext = reinterpret_cast<short*>(tr + rows * DT_WPR);
    short* ptime = ptext + rows + cols;
    int i = rows, j = cols, n = 0;
    while (i > 0 || j > 0) {
        ptext[n] = (short)(i - 1);
        ptime[n] = (short)(j - 1);
        n++;
        const uint32_t mv = i == 0 ? 2u : j == 0 ? 1u : (tr[(i - 1) * DT_WPR + ((j - 1) >> 4)] >> (2 * ((j - 1) & 15))) & 3u;
        if (mv == 0) {
            i--;
            j--;
        } else if (mv == 1) {
            i--;
        } else {
            j--;
        }
    }
    // align.rs:48-62, in the path's forward order (index n - 1 first): a row's time is that of its first entry
    int k_out = 0;
    for (int k = n - 1; k >= 0 && k_out < rows; k--)
        if (k == n - 1 || ptext[k] != ptext[k + 1]) out[k_out++] = __double2float_rn((double)ptime[k] * 0.02);
    const float last = k_out > 0 ? out[k_out - 1] : 0.f;
    for (; k_out < mt; k_out++) out[k_out] = k_out < rows ? last : 0.f;
}

static size_t dtw_smem_bytes(int mt) { return (size_t)mt * DT_WPR * 4 + (size_t)(mt + TENC) * 2 * 2; }

int launch_dtw_times(const void* cost, const int* rows, const int* cols, int n, int mt, void* times, cudaStream_t st) {
    if (n < 1 || mt < 1 || mt > DT_THREADS) return fail("dtw_times: bad shape (1 <= max_t <= 512)");
    if ((uintptr_t)cost & 15) return fail("dtw_times: cost must be 16-byte aligned");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    return check_pdl(launch_pdl(dtw_times_kernel, dim3(n), dim3(DT_THREADS), dtw_smem_bytes(mt), st,
                                (const float*)cost, rows, cols, mt, (float*)times),
                     "dtw_times");
}

void init_align_attrs() {
    cudaFuncSetAttribute(dtw_times_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dtw_smem_bytes(DT_THREADS));
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
