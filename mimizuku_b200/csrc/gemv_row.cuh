// The decoder's linear layers at m <= 8 sequences (src/gpu.rs:211-228: the reference's host uses its gemv kernels,
// kernels/whisper.cu:501-567, instead of cuBLAS up to 8 rows), shared by the library (gemv.cu) and the
// name-compatible image (dropin.cu): y[m][n] = rh(x[m] . W[n] + bias[n]).
//
// The arithmetic is the reference kernels', so the results are equal bit for bit: the output of column n comes from
// the 32 lanes of one warp, lane l accumulating the 8-element groups k = 256 i + 8 l .. 256 i + 8 l + 7 in increasing
// i with one fused multiply-add per element in order, then the xor butterfly over the lanes, then the bias added in
// fp32 before the single rounding. What is this library's is the data movement: a warp issues all of a block's
// weight loads (16 bytes per lane per column and group, a whole 512-byte row segment per warp instruction) before its
// arithmetic, the first block's before the wait for the kernel before (the weights do not depend on it), and x (at
// most 8 rows) is read through the read-only cache instead of being staged in shared memory behind block barriers.
// grid ceil(N / 32), block 256: warp w of block b owns the columns 32 b + 4 w .. + 3.
#pragma once
#include "common.cuh"

namespace mmz {
namespace gv {
constexpr int COLS = 4;   // columns per warp
constexpr int WARPS = 8;  // warps per block
constexpr int GB = 5;     // 8-element groups per lane per block of loads (K = 1280 in one block)
}  // namespace gv

template <int MR>
__device__ __forceinline__ void gemv_rows(const h16* __restrict__ x, int ldx, const h16* __restrict__ W,
                                          h16* __restrict__ y, int ldy, int M, int N, int K,
                                          const h16* __restrict__ bias) {
    using namespace gv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * WARPS + warp) * COLS;
    const int ng = K > 8 * lane ? (K - 8 * lane + 255) / 256 : 0;  // this lane's groups (K a multiple of 8)
    float acc[COLS][MR];
#pragma unroll
    for (int c = 0; c < COLS; c++)
#pragma unroll
        for (int m = 0; m < MR; m++) acc[c][m] = 0.f;
    uint4 wb[GB][COLS];
    auto load = [&](int i0) {
#pragma unroll
        for (int g = 0; g < GB; g++)
#pragma unroll
            for (int c = 0; c < COLS; c++) {
                const int i = i0 + g;
                wb[g][c] = i < ng && n0 + c < N
                               ? __ldg(reinterpret_cast<const uint4*>(W + (long)(n0 + c) * K + 256 * i + 8 * lane))
                               : make_uint4(0, 0, 0, 0);
            }
    };
    load(0);
    griddep_wait();  // x comes from the kernel before
    for (int i0 = 0; i0 < ng; i0 += GB) {
        if (i0 > 0) load(i0);
#pragma unroll
        for (int g = 0; g < GB; g++) {
            const int i = i0 + g;
            if (i >= ng) break;
            float w[COLS][8];
#pragma unroll
            for (int c = 0; c < COLS; c++) {
                const __half2* p = reinterpret_cast<const __half2*>(&wb[g][c]);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 v = __half22float2(p[j]);
                    w[c][2 * j] = v.x;
                    w[c][2 * j + 1] = v.y;
                }
            }
#pragma unroll
            for (int m = 0; m < MR; m++) {
                if (m < M) {
                    const uint4 u = __ldg(reinterpret_cast<const uint4*>(x + (long)m * ldx + 256 * i + 8 * lane));
                    const __half2* p = reinterpret_cast<const __half2*>(&u);
                    float xf[8];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float2 v = __half22float2(p[j]);
                        xf[2 * j] = v.x;
                        xf[2 * j + 1] = v.y;
                    }
#pragma unroll
                    for (int c = 0; c < COLS; c++)
#pragma unroll
                        for (int j = 0; j < 8; j++) acc[c][m] = __fmaf_rn(w[c][j], xf[j], acc[c][m]);
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < COLS; c++)
#pragma unroll
        for (int m = 0; m < MR; m++) {
            float v = acc[c][m];
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
            if (lane == m && m < M && n0 + c < N) y[(long)m * ldy + n0 + c] = h(bias ? v + f(bias[n0 + c]) : v);
        }
}

}  // namespace mmz
