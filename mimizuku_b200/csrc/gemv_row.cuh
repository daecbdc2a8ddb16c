// The decoder's linear layers at m <= 8 sequences (src/gpu.rs:211-228: the reference's host uses its gemv kernels,
// kernels/whisper.cu:501-567, instead of cuBLAS up to 8 rows): y[m][n] = rh(x[m] . W[n] + bias[n]). This header has
// what both of this library's forms share - the sums and the lane reduction - and the register-streaming form, which
// the name-compatible image (dropin.cu) exports with the reference's launch geometry and which the library (gemv.cu)
// falls back to when its shared-memory ring does not fit.
//
// The arithmetic is the reference kernels', so the results are equal bit for bit: the output of column n comes from
// the 32 lanes of one warp, lane l accumulating the 8-element groups k = 256 i + 8 l .. 256 i + 8 l + 7 in increasing
// i with one fused multiply-add per element in order, then the xor butterfly over offsets 16, 8, 4, 2, 1, then the
// bias added in fp32 before the single rounding. What is this library's:
//   - two sequences share one fp32x2 fused multiply-add (each half rounded on its own: the scalar sums);
//   - the lane reduction halves the values at each butterfly level (halving_reduce): the same tree of additions,
//     31 shuffles for 32 sums instead of 160;
//   - in the register form, a warp issues GB groups of weight loads for its 4 columns (16 bytes per lane, a whole
//     512-byte row segment per warp instruction) before their arithmetic, the first ones before the wait for the
//     kernel before (the weights do not depend on it), and reads x (at most 8 rows, written by the kernel before)
//     from L2 (ld.global.cg, not the non-coherent path: this kernel may be resident before x is written) instead of
//     staging it in shared memory behind block barriers.
// Register form: grid ceil(N / 32), block 256: warp w of block b owns the columns 32 b + 4 w .. + 3.
#pragma once
#include "common.cuh"

namespace mmz {
namespace gv {
constexpr int COLS = 4;   // columns per warp
constexpr int WARPS = 8;  // warps per block
constexpr int GB = 5;     // 8-element groups per lane per batch of weight loads (k = 1280 in one batch)
}  // namespace gv

__host__ __device__ constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

// The xor butterfly over the warp for NV values per lane, halving the values at each level: at offset o a lane keeps
// the half of its values selected by its bit o and adds its partner's copy of that half, so every value still gets
// v(l) + v(l ^ o) at every level, in the butterfly's order. After log2 NV levels the lane holds one value, the full
// sum of value index lane >> (5 - log2 NV) once the remaining levels have run on it.
template <int NV>
__device__ __forceinline__ float halving_reduce(float (&v)[NV], int lane) {
    static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "power of two up to 32");
    int o = 16;
#pragma unroll
    for (int half = NV / 2; half >= 1; half /= 2, o >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int j = 0; j < half; j++) {
            const float send = up ? v[j] : v[j + half];
            const float keep = up ? v[j + half] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffff, send, o);
        }
    }
    float r = v[0];
    for (; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffff, r, o);
    return r;
}

// w[c][0..7] (fp32) times the 8 x values of the group at xr(m) (a uint4 of 8 halves of row m), accumulated into
// acc[c][m] in element order; MR >= 2 pairs the rows (m, m + 1) in fp32x2 FMAs. Rows m >= M are neither read nor used.
template <int MR, int COLS, typename XRow>
__device__ __forceinline__ void gemv_group(const float (&w)[COLS][8], XRow xr, int M, float (&acc)[COLS][MR]) {
    if constexpr (MR == 1) {
        const uint4 u = xr(0);
        const __half2* p = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 f2 = __half22float2(p[j]);
#pragma unroll
            for (int c = 0; c < COLS; c++) {
                acc[c][0] = __fmaf_rn(w[c][2 * j], f2.x, acc[c][0]);
                acc[c][0] = __fmaf_rn(w[c][2 * j + 1], f2.y, acc[c][0]);
            }
        }
    } else {
        // every row pair's x first, then the products with j outermost, so that the COLS x MR / 2 accumulator pairs
        // form independent chains side by side (each still takes its 8 elements in order); rows m >= M read as zero
        float2 xp[MR / 2][8];
#pragma unroll
        for (int mp = 0; mp < MR / 2; mp++) {
            const uint4 z = make_uint4(0, 0, 0, 0);
            const uint4 u0 = 2 * mp < M ? xr(2 * mp) : z;
            const uint4 u1 = 2 * mp + 1 < M ? xr(2 * mp + 1) : z;
            const __half2* p0 = reinterpret_cast<const __half2*>(&u0);
            const __half2* p1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float2 a = __half22float2(p0[j]), b = __half22float2(p1[j]);
                xp[mp][2 * j] = make_float2(a.x, b.x);
                xp[mp][2 * j + 1] = make_float2(a.y, b.y);
            }
        }
        float2 a2[COLS][MR / 2];
#pragma unroll
        for (int c = 0; c < COLS; c++)
#pragma unroll
            for (int mp = 0; mp < MR / 2; mp++) a2[c][mp] = make_float2(acc[c][2 * mp], acc[c][2 * mp + 1]);
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int c = 0; c < COLS; c++) {
                const float2 wd = make_float2(w[c][j], w[c][j]);
#pragma unroll
                for (int mp = 0; mp < MR / 2; mp++) a2[c][mp] = ffma2(wd, xp[mp][j], a2[c][mp]);
            }
#pragma unroll
        for (int c = 0; c < COLS; c++)
#pragma unroll
            for (int mp = 0; mp < MR / 2; mp++) {
                acc[c][2 * mp] = a2[c][mp].x;
                acc[c][2 * mp + 1] = a2[c][mp].y;
            }
    }
}

// the 8 halves of a uint4 as fp32
__device__ __forceinline__ void halves8(const uint4& u, float (&o)[8]) {
    const __half2* p = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 f2 = __half22float2(p[j]);
        o[2 * j] = f2.x;
        o[2 * j + 1] = f2.y;
    }
}

// the lane reduction of a warp's COLS x MR sums and their store: columns n0 .. n0 + COLS - 1, rows m < M; gelu: the
// rounded value then goes through gelu_inplace's GELU and is rounded again (the fc1 product and the GELU after it,
// model.rs:708-709, in one kernel)
template <int MR, int COLS>
__device__ __forceinline__ void gemv_store(const float (&acc)[COLS][MR], int lane, int n0, h16* __restrict__ y,
                                           int ldy, int M, int N, const h16* __restrict__ bias, bool gelu = false) {
    float vals[COLS * MR];
#pragma unroll
    for (int c = 0; c < COLS; c++)
#pragma unroll
        for (int m = 0; m < MR; m++) vals[c * MR + m] = acc[c][m];
    const float r = halving_reduce<COLS * MR>(vals, lane);
    constexpr int LOGV = ilog2(COLS * MR);
    const int idx = lane >> (5 - LOGV), c = idx / MR, m = idx % MR;
    const bool lead = (lane & ((32 / (COLS * MR)) - 1)) == 0;  // one lane per value
    if (lead && m < M && n0 + c < N) {
        h16 v = h(bias ? r + f(bias[n0 + c]) : r);
        if (gelu) v = h(gelu_erf(f(v)));
        y[(long)m * ldy + n0 + c] = v;
    }
}

template <int MR, int GB = gv::GB>
__device__ __forceinline__ void gemv_rows(const h16* __restrict__ x, int ldx, const h16* __restrict__ W,
                                          h16* __restrict__ y, int ldy, int M, int N, int K,
                                          const h16* __restrict__ bias, bool gelu = false) {
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
            for (int c = 0; c < COLS; c++) halves8(wb[g][c], w[c]);
            const int k = 256 * i + 8 * lane;
            gemv_group<MR, COLS>(
                w, [&](int m) { return __ldcg(reinterpret_cast<const uint4*>(x + (long)m * ldx + k)); }, M, acc);
        }
    }
    gemv_store<MR, COLS>(acc, lane, n0, y, ldy, M, N, bias, gelu);
}

}  // namespace mmz
