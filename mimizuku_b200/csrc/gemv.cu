// The decoder's linear layers at m <= 8 sequences, bit-identical to the reference's gemv kernels (the arithmetic and
// the data movement are described in gemv_row.cuh). Launched as a programmatic dependent of the kernel before.
#include "common.cuh"
#include "gemv_row.cuh"
#include "launch.h"

namespace mmz {

template <int MR>
__global__ void __launch_bounds__(256) gemv_kernel(const h16* __restrict__ x, int ldx, const h16* __restrict__ W,
                                                   h16* __restrict__ y, int ldy, int M, int N, int K,
                                                   const h16* __restrict__ bias) {
    gemv_rows<MR>(x, ldx, W, y, ldy, M, N, K, bias);
}

int launch_gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
                cudaStream_t st) {
    if (m < 1 || m > 8 || n < 1 || k < 8 || k % 8 || ldx < k || ldy < n)
        return fail("gemv: 1 <= m <= 8, k a multiple of 8, ldx >= k, ldy >= n");
    if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ((long)ldx * 2) % 16)
        return fail("gemv: x and w 16-byte aligned, x rows a multiple of 16 bytes");
    const dim3 grid((n + gv::WARPS * gv::COLS - 1) / (gv::WARPS * gv::COLS));
    auto X = (const h16*)x;
    auto W = (const h16*)w;
    auto Y = (h16*)y;
    auto B = (const h16*)bias;
    cudaError_t e;
    if (m == 1) e = launch_pdl(gemv_kernel<1>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B);
    else if (m == 2) e = launch_pdl(gemv_kernel<2>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B);
    else if (m <= 4) e = launch_pdl(gemv_kernel<4>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B);
    else e = launch_pdl(gemv_kernel<8>, grid, dim3(256), 0, st, X, ldx, W, Y, ldy, m, n, k, B);
    return check_pdl(e, "gemv");
}

}  // namespace mmz
