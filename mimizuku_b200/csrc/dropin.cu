// Kernels under the reference's own names and argument lists, for sm_100a: an image (dropin_sm100a.fatbin) that the
// reference's host can load next to its own and launch by name through its unchanged Gpu::k (src/gpu.rs:187-201),
// with the launch geometry src/model.rs already uses. Only kernels whose new design fits that geometry are here:
//   layernorm, add_layernorm  grid (rows), block 128 (model.rs:529-537): the register-resident single pass of ln.cu
//                             (x read once, the reference's reduction tree), bit-identical to kernels/whisper.cu:66-82
//   kv_write                  grid (B), block 256 (model.rs:665): 16-byte copies of the current position's k and v
//                             into the caches (kernels/whisper.cu:310-317)
//   gemv_1, _2, _4, _8        grid ceil(N / 32), block 256 (gpu.rs:211-228; the shared memory it passes goes unused):
//                             gemv_row.cuh, bit-identical to kernels/whisper.cu:501-567
// The attention kernels need launch settings Gpu::k cannot express (a tensor map, 100+ KB of shared memory, other
// grids) and stay behind the C-ABI entry points.
#include "common.cuh"
#include "gemv_row.cuh"
#include "ln_row.cuh"

using namespace mmz;

namespace {

// rows of dim = 2 n2 values; the reference's dim is even and, for Whisper, at most 1280
template <bool ADD>
__device__ __forceinline__ void ln_dispatch(h16* x, const h16* d, const h16* w, const h16* bias, h16* out, int dim,
                                            float eps) {
    const int n2 = dim / 2, kp = (n2 + 127) / 128;
    auto X = reinterpret_cast<__half2*>(x);
    auto D = reinterpret_cast<const __half2*>(d);
    auto W = reinterpret_cast<const __half2*>(w);
    auto B = reinterpret_cast<const __half2*>(bias);
    auto Y = reinterpret_cast<__half2*>(out);
    switch (kp) {
        case 1: ln_block_row<1, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        case 2: ln_block_row<2, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        case 3: ln_block_row<3, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        case 4: ln_block_row<4, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        case 5: ln_block_row<5, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        case 6: ln_block_row<6, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        case 7: ln_block_row<7, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        case 8: ln_block_row<8, ADD>(X, D, W, B, Y, blockIdx.x, n2, eps); break;
        default: break;  // dim > 2048: not a Whisper width
    }
}

}  // namespace

extern "C" __global__ void __launch_bounds__(128) layernorm(const h16* x, const h16* w, const h16* bias, h16* out,
                                                            int dim, float eps) {
    ln_dispatch<false>(const_cast<h16*>(x), nullptr, w, bias, out, dim, eps);
}

extern "C" __global__ void __launch_bounds__(128) add_layernorm(h16* x, const h16* d, const h16* w, const h16* bias,
                                                                h16* out, int dim, float eps) {
    ln_dispatch<true>(x, d, w, bias, out, dim, eps);
}

extern "C" __global__ void kv_write(const h16* qkv, h16* kc, h16* vc, const int* ctr, int maxT, int d) {
    const int b = blockIdx.x, p = ctr[0];
    const long dst = ((long)b * maxT + p) * d, src = (long)b * 3 * d;
    const bool wide = d % 8 == 0 && !(((uintptr_t)qkv | (uintptr_t)kc | (uintptr_t)vc) & 15);
    if (wide) {  // 16-byte copies (qkv rows of 3d and cache rows of d values then start 16-byte aligned)
        for (int c = threadIdx.x; c < d / 8; c += blockDim.x) {
            reinterpret_cast<uint4*>(kc + dst)[c] = reinterpret_cast<const uint4*>(qkv + src + d)[c];
            reinterpret_cast<uint4*>(vc + dst)[c] = reinterpret_cast<const uint4*>(qkv + src + 2 * d)[c];
        }
    } else {
        for (int c = threadIdx.x; c < d; c += blockDim.x) {
            kc[dst + c] = qkv[src + d + c];
            vc[dst + c] = qkv[src + 2 * d + c];
        }
    }
}

#define MMZ_GEMV(MR)                                                                                                 \
    extern "C" __global__ void __launch_bounds__(256) gemv_##MR(const h16* x, int ldx, const h16* W, h16* y, int ldy, \
                                                                int M, int N, int K, const h16* bias) {               \
        gemv_rows<MR>(x, ldx, W, y, ldy, M, N, K, bias);                                                             \
    }
MMZ_GEMV(1)
MMZ_GEMV(2)
MMZ_GEMV(4)
MMZ_GEMV(8)
#undef MMZ_GEMV
