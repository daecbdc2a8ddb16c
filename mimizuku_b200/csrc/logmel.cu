// Log-mel features on the GPU for a whole batch (src/audio.rs:192-237; the host restatement is MelBank::features):
// windowed DFT of 400-sample frames every 160 samples (reflect padding of 200 at both ends), power spectrum, mel
// filterbank, log10 with a 1e-10 floor, then max(x, clip max - 8), (x + 4) / 4.
//
//   dft_power_kernel  the DFT as a 3000 x 400 by 400 x 402 product per clip in f64, one 64-frame x 32-bin tile per
//                     CTA: every (frame, bin) sums its 400 products in sample order with separate multiply and add
//                     roundings, as the host does (its file is built without contraction), so the f32 power
//                     spectrum equals the host's bit for bit
//   mel_log_kernel    16 frames per CTA: the filterbank sums in bin order in f32 (multiply and add rounded
//                     separately), log10 in f64 rounded to f32, frames past the audio at -10; per-CTA maximum
//   mel_finish_kernel the clip maximum from the per-CTA maxima and the final clamp and scale
//
// The windowed cos/sin bases and the filterbank are the host's own tables (MelBank), uploaded once per device and
// mel count.
#include <deque>
#include <mutex>

#include "common.cuh"
#include "host_cpu.h"
#include "launch.h"

namespace mmz {

constexpr int LM_TF = 64;                         // frames per DFT tile
constexpr int LM_TB = 32;                         // bins per DFT tile
constexpr int LM_KC = 16;                         // samples per K chunk
constexpr int LM_FPB = 16;                        // frames per mel CTA
constexpr int LM_NMB = (N_FRAMES + LM_FPB - 1) / LM_FPB;  // mel CTAs (and maxima) per clip

__device__ __forceinline__ int reflect_at(int i) {  // MelBank::features' sample index (before the length test)
    if (i < 0) i = -i;
    else if (i >= (int)N_SAMPLES) i = 2 * ((int)N_SAMPLES - 1) - i;
    return i;
}
__device__ __forceinline__ int live_frames(int n) {
    return min((n + N_FFT / 2 + HOP - 1) / HOP, N_FRAMES);
}

// grid (47 frame tiles, 7 bin tiles, clips), block 256: thread (tf, tb) owns frames 4 tf .. 4 tf + 3 and bins
// 2 tb, 2 tb + 1 of the tile. basis [2][N_BINS][N_FFT] f64: windowed cos, then sin. power [clips][3000][N_BINS] f32.
__global__ void __launch_bounds__(256) dft_power_kernel(const float* __restrict__ audio, const int* __restrict__ lens,
                                                        const double* __restrict__ basis, float* __restrict__ power) {
    __shared__ double sa[2][LM_TF][LM_KC + 1];
    __shared__ double sb[2][2][LM_TB][LM_KC + 1];
    griddep_wait();
    const int c = blockIdx.z, t0 = blockIdx.x * LM_TF, k0 = blockIdx.y * LM_TB, t = threadIdx.x;
    const int n = min(lens[c], (int)N_SAMPLES);
    const int live = live_frames(n);
    if (t0 >= live) return;
    const float* y = audio + (size_t)c * N_SAMPLES;
    const int tf = t >> 4, tb = t & 15;
    double re[4][2], im[4][2];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int q = 0; q < 2; q++) re[i][q] = im[i][q] = 0.0;
    auto load = [&](int buf, int j0) {
        for (int e = t; e < LM_TF * LM_KC; e += 256) {
            const int f = e / LM_KC, jj = e % LM_KC;
            const int i = reflect_at((t0 + f) * HOP + j0 + jj - N_FFT / 2);
            sa[buf][f][jj] = i < n ? (double)y[i] : 0.0;
        }
        for (int e = t; e < 2 * LM_TB * LM_KC; e += 256) {
            const int cs = e / (LM_TB * LM_KC), r = e % (LM_TB * LM_KC), kb = r / LM_KC, jj = r % LM_KC;
            const int k = k0 + kb;
            sb[buf][cs][kb][jj] = k < N_BINS ? basis[((size_t)cs * N_BINS + k) * N_FFT + j0 + jj] : 0.0;
        }
    };
    load(0, 0);
    __syncthreads();
    constexpr int NCH = N_FFT / LM_KC;
    for (int ch = 0; ch < NCH; ch++) {
        const int buf = ch & 1;
        if (ch + 1 < NCH) load(buf ^ 1, (ch + 1) * LM_KC);
#pragma unroll 4
        for (int jj = 0; jj < LM_KC; jj++) {
            double a[4], cb[2], sbv[2];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = sa[buf][tf * 4 + i][jj];
#pragma unroll
            for (int q = 0; q < 2; q++) {
                cb[q] = sb[buf][0][tb * 2 + q][jj];
                sbv[q] = sb[buf][1][tb * 2 + q][jj];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    re[i][q] = __dadd_rn(re[i][q], __dmul_rn(a[i], cb[q]));
                    im[i][q] = __dadd_rn(im[i][q], __dmul_rn(a[i], sbv[q]));
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int tt = t0 + tf * 4 + i;
        if (tt >= live) continue;
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const int k = k0 + tb * 2 + q;
            if (k < N_BINS)
                power[((size_t)c * N_FRAMES + tt) * N_BINS + k] =
                    __double2float_rn(__dadd_rn(__dmul_rn(re[i][q], re[i][q]), __dmul_rn(im[i][q], im[i][q])));
        }
    }
}

// grid (188, clips), block 128. filters [N_BINS][n_mels] f32; out [clips][n_mels][3000]; bmax [clips][188]
__global__ void __launch_bounds__(128) mel_log_kernel(const float* __restrict__ power, const int* __restrict__ lens,
                                                      const float* __restrict__ filters, int n_mels,
                                                      float* __restrict__ out, float* __restrict__ bmax) {
    __shared__ float pw[LM_FPB][N_BINS];
    __shared__ float wm[4];
    griddep_wait();
    const int c = blockIdx.y, t0 = blockIdx.x * LM_FPB, t = threadIdx.x;
    const int live = live_frames(min(lens[c], (int)N_SAMPLES));
    const int nf = max(0, min(LM_FPB, live - t0));
    for (int e = t; e < nf * N_BINS; e += 128)
        pw[e / N_BINS][e % N_BINS] = power[((size_t)c * N_FRAMES + t0) * N_BINS + e];
    __syncthreads();
    float mx = -INFINITY;
    for (int m = t; m < n_mels; m += 128) {
        float acc[LM_FPB];
#pragma unroll
        for (int f = 0; f < LM_FPB; f++) acc[f] = 0.f;
        if (nf > 0)
            for (int k = 0; k < N_BINS; k++) {
                const float w = __ldg(&filters[(size_t)k * n_mels + m]);
#pragma unroll
                for (int f = 0; f < LM_FPB; f++) acc[f] = __fadd_rn(acc[f], __fmul_rn(w, pw[f][k]));
            }
        float* o = out + ((size_t)c * n_mels + m) * N_FRAMES + t0;
#pragma unroll
        for (int f = 0; f < LM_FPB; f++) {
            if (t0 + f >= N_FRAMES) break;
            const float v = f < nf ? __double2float_rn(log10((double)fmaxf(acc[f], 1e-10f))) : -10.f;
            o[f] = v;
            mx = fmaxf(mx, v);
        }
    }
    for (int o2 = 16; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o2));
    if ((t & 31) == 0) wm[t >> 5] = mx;
    __syncthreads();
    if (t == 0) bmax[(size_t)c * LM_NMB + blockIdx.x] = fmaxf(fmaxf(wm[0], wm[1]), fmaxf(wm[2], wm[3]));
}

// grid (chunks, clips), block 256: out = (max(out, clip max - 8) + 4) / 4
__global__ void __launch_bounds__(256) mel_finish_kernel(float* __restrict__ out, const float* __restrict__ bmax,
                                                         int n_mels) {
    __shared__ float wm[8];
    griddep_wait();
    const int c = blockIdx.y, t = threadIdx.x;
    float mx = -INFINITY;
    for (int i = t; i < LM_NMB; i += 256) mx = fmaxf(mx, bmax[(size_t)c * LM_NMB + i]);
    for (int o2 = 16; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o2));
    if ((t & 31) == 0) wm[t >> 5] = mx;
    __syncthreads();
    mx = wm[0];
    for (int w = 1; w < 8; w++) mx = fmaxf(mx, wm[w]);
    const float lo = __fsub_rn(mx, 8.f);
    const size_t total = (size_t)n_mels * N_FRAMES;
    float* o = out + (size_t)c * total;
    for (size_t i = (size_t)blockIdx.x * 256 + t; i < total; i += (size_t)gridDim.x * 256)
        o[i] = __fdiv_rn(__fadd_rn(fmaxf(o[i], lo), 4.f), 4.f);
}

// ---------------------------------------------------------------- tables and launcher

namespace {
struct MelTables {
    int device = -1, n_mels = 0;
    double* basis = nullptr;  // [2][N_BINS][N_FFT]
    float* filters = nullptr; // [N_BINS][n_mels]
};
std::mutex g_mel_mu;
std::deque<MelTables> g_mel;  // push_back keeps the addresses of earlier entries

const MelTables* mel_tables(int n_mels) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_mel_mu);
    for (const MelTables& m : g_mel)
        if (m.device == dev && m.n_mels == n_mels) return &m;
    MelBank mb(n_mels);
    MelTables t;
    t.device = dev;
    t.n_mels = n_mels;
    const size_t nb = (size_t)N_BINS * N_FFT;
    if (cudaMalloc(&t.basis, 2 * nb * sizeof(double)) != cudaSuccess) return nullptr;
    if (cudaMalloc(&t.filters, mb.filters.size() * sizeof(float)) != cudaSuccess) {
        cudaFree(t.basis);
        return nullptr;
    }
    if (cudaMemcpy(t.basis, mb.cosb.data(), nb * sizeof(double), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(t.basis + nb, mb.sinb.data(), nb * sizeof(double), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(t.filters, mb.filters.data(), mb.filters.size() * sizeof(float), cudaMemcpyHostToDevice) !=
            cudaSuccess) {
        cudaFree(t.basis);
        cudaFree(t.filters);
        return nullptr;
    }
    g_mel.push_back(t);
    return &g_mel.back();
}
}  // namespace

size_t log_mel_work_bytes(int count) {
    return (size_t)count * N_FRAMES * N_BINS * 4 + (size_t)count * LM_NMB * 4;
}

int launch_log_mel(const float* audio, const int* lens, int count, int n_mels, float* out, void* work,
                   size_t work_bytes, cudaStream_t st) {
    if (count < 1 || n_mels < 1 || n_mels > 1024) return fail("log_mel_gpu: bad shape (1 <= n_mels <= 1024)");
    if (!work || work_bytes < log_mel_work_bytes(count) || ((uintptr_t)work & 15))
        return fail("log_mel_gpu: work missing, misaligned or smaller than mmz_log_mel_gpu_work_bytes");
    DevCtx& dc = dev_ctx();
    if (!dc.ok) return fail(dc.err);
    const MelTables* tb = mel_tables(n_mels);
    if (!tb) return fail("log_mel_gpu: could not upload the filterbank tables");
    float* power = (float*)work;
    float* bmax = power + (size_t)count * N_FRAMES * N_BINS;
    const dim3 g1((N_FRAMES + LM_TF - 1) / LM_TF, (N_BINS + LM_TB - 1) / LM_TB, count);
    if (check_pdl(launch_pdl(dft_power_kernel, g1, dim3(256), 0, st, audio, lens, (const double*)tb->basis, power),
                  "dft_power"))
        return -1;
    if (check_pdl(launch_pdl(mel_log_kernel, dim3(LM_NMB, count), dim3(128), 0, st, (const float*)power, lens,
                             (const float*)tb->filters, n_mels, out, bmax),
                  "mel_log"))
        return -1;
    return check_pdl(launch_pdl(mel_finish_kernel, dim3(32, count), dim3(256), 0, st, out, (const float*)bmax, n_mels),
                     "mel_finish");
}

}  // namespace mmz
