// CPU stages of the pipeline, restated in C++ from the reference's Rust: fp16 conversion (src/gpu.rs:79-119), token
// timestamps by median filter + dynamic time warping (src/align.rs:8-106), log-mel features (src/audio.rs:147-237),
// and the seeded synthetic clips the benchmark transcribes.
//
// Compiled with -ffp-contract=off: the reference's f32 arithmetic is never fused, and the DTW path must come out
// bit-identical.
#include <immintrin.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

#include "host_cpu.h"

namespace mmz {

// ---------------------------------------------------------------- fp16 (src/gpu.rs:79-119)

static inline float bits_f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
static inline uint32_t f_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}

float h2f(uint16_t hv) {
    const uint32_t s = (uint32_t)(hv >> 15) << 31, e = (hv >> 10) & 0x1f, m = hv & 0x3ff;
    if (e == 0) {
        const float v = (float)m / 16777216.0f;
        return s ? -v : v;
    }
    if (e == 31) return bits_f(s | 0x7f800000u | (m << 13));
    return bits_f(s | ((e + 112) << 23) | (m << 13));
}

uint16_t f2h(float x) {
    const uint32_t u = f_bits(x);
    const uint16_t s = (uint16_t)((u >> 16) & 0x8000);
    const uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return s | (a > 0x7f800000u ? 0x7e00 : 0x7c00);
    if (a >= 0x477ff000u) return s | 0x7c00;
    if (a < 0x38800000u) return s | (uint16_t)std::nearbyint(bits_f(a) * 16777216.0f);
    const uint32_t m = a & 0x7fffff;
    uint32_t hb = ((uint32_t)((int)(a >> 23) - 112) << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (hb & 1))) hb += 1;
    return s | (uint16_t)hb;
}

float rh(float x) { return h2f(f2h(x)); }

// ---------------------------------------------------------------- timestamps (src/align.rs)

// src/align.rs:65-106: float32 cost table, ties broken towards the horizontal move
int dtw(const double* m, int rows, int cols, int* text, int* time) {
    const long w = cols + 1;
    std::vector<float> cost((size_t)(rows + 1) * w, INFINITY);
    std::vector<int8_t> trace((size_t)(rows + 1) * w, -1);
    cost[0] = 0.f;
    for (int j = 1; j <= cols; j++)
        for (int i = 1; i <= rows; i++) {
            const float c0 = cost[(i - 1) * w + j - 1], c1 = cost[(i - 1) * w + j], c2 = cost[i * w + j - 1];
            float c;
            int8_t t;
            if (c0 < c1 && c0 < c2) {
                c = c0;
                t = 0;
            } else if (c1 < c0 && c1 < c2) {
                c = c1;
                t = 1;
            } else {
                c = c2;
                t = 2;
            }
            cost[i * w + j] = (float)(m[(long)(i - 1) * cols + j - 1] + (double)c);
            trace[i * w + j] = t;
        }
    for (long j = 0; j < w; j++) trace[j] = 2;
    for (int i = 0; i <= rows; i++) trace[i * w] = 1;
    int i = rows, j = cols, n = 0;
    while (i > 0 || j > 0) {
        text[n] = i - 1;
        time[n] = j - 1;
        n++;
        const int8_t t = trace[i * w + j];
        if (t == 0) {
            i--;
            j--;
        } else if (t == 1) {
            i--;
        } else {
            j--;
        }
    }
    std::reverse(text, text + n);
    std::reverse(time, time + n);
    return n;
}

// f32::total_cmp order as a signed key
static inline int32_t total_key(float x) {
    int32_t k;
    std::memcpy(&k, &x, 4);
    return k ^ (int32_t)(((uint32_t)(k >> 31)) >> 1);
}

static inline void cx(int32_t& a, int32_t& b) {
    const int32_t lo = a < b ? a : b, hi = a < b ? b : a;
    a = lo;
    b = hi;
}

// median of 7 keys: a 16-comparator sorting network (checked on every 0-1 input), branch-free
static inline int32_t median7(int32_t a0, int32_t a1, int32_t a2, int32_t a3, int32_t a4, int32_t a5, int32_t a6) {
    cx(a0, a6); cx(a2, a3); cx(a4, a5);
    cx(a0, a2); cx(a1, a4); cx(a3, a6);
    cx(a0, a1); cx(a2, a5); cx(a3, a4);
    cx(a1, a2); cx(a4, a6);
    cx(a2, a3); cx(a4, a5);
    cx(a1, a2); cx(a3, a4); cx(a5, a6);
    return a3;
}

// width-7 median filter of one row of keys with reflect padding; the interior loop has no branches
__attribute__((target("avx2"))) static void median7_row_avx2(const int32_t* k, int cols, int32_t* med) {
    for (int j = 3; j < cols - 3; j++) med[j] = median7(k[j - 3], k[j - 2], k[j - 1], k[j], k[j + 1], k[j + 2], k[j + 3]);
}
static void median7_row_plain(const int32_t* k, int cols, int32_t* med) {
    for (int j = 3; j < cols - 3; j++) med[j] = median7(k[j - 3], k[j - 2], k[j - 1], k[j], k[j + 1], k[j + 2], k[j + 3]);
}

static inline float key_to_f(int32_t k) {
    k ^= (int32_t)(((uint32_t)(k >> 31)) >> 1);  // the key map is its own inverse
    float v;
    std::memcpy(&v, &k, 4);
    return v;
}

// z-scores of one head: z[i][j] = rh(rh(w[i][j] - rh(mean_j)) / rh(std_j)), 0 where std_j = 0 (src/align.rs:16-25).
// Column statistics accumulate over the rows in order, exactly as the reference's per-column sums do.
static void zscore_plain(const float* w, int rows, int heads, int a, int cols_full, int cols, float* z, float* mean,
                         float* sd, int j0 = 0) {
    auto at = [&](int i, int j) { return w[((long)i * heads + a) * cols_full + j]; };
    for (int j = j0; j < cols; j++) {
        float sum = -0.0f;  // Rust's f32 Sum starts from -0.0
        for (int i = 0; i < rows; i++) sum += at(i, j);
        const float mean_f = sum / (float)rows;
        float vs = -0.0f;
        for (int i = 0; i < rows; i++) {
            const float t = at(i, j) - mean_f;
            vs += t * t;
        }
        mean[j] = rh(mean_f);
        sd[j] = rh(std::sqrt(vs / (float)rows));
        // a constant column (always so for a single row) scores 0 (src/align.rs:22-23)
        for (int i = 0; i < rows; i++) z[(long)i * cols + j] = sd[j] > 0.f ? rh(rh(at(i, j) - mean[j]) / sd[j]) : 0.f;
    }
}

// The same with 8 columns per AVX2 lane group and the hardware's round-to-nearest-even fp16 conversion, which equals
// f2h / h2f for every finite value (the caller takes the plain path when the input holds a non-finite value).
__attribute__((target("avx2,f16c"))) static inline __m256 rh8(__m256 x) {
    return _mm256_cvtph_ps(_mm256_cvtps_ph(x, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
}
__attribute__((target("avx2,f16c"))) static void zscore_avx2(const float* w, int rows, int heads, int a,
                                                             int cols_full, int cols, float* z, float* mean,
                                                             float* sd, float* acc) {
    const int c8 = cols / 8 * 8;
    const __m256 rows_f = _mm256_set1_ps((float)rows), zero = _mm256_setzero_ps();
    for (int j = 0; j < c8; j += 8) _mm256_storeu_ps(acc + j, _mm256_set1_ps(-0.0f));
    for (int i = 0; i < rows; i++) {
        const float* r = w + ((long)i * heads + a) * cols_full;
        for (int j = 0; j < c8; j += 8) _mm256_storeu_ps(acc + j, _mm256_add_ps(_mm256_loadu_ps(acc + j), _mm256_loadu_ps(r + j)));
    }
    for (int j = 0; j < c8; j += 8) _mm256_storeu_ps(mean + j, _mm256_div_ps(_mm256_loadu_ps(acc + j), rows_f));
    for (int j = 0; j < c8; j += 8) _mm256_storeu_ps(acc + j, _mm256_set1_ps(-0.0f));
    for (int i = 0; i < rows; i++) {
        const float* r = w + ((long)i * heads + a) * cols_full;
        for (int j = 0; j < c8; j += 8) {
            const __m256 t = _mm256_sub_ps(_mm256_loadu_ps(r + j), _mm256_loadu_ps(mean + j));
            _mm256_storeu_ps(acc + j, _mm256_add_ps(_mm256_loadu_ps(acc + j), _mm256_mul_ps(t, t)));
        }
    }
    for (int j = 0; j < c8; j += 8) {
        _mm256_storeu_ps(sd + j, rh8(_mm256_sqrt_ps(_mm256_div_ps(_mm256_loadu_ps(acc + j), rows_f))));
        _mm256_storeu_ps(mean + j, rh8(_mm256_loadu_ps(mean + j)));
    }
    for (int i = 0; i < rows; i++) {
        const float* r = w + ((long)i * heads + a) * cols_full;
        float* zr = z + (long)i * cols;
        for (int j = 0; j < c8; j += 8) {
            const __m256 s8 = _mm256_loadu_ps(sd + j);
            const __m256 v = rh8(_mm256_div_ps(rh8(_mm256_sub_ps(_mm256_loadu_ps(r + j), _mm256_loadu_ps(mean + j))), s8));
            _mm256_storeu_ps(zr + j, _mm256_blendv_ps(zero, v, _mm256_cmp_ps(s8, zero, _CMP_GT_OQ)));
        }
    }
    if (c8 < cols) zscore_plain(w, rows, heads, a, cols_full, cols, z, mean, sd, c8);  // the last columns
}

// src/align.rs:6-63: w [rows][heads][cols_full]; one start time per row
void jump_times(const float* w, int rows, int heads, int cols_full, int cols, int width, float* out) {
    if (cols == 0) {
        std::fill(out, out + rows, 0.f);
        return;
    }
    const int pad = width / 2;
    static const bool avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("f16c");
    bool finite = true;
    for (long i = 0; i < (long)rows * heads * cols_full && finite; i++) finite = std::isfinite(w[i]);
    const bool fast = avx2 && finite;
    std::vector<float> avg((size_t)rows * cols, 0.f), z((size_t)rows * cols, 0.f);
    std::vector<float> mean(cols), sd(cols), acc(cols);
    std::vector<int32_t> win(width), keys(cols), med(cols);
    for (int a = 0; a < heads; a++) {
        if (fast) zscore_avx2(w, rows, heads, a, cols_full, cols, z.data(), mean.data(), sd.data(), acc.data());
        else zscore_plain(w, rows, heads, a, cols_full, cols, z.data(), mean.data(), sd.data());
        for (int i = 0; i < rows; i++) {
            const float* row = &z[(long)i * cols];
            float* dst = &avg[(long)i * cols];
            if (cols <= pad) {
                for (int j = 0; j < cols; j++) dst[j] += row[j];
                continue;
            }
            // the median of the width-wide window with reflect padding, in f32::total_cmp order
            for (int j = 0; j < cols; j++) keys[j] = total_key(row[j]);
            int lo = cols, hi = cols;  // columns [lo, hi) take the branch-free interior path
            if (width == 7 && cols > 6) {
                lo = 3;
                hi = cols - 3;
                if (fast) median7_row_avx2(keys.data(), cols, med.data());
                else median7_row_plain(keys.data(), cols, med.data());
            }
            for (int j = 0; j < cols; j++) {
                int32_t kmed;
                if (j >= lo && j < hi) {
                    kmed = med[j];
                } else {
                    for (int k = 0; k < width; k++) {
                        long t = (long)j + k - pad;
                        if (t < 0) t = -t;
                        else if (t >= cols) t = 2 * ((long)cols - 1) - t;
                        win[k] = keys[t];
                    }
                    std::nth_element(win.begin(), win.begin() + pad, win.end());
                    kmed = win[pad];
                }
                dst[j] += key_to_f(kmed);
            }
        }
    }
    for (size_t k = 0; k < avg.size(); k++) avg[k] = rh(avg[k] / (float)heads);
    times_from_cost(avg.data(), rows, cols, cols, out);
}

// src/align.rs:44-63: the DTW over -cost and the start time of each token row
void times_from_cost(const float* cost, int rows, int cols, int ld, float* out) {
    if (cols == 0) {
        std::fill(out, out + rows, 0.f);
        return;
    }
    std::vector<double> m((size_t)rows * cols);
    for (int i = 0; i < rows; i++)
        for (int j = 0; j < cols; j++) m[(size_t)i * cols + j] = -(double)cost[(size_t)i * ld + j];
    std::vector<int> text(rows + cols + 2), time(rows + cols + 2);
    const int n = dtw(m.data(), rows, cols, text.data(), time.data());
    int k_out = 0;
    for (int k = 0; k < n && k_out < rows; k++)
        if (k == 0 || text[k] != text[k - 1]) out[k_out++] = (float)((double)time[k] * 0.02);
    const float last = k_out > 0 ? out[k_out - 1] : 0.f;
    for (; k_out < rows; k_out++) out[k_out] = last;
}

// ---------------------------------------------------------------- log-mel features (src/audio.rs:147-237)

static double hz_to_mel(double f) {
    const double logstep = 27.0 / std::log(6.4);
    return f >= 1000.0 ? 15.0 + std::log(f / 1000.0) * logstep : 3.0 * f / 200.0;
}
static double mel_to_hz(double m) {
    const double logstep = std::log(6.4) / 27.0;
    return m >= 15.0 ? 1000.0 * std::exp(logstep * (m - 15.0)) : 200.0 * m / 3.0;
}

MelBank::MelBank(int n_mels_) : n_mels(n_mels_) {
    const double pi = 3.14159265358979323846;
    std::vector<double> fft_freqs(N_BINS);
    for (int i = 0; i < N_BINS; i++) fft_freqs[i] = i * (SR / 2.0) / (N_BINS - 1);
    const double m0 = hz_to_mel(0.0), m1 = hz_to_mel(8000.0);
    std::vector<double> ff(n_mels + 2);
    for (int i = 0; i < n_mels + 2; i++) ff[i] = mel_to_hz(m0 + (m1 - m0) * i / (n_mels + 1));
    filters.assign((size_t)N_BINS * n_mels, 0.f);
    for (int k = 0; k < N_BINS; k++)
        for (int m = 0; m < n_mels; m++) {
            const double down = (fft_freqs[k] - ff[m]) / (ff[m + 1] - ff[m]);
            const double up = (ff[m + 2] - fft_freqs[k]) / (ff[m + 2] - ff[m + 1]);
            const double enorm = 2.0 / (ff[m + 2] - ff[m]);
            filters[(size_t)k * n_mels + m] = (float)(std::max(std::min(down, up), 0.0) * enorm);
        }
    std::vector<double> win(N_FFT);
    for (int n = 0; n < N_FFT; n++) win[n] = 0.5 - 0.5 * std::cos(2.0 * pi * n / N_FFT);
    cosb.assign((size_t)N_BINS * N_FFT, 0.0);
    sinb.assign((size_t)N_BINS * N_FFT, 0.0);
    for (int k = 0; k < N_BINS; k++)
        for (int n = 0; n < N_FFT; n++) {
            const double a = 2.0 * pi * (double)((k * n) % N_FFT) / N_FFT;
            cosb[(size_t)k * N_FFT + n] = win[n] * std::cos(a);
            sinb[(size_t)k * N_FFT + n] = win[n] * std::sin(a);
        }
}

// log-mel [n_mels][3000] of the first 30 s of y and the number of 10 ms frames that hold audio
int MelBank::features(const float* y, long ny, float* out) const {
    const long n = std::min<long>(ny, N_SAMPLES);
    auto at = [&](long i) -> double {
        if (i < 0) i = -i;
        else if (i >= N_SAMPLES) i = 2 * ((long)N_SAMPLES - 1) - i;
        return i < n ? (double)y[i] : 0.0;
    };
    const long live = std::min<long>((n + N_FFT / 2 + HOP - 1) / HOP, N_FRAMES);
    std::fill(out, out + (size_t)n_mels * N_FRAMES, -10.f);
    double frame[N_FFT];
    float power[N_BINS];
    for (long t = 0; t < live; t++) {
        for (int j = 0; j < N_FFT; j++) frame[j] = at(t * HOP + j - N_FFT / 2);
        for (int k = 0; k < N_BINS; k++) {
            const double* c = &cosb[(size_t)k * N_FFT];
            const double* s = &sinb[(size_t)k * N_FFT];
            double re = 0.0, im = 0.0;
            for (int j = 0; j < N_FFT; j++) {
                re += frame[j] * c[j];
                im += frame[j] * s[j];
            }
            power[k] = (float)(re * re + im * im);
        }
        for (int m = 0; m < n_mels; m++) {
            float acc = 0.f;
            for (int k = 0; k < N_BINS; k++) acc += filters[(size_t)k * n_mels + m] * power[k];
            out[(size_t)m * N_FRAMES + t] = std::log10(std::max(acc, 1e-10f));
        }
    }
    float mx = -INFINITY;
    for (size_t i = 0; i < (size_t)n_mels * N_FRAMES; i++) mx = std::max(mx, out[i]);
    for (size_t i = 0; i < (size_t)n_mels * N_FRAMES; i++) out[i] = (std::max(out[i], mx - 8.f) + 4.f) / 4.f;
    return (int)std::min<long>((n + HOP - 1) / HOP, N_FRAMES);
}

// ---------------------------------------------------------------- synthetic clips

// 30 s at 16 kHz: a sum of k ~ U{1..8} sinusoids with f ~ U(80, 4000) Hz, random phase and amplitude, plus Gaussian
// noise at 10 dB SNR; seeded per clip
void synth_clip(unsigned long long seed, float* y, long n) {
    std::mt19937_64 rng(seed);
    std::uniform_int_distribution<int> nk(1, 8);
    std::uniform_real_distribution<double> fq(80.0, 4000.0), ph(0.0, 2.0 * 3.14159265358979323846), amp(0.1, 1.0);
    const int k = nk(rng);
    double f[8], p[8], a[8];
    for (int i = 0; i < k; i++) {
        f[i] = fq(rng);
        p[i] = ph(rng);
        a[i] = amp(rng);
    }
    double power = 0.0;
    for (long t = 0; t < n; t++) {
        double v = 0.0;
        for (int i = 0; i < k; i++) v += a[i] * std::sin(2.0 * 3.14159265358979323846 * f[i] * t / SR + p[i]);
        y[t] = (float)v;
        power += v * v;
    }
    power /= (double)std::max<long>(n, 1);
    std::normal_distribution<double> noise(0.0, std::sqrt(power / 10.0));  // 10 dB below the signal
    double peak = 0.0;
    for (long t = 0; t < n; t++) {
        y[t] = (float)(y[t] + noise(rng));
        peak = std::max(peak, (double)std::fabs(y[t]));
    }
    if (peak > 0.99)
        for (long t = 0; t < n; t++) y[t] = (float)(y[t] * (0.99 / peak));
}

void features_parallel(const MelBank& mb, const float* const* clips, const long* lens, int n, float* out, int* frames,
                       int nthreads) {
    if (nthreads < 1) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
    nthreads = std::min(nthreads, std::max(n, 1));
    std::vector<std::thread> th;
    for (int w = 0; w < nthreads; w++)
        th.emplace_back([&, w] {
            for (int i = w; i < n; i += nthreads)
                frames[i] = mb.features(clips[i], lens[i], out + (size_t)i * mb.n_mels * N_FRAMES);
        });
    for (auto& t : th) t.join();
}

}  // namespace mmz
