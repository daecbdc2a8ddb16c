// CPU stages of the pipeline (fp16 conversion, token timestamps, log-mel features, synthetic clips).
#pragma once
#include <cstdint>
#include <vector>

namespace mmz {

constexpr int SR = 16000;
constexpr long N_SAMPLES = 30L * SR;
constexpr int N_FRAMES = 3000;
constexpr int N_FFT = 400;
constexpr int HOP = 160;
constexpr int N_BINS = N_FFT / 2 + 1;

float h2f(uint16_t h);
uint16_t f2h(float x);
float rh(float x);

int dtw(const double* m, int rows, int cols, int* text, int* time);
void jump_times(const float* w, int rows, int heads, int cols_full, int cols, int width, float* out);
// src/align.rs:44-63 alone: cost [rows][ld] holds rh(mean over heads of the median-filtered z-scores) (the DTW runs
// on -cost); writes rows start times
void times_from_cost(const float* cost, int rows, int cols, int ld, float* out);

struct MelBank {
    int n_mels;
    std::vector<float> filters;      // [N_BINS][n_mels]
    std::vector<double> cosb, sinb;  // windowed DFT bases [N_BINS][N_FFT]
    explicit MelBank(int n_mels);
    int features(const float* y, long n, float* out) const;
};

void synth_clip(unsigned long long seed, float* y, long n);
void features_parallel(const MelBank& mb, const float* const* clips, const long* lens, int n, float* out, int* frames,
                       int nthreads);

}  // namespace mmz
