/*
 * TEST INFRASTRUCTURE ONLY: the multithreaded f32 CPU attention that bench.py times as its cpu_baseline (the
 * reference has no CPU attention path, so this restates its GPU kernels' math on the host cores). Compiled with
 * reassociation allowed so that the dot products vectorise; it is a timing baseline, not a parity checker (the
 * strict checkers are in oracle.c).
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    const uint16_t* qkv;
    uint16_t* out;
    int g, d, heads, rows;
    int next;
    pthread_mutex_t mu;
} job_t;

static int take(job_t* j) {
    pthread_mutex_lock(&j->mu);
    int t = j->next++;
    pthread_mutex_unlock(&j->mu);
    return t;
}

/* kernels/whisper.cu:209-299 per query row: 64-key tiles (AT, :171), fp32 scores times 0.125 (:252), running max and
 * rescale by expf(m_old - m_new) (:257-267), P rounded to fp16 for the product while l sums the unrounded p
 * (:269-277), O / l rounded to fp16 (:297). Work unit: one (clip, head) over the first `rows` query rows. */
static void* enc_worker(void* arg) {
    job_t* j = (job_t*)arg;
    int nh = j->d / ORC_HD, d3 = 3 * j->d;
    float* kf = (float*)malloc(sizeof(float) * ORC_TENC * ORC_HD * 2);
    for (;;) {
        int t = take(j);
        if (t >= j->g * j->heads) break;
        int g = t / j->heads, hh = t % j->heads;
        if (hh >= nh) continue;
        const uint16_t* base = j->qkv + (long)g * ORC_TENC * d3 + hh * ORC_HD;
        float* vf = kf + ORC_TENC * ORC_HD;
        for (int r = 0; r < ORC_TENC; r++)
            for (int c = 0; c < ORC_HD; c++) {
                kf[r * ORC_HD + c] = orc_h2f(base[(long)r * d3 + j->d + c]);
                vf[r * ORC_HD + c] = orc_h2f(base[(long)r * d3 + 2 * j->d + c]);
            }
        for (int row = 0; row < j->rows; row++) {
            float q[ORC_HD];
            for (int c = 0; c < ORC_HD; c++) q[c] = orc_h2f(base[(long)row * d3 + c]);
            float m = -INFINITY, l = 0.f, o[ORC_HD];
            for (int c = 0; c < ORC_HD; c++) o[c] = 0.f;
            for (int k0 = 0; k0 < ORC_TENC; k0 += 64) {
                int n = ORC_TENC - k0 < 64 ? ORC_TENC - k0 : 64;
                float s[64], tmax = -INFINITY;
                for (int k = 0; k < n; k++) {
                    const float* kr = kf + (k0 + k) * ORC_HD;
                    float a = 0.f;
                    for (int c = 0; c < ORC_HD; c++) a += q[c] * kr[c];
                    s[k] = a * 0.125f;
                    tmax = fmaxf(tmax, s[k]);
                }
                float mn = fmaxf(m, tmax), corr = expf(m - mn);
                m = mn;
                l *= corr;
                for (int c = 0; c < ORC_HD; c++) o[c] *= corr;
                for (int k = 0; k < n; k++) {
                    float p = expf(s[k] - m);
                    l += p;
                    float ph = orc_rh(p);
                    const float* vr = vf + (k0 + k) * ORC_HD;
                    for (int c = 0; c < ORC_HD; c++) o[c] += ph * vr[c];
                }
            }
            uint16_t* dst = j->out + ((long)g * ORC_TENC + row) * j->d + hh * ORC_HD;
            for (int c = 0; c < ORC_HD; c++) dst[c] = orc_f2h(o[c] / l);
        }
    }
    free(kf);
    return NULL;
}

/* Encoder attention of `heads` heads (<= d/64) of g clips over the first `rows` query rows; returns nothing, the
 * caller times it. */
void orc_cpu_enc_attn(const uint16_t* qkv, uint16_t* out, int g, int d, int heads, int rows, int nthreads) {
    job_t j = {qkv, out, g, d, heads, rows, 0, PTHREAD_MUTEX_INITIALIZER};
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, enc_worker, &j);
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
}

/* One decoder step's cross-attention (kernels/whisper.cu:368-449) for one sequence and nh heads over 1500 positions:
 * kv [2][nh][1500][64] (this sequence and layer). Returns the sum of the outputs so the work cannot be elided. */
double orc_cpu_cross_step(const uint16_t* q, const uint16_t* kv, uint16_t* out, int nh) {
    double chk = 0.0;
    float S[ORC_TENC];
    for (int hh = 0; hh < nh; hh++) {
        float qs[ORC_HD];
        for (int t = 0; t < ORC_HD; t++) qs[t] = orc_rh(orc_h2f(q[hh * ORC_HD + t]) * 0.125f);
        const uint16_t* K = kv + (long)hh * ORC_TENC * ORC_HD;
        const uint16_t* V = kv + (long)(nh + hh) * ORC_TENC * ORC_HD;
        float m = -INFINITY;
        for (int j = 0; j < ORC_TENC; j++) {
            float a = 0.f;
            for (int t = 0; t < ORC_HD; t++) a += qs[t] * orc_h2f(K[(long)j * ORC_HD + t]);
            S[j] = orc_rh(a);
            m = fmaxf(m, S[j]);
        }
        float sum = 0.f;
        for (int j = 0; j < ORC_TENC; j++) sum += expf(S[j] - m);
        float o[ORC_HD];
        for (int t = 0; t < ORC_HD; t++) o[t] = 0.f;
        for (int j = 0; j < ORC_TENC; j++) {
            float pj = orc_rh(expf(S[j] - m) / sum);
            for (int t = 0; t < ORC_HD; t++) o[t] += pj * orc_h2f(V[(long)j * ORC_HD + t]);
        }
        for (int t = 0; t < ORC_HD; t++) { out[hh * ORC_HD + t] = orc_f2h(o[t]); chk += o[t]; }
    }
    return chk;
}
