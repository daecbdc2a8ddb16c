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
#include <time.h>
#include <sys/mman.h>
#include <immintrin.h>

typedef struct {
    const uint16_t* qkv;
    uint16_t* out;
    int g, d, heads, rows;
    int next;
    pthread_mutex_t mu;
} job_t;

#define ENC_RB 128 /* query rows per work unit */

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
    const int nrb = (j->rows + ENC_RB - 1) / ENC_RB;
    for (;;) {
        int t = take(j);
        if (t >= j->g * j->heads * nrb) break;
        const int rb = t % nrb;
        t /= nrb;
        int g = t / j->heads, hh = t % j->heads;
        if (hh >= nh) continue;
        const uint16_t* base = j->qkv + (long)g * ORC_TENC * d3 + hh * ORC_HD;
        float* vf = kf + ORC_TENC * ORC_HD;
        for (int r = 0; r < ORC_TENC; r++)
            for (int c = 0; c < ORC_HD; c++) {
                kf[r * ORC_HD + c] = orc_h2f(base[(long)r * d3 + j->d + c]);
                vf[r * ORC_HD + c] = orc_h2f(base[(long)r * d3 + 2 * j->d + c]);
            }
        const int r1 = (rb + 1) * ENC_RB < j->rows ? (rb + 1) * ENC_RB : j->rows;
        for (int row = rb * ENC_RB; row < r1; row++) {
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

/* Encoder attention of `heads` heads (<= d/64) of g clips over the first `rows` query rows, work units of one
 * (clip, head) and 128 query rows shared among the threads; returns nothing, the caller times it. */
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

/* ------------------------------------------------------------------------------------------------------------------
 * Whole-clip decoder attention on the host: what the decoding steps of one clip ask of attention (src/model.rs:660-705
 * per layer: kv_write + self_attn, then cross_scores / cross_pv / cross_combine over the 1500 encoder positions), with
 * the reference kernels' rounding points (q * 0.125, scores and probabilities rounded to fp16; kernels/whisper.cu:
 * 321-353, 368-449), vectorised with AVX2 / F16C / FMA. fp16 storage as on the GPU. One sequence per thread. */

/* 2^x for x <= 0, eight lanes: x = n + f with n = round(x), 2^f by a degree-4 polynomial (least-squares fit of 2^f on
 * [-0.5, 0.5], constant term 1; max relative error 5.4e-6), 2^n added into the exponent. Inputs below -126 give
 * 2^-126. */
static inline __m256 exp2_v(__m256 x) {
    x = _mm256_max_ps(x, _mm256_set1_ps(-126.f));
    const __m256 n = _mm256_round_ps(x, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    const __m256 f = _mm256_sub_ps(x, n);
    __m256 p = _mm256_set1_ps(0.009550929069519043f);
    p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(0.055833350867033005f));
    p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(0.24024498462677002f));
    p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(0.6931373476982117f));
    p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(1.f));
    const __m256i e = _mm256_slli_epi32(_mm256_cvtps_epi32(n), 23);
    return _mm256_castsi256_ps(_mm256_add_epi32(_mm256_castps_si256(p), e));
}
static inline __m256 exp_v(__m256 x) { return exp2_v(_mm256_mul_ps(x, _mm256_set1_ps(1.4426950408889634f))); }
static inline __m256 rh_v(__m256 x) { return _mm256_cvtph_ps(_mm256_cvtps_ph(x, _MM_FROUND_TO_NEAREST_INT)); }
static inline __m256 ld8h(const uint16_t* p) { return _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)p)); }
static inline float hsum8(__m256 v) {
    __m128 a = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    a = _mm_add_ps(a, _mm_movehl_ps(a, a));
    a = _mm_add_ss(a, _mm_movehdup_ps(a));
    return _mm_cvtss_f32(a);
}

/* softmax(rh(rh(q * 0.125) . k_j)) . v over n keys (rows of stride ld halfs), probabilities rounded to fp16;
 * o[64] receives the f32 output. s: scratch of n + 8 floats. */
static void attend_row(const uint16_t* q, const uint16_t* K, const uint16_t* V, long ld, int n, float* s, float* o) {
    __m256 qv[8];
    for (int c = 0; c < 8; c++) qv[c] = rh_v(_mm256_mul_ps(ld8h(q + 8 * c), _mm256_set1_ps(0.125f)));
    for (int j = 0; j < n; j++) {
        const uint16_t* kr = K + (long)j * ld;
        __m256 a0 = _mm256_mul_ps(qv[0], ld8h(kr)), a1 = _mm256_mul_ps(qv[1], ld8h(kr + 8));
        a0 = _mm256_fmadd_ps(qv[2], ld8h(kr + 16), a0);
        a1 = _mm256_fmadd_ps(qv[3], ld8h(kr + 24), a1);
        a0 = _mm256_fmadd_ps(qv[4], ld8h(kr + 32), a0);
        a1 = _mm256_fmadd_ps(qv[5], ld8h(kr + 40), a1);
        a0 = _mm256_fmadd_ps(qv[6], ld8h(kr + 48), a0);
        a1 = _mm256_fmadd_ps(qv[7], ld8h(kr + 56), a1);
        s[j] = hsum8(_mm256_add_ps(a0, a1));
    }
    const int n8 = n & ~7;
    __m256 mv = _mm256_set1_ps(-INFINITY);
    for (int j = 0; j < n8; j += 8) {
        const __m256 v = rh_v(_mm256_loadu_ps(s + j));
        _mm256_storeu_ps(s + j, v);
        mv = _mm256_max_ps(mv, v);
    }
    float m = -INFINITY;
    {
        float t[8];
        _mm256_storeu_ps(t, mv);
        for (int i = 0; i < 8; i++) m = fmaxf(m, t[i]);
        for (int j = n8; j < n; j++) {
            s[j] = orc_rh(s[j]);
            m = fmaxf(m, s[j]);
        }
    }
    for (int j = n; j < n8 + 8; j++) s[j] = -INFINITY;
    const __m256 m8 = _mm256_set1_ps(m);
    __m256 sv = _mm256_setzero_ps();
    for (int j = 0; j < n; j += 8) {
        const __m256 e = exp_v(_mm256_sub_ps(_mm256_loadu_ps(s + j), m8));
        _mm256_storeu_ps(s + j, e);
        sv = _mm256_add_ps(sv, e);
    }
    const __m256 inv = _mm256_set1_ps(1.f / hsum8(sv));
    for (int j = 0; j < n; j += 8) _mm256_storeu_ps(s + j, rh_v(_mm256_mul_ps(_mm256_loadu_ps(s + j), inv)));
    __m256 ov[8];
    for (int c = 0; c < 8; c++) ov[c] = _mm256_setzero_ps();
    for (int j = 0; j < n; j++) {
        const __m256 pj = _mm256_set1_ps(s[j]);
        const uint16_t* vr = V + (long)j * ld;
        for (int c = 0; c < 8; c++) ov[c] = _mm256_fmadd_ps(pj, ld8h(vr + 8 * c), ov[c]);
    }
    for (int c = 0; c < 8; c++) _mm256_storeu_ps(o + 8 * c, ov[c]);
}

typedef struct {
    int nl, nh, np, steps, max_t, nseq;
    const uint16_t* kv; /* cross k/v [nl][2][nh][1500][64], shared by the threads (read only) */
    pthread_barrier_t bar;
    pthread_mutex_t mu;
    double chk, t0, t1;
} dec_job_t;

static void fill_h(uint16_t* p, size_t n, uint64_t seed) {
    /* random fp16 bit patterns of magnitude below 1 (sign, exponent field <= 14, any mantissa); timing inputs only */
    uint64_t x = seed * 6364136223846793005ull + 1442695040888963407ull;
    for (size_t i = 0; i < n; i++) {
        x = x * 6364136223846793005ull + 1442695040888963407ull;
        p[i] = (uint16_t)((x >> 40) & 0xBBFFu);
    }
}

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

typedef struct {
    dec_job_t* j;
    int seq;
} dec_arg_t;

/* a large buffer backed by transparent huge pages where the system allows (fewer page faults) */
static void* big_alloc(size_t bytes) {
    void* p = NULL;
    const size_t align = (size_t)2 << 20;
    bytes = (bytes + align - 1) & ~(align - 1);
    if (posix_memalign(&p, align, bytes) != 0) return NULL;
    madvise(p, bytes, MADV_HUGEPAGE);
    return p;
}

static void* dec_worker(void* arg) {
    dec_job_t* j = ((dec_arg_t*)arg)->j;
    const int seq = ((dec_arg_t*)arg)->seq;
    const int nl = j->nl, nh = j->nh, d = nh * ORC_HD, mt = j->max_t;
    const int used = j->np + j->steps < mt ? j->np + j->steps : mt; /* cache rows the steps touch */
    uint16_t* kc = (uint16_t*)big_alloc((size_t)nl * mt * d * 2);
    uint16_t* vc = (uint16_t*)big_alloc((size_t)nl * mt * d * 2);
    uint16_t* q = (uint16_t*)malloc((size_t)d * 2 * 2);
    float* s = (float*)malloc(sizeof(float) * (ORC_TENC + 16));
    float o[ORC_HD];
    double chk = 0.0;
    for (int l = 0; l < nl; l++) {
        fill_h(kc + (size_t)l * mt * d, (size_t)used * d, 1000 * seq + 2 * l + 1);
        fill_h(vc + (size_t)l * mt * d, (size_t)used * d, 1000 * seq + 2 * l + 2);
    }
    fill_h(q, (size_t)d * 2, 7 * seq + 5);
    /* each thread starts at its own layer, so that at any moment the threads stream different slices of the shared
     * cross k/v (from memory, as separate clips' buffers would be) rather than one slice through the cache */
    const int l0 = (int)((long)seq * nl / j->nseq);
    pthread_barrier_wait(&j->bar); /* inputs in place: the timed part starts */
    if (seq == 0) j->t0 = now_s();
    for (int st = 0; st < j->steps; st++) {
        const int p = j->np - 1 + st; /* position of the step's input token */
        for (int li = 0; li < nl; li++) {
            const int l = (l0 + li) % nl;
            uint16_t* K = kc + (size_t)l * mt * d;
            uint16_t* V = vc + (size_t)l * mt * d;
            /* kv_write of position p, then causal self-attention over 0..p */
            memcpy(K + (size_t)p * d, q, (size_t)d * 2);
            memcpy(V + (size_t)p * d, q + d, (size_t)d * 2);
            for (int h = 0; h < nh; h++) {
                attend_row(q + h * ORC_HD, K + h * ORC_HD, V + h * ORC_HD, d, p + 1, s, o);
                for (int c = 0; c < ORC_HD; c++) chk += o[c];
            }
            /* cross-attention over the 1500 encoder positions of this layer */
            const uint16_t* X = j->kv + (size_t)l * 2 * nh * ORC_TENC * ORC_HD;
            for (int h = 0; h < nh; h++) {
                attend_row(q + d + h * ORC_HD, X + (size_t)h * ORC_TENC * ORC_HD,
                           X + (size_t)(nh + h) * ORC_TENC * ORC_HD, ORC_HD, ORC_TENC, s, o);
                for (int c = 0; c < ORC_HD; c++) chk += o[c];
            }
        }
    }
    pthread_barrier_wait(&j->bar);
    if (seq == 0) j->t1 = now_s();
    pthread_mutex_lock(&j->mu);
    j->chk += chk;
    pthread_mutex_unlock(&j->mu);
    free(kc);
    free(vc);
    free(q);
    free(s);
    return NULL;
}

/* The decoder attention of nseq whole clips on nseq threads, one clip each (steps decoding steps after an np-token
 * prompt, nl layers of nh heads, self-attention caches of max_t rows); synthetic inputs filled before the timed part:
 * one cross k/v of nl x 2 x nh x 1500 x 64 fp16 shared by the threads (read only; each thread starts at another
 * layer), self-attention caches per thread. *seconds receives the wall time of the attention work alone (all threads
 * between two barriers). Returns a checksum of the outputs. */
double orc_cpu_dec_attn_clips(int nseq, int nl, int nh, int np, int steps, int max_t, double* seconds) {
    dec_job_t j;
    memset(&j, 0, sizeof j);
    j.nl = nl;
    j.nh = nh;
    j.np = np;
    j.steps = steps;
    j.max_t = max_t;
    if (nseq < 1) nseq = 1;
    j.nseq = nseq;
    const size_t xkv = (size_t)nl * 2 * nh * ORC_TENC * ORC_HD;
    uint16_t* kv = (uint16_t*)big_alloc(xkv * 2);
    if (!kv) return 0.0;
    fill_h(kv, xkv, 12345);
    j.kv = kv;
    pthread_mutex_init(&j.mu, NULL);
    pthread_barrier_init(&j.bar, NULL, (unsigned)nseq);
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nseq);
    dec_arg_t* args = (dec_arg_t*)malloc(sizeof(dec_arg_t) * nseq);
    for (int i = 0; i < nseq; i++) {
        args[i].j = &j;
        args[i].seq = i;
        pthread_create(&th[i], NULL, dec_worker, &args[i]);
    }
    for (int i = 0; i < nseq; i++) pthread_join(th[i], NULL);
    free(th);
    free(args);
    free(kv);
    pthread_barrier_destroy(&j.bar);
    pthread_mutex_destroy(&j.mu);
    if (seconds) *seconds = j.t1 - j.t0;
    return j.chk;
}
