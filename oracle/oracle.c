/*
 * TEST INFRASTRUCTURE ONLY: the CPU parity oracle for the mimizuku attention hot path (see oracle.h). Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it; the product never does.
 *
 * Built with -ffp-contract=off so that f32 expressions round exactly as written (the reference's Rust code never
 * fuses multiply-adds), which the bit-exact align.rs restatement depends on.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- fp16 (src/gpu.rs:79-119) */

static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* src/gpu.rs:79-91 */
float orc_h2f(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    if (e == 0) {
        float v = (float)m / 16777216.0f; /* subnormal: m * 2^-24 */
        return s ? -v : v;
    }
    if (e == 31) return bits_f(s | 0x7f800000u | (m << 13));
    return bits_f(s | ((e + 112) << 23) | (m << 13));
}

/* src/gpu.rs:93-114: round to nearest even, like __float2half_rn */
uint16_t orc_f2h(float x) {
    uint32_t u = f_bits(x);
    uint16_t s = (uint16_t)((u >> 16) & 0x8000);
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return s | (a > 0x7f800000u ? 0x7e00 : 0x7c00);
    if (a >= 0x477ff000u) return s | 0x7c00; /* >= 65520 rounds to infinity */
    if (a < 0x38800000u) return s | (uint16_t)nearbyintf(bits_f(a) * 16777216.0f); /* subnormal, ties to even */
    uint32_t m = a & 0x7fffff;
    uint32_t hb = ((uint32_t)((int)(a >> 23) - 112) << 10) | (m >> 13);
    uint32_t rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (hb & 1))) hb += 1;
    return s | (uint16_t)hb;
}

/* src/gpu.rs:116-119 */
float orc_rh(float x) { return orc_h2f(orc_f2h(x)); }

void orc_f2h_array(const float* x, uint16_t* out, long n) { for (long i = 0; i < n; i++) out[i] = orc_f2h(x[i]); }
void orc_h2f_array(const uint16_t* x, float* out, long n) { for (long i = 0; i < n; i++) out[i] = orc_h2f(x[i]); }

#define F(x) orc_h2f(x)
#define H(x) orc_f2h(x)
#define RH(x) orc_rh(x)

/* ---------------------------------------------------------------- layer norm (kernels/whisper.cu:48-82) */

/* kernels/whisper.cu:49-63: mean, then the centred variance, rstd = 1/sqrt(var + eps), y = h((x-mean)*rstd*w + b).
 * The statistics are accumulated in double (the reference's block reduction order is not reproducible). */
static void ln_row(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* y, int dim, float eps) {
    double s = 0.0;
    for (int i = 0; i < dim; i++) s += F(x[i]);
    float mean = (float)(s / dim);
    double v = 0.0;
    for (int i = 0; i < dim; i++) { double t = (double)F(x[i]) - mean; v += t * t; }
    float rstd = (float)(1.0 / sqrt((double)(float)(v / dim) + eps));
    for (int i = 0; i < dim; i++) y[i] = H((F(x[i]) - mean) * rstd * F(w[i]) + F(b[i]));
}

/* kernels/whisper.cu:66-69 */
void orc_layernorm(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* out, int rows, int dim, float eps) {
    for (int r = 0; r < rows; r++) ln_row(x + (long)r * dim, w, b, out + (long)r * dim, dim, eps);
}

/* kernels/whisper.cu:72-82: x = h(x + d) in place, then out = layernorm(x) */
void orc_add_layernorm(uint16_t* x, const uint16_t* d, const uint16_t* w, const uint16_t* b, uint16_t* out, int rows,
                       int dim, float eps) {
    for (int r = 0; r < rows; r++) {
        uint16_t* xr = x + (long)r * dim;
        const uint16_t* dr = d + (long)r * dim;
        for (int i = 0; i < dim; i++) xr[i] = H(F(xr[i]) + F(dr[i]));
        ln_row(xr, w, b, out + (long)r * dim, dim, eps);
    }
}

/* ---------------------------------------------------------------- encoder attention (kernels/whisper.cu:168-299) */

typedef struct {
    const uint16_t* qkv;
    void* out;
    int g, d, r0, nr;
    int next; /* shared work counter */
    pthread_mutex_t mu;
} enc_job;

static int take(enc_job* j) {
    pthread_mutex_lock(&j->mu);
    int t = j->next++;
    pthread_mutex_unlock(&j->mu);
    return t;
}

/* Q, K, V of head hh of clip g: rows of the interleaved [TENC][3d] buffer at column offsets hh*64, d+hh*64, 2d+hh*64
 * (kernels/whisper.cu:215) */
static void* enc_f64_worker(void* arg) {
    enc_job* j = (enc_job*)arg;
    int nh = j->d / ORC_HD, d3 = 3 * j->d;
    double* sc = (double*)malloc(sizeof(double) * ORC_TENC);
    float* kf = (float*)malloc(sizeof(float) * ORC_TENC * ORC_HD * 2);
    for (;;) {
        int t = take(j);
        if (t >= j->g * nh) break;
        int g = t / nh, hh = t % nh;
        const uint16_t* base = j->qkv + (long)g * ORC_TENC * d3 + hh * ORC_HD;
        float* vf = kf + ORC_TENC * ORC_HD;
        for (int r = 0; r < ORC_TENC; r++)
            for (int c = 0; c < ORC_HD; c++) {
                kf[r * ORC_HD + c] = F(base[(long)r * d3 + j->d + c]);
                vf[r * ORC_HD + c] = F(base[(long)r * d3 + 2 * j->d + c]);
            }
        for (int row = j->r0; row < j->r0 + j->nr && row < ORC_TENC; row++) {
            double q[ORC_HD];
            for (int c = 0; c < ORC_HD; c++) q[c] = F(base[(long)row * d3 + c]);
            double m = -INFINITY;
            for (int k = 0; k < ORC_TENC; k++) {
                double a = 0.0;
                for (int c = 0; c < ORC_HD; c++) a += q[c] * kf[k * ORC_HD + c];
                sc[k] = a * 0.125;
                if (sc[k] > m) m = sc[k];
            }
            double l = 0.0, o[ORC_HD] = {0};
            for (int k = 0; k < ORC_TENC; k++) {
                double p = exp(sc[k] - m);
                l += p;
                for (int c = 0; c < ORC_HD; c++) o[c] += p * vf[k * ORC_HD + c];
            }
            double* dst = (double*)j->out + ((long)g * ORC_TENC + row) * j->d + hh * ORC_HD;
            for (int c = 0; c < ORC_HD; c++) dst[c] = o[c] / l;
        }
    }
    free(sc);
    free(kf);
    return NULL;
}

static void run_enc(void* (*fn)(void*), const uint16_t* qkv, void* out, int g, int d, int r0, int nr, int nthreads) {
    enc_job j = {qkv, out, g, d, r0, nr, 0, PTHREAD_MUTEX_INITIALIZER};
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, fn, &j);
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
}

void orc_enc_attn_f64(const uint16_t* qkv, double* out, int g, int d, int r0, int nr, int nthreads) {
    run_enc(enc_f64_worker, qkv, out, g, d, r0, nr, nthreads);
}


/* ---------------------------------------------------------------- decoder self-attention (kernels/whisper.cu:309-353) */

void orc_self_attn(const uint16_t* qkv, uint16_t* kc, uint16_t* vc, uint16_t* out, int p, const int* done, int B,
                   int maxT, int d) {
    int nh = d / ORC_HD, L = p + 1;
    /* kernels/whisper.cu:310-317: k and v of position p into the caches, for every sequence */
    for (int b = 0; b < B; b++)
        for (int c = 0; c < d; c++) {
            kc[((long)b * maxT + p) * d + c] = qkv[(long)b * 3 * d + d + c];
            vc[((long)b * maxT + p) * d + c] = qkv[(long)b * 3 * d + 2 * d + c];
        }
    float* sc = (float*)malloc(sizeof(float) * L);
    for (int b = 0; b < B; b++) {
        if (done[b]) continue; /* :326 */
        for (int hh = 0; hh < nh; hh++) {
            float q[ORC_HD];
            for (int t = 0; t < ORC_HD; t++) q[t] = RH(F(qkv[(long)b * 3 * d + hh * ORC_HD + t]) * 0.125f); /* :327 */
            const uint16_t* K = kc + (long)b * maxT * d + hh * ORC_HD;
            const uint16_t* V = vc + (long)b * maxT * d + hh * ORC_HD;
            float m = -INFINITY;
            for (int j = 0; j < L; j++) {
                double a = 0.0;
                for (int t = 0; t < ORC_HD; t++) a += (double)q[t] * F(K[(long)j * d + t]);
                sc[j] = RH((float)a); /* :335 */
                m = fmaxf(m, sc[j]);
            }
            double s = 0.0;
            for (int j = 0; j < L; j++) s += expf(sc[j] - m);
            for (int j = 0; j < L; j++) sc[j] = RH(expf(sc[j] - m) / (float)s); /* :344 */
            for (int c = 0; c < ORC_HD; c++) {
                double a = 0.0;
                for (int j = 0; j < L; j++) a += (double)sc[j] * F(V[(long)j * d + c]);
                out[(long)b * d + hh * ORC_HD + c] = H((float)a); /* :352 */
            }
        }
    }
    free(sc);
}

void orc_self_attn_f64(const uint16_t* qkv, const uint16_t* kc, const uint16_t* vc, double* out, int p,
                       const int* done, int B, int maxT, int d) {
    int nh = d / ORC_HD, L = p + 1;
    double* sc = (double*)malloc(sizeof(double) * L);
    for (int b = 0; b < B; b++) {
        if (done[b]) continue;
        for (int hh = 0; hh < nh; hh++) {
            const uint16_t* qr = qkv + (long)b * 3 * d + hh * ORC_HD;
            double m = -INFINITY;
            for (int j = 0; j < L; j++) {
                const uint16_t* kr = j == p ? qkv + (long)b * 3 * d + d + hh * ORC_HD
                                            : kc + ((long)b * maxT + j) * d + hh * ORC_HD;
                double a = 0.0;
                for (int t = 0; t < ORC_HD; t++) a += (double)F(qr[t]) * F(kr[t]);
                sc[j] = a * 0.125;
                if (sc[j] > m) m = sc[j];
            }
            double l = 0.0;
            for (int j = 0; j < L; j++) { sc[j] = exp(sc[j] - m); l += sc[j]; }
            for (int c = 0; c < ORC_HD; c++) {
                double a = 0.0;
                for (int j = 0; j < L; j++) {
                    const uint16_t* vr = j == p ? qkv + (long)b * 3 * d + 2 * d + hh * ORC_HD
                                                : vc + ((long)b * maxT + j) * d + hh * ORC_HD;
                    a += sc[j] * F(vr[c]);
                }
                out[(long)b * d + hh * ORC_HD + c] = a / l;
            }
        }
    }
    free(sc);
}

/* ---------------------------------------------------------------- decoder cross-attention (kernels/whisper.cu:355-449) */

#define XCH 64
#define NCH ((ORC_TENC + XCH - 1) / XCH)

/* kernels/whisper.cu:362-364 */
static long xkv_off(int b, int layer, int kv, int hh, int nl, int nh) {
    return ((((long)b * nl + layer) * 2 + kv) * nh + hh) * (long)ORC_TENC * ORC_HD;
}

void orc_cross_attn(const uint16_t* q, const uint16_t* kv, uint16_t* out, uint16_t* align, const int* aslot, int p,
                    const int* done, int B, int layer, int nl, int d, int na, int maxT) {
    int nh = d / ORC_HD;
    float S[ORC_TENC];
    for (int b = 0; b < B; b++) {
        if (done[b]) continue; /* :372, :412, :445 */
        for (int hh = 0; hh < nh; hh++) {
            float qs[ORC_HD];
            for (int t = 0; t < ORC_HD; t++) qs[t] = RH(F(q[(long)b * d + hh * ORC_HD + t]) * 0.125f); /* :373 */
            const uint16_t* K = kv + xkv_off(b, layer, 0, hh, nl, nh);
            const uint16_t* V = kv + xkv_off(b, layer, 1, hh, nl, nh);
            for (int j = 0; j < ORC_TENC; j++) {
                double a = 0.0;
                for (int t = 0; t < ORC_HD; t++) a += (double)qs[t] * F(K[(long)j * ORC_HD + t]);
                S[j] = RH((float)a); /* :388 */
            }
            /* chunk statistics (:394-401) combined as at :414-417 */
            float cm[NCH], cs[NCH];
            for (int c = 0; c < NCH; c++) {
                float m = -INFINITY;
                for (int j = c * XCH; j < (c + 1) * XCH && j < ORC_TENC; j++) m = fmaxf(m, S[j]);
                double s = 0.0;
                for (int j = c * XCH; j < (c + 1) * XCH && j < ORC_TENC; j++) s += expf(S[j] - m);
                cm[c] = m;
                cs[c] = (float)s;
            }
            float m = -INFINITY, sum = 0.f;
            for (int c = 0; c < NCH; c++) m = fmaxf(m, cm[c]);
            for (int c = 0; c < NCH; c++) sum += cs[c] * expf(cm[c] - m);
            int slot = aslot[layer * nh + hh];
            double o[ORC_HD] = {0};
            for (int j = 0; j < ORC_TENC; j++) {
                float pj = RH(expf(S[j] - m) / sum); /* :419 */
                if (slot >= 0) align[(((long)b * maxT + p) * na + slot) * ORC_TENC + j] = H(pj); /* :440 */
                for (int t = 0; t < ORC_HD; t++) o[t] += (double)pj * F(V[(long)j * ORC_HD + t]);
            }
            for (int t = 0; t < ORC_HD; t++) out[(long)b * d + hh * ORC_HD + t] = H((float)o[t]); /* :448 */
        }
    }
}

void orc_cross_attn_f64(const uint16_t* q, const uint16_t* kv, double* out, double* probs, const int* done, int B,
                        int layer, int nl, int d) {
    int nh = d / ORC_HD;
    double S[ORC_TENC];
    for (int b = 0; b < B; b++) {
        if (done[b]) continue;
        for (int hh = 0; hh < nh; hh++) {
            const uint16_t* qr = q + (long)b * d + hh * ORC_HD;
            const uint16_t* K = kv + xkv_off(b, layer, 0, hh, nl, nh);
            const uint16_t* V = kv + xkv_off(b, layer, 1, hh, nl, nh);
            double m = -INFINITY, l = 0.0;
            for (int j = 0; j < ORC_TENC; j++) {
                double a = 0.0;
                for (int t = 0; t < ORC_HD; t++) a += (double)F(qr[t]) * F(K[(long)j * ORC_HD + t]);
                S[j] = a * 0.125;
                if (S[j] > m) m = S[j];
            }
            for (int j = 0; j < ORC_TENC; j++) { S[j] = exp(S[j] - m); l += S[j]; }
            double o[ORC_HD] = {0};
            for (int j = 0; j < ORC_TENC; j++) {
                double pj = S[j] / l;
                if (probs) probs[((long)b * nh + hh) * ORC_TENC + j] = pj;
                for (int t = 0; t < ORC_HD; t++) o[t] += pj * F(V[(long)j * ORC_HD + t]);
            }
            for (int t = 0; t < ORC_HD; t++) out[(long)b * d + hh * ORC_HD + t] = o[t];
        }
    }
}

/* ---------------------------------------------------------------- timestamps (src/align.rs) */

/* src/align.rs:65-106: f32 cost table, ties broken towards the horizontal move */
int orc_dtw(const double* m, int rows, int cols, int* text, int* time) {
    int w = cols + 1;
    float* cost = (float*)malloc(sizeof(float) * (size_t)(rows + 1) * w);
    signed char* trace = (signed char*)malloc((size_t)(rows + 1) * w);
    for (long k = 0; k < (long)(rows + 1) * w; k++) { cost[k] = INFINITY; trace[k] = -1; }
    cost[0] = 0.f;
    for (int j = 1; j <= cols; j++)
        for (int i = 1; i <= rows; i++) {
            float c0 = cost[(long)(i - 1) * w + j - 1], c1 = cost[(long)(i - 1) * w + j], c2 = cost[(long)i * w + j - 1];
            float c;
            signed char t;
            if (c0 < c1 && c0 < c2) { c = c0; t = 0; }
            else if (c1 < c0 && c1 < c2) { c = c1; t = 1; }
            else { c = c2; t = 2; }
            cost[(long)i * w + j] = (float)(m[(long)(i - 1) * cols + j - 1] + (double)c);
            trace[(long)i * w + j] = t;
        }
    for (int j = 0; j < w; j++) trace[j] = 2;
    for (int i = 0; i <= rows; i++) trace[(long)i * w] = 1;
    int i = rows, j = cols, n = 0;
    while (i > 0 || j > 0) {
        text[n] = i - 1;
        time[n] = j - 1;
        n++;
        signed char t = trace[(long)i * w + j];
        if (t == 0) { i--; j--; }
        else if (t == 1) i--;
        else j--;
    }
    for (int a = 0, b = n - 1; a < b; a++, b--) {
        int x = text[a]; text[a] = text[b]; text[b] = x;
        x = time[a]; time[a] = time[b]; time[b] = x;
    }
    free(cost);
    free(trace);
    return n;
}

/* f32::total_cmp as a signed integer key */
static int32_t total_key(float x) {
    int32_t k;
    memcpy(&k, &x, 4);
    k ^= (int32_t)(((uint32_t)(k >> 31)) >> 1);
    return k;
}

static void sort7(float* v, int n) {
    for (int a = 1; a < n; a++) {
        float x = v[a];
        int b = a - 1;
        while (b >= 0 && total_key(v[b]) > total_key(x)) { v[b + 1] = v[b]; b--; }
        v[b + 1] = x;
    }
}

/* src/align.rs:6-63 */
/* src/align.rs:6-43 up to the DTW cost: cost[i * cols + j] = rh(mean over heads of the width-wide median (reflect
   padding, total order) of the per-column z-scores) -- the DTW runs on -cost. */
void orc_align_cost(const float* w, int rows, int heads, int cols_full, int cols, int width, float* cost) {
#define AT(i, a, j) w[((long)(i) * heads + (a)) * cols_full + (j)]
    float* avg = (float*)calloc((size_t)rows * cols, sizeof(float));
    float* z = (float*)calloc((size_t)rows * cols, sizeof(float));
    float win[64];
    int pad = width / 2;
    for (int a = 0; a < heads; a++) {
        for (int j = 0; j < cols; j++) {
            float sum = -0.0f; /* Rust's f32 Sum starts from -0.0 */
            for (int i = 0; i < rows; i++) sum += AT(i, a, j);
            float mean_f = sum / (float)rows;
            float vs = -0.0f;
            for (int i = 0; i < rows; i++) { float t = AT(i, a, j) - mean_f; vs += t * t; }
            float var = vs / (float)rows;
            float mean = orc_rh(mean_f), sd = orc_rh(sqrtf(var));
            for (int i = 0; i < rows; i++)
                z[(long)i * cols + j] = sd > 0.f ? orc_rh(orc_rh(AT(i, a, j) - mean) / sd) : 0.f;
        }
        for (int i = 0; i < rows; i++) {
            const float* row = z + (long)i * cols;
            for (int j = 0; j < cols; j++) {
                float v;
                if (cols <= pad) {
                    v = row[j];
                } else {
                    for (int k = 0; k < width; k++) {
                        long t = (long)j + k - pad;
                        if (t < 0) t = -t;
                        else if (t >= cols) t = 2 * ((long)cols - 1) - t;
                        win[k] = row[t];
                    }
                    sort7(win, width);
                    v = win[pad];
                }
                avg[(long)i * cols + j] += v;
            }
        }
    }
#undef AT
    for (long k = 0; k < (long)rows * cols; k++) cost[k] = orc_rh(avg[k] / (float)heads);
    free(avg); free(z);
}

/* src/align.rs:44-63: DTW over -cost ([rows][cols], row stride ld) and the start time of each token row */
void orc_times_from_cost(const float* cost, int rows, int cols, int ld, float* out) {
    if (cols == 0) {
        for (int i = 0; i < rows; i++) out[i] = 0.f;
        return;
    }
    double* m = (double*)malloc(sizeof(double) * (size_t)rows * cols);
    for (int i = 0; i < rows; i++)
        for (int j = 0; j < cols; j++) m[(long)i * cols + j] = -(double)cost[(long)i * ld + j];
    int* text = (int*)malloc(sizeof(int) * (size_t)(rows + cols + 2));
    int* time = (int*)malloc(sizeof(int) * (size_t)(rows + cols + 2));
    int n = orc_dtw(m, rows, cols, text, time);
    int k_out = 0;
    for (int k = 0; k < n && k_out < rows; k++)
        if (k == 0 || text[k] != text[k - 1]) out[k_out++] = (float)((double)time[k] * 0.02);
    float last = k_out > 0 ? out[k_out - 1] : 0.f;
    for (; k_out < rows; k_out++) out[k_out] = last;
    free(m); free(text); free(time);
}

void orc_jump_times(const float* w, int rows, int heads, int cols_full, int cols, int width, float* out) {
    if (cols == 0) {
        for (int i = 0; i < rows; i++) out[i] = 0.f;
        return;
    }
    float* cost = (float*)malloc(sizeof(float) * (size_t)rows * cols);
    orc_align_cost(w, rows, heads, cols_full, cols, width, cost);
    orc_times_from_cost(cost, rows, cols, cols, out);
    free(cost);
}
