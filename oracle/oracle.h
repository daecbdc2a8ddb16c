/*
 * TEST INFRASTRUCTURE ONLY. A CPU restatement of hayatree/mimizuku's attention hot path, used as the parity
 * checker by tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py. Nothing in the product
 * (mimizuku_b200/) includes, links or calls this code.
 *
 * Parity pins: the fp16 helpers and the align.rs known-answer tests are restated as golden vectors in
 * tests/golden/; the attention and layer-norm routines are pinned against the reference's own whisper.cu kernels
 * (compiled from source into oracle/_ref/ and run on a B200) through the fixtures in tests/golden/ and the -m gpu
 * differential tests.
 *
 * fp16 values are passed as their uint16 bit patterns. Every routine names the reference file:line it follows
 * (paths inside the hayatree/mimizuku project).
 */
#ifndef MMZ_ORACLE_H
#define MMZ_ORACLE_H
#include <stdint.h>

#define ORC_HD 64
#define ORC_TENC 1500

#ifdef __cplusplus
extern "C" {
#endif

/* src/gpu.rs:79-119 */
float orc_h2f(uint16_t h);
uint16_t orc_f2h(float x);
float orc_rh(float x);
void orc_f2h_array(const float* x, uint16_t* out, long n);
void orc_h2f_array(const uint16_t* x, float* out, long n);

/* kernels/whisper.cu:48-82: y = h((x - mean) * rstd * w + b) per row; add_layernorm first stores x = h(x + d). */
void orc_layernorm(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* out, int rows, int dim, float eps);
void orc_add_layernorm(uint16_t* x, const uint16_t* d, const uint16_t* w, const uint16_t* b, uint16_t* out, int rows,
                       int dim, float eps);

/* kernels/whisper.cu:209-299, exact softmax in double: out[g][row][d] (head h at columns h*64..) for query rows
 * [r0, r0 + nr) of every (clip, head), no fp16 rounding of anything but the inputs. */
void orc_enc_attn_f64(const uint16_t* qkv, double* out, int g, int d, int r0, int nr, int nthreads);
/* oracle_fast.c: the multithreaded f32 CPU attention timed as bench.py's cpu_baseline (kernels/whisper.cu:209-299
 * restated with its 64-key tiles and rounding points), for `heads` heads and the first `rows` query rows. */
void orc_cpu_enc_attn(const uint16_t* qkv, uint16_t* out, int g, int d, int heads, int rows, int nthreads);
/* oracle_fast.c: one sequence's cross-attention step (kernels/whisper.cu:368-449), kv [2][nh][1500][64] */
double orc_cpu_cross_step(const uint16_t* q, const uint16_t* kv, uint16_t* out, int nh);
/* oracle_fast.c: the decoder attention of nseq whole clips on nseq threads (steps decoding steps after an np-token
 * prompt; per step and layer kv_write + causal self-attention and the cross-attention over 1500 positions,
 * src/model.rs:660-705, with kernels/whisper.cu's rounding points), AVX2/F16C/FMA, synthetic fp16 inputs filled
 * before the timed part (one cross k/v shared read-only, each thread starting at another layer; caches per thread);
 * *seconds = wall time of the attention work; returns a checksum of the outputs. */
double orc_cpu_dec_attn_clips(int nseq, int nl, int nh, int np, int steps, int max_t, double* seconds);

/* kernels/whisper.cu:310-353 (kv_write then self_attn) at position p = ctr[0]: the caches hold rows 0..p-1, row p
 * is taken from qkv and also written to the caches. Rounds q*0.125, scores and probabilities to fp16. */
void orc_self_attn(const uint16_t* qkv, uint16_t* kc, uint16_t* vc, uint16_t* out, int p, const int* done, int B,
                   int maxT, int d);
/* the same attention in double with no intermediate rounding (q*0.125 exact); out [B][d] */
void orc_self_attn_f64(const uint16_t* qkv, const uint16_t* kc, const uint16_t* vc, double* out, int p,
                       const int* done, int B, int maxT, int d);

/* kernels/whisper.cu:355-449 (cross_scores, cross_pv, cross_combine) for one decoder layer at position p.
 * kv: [B][nl][2][nh][1500][64]; align: [B][maxT][na][1500]; aslot: [nl * nh] (slot or -1). */
void orc_cross_attn(const uint16_t* q, const uint16_t* kv, uint16_t* out, uint16_t* align, const int* aslot, int p,
                    const int* done, int B, int layer, int nl, int d, int na, int maxT);
/* the same in double, no intermediate rounding; out [B][d], probs [B][nh][1500] (may be NULL) */
void orc_cross_attn_f64(const uint16_t* q, const uint16_t* kv, double* out, double* probs, const int* done, int B,
                        int layer, int nl, int d);

/* src/align.rs:66-106: m [rows][cols]; writes the path (text, time) and returns its length (<= rows + cols). */
int orc_dtw(const double* m, int rows, int cols, int* text, int* time);
/* src/align.rs:8-63: w [rows][heads][cols_full]; writes rows start times. */
void orc_jump_times(const float* w, int rows, int heads, int cols_full, int cols, int width, float* out);
/* the two halves of orc_jump_times: the DTW cost (align.rs:6-43) and the DTW with the token start times (:44-63) */
void orc_align_cost(const float* w, int rows, int heads, int cols_full, int cols, int width, float* cost);
void orc_times_from_cost(const float* cost, int rows, int cols, int ld, float* out);

#ifdef __cplusplus
}
#endif
#endif
