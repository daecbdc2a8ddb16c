/*
 * mimizuku_b200: the B200-native (sm_100a) attention hot path of the mimizuku Whisper engine, as a C-ABI library.
 *
 * Conventions
 *   - Device buffers are plain CUDA device pointers; fp16 tensors are IEEE binary16 (`uint16_t` bit patterns on the
 *     host side). Layouts are the reference engine's (paths below are inside the hayatree/mimizuku project).
 *   - `stream` is a cudaStream_t / CUstream (NULL = legacy default stream). Kernel entry points are asynchronous and
 *     never allocate, so they may be captured in a CUDA graph; call mmz_init on the device first.
 *   - Every function returns 0 on success and a negative value on error; mmz_last_error() then describes the error
 *     (thread-local). Asynchronous kernel faults surface at the next synchronisation, as in the reference
 *     (src/gpu.rs:187-201 checks only the launch).
 *   - In-kernel waits are bounded; a wait that gives up records a code in the device status word (mmz_status).
 */
#ifndef MIMIZUKU_B200_H
#define MIMIZUKU_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- library */

/* Initialises the library on `device` and makes it current (status word, kernel attributes, the static scratch of
 * mmz_cross_attn_noalloc). Calling it again re-resolves those device addresses, as is needed after a
 * cudaDeviceReset. Replaces the set-up part of Gpu::new (src/gpu.rs:122-137). */
int mmz_init(int device);
const char* mmz_last_error(void);
/* Reads and clears the device status word of the current device: code[0] error (0 none, 1 wait timed out,
 * 2 misaligned shared memory, 3 bad argument), code[1] kernel (1 enc_flash, 2 self_attn, 3 cross_attn, 4 layernorm,
 * 5 dec_linear, 6 the wait self-test, 7 logits_argmax, 8 gemm_bias), code[2] site.
 * Synchronises the device. No reference counterpart (the reference has no in-kernel failure detection). */
int mmz_status(int code[3]);
/* Sets the bound on every in-kernel wait, in milliseconds (default 1000). */
int mmz_set_wait_limit_ms(int device, int ms);
/* Failure-detection self-test: launches a kernel that waits on a barrier nothing arrives on, with a limit of
 * limit_ms (1..10000). Its bounded waits give up, record (1 = timeout, 6 = self-test, site) in the status word that
 * mmz_status reads, and the kernel returns; the context stays usable. No reference counterpart (the reference has no
 * in-kernel failure detection). */
int mmz_selftest_wait(int limit_ms, void* stream);

/* ---------------------------------------------------------------- fp16 helpers (src/gpu.rs:79-119) */

float mmz_h2f(uint16_t h);      /* src/gpu.rs:79-91 */
uint16_t mmz_f2h(float x);      /* src/gpu.rs:93-114, round to nearest even */
float mmz_rh(float x);          /* src/gpu.rs:116-119 */

/* ---------------------------------------------------------------- attention hot path (device pointers) */

/* Encoder self-attention, non-causal, over the 1500 encoder positions of `groups` clips:
 * qkv [groups][1500][3d] fp16 (Q at column h*64, K at d + h*64, V at 2d + h*64), out [groups][1500][d] fp16.
 * tcgen05 / TMEM / TMA flash attention. Replaces the enc_flash launch (kernels/whisper.cu:209,
 * src/model.rs:566: grid (24, heads, groups), block 128). qkv and out 16-byte aligned. */
int mmz_enc_flash(const void* qkv, void* out, int groups, int d, void* stream);

/* Causal decoder self-attention at position p = ctr[0] over the per-layer caches kc, vc [batch][max_t][d], with the
 * cache write of position p folded in: k and v of p are read from qkv [batch][3d] and stored into the caches.
 * Sequences with done[b] != 0 only get the cache write. out [batch][d]. Replaces kv_write + self_attn
 * (kernels/whisper.cu:310, :321; src/model.rs:665-672). max_t <= 512. Outputs equal the reference kernel's bit for
 * bit. Launched as a programmatic dependent of the kernel before it on the stream: ctr, done and the cache rows
 * before ctr[0] are read before that kernel has finished (in the reference's decoding step they come from earlier
 * steps), so they must not be written by the kernel immediately before this call; qkv may be. */
int mmz_self_attn(const void* qkv, void* kc, void* vc, void* out, const int* ctr, const int* done, int batch,
                  int max_t, int d, void* stream);

/* kv_write alone (kernels/whisper.cu:310; src/model.rs:665): k, v of position ctr[0] from qkv into the caches. */
int mmz_kv_write(const void* qkv, void* kc, void* vc, const int* ctr, int batch, int max_t, int d, void* stream);

/* Decoder cross-attention of one layer over the 1500 encoder positions: q [batch][d] (the xq projection), kv the
 * head-contiguous cross k/v buffer [batch][nl][k|v][heads][1500][64], out [batch][d]. For the heads with
 * aslot[layer * heads + head] = s >= 0, the fp16 probabilities are also stored into align[b][ctr[0]][s][1500]
 * (align is [batch][max_t][na][1500]). Sequences with done[b] != 0 are skipped.
 * Three kernels chained by programmatic dependent launches: split-KV scores and 64-position chunk statistics; then
 * probabilities and per-chunk P.V partials; then the in-order combine of the 24 chunk partials of each
 * (sequence, head). Replaces cross_scores + cross_pv + cross_combine (kernels/whisper.cu:368, :407, :443;
 * src/model.rs:676-705), whose S / stat / part buffers (model.rs:452-454) become `scratch`: a device buffer of at
 * least mmz_cross_attn_scratch_bytes(batch, d) bytes, 16-byte aligned, with no initial contents required.
 * Launches that share a scratch buffer must not overlap on the GPU. kv 16-byte aligned. Launched as a programmatic
 * dependent of the kernel before it on the stream: kv and done are read before that kernel has finished (in the
 * reference's decoding step they come from the encoder and from earlier steps), so they must not be written by the
 * kernel immediately before this call; q may be. */
int mmz_cross_attn(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                   const int* done, int batch, int layer, int nl, int d, int na, int max_t, void* scratch,
                   unsigned long long scratch_bytes, void* stream);
unsigned long long mmz_cross_attn_scratch_bytes(int batch, int d);
/* mmz_cross_attn for callers that cannot allocate device memory (a host that owns a fixed device-memory budget and
 * forbids cudaMalloc after start-up, or a loop that cannot take cudaMalloc's implicit synchronisation): the same
 * kernels and results, with the scratch in a static device array of the library (7.9 MB per device that loads the
 * library, held until the process exits) instead of a caller buffer. It allocates nothing. Limit: batch x heads <= 640
 * (32 sequences of a 20-head model); larger calls return an error. mmz_init resolves the array's device address
 * and caches it (a call on a device without a prior mmz_init resolves it itself, which should then come before any
 * stream capture); after a cudaDeviceReset the cached address is invalid until mmz_init is called again on that
 * device. Every call shares the array, which keeps the last call's contents; calls that overlap on the GPU race on
 * it and must be serialised by the caller. No counterpart in the reference. */
int mmz_cross_attn_noalloc(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                           const int* done, int batch, int layer, int nl, int d, int na, int max_t, void* stream);

/* out = layernorm(x) per row of `dim` (even, <= 2048) fp16 values, fp32 statistics, eps as given.
 * Replaces layernorm (kernels/whisper.cu:66; src/model.rs:529-531). */
int mmz_layernorm(const void* x, const void* w, const void* b, void* out, int rows, int dim, float eps, void* stream);
/* x = h(x + d) in place, then out = layernorm(x); out may be d. Replaces add_layernorm (kernels/whisper.cu:72;
 * src/model.rs:533-537). */
int mmz_add_layernorm(void* x, const void* d, const void* w, const void* b, void* out, int rows, int dim, float eps,
                      void* stream);

/* The encoder's linear layers and cross-K/V projection on the tensor cores: C = rh(A W^T + bias) (A [m][lda] fp16,
 * W [n][k] fp16, bias [n] fp16 or NULL, fp32 accumulation, the bias added in fp32 before the one rounding), with the
 * work around the product in its epilogue: mode 0 stores C [m][ldc]; mode 1 applies the exact-erf GELU to the
 * rounded value first (lin + gelu_inplace, kernels/whisper.cu:107-112); mode 2 stores C[i][j] at
 * c + (j / 64) * blk + i * 64 + j % 64, the decoder's head-contiguous cross k/v layout ([layer][k|v][head][1500][64]
 * with blk = 1500 * 64: model.rs:614-623 and fill_bias_heads, whisper.cu:99-104). n a multiple of 128, k of 64,
 * 16-byte aligned operands and row pitches. Where n is a multiple of 256 and m > 128 the tiles are 256 x 256 on pairs of
 * CTAs (thread-block clusters of two), else 128 x 256 or 128 x 128 on one CTA. Replaces the encoder's cuBLAS GEMMs onto
 * bias images (src/gpu.rs:208-236); the summation order differs from cuBLAS's, so results agree to fp32 rounding
 * before the final fp16 rounding. */
int mmz_gemm_bias(const void* a, int lda, const void* w, const void* bias, void* c, long long ldc, int m, int n, int k,
                  int mode, long long blk, void* stream);

/* Row softmax in place: each of `rows` rows of n <= 2048 fp16 values becomes rh(exp(s - max) / sum) (fp32 inside);
 * rows 8-byte aligned (n a multiple of 4 when rows > 1). Replaces softmax_rows (kernels/whisper.cu:141-166), which
 * the unfused encoder attention launches (src/model.rs:588); its sum associates differently, so a probability may
 * differ from the reference kernel's in the last fp16 bit. */
int mmz_softmax_rows(void* s, long rows, int n, void* stream);

/* Decoder linear layer at 1 <= m <= 8 sequences: y[m][n] = rh(x[m][:k] . w[n][:k] + bias[n]) (bias may be NULL),
 * equal bit for bit to the reference's gemv kernels (kernels/whisper.cu:501-567), which its host uses instead of
 * cuBLAS up to 8 rows (src/gpu.rs:211-228): the same per-lane sums and lane butterfly, the weights streamed before the
 * wait for the kernel before. k a multiple of 8, x and w 16-byte aligned, ldx a multiple of 8. */
int mmz_gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
             void* stream);

/* The decoder's fc1 product and the GELU after it (src/model.rs:708-709: Gpu::gemm of fc1, then gelu_inplace over
 * its b x ff values, kernels/whisper.cu:106-113) in one launch at 1 <= m <= 8: mmz_gemv's rounded value, then
 * rh(GELU) of it, equal bit for bit to the two reference kernels. Arguments and rules as mmz_gemv. */
int mmz_gemv_gelu(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
                  void* stream);

/* The encoder front end's data movement, with the reference kernels' arguments (kernels/whisper.cu:115-139, launched
 * at src/model.rs:553-559): im2col1 writes conv1's operand X[g][t][ci * 3 + k] = mel[g][ci][t + k - 1] (zero outside
 * the 3000 frames) for the n = groups x 3000 x 3 nm values; im2col2 writes conv2's X[g][t][ci * 3 + k] =
 * h1[g][2t + k - 1][ci] for the n = groups x 1500 x 3d values; add_pos adds pos[r % period] to each of the `rows` rows
 * of x [rows][n] in place (f32 sum, one rounding). The same values as the reference kernels', bit for bit. */
int mmz_im2col1(const void* mel, void* X, long long n, int nm, void* stream);
int mmz_im2col2(const void* h1, void* X, long long n, int d, void* stream);
int mmz_add_pos(void* x, const void* pos, long long rows, int n, int period, void* stream);

/* Decoder linear layer at m <= 32 sequences: y[m][n] = rh(x[m][:k] . w[n][:k] + bias[n]) (fp16 in and out, fp32
 * accumulation; bias may be NULL), then GELU when gelu != 0 (fc1 followed by gelu_inplace, kernels/whisper.cu:107-112). x [m][ldx],
 * w [n][k], y [m][ldy]; k a multiple of 64, x and w 16-byte aligned. Replaces the decoder step's cuBLAS GEMMs onto
 * the bias image (src/gpu.rs:208-247, src/model.rs:664-714); the summation order differs from cuBLAS's, so results
 * agree to fp32 rounding before the final fp16 rounding. */
int mmz_dec_linear(const void* x, int ldx, const void* w, const void* bias, void* y, int ldy, int m, int n, int k,
                   int gelu, void* stream);

/* The decoding step's logits fused with the greedy choice: for m <= 32 sequences, logits = rh(x . emb^T) over the
 * vocabulary (x [m][ldx] fp16, emb [vocab][d] fp16, d a multiple of 64 up to 1280; the product of src/model.rs:714-716)
 * and token p + 1 = argmax_tok's choice at p = ctr[0] (kernels/whisper.cu:451-493): suppressed ids (sup[id] != 0, and
 * bs1 / bs2 at the first generated position p + 1 == prompt_len) never chosen, ties to the lower id, a finished
 * sequence (done != 0) or one with no candidate gets eos, and eos sets done; nothing is chosen when
 * p + 1 < prompt_len or p + 1 >= max_t. tok [m][max_t], done [m]. advance != 0 also sets ctr[0] = p + 1 (advance,
 * kernels/whisper.cu:495). The logits are not written to memory unless `logits` ([m][vocab] fp16) is given, and then
 * only at steps that choose a token. Replaces the logits GEMM + argmax_tok + advance launches of src/model.rs:714-735;
 * each logit is the fp16 rounding of one fp32 accumulation in K order, as mmz_dec_linear computes it (bias NULL) when
 * it does not split K (vocabularies of more than 128 x SM-count ids, every Whisper vocabulary on a B200), so the tokens
 * equal argmax_tok's on mmz_dec_linear's logits there. scratch: a
 * device buffer of mmz_logits_argmax_scratch_bytes() bytes, 16-byte aligned, zero-filled once before the first call
 * (every call leaves it zero again); launches that share it must not overlap on the GPU. */
unsigned long long mmz_logits_argmax_scratch_bytes(void);
int mmz_logits_argmax(const void* x, int ldx, const void* emb, int vocab, int d, int m, const unsigned char* sup,
                      int* tok, int* done, int* ctr, int max_t, int prompt_len, int eos, int bs1, int bs2, void* logits,
                      int advance, void* scratch, unsigned long long scratch_bytes, void* stream);

/* ---------------------------------------------------------------- token timestamps (host, src/align.rs) */

/* w [rows][heads][cols_full] alignment-head probabilities -> out [rows] start times in seconds (cols = audio frames
 * / 2, width = median filter width, 7 in the reference). src/align.rs:8-63. */
int mmz_jump_times(const float* w, int rows, int heads, int cols_full, int cols, int width, float* out);
/* The two halves of mmz_jump_times, the first on the GPU for a whole batch.
 * mmz_align_cost: align [n][max_t][na][1500] fp16 (the decoder's alignment-head probabilities, token row i of clip s
 * at position np + i) -> cost [n][max_t][1500] f32, row i at index i: rh(mean over the heads of the width-7 median of
 * the per-column z-scores), bit-identical to src/align.rs:6-43 (the DTW runs on -cost). rows [n], cols [n] are device
 * arrays: token rows (<= max_t - np) and frame columns (<= 1500) per clip. na <= 16. Asynchronous on `stream`.
 * mmz_dtw_times: the DTW over -cost and the start time of each token row (src/align.rs:44-106) for the whole batch
 * on the GPU: cost [n][max_t][1500] as mmz_align_cost writes it, rows / cols the same device arrays, times [n][max_t]
 * f32 (entry i < rows[s] = start of token row i in seconds, 0 past it), bit-identical to mmz_times_from_cost with
 * ld = 1500. max_t <= 512. Asynchronous on `stream`.
 * mmz_times_from_cost: the same DTW for one clip on the host (cost [rows][ld]). */
int mmz_align_cost(const void* align, const int* rows, const int* cols, int n, int np, int max_t, int na, void* cost,
                   void* stream);
int mmz_dtw_times(const void* cost, const int* rows, const int* cols, int n, int max_t, void* times, void* stream);
int mmz_times_from_cost(const float* cost, int rows, int cols, int ld, float* out);
/* DTW over cost m [rows][cols]; writes the path into text, time (rows + cols entries each) and its length into
 * *len. src/align.rs:66-106. */
int mmz_dtw(const double* m, int rows, int cols, int* text, int* time, int* len);

/* ---------------------------------------------------------------- features (host, src/audio.rs) */

/* Log-mel [n_mels][3000] of the first 30 s of 16 kHz samples y[n]; *frames = 10 ms frames that hold audio.
 * src/audio.rs:192-237. */
int mmz_log_mel(const float* y, long n, int n_mels, float* out, int* frames);
/* The same for `count` clips on `threads` host threads (src/transcribe.rs:25-56); out [count][n_mels][3000]. */
/* The same features for a batch on the GPU: audio [count][480000] f32 device (each clip's first 30 s; samples past
 * lens[s] are ignored), lens [count] int32 device (samples that hold audio), out [count][n_mels][3000] f32 device;
 * work: mmz_log_mel_gpu_work_bytes(count) device bytes, 16-byte aligned. The DFT runs in f64 with the host's summation
 * order and roundings, so the power spectra equal mmz_log_mel_batch's bit for bit; log10 is taken in f64 and rounded.
 * The first call per (device, n_mels) uploads the host's filterbank tables (1.4 MB, synchronously); later calls are
 * asynchronous on `stream`. The frame counts are the host's: min((lens[s] + 159) / 160, 3000). */
size_t mmz_log_mel_gpu_work_bytes(int count);
int mmz_log_mel_gpu(const float* audio, const int* lens, int count, int n_mels, float* out, void* work,
                    size_t work_bytes, void* stream);
int mmz_log_mel_batch(const float* const* ys, const long* ns, int count, int n_mels, int threads, float* out,
                      int* frames);
/* A seeded synthetic 30 s clip: 1-8 sinusoids in 80-4000 Hz plus Gaussian noise at 10 dB SNR. */
int mmz_synth_clip(unsigned long long seed, float* y, long n);

/* ---------------------------------------------------------------- engine (src/model.rs, src/transcribe.rs) */

typedef struct mmz_engine mmz_engine;

/* src/model.rs:14-25 Dims */
typedef struct {
    int d, ff, heads, enc_layers, dec_layers, n_mels, vocab, max_t;
} mmz_dims;

/* src/model.rs:64-76 GenCfg (the prompt tokens are passed to mmz_engine_transcribe) */
typedef struct {
    int eos;
    const int* suppress;     /* token ids never chosen */
    int n_suppress;
    int begin_suppress[2];   /* suppressed at the first generated position; -1 = none */
    const int* align_heads;  /* n_align (decoder layer, head) pairs */
    int n_align;
} mmz_gencfg;

/* Engine::new (src/model.rs:333-514) with seeded random-init weights in the reference's fused layouts, for up to
 * bmax sequences and eg clips per encoder pass, on `device`. kernel_image NULL runs this library's sm_100a kernels;
 * a path loads a fatbin exporting the reference's 23 kernel names (src/gpu.rs:16-40) and launches them by name with
 * the reference's grid geometry. Returns NULL on error (mmz_last_error). */
mmz_engine* mmz_engine_create(const mmz_dims* dims, const mmz_gencfg* gc, int bmax, int eg, int device,
                              const char* kernel_image, unsigned long long seed);
void mmz_engine_destroy(mmz_engine* e);
/* transcribe (src/transcribe.rs:104-167) for n <= bmax clips: mel host [n][n_mels][3000] fp32, frames [n];
 * prompt [np] tokens for every clip; at most max_steps decoding steps (<= max_t - 1; 0 = max_t - 1), stopping when
 * every sequence has produced eos; use_graph replays one captured CUDA graph per step. Outputs: tokens [n][max_t],
 * lens [n] (sequence lengths), times [n][max_t] (token start times, s); stage_s [3] = encode, decode, timestamps
 * seconds (may be NULL). */
int mmz_engine_transcribe(mmz_engine* e, const float* mel, const int* frames, int n, const int* prompt, int np,
                          int max_steps, int use_graph, int threads, int* tokens, int* lens, float* times,
                          double* stage_s);
/* The whole of src/transcribe.rs:25-167 from host audio: ys[s] holds ns[s] samples at 16 kHz (the first 30 s are
 * used); the log-mel features are computed on the GPU (mmz_log_mel_gpu) group by group and fed to the encoder, then as
 * mmz_engine_transcribe. frames [n] receives each clip's 10 ms frames that hold audio (as mmz_log_mel_batch returns
 * them); stage_s[0] covers the features and the encoder. Native kernel image only. */
int mmz_engine_transcribe_audio(mmz_engine* e, const float* const* ys, const long* ns, int n, const int* prompt, int np,
                                int max_steps, int use_graph, int threads, int* tokens, int* lens, float* times,
                                int* frames, double* stage_s);
/* Engine::encode (src/model.rs:545-625) for gn <= eg clips of fp16 log-mel already on the device. */
int mmz_engine_encode(mmz_engine* e, const void* mel16, int gn, int slot0);
/* Engine::reset (src/model.rs:628-637): prompts [b][np]. */
int mmz_engine_reset(mmz_engine* e, const int* prompts, int b, int np);
/* Engine::step (src/model.rs:650-736), launched eagerly. */
int mmz_engine_step(mmz_engine* e, int b, int prompt_len);
/* Captures Engine::step as a CUDA graph (src/transcribe.rs:122-131); mmz_engine_replay launches it once. */
int mmz_engine_capture(mmz_engine* e, int b, int prompt_len);
int mmz_engine_replay(mmz_engine* e);
/* Decoder-step lanes (no counterpart in the reference, whose Rust host decodes on one stream): 1 runs every layer of
 * the step for the whole batch on the engine's stream, as src/model.rs:648-736 does; 2 (the default of the native
 * image) runs the layers of the two halves of a 32-sequence batch on two streams, forked after the embedding and
 * joined before the logits, so that the launch- and latency-bound kernels of one half overlap the other half's. The
 * step's kernels work sequence by sequence, so both settings give identical results as long as cuBLAS returns the
 * same rows for 16 sequences as for 32: the engine checks that once when it is created (the four decoder GEMM shapes,
 * bit for bit) and otherwise starts on one lane and refuses 2. Other batch sizes always decode on one lane. Engines
 * on a fatbin image, and engines created for fewer than 32 sequences (bmax < 32), have no second lane and accept
 * only 1. Takes effect at the next step or capture. */
int mmz_engine_set_lanes(mmz_engine* e, int lanes);
int mmz_engine_lanes(mmz_engine* e);
/* Encoder attention of the engine: 0 (the default) the image's fused kernel (this library's mmz_enc_flash, or the
 * reference's enc_flash on a fatbin image); 1 the unfused comparison path of src/model.rs:567-604 (--enc-attn cublas,
 * src/main.rs:37, 179): per clip the scores 0.125 K Q^T of every head into a [heads][1500][1500] fp16 buffer (one
 * cuBLAS strided-batched GEMM; the buffer, 90 MB for 20 heads, is allocated at the first encode in this mode), the row
 * softmax in place (this library's kernel, or the reference's softmax_rows on a fatbin image), then P.V (cuBLAS).
 * Takes effect at the next encode. */
int mmz_engine_set_enc_attn(mmz_engine* e, int unfused);
int mmz_engine_enc_attn(mmz_engine* e);
/* Encoder GEMMs of an engine on this library's kernels: 0 cuBLASLt for every linear layer (the bias in its epilogue,
 * GELU as a separate kernel, the cross k/v as strided-batched products onto the head blocks); 1 (the default) this
 * library's tensor-core GEMM (mmz_gemm_bias) for the qkv projection, fc1 with GELU in its epilogue and the cross k/v
 * projection stored straight into the [layer][k|v][head][1500][64] blocks, cuBLASLt for the others. The sums associate differently
 * from cuBLAS's, so the encoder output agrees with the other setting to fp32 rounding. No effect on a fatbin image.
 * Takes effect at the next encode. */
int mmz_engine_set_enc_gemm(mmz_engine* e, int mode);
int mmz_engine_enc_gemm(mmz_engine* e);
/* Device address of an engine buffer: "tok", "done", "ctr", "align", "logits", "eh", "eqkv", "eatt", "xkv", "mel",
 * "kc", "vc", "x", "hb", "att", "aslot"; NULL if unknown. */
void* mmz_engine_buffer(mmz_engine* e, const char* name);
void* mmz_engine_stream(mmz_engine* e);
int mmz_engine_sync(mmz_engine* e);
/* Device bytes the engine allocated. */
long long mmz_engine_allocated(mmz_engine* e);
/* Kernels of the engine's kernel image launched so far (each graph replay counts every kernel of the captured step;
 * cuBLAS GEMMs are not counted). */
long long mmz_engine_launches(mmz_engine* e);
/* bytes the last mmz_engine_transcribe copied device -> host (tokens and the timestamp inputs). No reference
 * counterpart. */
unsigned long long mmz_engine_d2h_bytes(mmz_engine* e);

#ifdef __cplusplus
}
#endif
#endif
