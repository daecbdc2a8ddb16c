// The C-ABI of include/mimizuku_b200.h over the launchers, the engine and the CPU stages.
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/mimizuku_b200.h"
#include "engine.h"
#include "host_cpu.h"
#include "launch.h"

using namespace mmz;

struct mmz_engine {
    Engine* e;
};

static cudaStream_t S(void* s) { return (cudaStream_t)s; }

extern "C" {

int mmz_init(int device) {
    if (cudaSetDevice(device) != cudaSuccess) return failf("cudaSetDevice(%d) failed", device);
    DevCtx& c = dev_ctx_refresh();
    if (!c.ok) return fail(c.err);
    return noalloc_resolve();
}

const char* mmz_last_error(void) { return last_error(); }

int mmz_status(int code[3]) {
    DevCtx& c = dev_ctx();
    if (!c.ok) return fail(c.err);
    unsigned st[4];
    if (cudaDeviceSynchronize() != cudaSuccess) return fail("cudaDeviceSynchronize failed");
    if (cudaMemcpy(st, c.status, sizeof st, cudaMemcpyDeviceToHost) != cudaSuccess) return fail("status read failed");
    unsigned z[4] = {0, 0, 0, 0};
    if (cudaMemcpy(c.status, z, sizeof z, cudaMemcpyHostToDevice) != cudaSuccess) return fail("status clear failed");
    for (int i = 0; i < 3; i++) code[i] = (int)st[i];
    return 0;
}

int mmz_selftest_wait(int limit_ms, void* stream) { return launch_wait_selftest(limit_ms, S(stream)); }

int mmz_set_wait_limit_ms(int device, int ms) {
    if (cudaSetDevice(device) != cudaSuccess) return fail("cudaSetDevice failed");
    DevCtx& c = dev_ctx();
    if (!c.ok) return fail(c.err);
    if (ms < 1) return fail("wait limit must be >= 1 ms");
    c.limit_ns = (unsigned long long)ms * 1000000ull;
    return 0;
}

float mmz_h2f(uint16_t h) { return h2f(h); }
uint16_t mmz_f2h(float x) { return f2h(x); }
float mmz_rh(float x) { return rh(x); }

int mmz_enc_flash(const void* qkv, void* out, int groups, int d, void* stream) {
    return launch_enc_flash(qkv, out, groups, d, S(stream));
}

int mmz_self_attn(const void* qkv, void* kc, void* vc, void* out, const int* ctr, const int* done, int batch, int max_t,
                  int d, void* stream) {
    return launch_self_attn(qkv, kc, vc, out, ctr, done, batch, max_t, d, S(stream));
}

int mmz_kv_write(const void* qkv, void* kc, void* vc, const int* ctr, int batch, int max_t, int d, void* stream) {
    return launch_kv_write(qkv, kc, vc, ctr, batch, max_t, d, S(stream));
}

int mmz_cross_attn(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                   const int* done, int batch, int layer, int nl, int d, int na, int max_t, void* scratch,
                   unsigned long long scratch_bytes, void* stream) {
    return launch_cross_attn(q, kv, out, align, aslot, ctr, done, batch, layer, nl, d, na, max_t, scratch,
                             (size_t)scratch_bytes, S(stream));
}

unsigned long long mmz_cross_attn_scratch_bytes(int batch, int d) {
    return batch < 1 || d < 64 ? 0 : (unsigned long long)cross_attn_scratch_bytes(batch, d);
}

int mmz_layernorm(const void* x, const void* w, const void* b, void* out, int rows, int dim, float eps, void* stream) {
    return launch_layernorm(x, w, b, out, rows, dim, eps, S(stream));
}

int mmz_add_layernorm(void* x, const void* d, const void* w, const void* b, void* out, int rows, int dim, float eps,
                      void* stream) {
    return launch_add_layernorm(x, d, w, b, out, rows, dim, eps, S(stream));
}

int mmz_jump_times(const float* w, int rows, int heads, int cols_full, int cols, int width, float* out) {
    if (rows < 1 || heads < 1 || cols < 0 || cols > cols_full || width < 1 || width > 63 || !(width & 1))
        return fail("jump_times: bad shape (odd width < 64, cols <= cols_full)");
    jump_times(w, rows, heads, cols_full, cols, width, out);
    return 0;
}

int mmz_dec_linear(const void* x, int ldx, const void* w, const void* bias, void* y, int ldy, int m, int n, int k,
                   int gelu, void* stream) {
    return launch_dec_linear(x, ldx, w, bias, y, ldy, m, n, k, gelu != 0, S(stream));
}

int mmz_gemm_bias(const void* a, int lda, const void* w, const void* bias, void* c, long long ldc, int m, int n, int k,
                  int mode, long long blk, void* stream) {
    return launch_gemm_bias(a, lda, w, bias, c, (long)ldc, m, n, k, mode, (long)blk, S(stream));
}

int mmz_softmax_rows(void* s, long rows, int n, void* stream) { return launch_softmax_rows(s, rows, n, S(stream)); }

int mmz_gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
             void* stream) {
    return launch_gemv(x, ldx, w, y, ldy, m, n, k, bias, false, S(stream));
}
int mmz_gemv_gelu(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
                  void* stream) {
    return launch_gemv(x, ldx, w, y, ldy, m, n, k, bias, true, S(stream));
}
int mmz_im2col1(const void* mel, void* X, long long n, int nm, void* stream) {
    if (n < 0 || nm < 1) return fail("im2col1: bad shape");
    return launch_im2col1(mel, X, (long)n, nm, S(stream));
}
int mmz_im2col2(const void* h1, void* X, long long n, int d, void* stream) {
    if (n < 0 || d < 1) return fail("im2col2: bad shape");
    return launch_im2col2(h1, X, (long)n, d, S(stream));
}
int mmz_add_pos(void* x, const void* pos, long long rows, int n, int period, void* stream) {
    if (rows < 0 || n < 1 || period < 1) return fail("add_pos: bad shape");
    return launch_add_pos(x, pos, (long)rows, n, period, S(stream));
}

unsigned long long mmz_logits_argmax_scratch_bytes(void) { return logits_argmax_scratch_bytes(); }

int mmz_logits_argmax(const void* x, int ldx, const void* emb, int vocab, int d, int m, const unsigned char* sup,
                      int* tok, int* done, int* ctr, int max_t, int prompt_len, int eos, int bs1, int bs2, void* logits,
                      int advance, void* scratch, unsigned long long scratch_bytes, void* stream) {
    return launch_logits_argmax(x, ldx, emb, vocab, d, m, sup, tok, done, ctr, max_t, prompt_len, eos, bs1, bs2, logits,
                                advance != 0, scratch, (size_t)scratch_bytes, S(stream));
}

int mmz_align_cost(const void* align, const int* rows, const int* cols, int n, int np, int max_t, int na, void* cost,
                   void* stream) {
    return launch_align_cost(align, rows, cols, n, np, max_t, na, cost, S(stream));
}

int mmz_dtw_times(const void* cost, const int* rows, const int* cols, int n, int max_t, void* times, void* stream) {
    return launch_dtw_times(cost, rows, cols, n, max_t, times, S(stream));
}

int mmz_times_from_cost(const float* cost, int rows, int cols, int ld, float* out) {
    if (rows < 1 || cols < 0 || ld < cols) return fail("times_from_cost: bad shape (cols <= ld)");
    times_from_cost(cost, rows, cols, ld, out);
    return 0;
}

int mmz_dtw(const double* m, int rows, int cols, int* text, int* time, int* len) {
    if (rows < 0 || cols < 0) return fail("dtw: bad shape");
    *len = dtw(m, rows, cols, text, time);
    return 0;
}

int mmz_log_mel(const float* y, long n, int n_mels, float* out, int* frames) {
    if (n_mels < 1 || n < 0) return fail("log_mel: bad shape");
    MelBank mb(n_mels);
    *frames = mb.features(y, n, out);
    return 0;
}

int mmz_log_mel_batch(const float* const* ys, const long* ns, int count, int n_mels, int threads, float* out,
                      int* frames) {
    if (n_mels < 1 || count < 0) return fail("log_mel_batch: bad shape");
    MelBank mb(n_mels);
    features_parallel(mb, ys, ns, count, out, frames, threads);
    return 0;
}

size_t mmz_log_mel_gpu_work_bytes(int count) { return count < 1 ? 0 : log_mel_work_bytes(count); }

int mmz_log_mel_gpu(const float* audio, const int* lens, int count, int n_mels, float* out, void* work,
                    size_t work_bytes, void* stream) {
    return launch_log_mel(audio, lens, count, n_mels, out, work, work_bytes, S(stream));
}

int mmz_synth_clip(unsigned long long seed, float* y, long n) {
    if (n < 0) return fail("synth_clip: bad length");
    synth_clip(seed, y, n);
    return 0;
}

mmz_engine* mmz_engine_create(const mmz_dims* dims, const mmz_gencfg* gc, int bmax, int eg, int device,
                              const char* kernel_image, unsigned long long seed) {
    if (!dims || !gc) {
        fail("engine_create: null argument");
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        failf("cudaSetDevice(%d) failed", device);
        return nullptr;
    }
    Dims dm{dims->d, dims->ff, dims->heads, dims->enc_layers, dims->dec_layers, dims->n_mels, dims->vocab, dims->max_t};
    GenCfg g;
    g.sot = 0;
    g.no_timestamps = 0;
    g.eos = gc->eos;
    if (gc->eos < 0 || gc->eos >= dims->vocab) {
        fail("engine_create: eos out of range");
        return nullptr;
    }
    for (int i = 0; i < gc->n_suppress; i++) g.suppress.push_back(gc->suppress[i]);
    g.bs[0] = gc->begin_suppress[0];
    g.bs[1] = gc->begin_suppress[1];
    for (int i = 0; i < gc->n_align; i++) g.align_heads.push_back({gc->align_heads[2 * i], gc->align_heads[2 * i + 1]});
    Engine* e = new Engine(dm, g, bmax, eg, kernel_image, seed);
    if (!e->ok()) {
        std::string msg = "engine_create: " + e->error();
        delete e;
        fail(msg.c_str());
        return nullptr;
    }
    return new mmz_engine{e};
}

void mmz_engine_destroy(mmz_engine* e) {
    if (!e) return;
    delete e->e;
    delete e;
}

int mmz_engine_transcribe(mmz_engine* e, const float* mel, const int* frames, int n, const int* prompt, int np,
                          int max_steps, int use_graph, int threads, int* tokens, int* lens, float* times,
                          double* stage_s) {
    if (!e) return fail("null engine");
    return e->e->transcribe(mel, frames, n, prompt, np, max_steps, use_graph != 0, threads, tokens, lens, times, stage_s);
}

int mmz_engine_transcribe_audio(mmz_engine* e, const float* const* ys, const long* ns, int n, const int* prompt, int np,
                                int max_steps, int use_graph, int threads, int* tokens, int* lens, float* times,
                                int* frames, double* stage_s) {
    if (!e) return fail("null engine");
    if (!ys || !ns || !frames) return fail("transcribe_audio: null clip, length or frames array");
    return e->e->transcribe_audio(ys, ns, n, prompt, np, max_steps, use_graph != 0, threads, tokens, lens, times,
                                  frames, stage_s);
}

int mmz_engine_encode(mmz_engine* e, const void* mel16, int gn, int slot0) {
    return e ? e->e->encode_dev(mel16, gn, slot0) : fail("null engine");
}
int mmz_engine_reset(mmz_engine* e, const int* prompts, int b, int np) {
    return e ? e->e->reset(prompts, b, np) : fail("null engine");
}
int mmz_engine_step(mmz_engine* e, int b, int prompt_len) { return e ? e->e->step(b, prompt_len) : fail("null engine"); }
int mmz_engine_capture(mmz_engine* e, int b, int prompt_len) {
    return e ? e->e->capture(b, prompt_len) : fail("null engine");
}
int mmz_engine_replay(mmz_engine* e) { return e ? e->e->replay() : fail("null engine"); }
int mmz_engine_set_lanes(mmz_engine* e, int lanes) { return e ? e->e->set_lanes(lanes) : fail("null engine"); }
int mmz_engine_lanes(mmz_engine* e) { return e ? e->e->lanes() : 0; }
int mmz_engine_set_enc_attn(mmz_engine* e, int unfused) { return e ? e->e->set_enc_attn(unfused) : fail("null engine"); }
int mmz_engine_enc_attn(mmz_engine* e) { return e ? e->e->enc_attn() : -1; }
int mmz_engine_set_enc_gemm(mmz_engine* e, int mode) { return e ? e->e->set_enc_gemm(mode) : fail("null engine"); }
int mmz_engine_enc_gemm(mmz_engine* e) { return e ? e->e->enc_gemm() : -1; }
void* mmz_engine_buffer(mmz_engine* e, const char* name) { return e && name ? e->e->buffer(name) : nullptr; }
void* mmz_engine_stream(mmz_engine* e) { return e ? (void*)e->e->stream() : nullptr; }
int mmz_engine_sync(mmz_engine* e) {
    if (!e) return fail("null engine");
    cudaError_t r = cudaStreamSynchronize(e->e->stream());
    return r == cudaSuccess ? 0 : failf("engine stream: %s", cudaGetErrorString(r));
}
long long mmz_engine_allocated(mmz_engine* e) { return e ? (long long)e->e->allocated() : 0; }
long long mmz_engine_launches(mmz_engine* e) { return e ? e->e->launches() : 0; }
unsigned long long mmz_engine_d2h_bytes(mmz_engine* e) { return e ? e->e->last_d2h_bytes() : 0; }

}  // extern "C"
