// Host-side helpers shared by the kernel launchers: per-device context (status word, wait limit, kernel attributes),
// error recording, and TMA tensor-map encoding through the driver entry point (the library does not link libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mmz {

struct DevCtx {
    bool inited = false;
    bool ok = false;
    const char* err = "device context not initialised";
    unsigned* status = nullptr;            // device address of the status word (4 x u32)
    unsigned long long limit_ns = 1000000000ull;  // bound on every in-kernel wait
    int sms = 0;
    int gemm_pairs = 0;  // clusters of two gemm_pair_kernel CTAs that fit the device at once (0: none)
};

// context of the current device, initialised on first use (call mmz_init before any stream capture)
DevCtx& dev_ctx();
// the same, initialised again (device addresses re-resolved: after a cudaDeviceReset they change); mmz_init calls it
DevCtx& dev_ctx_refresh();
// resolves the device address of mmz_cross_attn_noalloc's static scratch array on the current device (cross_noalloc.cu)
int noalloc_resolve();
// records msg as the calling thread's last error and returns -1
int fail(const char* msg);
int failf(const char* fmt, ...);
// the calling thread's last error message
const char* last_error();
// cudaGetLastError after a launch: 0 or fail
int check_launch(const char* what);

// fp16 tensor maps; swizzle: 0 (none), 64 or 128 (bytes)
int make_tmap_2d(CUtensorMap* map, const void* base, const uint64_t dims[2], const uint64_t strides[1],
                 const uint32_t box[2], int swizzle);
int make_tmap_3d(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                 const uint32_t box[3], int swizzle);

// Launches `kernel` as a programmatic dependent of the previous kernel in the stream, so that its launch overlaps that
// kernel's tail; the kernel runs griddep_wait() before it touches memory.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
// launch_pdl, then the same check as check_launch
int check_pdl(cudaError_t e, const char* what);

void init_dec_attn_attrs(DevCtx& c);
void init_gemv_attrs();
// a kernel whose bounded wait runs out on purpose (runtime.cu)
int launch_wait_selftest(int limit_ms, cudaStream_t st);
void init_enc_attn_attrs();
void init_dec_linear_attrs();
void init_logits_argmax_attrs();
void init_gemm_attrs(DevCtx& c);
void init_align_attrs();

// launchers (device pointers, asynchronous on `st`); 0 on success, -1 with the last error set
size_t cross_attn_scratch_bytes(int batch, int d);
// launch_cross_attn's three kernels as one launch on clusters of 8 CTAs, no scratch (dec_attn.cu), bit-identical
int launch_cross_fused(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                       const int* done, int batch, int layer, int nl, int d, int na, int maxT, cudaStream_t st);
int launch_cross_attn(const void* q, const void* kv, void* out, void* align, const int* aslot, const int* ctr,
                      const int* done, int batch, int layer, int nl, int d, int na, int maxT, void* scratch,
                      size_t scratch_bytes, cudaStream_t st);
int launch_self_attn(const void* qkv, void* kc, void* vc, void* out, const int* ctr, const int* done, int batch,
                     int maxT, int d, cudaStream_t st);
int launch_kv_write(const void* qkv, void* kc, void* vc, const int* ctr, int batch, int maxT, int d, cudaStream_t st);
int launch_enc_flash(const void* qkv, void* out, int groups, int d, cudaStream_t st);
int launch_layernorm(const void* x, const void* w, const void* b, void* out, int rows, int dim, float eps,
                     cudaStream_t st);
int launch_add_layernorm(void* x, const void* d, const void* w, const void* b, void* out, int rows, int dim, float eps,
                         cudaStream_t st);

// y[m][n] = rh(x[m] . W[n] + b[n]) (b may be null; GELU after the rounding when gelu), m <= 32, k a multiple of 64
// (dec_linear.cu)
int launch_dec_linear(const void* x, int ldx, const void* w, const void* bias, void* y, int ldy, int m, int n, int k,
                      bool gelu, cudaStream_t st);

// logits of m <= 32 sequences (x [m][ldx], emb [V][k], k <= 1280) fused with argmax_tok's choice of token ctr[0] + 1
// (and ctr[0] += 1 when advance); logits [m][V] fp16 written only when not null; scratch of
// logits_argmax_scratch_bytes(), zero before the first launch and left zero by every launch (logits_argmax.cu)
size_t logits_argmax_scratch_bytes();
int launch_logits_argmax(const void* x, int ldx, const void* emb, int V, int k, int m, const unsigned char* sup,
                         int* tok, int* done, int* ctr, int maxT, int prompt_len, int eos, int bs1, int bs2,
                         void* logits, bool advance, void* scratch, size_t scratch_bytes, cudaStream_t st);

// C = rh(A B^T + bias) on the tensor cores (gemm.cu): A [M][lda], B [N][K] (weights), bias [N] (may be null);
// mode 0 C [M][ldc]; 1 the same after the exact-erf GELU; 2 head blocks: C[m][n] at c + (n / 64) blk + m 64 + n % 64.
// N a multiple of 128, K of 64, 16-byte aligned operands and row pitches.
int launch_gemm_bias(const void* a, int lda, const void* w, const void* bias, void* c, long ldc, int M, int N, int K,
                     int mode, long blk, cudaStream_t st);

// the DTW cost of the token timestamps for a batch of clips (align.cu)
int launch_align_cost(const void* align, const int* rows, const int* cols, int n, int np, int mt, int na, void* cost,
                      cudaStream_t st);
int launch_dtw_times(const void* cost, const int* rows, const int* cols, int n, int mt, void* times, cudaStream_t st);
size_t log_mel_work_bytes(int count);
int launch_log_mel(const float* audio, const int* lens, int count, int n_mels, float* out, void* work,
                   size_t work_bytes, cudaStream_t st);

// engine-side elementwise and token kernels (misc.cu)
int launch_embed(const int* tok, const int* ctr, const void* emb, const void* pe, void* x, int batch, int maxT, int d,
                 cudaStream_t st);
int launch_argmax_tok(const void* logits, int V, const unsigned char* sup, int* tok, int* done, const int* ctr,
                      int batch, int maxT, int prompt_len, int eos, int bs1, int bs2, cudaStream_t st);
int launch_advance(int* ctr, cudaStream_t st);
// row softmax in place, rows of n <= 2048 fp16 values (8-byte aligned rows): the unfused encoder attention's
int launch_softmax_rows(void* s, long rows, int n, cudaStream_t st);
// y[m][n] = rh(x[m] . W[n] + bias[n]) for m <= 8, bit-identical to the reference's gemv kernels (gemv.cu); gelu: then
// rh(GELU(y)), as gelu_inplace after it
int launch_gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
                bool gelu, cudaStream_t st);
int launch_im2col1(const void* mel, void* X, long n, int nm, cudaStream_t st);
int launch_im2col2(const void* h1, void* X, long n, int d, cudaStream_t st);
int launch_gelu(void* x, long n, cudaStream_t st);
int launch_add_pos(void* x, const void* pos, long rows, int n, int period, cudaStream_t st);
int launch_fill_bias(void* y, const void* bias, long rows, int n, long ld, cudaStream_t st);
int launch_fill_bias_heads(void* y, const void* bias, long n8, cudaStream_t st);
int launch_fill_normal(void* p, long n, unsigned long long seed, float mean, float std, cudaStream_t st);
int launch_f32_to_f16(const float* src, void* dst, long n, cudaStream_t st);

}  // namespace mmz
