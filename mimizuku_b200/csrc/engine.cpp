// The Whisper engine (see engine.h): weights, buffers and the encoder / decoder-step launch sequences of the
// reference's src/model.rs, the batch driver of src/transcribe.rs, and the two kernel images it can run on.
#include "engine.h"

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <thread>

#include "host_cpu.h"
#include "launch.h"

namespace mmz {

constexpr int HDIM = 64;
constexpr int TENC_ = 1500;
constexpr int NFRAMES = 3000;
constexpr int NCH = (TENC_ + 63) / 64;
constexpr float EPS = 1e-5f;            // model.rs:12
constexpr size_t WS_BYTES = 64u << 20;  // fixed cuBLAS workspace: no allocation during graph capture (gpu.rs:41)
// Two decoder lanes split a batch of exactly 32 sequences into halves of 16: the one split for which cuBLAS's decoder
// GEMMs (cublasGemmStridedBatchedEx, T/N, fp16, fp32 compute; every large-v3 and tiny shape) return the same rows for
// 16 sequences as for 32. Smaller halves do not (4 + 5 of 9 and 12 + 12 of 24 differ in some shapes), so other batch
// sizes decode on one lane.
constexpr int LANE_ROWS = 16;

// ============================================================================ kernel images

class Kernels {
   public:
    long long launches = 0;  // kernels of this image launched (or replayed) so far
    virtual ~Kernels() {}
    virtual bool native() const = 0;
    virtual int layernorm(const void* x, const Ln& l, void* y, int rows, int d, cudaStream_t st) = 0;
    virtual int add_layernorm(void* x, const void* dx, const Ln& l, void* y, int rows, int d, cudaStream_t st) = 0;
    virtual int enc_attn(const void* qkv, void* out, int gn, int d, int nh, cudaStream_t st) = 0;
    // row softmax in place of the unfused encoder attention (kernels/whisper.cu:141-166)
    virtual int softmax_rows(void* s, long rows, int n, cudaStream_t st) = 0;
    virtual int self_attn(const void* qkv, void* kc, void* vc, void* att, const int* ctr, const int* done, int b,
                          int maxT, int d, int nh, cudaStream_t st) = 0;
    virtual int cross_attn(const void* xq, const void* kv, void* s, void* stat, void* part, void* att, void* align,
                           const int* aslot, const int* ctr, const int* done, int b, int layer, int nl, int d, int nh,
                           int na, int maxT, cudaStream_t st) = 0;
    virtual int embed(const int* tok, const int* ctr, const void* emb, const void* dpos, void* x, int b, int maxT,
                      int d, cudaStream_t st) = 0;
    virtual int argmax_tok(const void* logits, int V, const unsigned char* sup, int* tok, int* done, const int* ctr,
                           int b, int maxT, int prompt_len, int eos, int bs1, int bs2, cudaStream_t st) = 0;
    virtual int advance(int* ctr, cudaStream_t st) = 0;
    virtual int im2col1(const void* mel, void* X, long n, int nm, cudaStream_t st) = 0;
    virtual int im2col2(const void* h1, void* X, long n, int d, cudaStream_t st) = 0;
    virtual int gelu(void* x, long n, cudaStream_t st) = 0;
    virtual int add_pos(void* x, const void* pos, long rows, int n, int period, cudaStream_t st) = 0;
    virtual int fill_bias(void* y, const void* bias, long rows, int n, long ld, cudaStream_t st) = 0;
    virtual int fill_bias_heads(void* y, const void* bias, long n8, cudaStream_t st) = 0;
    // y = x W^T + bias for m <= 8 rows, or -2 when the image has no such kernel
    virtual int gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
                     cudaStream_t st) = 0;
    // the same followed by gelu_inplace's GELU, in one kernel, or -2 when the image has none
    virtual int gemv_gelu(const void*, int, const void*, void*, int, int, int, int, const void*, cudaStream_t) {
        return -2;
    }
    // the logits product hb emb^T (model.rs:714-716) where the image has a kernel for it; -2: use cuBLAS
    virtual int logits(const void*, int, const void*, void*, int, int, int, cudaStream_t) { return -2; }
    // the logits product, argmax_tok and advance as one kernel (model.rs:714-735) where the image has one; -2: no
    virtual int logits_argmax(const void*, int, const void*, int, int, const unsigned char*, int*, int*, int*, int,
                              int, int, int, int, cudaStream_t) {
        return -2;
    }
};

// ---------------------------------------------------------------- native sm_100a kernels

class NativeKernels : public Kernels {
   public:
    void* xscratch = nullptr;  // cross-attention scratch (the reference's S / stat / part, model.rs:452-454)
    size_t xscratch_bytes = 0;
    bool native() const override { return true; }
    int layernorm(const void* x, const Ln& l, void* y, int rows, int d, cudaStream_t st) override {
        return ++launches, launch_layernorm(x, l.w, l.b, y, rows, d, EPS, st);
    }
    int add_layernorm(void* x, const void* dx, const Ln& l, void* y, int rows, int d, cudaStream_t st) override {
        return ++launches, launch_add_layernorm(x, dx, l.w, l.b, y, rows, d, EPS, st);
    }
    int enc_attn(const void* qkv, void* out, int gn, int d, int, cudaStream_t st) override {
        return ++launches, launch_enc_flash(qkv, out, gn, d, st);
    }
    int softmax_rows(void* s, long rows, int n, cudaStream_t st) override {
        return ++launches, launch_softmax_rows(s, rows, n, st);
    }
    // kv_write is folded into the self-attention kernel
    int self_attn(const void* qkv, void* kc, void* vc, void* att, const int* ctr, const int* done, int b, int maxT,
                  int d, int, cudaStream_t st) override {
        return ++launches, launch_self_attn(qkv, kc, vc, att, ctr, done, b, maxT, d, st);
    }
    // three kernels chained by programmatic dependent launches, on the engine's cross-attention scratch
    // (s: where this call's scratch starts inside the engine's, so that two decoder lanes use disjoint parts)
    int cross_attn(const void* xq, const void* kv, void* s, void*, void*, void* att, void* align, const int* aslot,
                   const int* ctr, const int* done, int b, int layer, int nl, int d, int, int na, int maxT,
                   cudaStream_t st) override {
        if (b <= cross_fused_max) {  // small batches: the three kernels as one launch on clusters, no scratch
            ++launches;
            return launch_cross_fused(xq, kv, att, align, aslot, ctr, done, b, layer, nl, d, na, maxT, st);
        }
        char* base = s ? (char*)s : (char*)xscratch;
        const size_t used = (size_t)(base - (char*)xscratch);
        if (used > xscratch_bytes) return fail("cross_attn: scratch offset out of range");
        launches += 3;
        return launch_cross_attn(xq, kv, att, align, aslot, ctr, done, b, layer, nl, d, na, maxT, base,
                                 xscratch_bytes - used, st);
    }
    int embed(const int* tok, const int* ctr, const void* emb, const void* dpos, void* x, int b, int maxT, int d,
              cudaStream_t st) override {
        return ++launches, launch_embed(tok, ctr, emb, dpos, x, b, maxT, d, st);
    }
    int argmax_tok(const void* logits, int V, const unsigned char* sup, int* tok, int* done, const int* ctr, int b,
                   int maxT, int prompt_len, int eos, int bs1, int bs2, cudaStream_t st) override {
        return ++launches, launch_argmax_tok(logits, V, sup, tok, done, ctr, b, maxT, prompt_len, eos, bs1, bs2, st);
    }
    int advance(int* ctr, cudaStream_t st) override { return ++launches, launch_advance(ctr, st); }
    int im2col1(const void* mel, void* X, long n, int nm, cudaStream_t st) override {
        return ++launches, launch_im2col1(mel, X, n, nm, st);
    }
    int im2col2(const void* h1, void* X, long n, int d, cudaStream_t st) override {
        return ++launches, launch_im2col2(h1, X, n, d, st);
    }
    int gelu(void* x, long n, cudaStream_t st) override { return ++launches, launch_gelu(x, n, st); }
    int add_pos(void* x, const void* pos, long rows, int n, int period, cudaStream_t st) override {
        return ++launches, launch_add_pos(x, pos, rows, n, period, st);
    }
    int fill_bias(void* y, const void* bias, long rows, int n, long ld, cudaStream_t st) override {
        return ++launches, launch_fill_bias(y, bias, rows, n, ld, st);
    }
    int fill_bias_heads(void* y, const void* bias, long n8, cudaStream_t st) override {
        return ++launches, launch_fill_bias_heads(y, bias, n8, st);
    }
    int gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
             cudaStream_t st) override {
        return ++launches, launch_gemv(x, ldx, w, y, ldy, m, n, k, bias, false, st);
    }
    int gemv_gelu(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int k, const void* bias,
                  cudaStream_t st) override {
        return ++launches, launch_gemv(x, ldx, w, y, ldy, m, n, k, bias, true, st);
    }
    // split-K tensor-core product streaming the 133 MB embedding (8 < m <= 32; up to 8 sequences the reference's host
    // takes its gemv kernels, gpu.rs:211-228, and so does this engine, for the same logits bit for bit)
    int logits(const void* hb, int d, const void* emb, void* out, int vocab, int b, int, cudaStream_t st) override {
        if (b <= 8 || b > 32) return -2;
        return ++launches, launch_dec_linear(hb, d, emb, nullptr, out, vocab, b, vocab, d, false, st);
    }
    // the logits streamed once and reduced to each sequence's token on the GPU, no [b][vocab] logits in memory
    // (8 < m <= 32, d <= 1280); lgscratch: its zero-initialised scratch, owned by the engine
    // up to this many sequences the cross-attention is one launch (cross_fused_kernel); a test hook,
    // MMZ_CROSS_FUSED_MAX=<n>, moves the limit (0: always the three kernels)
    int cross_fused_max = 8;
    void* lgscratch = nullptr;
    size_t lgscratch_bytes = 0;
    bool fused_logits = true;
    int logits_argmax(const void* hb, int d, const void* emb, int vocab, int b, const unsigned char* sup, int* tok,
                      int* done, int* ctr, int maxT, int prompt_len, int eos, int bs1, int bs2,
                      cudaStream_t st) override {
        if (!fused_logits || b <= 8 || b > 32 || d > 1280 || !lgscratch) return -2;
        return ++launches, launch_logits_argmax(hb, d, emb, vocab, d, b, sup, tok, done, ctr, maxT, prompt_len, eos,
                                                bs1, bs2, nullptr, true, lgscratch, lgscratch_bytes, st);
    }
};

// ---------------------------------------------------------------- a fatbin with the reference's kernel names

typedef CUresult (*PfnModuleLoadData)(CUmodule*, const void*);
typedef CUresult (*PfnModuleUnload)(CUmodule);
typedef CUresult (*PfnModuleGetFunction)(CUfunction*, CUmodule, const char*);
typedef CUresult (*PfnLaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                                    CUstream, void**, void**);

static void* driver_fn(const char* name) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return nullptr;
    return p;
}

// One launch argument as the reference's host passes it (gpu.rs:44-50): u64 pointer, i32, i64 or f32.
struct Arg {
    union {
        uint64_t p;
        int32_t i;
        int64_t l;
        float f;
    } v;
    static Arg P(const void* x) { Arg a; a.v.p = (uint64_t)(uintptr_t)x; return a; }
    static Arg I(int x) { Arg a; a.v.l = 0; a.v.i = x; return a; }
    static Arg L(long long x) { Arg a; a.v.l = x; return a; }
    static Arg F(float x) { Arg a; a.v.l = 0; a.v.f = x; return a; }
};

class FatbinKernels : public Kernels {
   public:
    std::string err;
    explicit FatbinKernels(const char* path) {
        load_ = (PfnModuleLoadData)driver_fn("cuModuleLoadData");
        unload_ = (PfnModuleUnload)driver_fn("cuModuleUnload");
        getfn_ = (PfnModuleGetFunction)driver_fn("cuModuleGetFunction");
        launch_ = (PfnLaunchKernel)driver_fn("cuLaunchKernel");
        if (!load_ || !getfn_ || !launch_ || !unload_) {
            err = "driver entry points unavailable";
            return;
        }
        std::ifstream f(path, std::ios::binary);
        if (!f) {
            err = std::string("cannot read kernel image ") + path;
            return;
        }
        image_.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
        if (load_(&mod_, image_.data()) != CUDA_SUCCESS) {
            err = std::string("cuModuleLoadData failed for ") + path;
            return;
        }
        // gpu.rs:16-40: a missing name is an error at start-up
        static const char* names[] = {"layernorm", "add_layernorm", "add_inplace", "fill_bias", "fill_bias_heads",
                                      "gelu_inplace", "add_pos", "im2col1", "im2col2", "softmax_rows", "enc_flash",
                                      "embed", "kv_write", "self_attn", "cross_scores", "cross_pv", "cross_combine",
                                      "argmax_tok", "advance", "gemv_1", "gemv_2", "gemv_4", "gemv_8"};
        for (const char* n : names) {
            CUfunction fn;
            if (getfn_(&fn, mod_, n) != CUDA_SUCCESS) {
                err = std::string("kernel image has no function ") + n;
                return;
            }
            fns_.push_back({n, fn});
        }
    }
    ~FatbinKernels() override {
        if (mod_ && unload_) unload_(mod_);
    }
    bool native() const override { return false; }

    // gpu.rs:187-201
    int k(const char* name, unsigned gx, unsigned gy, unsigned gz, unsigned block, unsigned smem, cudaStream_t st,
          std::initializer_list<Arg> args) {
        CUfunction fn = nullptr;
        for (auto& e : fns_)
            if (!strcmp(e.first, name)) fn = e.second;
        if (!fn) return failf("no kernel %s", name);
        std::vector<Arg> vals(args);
        std::vector<void*> ptrs;
        for (auto& a : vals) ptrs.push_back(&a.v);
        CUresult r = launch_(fn, gx, gy, gz, block, 1, 1, smem, (CUstream)st, ptrs.data(), nullptr);
        ++launches;
        return r == CUDA_SUCCESS ? 0 : failf("%s: cuLaunchKernel failed (%d)", name, (int)r);
    }
    // elementwise launch over n items (gpu.rs:203-206)
    int k1(const char* name, long n, cudaStream_t st, std::initializer_list<Arg> args) {
        return k(name, (unsigned)((n + 255) / 256), 1, 1, 256, 0, st, args);
    }

    int layernorm(const void* x, const Ln& l, void* y, int rows, int d, cudaStream_t st) override {
        return k("layernorm", rows, 1, 1, 128, 0, st, {Arg::P(x), Arg::P(l.w), Arg::P(l.b), Arg::P(y), Arg::I(d), Arg::F(EPS)});
    }
    int add_layernorm(void* x, const void* dx, const Ln& l, void* y, int rows, int d, cudaStream_t st) override {
        return k("add_layernorm", rows, 1, 1, 128, 0, st,
                 {Arg::P(x), Arg::P(dx), Arg::P(l.w), Arg::P(l.b), Arg::P(y), Arg::I(d), Arg::F(EPS)});
    }
    // model.rs:566
    int enc_attn(const void* qkv, void* out, int gn, int d, int nh, cudaStream_t st) override {
        return k("enc_flash", (TENC_ + 63) / 64, nh, gn, 128, 0, st, {Arg::P(qkv), Arg::P(out), Arg::I(d)});
    }
    // model.rs:588
    int softmax_rows(void* s, long rows, int n, cudaStream_t st) override {
        return k("softmax_rows", (unsigned)rows, 1, 1, 256, 0, st, {Arg::P(s), Arg::I(n)});
    }
    // model.rs:665-672
    int self_attn(const void* qkv, void* kc, void* vc, void* att, const int* ctr, const int* done, int b, int maxT,
                  int d, int nh, cudaStream_t st) override {
        if (k("kv_write", b, 1, 1, 256, 0, st, {Arg::P(qkv), Arg::P(kc), Arg::P(vc), Arg::P(ctr), Arg::I(maxT), Arg::I(d)}))
            return -1;
        return k("self_attn", b, nh, 1, 128, 0, st,
                 {Arg::P(qkv), Arg::P(kc), Arg::P(vc), Arg::P(att), Arg::P(ctr), Arg::P(done), Arg::I(maxT), Arg::I(d)});
    }
    // model.rs:676-705
    int cross_attn(const void* xq, const void* kv, void* s, void* stat, void* part, void* att, void* align,
                   const int* aslot, const int* ctr, const int* done, int b, int layer, int nl, int d, int nh, int na,
                   int maxT, cudaStream_t st) override {
        if (k("cross_scores", b * nh, NCH, 1, 128, 0, st,
              {Arg::P(xq), Arg::P(kv), Arg::P(s), Arg::P(stat), Arg::P(done), Arg::I(layer), Arg::I(nl), Arg::I(d)}))
            return -1;
        if (k("cross_pv", b * nh, NCH, 1, 128, 0, st,
              {Arg::P(s), Arg::P(stat), Arg::P(kv), Arg::P(part), Arg::P(align), Arg::P(aslot), Arg::P(ctr),
               Arg::P(done), Arg::I(layer), Arg::I(nl), Arg::I(d), Arg::I(na), Arg::I(maxT)}))
            return -1;
        return k("cross_combine", b * nh, 1, 1, HDIM, 0, st, {Arg::P(part), Arg::P(att), Arg::P(done), Arg::I(d)});
    }
    int embed(const int* tok, const int* ctr, const void* emb, const void* dpos, void* x, int b, int maxT, int d,
              cudaStream_t st) override {
        return k("embed", b, 1, 1, 256, 0, st,
                 {Arg::P(tok), Arg::P(ctr), Arg::P(emb), Arg::P(dpos), Arg::P(x), Arg::I(maxT), Arg::I(d)});
    }
    int argmax_tok(const void* logits, int V, const unsigned char* sup, int* tok, int* done, const int* ctr, int b,
                   int maxT, int prompt_len, int eos, int bs1, int bs2, cudaStream_t st) override {
        return k("argmax_tok", b, 1, 1, 1024, 0, st,
                 {Arg::P(logits), Arg::I(V), Arg::P(sup), Arg::P(tok), Arg::P(done), Arg::P(ctr), Arg::I(maxT),
                  Arg::I(prompt_len), Arg::I(eos), Arg::I(bs1), Arg::I(bs2)});
    }
    int advance(int* ctr, cudaStream_t st) override { return k("advance", 1, 1, 1, 1, 0, st, {Arg::P(ctr)}); }
    int im2col1(const void* mel, void* X, long n, int nm, cudaStream_t st) override {
        return k1("im2col1", n, st, {Arg::P(mel), Arg::P(X), Arg::L(n), Arg::I(nm)});
    }
    int im2col2(const void* h1, void* X, long n, int d, cudaStream_t st) override {
        return k1("im2col2", n, st, {Arg::P(h1), Arg::P(X), Arg::L(n), Arg::I(d)});
    }
    int gelu(void* x, long n, cudaStream_t st) override {
        return k1("gelu_inplace", n / 2, st, {Arg::P(x), Arg::L(n / 2)});
    }
    int add_pos(void* x, const void* pos, long rows, int n, int period, cudaStream_t st) override {
        return k1("add_pos", rows * n, st, {Arg::P(x), Arg::P(pos), Arg::L(rows), Arg::I(n), Arg::I(period)});
    }
    int fill_bias(void* y, const void* bias, long rows, int n, long ld, cudaStream_t st) override {
        return k1("fill_bias", rows * n / 8, st, {Arg::P(y), Arg::P(bias), Arg::L(rows), Arg::I(n), Arg::L(ld)});
    }
    int fill_bias_heads(void* y, const void* bias, long n8, cudaStream_t st) override {
        return k1("fill_bias_heads", n8, st, {Arg::P(y), Arg::P(bias), Arg::L(n8)});
    }
    // gpu.rs:211-228
    int gemv(const void* x, int ldx, const void* w, void* y, int ldy, int m, int n, int kk, const void* bias,
             cudaStream_t st) override {
        const char* name;
        int mr, kc;
        if (m == 1) { name = "gemv_1"; mr = 1; kc = 2048; }
        else if (m == 2) { name = "gemv_2"; mr = 2; kc = 2048; }
        else if (m <= 4) { name = "gemv_4"; mr = 4; kc = 1024; }
        else { name = "gemv_8"; mr = 8; kc = 1024; }
        const int per_block = 8 * 4;
        return k(name, (n + per_block - 1) / per_block, 1, 1, 256, mr * kc * 2, st,
                 {Arg::P(x), Arg::I(ldx), Arg::P(w), Arg::P(y), Arg::I(ldy), Arg::I(m), Arg::I(n), Arg::I(kk), Arg::P(bias)});
    }

   private:
    PfnModuleLoadData load_ = nullptr;
    PfnModuleUnload unload_ = nullptr;
    PfnModuleGetFunction getfn_ = nullptr;
    PfnLaunchKernel launch_ = nullptr;
    CUmodule mod_ = nullptr;
    std::vector<char> image_;
    std::vector<std::pair<const char*, CUfunction>> fns_;
};

// ============================================================================ engine

#define CK(x)                                        \
    do {                                             \
        if ((x) != 0) return -1;                     \
    } while (0)
#define CUDA_CK(x)                                                                                  \
    do {                                                                                            \
        cudaError_t e_ = (x);                                                                       \
        if (e_ != cudaSuccess) return failf("%s:%d: %s", __FILE__, __LINE__, cudaGetErrorString(e_)); \
    } while (0)

void* Engine::alloc(size_t bytes) {
    void* p = nullptr;
    bytes = bytes < 16 ? 16 : bytes;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    cudaMemsetAsync(p, 0, bytes, st_);
    allocs_.push_back(p);
    allocated_ += bytes;
    return p;
}

Engine::Engine(const Dims& dims, const GenCfg& gc, int bmax, int eg, const char* kernel_image, unsigned long long seed)
    : dm_(dims), gc_(gc), bmax_(bmax), eg_(eg) {
    const int d = dm_.d, ff = dm_.ff, nh = dm_.nh, nl = dm_.dec_layers, mt = dm_.max_t;
    // model.rs:47-59
    if (nh * HDIM != d || d % 128 || ff % 8 || mt < 16 || mt > 448 || dm_.enc_layers < 1 || dm_.enc_layers > 64 ||
        nl < 1 || nl > 64 || bmax < 1 || eg < 1 || eg > bmax || dm_.vocab < 1 || dm_.n_mels < 1) {
        err_ = "unsupported shape";
        return;
    }
    for (auto& ah : gc_.align_heads)
        if (ah.first < 0 || ah.first >= nl || ah.second < 0 || ah.second >= nh) {
            err_ = "alignment head out of range";
            return;
        }
    if (gc_.align_heads.empty()) {
        err_ = "no alignment heads";
        return;
    }
    if (cudaGetDevice(&dev_) != cudaSuccess) {
        err_ = "no CUDA device";
        return;
    }
    if (kernel_image && *kernel_image) {
        auto fk = new FatbinKernels(kernel_image);
        k_.reset(fk);
        if (!fk->err.empty()) {
            err_ = fk->err;
            return;
        }
    } else {
        DevCtx& dc = dev_ctx();
        if (!dc.ok) {
            err_ = dc.err;
            return;
        }
        k_.reset(new NativeKernels());
    }
    if (cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking) != cudaSuccess || cublasCreate(&blas_) != CUBLAS_STATUS_SUCCESS ||
        cublasSetStream(blas_, st_) != CUBLAS_STATUS_SUCCESS) {
        err_ = "stream / cuBLAS setup failed";
        return;
    }
    ws_ = alloc(WS_BYTES);
    if (cudaMallocHost(&done_host_, (size_t)bmax_ * 4) != cudaSuccess ||
        cudaEventCreateWithFlags(&poll_ev_, cudaEventDisableTiming) != cudaSuccess) {
        err_ = "pinned poll buffer / event setup failed";
        return;
    }
    if (k_->native() && cublasLtCreate(&lt_) != CUBLAS_STATUS_SUCCESS) {
        err_ = "cuBLASLt setup failed";
        return;
    }
    if (!ws_ || cublasSetWorkspace(blas_, ws_, WS_BYTES) != CUBLAS_STATUS_SUCCESS) {
        err_ = "cuBLAS workspace";
        return;
    }
    if (k_->native() && bmax_ >= 2 * LANE_ROWS) {  // the second decoder lane: its own stream, cuBLAS handle, workspace
        ws2_ = alloc(WS_BYTES);
        if (!ws2_ || cudaStreamCreateWithFlags(&st2_, cudaStreamNonBlocking) != cudaSuccess ||
            cublasCreate(&blas2_) != CUBLAS_STATUS_SUCCESS || cublasSetStream(blas2_, st2_) != CUBLAS_STATUS_SUCCESS ||
            cublasSetWorkspace(blas2_, ws2_, WS_BYTES) != CUBLAS_STATUS_SUCCESS ||
            cudaEventCreateWithFlags(&fork_ev_, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&join_ev_, cudaEventDisableTiming) != cudaSuccess) {
            err_ = "second decoder lane setup failed";
            return;
        }
    }
    const int na = (int)gc_.align_heads.size();
    auto H = [&](size_t n) { return alloc(n * 2); };
    const size_t r1 = (size_t)eg * NFRAMES, r2 = (size_t)eg * TENC_;
    mel_ = H((size_t)eg * dm_.n_mels * NFRAMES);
    mel32_ = (float*)alloc((size_t)eg * dm_.n_mels * NFRAMES * 4);
    x1_ = H(r1 * 3 * dm_.n_mels);
    h1_ = H(r1 * d);
    x2_ = H(r2 * 3 * d);
    ex_ = H(r2 * d);
    eh_ = H(r2 * d);
    eqkv_ = H(r2 * 3 * d);
    eatt_ = H(r2 * d);
    ef_ = H(r2 * ff);
    const size_t b = bmax;
    xkv_buf_ = H(b * nl * 2 * d * TENC_);
    tok_ = (int*)alloc(b * mt * 4);
    done_ = (int*)alloc(b * 4);
    ctr_ = (int*)alloc(16);
    x_ = H(b * d);
    hb_ = H(b * d);
    att_ = H(b * d);
    dout_ = H((size_t)nl * b * (7 * d + ff));
    dbias_ = H((size_t)nl * b * (7 * d + ff));
    logits_ = H(b * dm_.vocab);
    kc_ = H((size_t)nl * b * mt * d);
    vc_ = H((size_t)nl * b * mt * d);
    if (!k_->native()) {  // the reference's split cross-attention scratch (model.rs:452-454)
        s_ = alloc(b * nh * TENC_ * 4);
        stat_ = alloc(b * nh * NCH * 8);
        part_ = alloc(b * nh * NCH * HDIM * 4);
    } else {  // the native kernels' scratch for the same role
        NativeKernels* nk = static_cast<NativeKernels*>(k_.get());
        nk->xscratch_bytes = cross_attn_scratch_bytes(bmax, d);
        nk->xscratch = alloc(nk->xscratch_bytes);
        nk->lgscratch_bytes = logits_argmax_scratch_bytes();
        nk->lgscratch = alloc(nk->lgscratch_bytes);  // zero-filled by alloc, as the fused logits kernel needs
        // a test hook: MMZ_TEST_UNFUSED_LOGITS=1 keeps the logits product, argmax_tok and advance as three launches, so
        // that the two paths can be compared
        if (const char* t = getenv("MMZ_TEST_UNFUSED_LOGITS")) nk->fused_logits = t[0] != '1';
        if (const char* t = getenv("MMZ_CROSS_FUSED_MAX")) nk->cross_fused_max = atoi(t);
        s_ = nk->xscratch;
        stat_ = part_ = nullptr;
    }
    align_ = H(b * mt * na * TENC_);
    if (k_->native()) {
        cost_ = (float*)alloc(b * mt * TENC_ * 4);
        rc_ = (int*)alloc(b * 2 * 4);
        tms_ = (float*)alloc(b * mt * 4);
        if (!cost_ || !rc_ || !tms_) {
            err_ = "device memory allocation failed";
            return;
        }
    }
    for (void* p : {s_, mel_, (void*)mel32_, x1_, h1_, x2_, ex_, eh_, eqkv_, eatt_, ef_, xkv_buf_, (void*)tok_, (void*)done_, (void*)ctr_,
                    x_, hb_, att_, dout_, dbias_, logits_, kc_, vc_, align_})
        if (!p) {
            err_ = "device memory allocation failed";
            return;
        }
    // suppress mask and alignment slots (model.rs:411-425)
    std::vector<unsigned char> sup(dm_.vocab, 0);
    for (int t : gc_.suppress)
        if (t >= 0 && t < dm_.vocab) sup[t] = 1;
    sup_ = (unsigned char*)alloc(dm_.vocab);
    std::vector<int> slots(nl * nh, -1);
    for (int s = 0; s < na; s++) slots[gc_.align_heads[s].first * nh + gc_.align_heads[s].second] = s;
    aslot_ = (int*)alloc(slots.size() * 4);
    if (!sup_ || !aslot_) {
        err_ = "device memory allocation failed";
        return;
    }
    cudaMemcpyAsync(sup_, sup.data(), sup.size(), cudaMemcpyHostToDevice, st_);
    cudaMemcpyAsync(aslot_, slots.data(), slots.size() * 4, cudaMemcpyHostToDevice, st_);
    cudaStreamSynchronize(st_);
    if (init_weights(seed)) {
        err_ = std::string("weight initialisation failed: ") + last_error();
        return;
    }
    // bias images of every decoder layer's outputs (model.rs:505-511)
    for (int i = 0; i < nl; i++) {
        const DecLayer& l = dec_[i];
        const std::pair<int, const Lin*> outs[6] = {{3 * d, &l.qkv}, {d, &l.o}, {d, &l.xq}, {d, &l.xo}, {ff, &l.fc1}, {d, &l.fc2}};
        for (int o = 0; o < 6; o++) {
            void* dst = (char*)dbias_ + ((char*)dec_out(i, o) - (char*)dout_);
            if (k_->fill_bias(dst, outs[o].second->b, bmax, outs[o].first, outs[o].first, st_)) {
                err_ = last_error();
                return;
            }
        }
    }
    if (cudaStreamSynchronize(st_) != cudaSuccess) {
        err_ = "engine set-up failed";
        return;
    }
    if (st2_) {
        const int r = lanes_rows_match();
        if (r < 0) {
            err_ = std::string("decoder lane check failed: ") + last_error();
            return;
        }
        lanes_ok_ = r == 1;
        lanes_ = lanes_ok_ ? 2 : 1;
    }
}

// The two decoder lanes give the one-lane results only if cuBLAS returns, for 16 rows, the rows it returns for 32.
// Checked once per engine on this GPU and library for the four decoder GEMM shapes, with layer 0's weights, seeded
// inputs and the same call as the decoding step (each half on its own lane's handle): 1 if every output is equal bit
// for bit, 0 if not, -1 on an error.
int Engine::lanes_rows_match() {
    // a test hook: MMZ_TEST_LANES_DIFFER=1 makes the check report different rows, so that the one-lane fallback can be
    // exercised on hardware where cuBLAS does return equal rows
    if (const char* t = getenv("MMZ_TEST_LANES_DIFFER"))
        if (t[0] == '1') return 0;
    // the probe buffers live only for the check (plain allocations, freed on every return path)
    struct Probe {
        void* p[3] = {nullptr, nullptr, nullptr};
        ~Probe() { for (void* q : p) if (q) cudaFree(q); }
    } pb;
    const int d = dm_.d, ff = dm_.ff, kmax = ff > d ? ff : d, nmax = 3 * d > ff ? 3 * d : ff;
    const int rows = 2 * LANE_ROWS;
    if (cudaMalloc(&pb.p[0], (size_t)rows * kmax * 2) != cudaSuccess ||
        cudaMalloc(&pb.p[1], (size_t)rows * nmax * 2) != cudaSuccess ||
        cudaMalloc(&pb.p[2], (size_t)rows * nmax * 2) != cudaSuccess)
        return fail("device memory allocation failed");
    void *x = pb.p[0], *y1 = pb.p[1], *y2 = pb.p[2];
    if (launch_fill_normal(x, (long)rows * kmax, 0x5eedull, 0.f, 1.f, st_)) return -1;
    const DecLayer& l = dec_[0];
    const struct { const void* w; int n, k; } shapes[4] = {{l.qkv.w, 3 * d, d}, {l.o.w, d, d}, {l.fc1.w, ff, d}, {l.fc2.w, d, ff}};
    std::vector<uint16_t> a((size_t)rows * nmax), b((size_t)rows * nmax);
    for (const auto& sh : shapes) {
        const size_t bytes = (size_t)rows * sh.n * 2;
        CUDA_CK(cudaMemsetAsync(y1, 0, bytes, st_));
        CUDA_CK(cudaMemsetAsync(y2, 0, bytes, st_));
        CK(matmul(true, false, sh.n, rows, sh.k, 1.f, sh.w, sh.k, 0, x, sh.k, 0, 1.f, y1, sh.n, 0, 1, blas_));
        CK(matmul(true, false, sh.n, LANE_ROWS, sh.k, 1.f, sh.w, sh.k, 0, x, sh.k, 0, 1.f, y2, sh.n, 0, 1, blas_));
        CUDA_CK(cudaStreamSynchronize(st_));
        CK(matmul(true, false, sh.n, LANE_ROWS, sh.k, 1.f, sh.w, sh.k, 0, (const char*)x + (size_t)LANE_ROWS * sh.k * 2,
                  sh.k, 0, 1.f, (char*)y2 + (size_t)LANE_ROWS * sh.n * 2, sh.n, 0, 1, blas2_));
        CUDA_CK(cudaStreamSynchronize(st2_));
        CUDA_CK(cudaMemcpy(a.data(), y1, bytes, cudaMemcpyDeviceToHost));
        CUDA_CK(cudaMemcpy(b.data(), y2, bytes, cudaMemcpyDeviceToHost));
        if (std::memcmp(a.data(), b.data(), bytes) != 0) return 0;
    }
    return 1;
}

Engine::~Engine() {
    if (graph_) cudaGraphExecDestroy(graph_);
    if (st_) cudaStreamSynchronize(st_);
    k_.reset();
    for (void* p : allocs_) cudaFree(p);
    if (st2_) cudaStreamSynchronize(st2_);
    if (blas_) cublasDestroy(blas_);
    if (blas2_) cublasDestroy(blas2_);
    if (lt_) cublasLtDestroy(lt_);
    if (fork_ev_) cudaEventDestroy(fork_ev_);
    if (join_ev_) cudaEventDestroy(join_ev_);
    if (st2_) cudaStreamDestroy(st2_);
    if (poll_ev_) cudaEventDestroy(poll_ev_);
    if (done_host_) cudaFreeHost(done_host_);
    if (st_) cudaStreamDestroy(st_);
}

// Random-init weights with the fused layouts of model.rs:253-264 (qkv [3d][d], bias [q, 0, v]) and :387-399 (every
// decoder layer's cross k/v projection fused: [nl * 2d][d], bias [0, v] per layer). Linear weights and embeddings
// N(0, 0.02), biases N(0, 0.02), layer-norm weights N(1, 0.02) and biases N(0, 0.02); the encoder positions are
// Whisper's sinusoids. One allocation per tensor class, seeded per tensor.
int Engine::init_weights(unsigned long long seed) {
    const int d = dm_.d, ff = dm_.ff, nm = dm_.n_mels, nl = dm_.dec_layers;
    unsigned long long tid = 0;
    auto normal = [&](size_t n, float mean, float std) -> void* {
        void* p = alloc(n * 2);
        if (!p) return nullptr;
        if (launch_fill_normal(p, (long)n, seed * 1000003ull + (++tid), mean, std, st_)) return nullptr;
        return p;
    };
    auto ln = [&](Ln& l) { l.w = normal(d, 1.f, 0.02f); l.b = normal(d, 0.f, 0.02f); return l.w && l.b; };
    auto lin = [&](Lin& l, size_t n, size_t k) { l.w = normal(n * k, 0.f, 0.02f); l.b = normal(n, 0.f, 0.02f); return l.w && l.b; };
    auto qkv = [&](Lin& l) {
        if (!lin(l, 3 * (size_t)d, d)) return false;
        return cudaMemsetAsync((char*)l.b + (size_t)d * 2, 0, (size_t)d * 2, st_) == cudaSuccess;  // k_proj has no bias
    };
    enc_.resize(dm_.enc_layers);
    for (auto& l : enc_)
        if (!ln(l.ln1) || !qkv(l.qkv) || !lin(l.o, d, d) || !ln(l.ln2) || !lin(l.fc1, ff, d) || !lin(l.fc2, d, ff)) return -1;
    dec_.resize(nl);
    for (auto& l : dec_)
        if (!ln(l.ln1) || !qkv(l.qkv) || !lin(l.o, d, d) || !ln(l.lnx) || !lin(l.xq, d, d) || !lin(l.xo, d, d) ||
            !ln(l.ln3) || !lin(l.fc1, ff, d) || !lin(l.fc2, d, ff))
            return -1;
    if (!lin(xkv_, (size_t)nl * 2 * d, d)) return -1;
    for (int i = 0; i < nl; i++) cudaMemsetAsync((char*)xkv_.b + (size_t)i * 2 * d * 2, 0, (size_t)d * 2, st_);
    if (!lin(conv1_, d, (size_t)nm * 3) || !lin(conv2_, d, (size_t)d * 3) || !ln(eln_) || !ln(dln_)) return -1;
    emb_ = normal((size_t)dm_.vocab * d, 0.f, 0.02f);
    dpos_ = normal((size_t)dm_.max_t * d, 0.f, 0.02f);
    if (!emb_ || !dpos_) return -1;
    // sinusoids(1500, d): [sin(t * inc_i) | cos(t * inc_i)], inc_i = exp(-log(10000) / (d/2 - 1) * i)
    std::vector<uint16_t> pos((size_t)TENC_ * d);
    const int half = d / 2;
    for (int t = 0; t < TENC_; t++)
        for (int i = 0; i < half; i++) {
            const double inv = std::exp(-std::log(10000.0) / (half - 1) * i);
            pos[(size_t)t * d + i] = f2h((float)std::sin(t * inv));
            pos[(size_t)t * d + half + i] = f2h((float)std::cos(t * inv));
        }
    epos_ = alloc(pos.size() * 2);
    if (!epos_) return -1;
    CUDA_CK(cudaMemcpyAsync(epos_, pos.data(), pos.size() * 2, cudaMemcpyHostToDevice, st_));
    CUDA_CK(cudaStreamSynchronize(st_));
    return 0;
}

// decoder layer i's output `which` (qkv, o, xq, xo, fc1, fc2) inside dout, [bmax][n] each (model.rs:516-522)
void* Engine::dec_out(int i, int which) const {
    const size_t d = dm_.d, ff = dm_.ff, b = bmax_;
    const size_t offs[6] = {0, 3 * d, 4 * d, 5 * d, 6 * d, 6 * d + ff};
    return (char*)dout_ + 2 * (i * b * (7 * d + ff)) + 2 * b * offs[which];
}

// column-major strided-batched fp16 GEMM, fp32 accumulation (gpu.rs:254-286)
int Engine::matmul(bool ta, bool tb, int m, int n, int k, float alpha, const void* a, int lda, long long sa,
                   const void* b, int ldb, long long sb, float beta, void* c, int ldc, long long sc, int batch,
                   cublasHandle_t h) {
    cublasStatus_t r = cublasGemmStridedBatchedEx(
        h ? h : blas_, ta ? CUBLAS_OP_T : CUBLAS_OP_N, tb ? CUBLAS_OP_T : CUBLAS_OP_N, m, n, k, &alpha, a, CUDA_R_16F, lda, sa,
        b, CUDA_R_16F, ldb, sb, &beta, c, CUDA_R_16F, ldc, sc, batch, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    return r == CUBLAS_STATUS_SUCCESS ? 0 : failf("cublasGemmStridedBatchedEx failed (%d)", (int)r);
}

// y = x W^T + bias: bias first, then the GEMM accumulates onto it (beta = 1), one rounding of acc + bias
// (gpu.rs:208-236); m <= 8 goes to the image's gemv kernels where it has them
int Engine::lin(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k) {
    if (m <= 8) {
        int r = k_->gemv(x, ldx, l.w, y, ldy, m, n, k, l.b, st_);
        if (r != -2) return r;
    }
    CK(k_->fill_bias(y, l.b, m, n, ldy, st_));
    return matmul(true, false, n, m, k, 1.f, l.w, k, 0, x, ldx, 0, 1.f, y, ldy, 0, 1);
}

// the same for a y that already holds the bias (gpu.rs:238-247)
int Engine::lin_onto_bias(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k) {
    return lin_onto_bias_on(x, ldx, l, y, ldy, m, n, k, st_, blas_);
}

int Engine::lin_onto_bias_on(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k,
                             cudaStream_t st, cublasHandle_t h) {
    if (m <= 8) {
        int r = k_->gemv(x, ldx, l.w, y, ldy, m, n, k, l.b, st);
        if (r != -2) return r;
    }
    return matmul(true, false, n, m, k, 1.f, l.w, k, 0, x, ldx, 0, 1.f, y, ldy, 0, 1, h);
}

// The native encoder's linear layers take their bias in the GEMM's epilogue instead of a bias image that the GEMM
// reads back (model.rs:543-623 writes the image, then accumulates onto it): one write of y instead of two writes and a
// read. The fp32 accumulator plus the bias is rounded once either way; the algorithm is cuBLASLt's first heuristic
// choice for the shape, so the sums may associate differently from cublasGemmEx's (the encoder is compared with the
// reference's within tolerance, not bit for bit).
int Engine::gemm_bias(const void* x, int ldx, const void* w, long long sw, const void* bias, void* y, int ldy,
                      long long sy, int m, int n, int k, int batch) {
    if (!lt_) return -2;
    const long long key[8] = {m, n, k, batch, ldx, ldy, sw, sy};
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
    int rc = -2;
    const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
    const cublasLtEpilogue_t epi = CUBLASLT_EPILOGUE_BIAS;
    const cudaDataType_t bt = CUDA_R_16F;
    const long long bstride = n, zero = 0;
    const float one = 1.f, nil = 0.f;
    auto ok = [](cublasStatus_t s) { return s == CUBLAS_STATUS_SUCCESS; };
    if (ok(cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F)) &&
        ok(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA))) &&
        ok(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB))) &&
        ok(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_EPILOGUE, &epi, sizeof(epi))) &&
        ok(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof(bias))) &&
        ok(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_DATA_TYPE, &bt, sizeof(bt))) &&
        (batch == 1 || ok(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_BATCH_STRIDE, &bstride,
                                                          sizeof(bstride)))) &&
        // column-major: W^T (n x k, stored k x n), x^T (k x m), y^T (n x m)
        ok(cublasLtMatrixLayoutCreate(&la, CUDA_R_16F, k, n, k)) && ok(cublasLtMatrixLayoutCreate(&lb, CUDA_R_16F, k, m, ldx)) &&
        ok(cublasLtMatrixLayoutCreate(&lc, CUDA_R_16F, n, m, ldy))) {
        bool lay = true;
        if (batch > 1)
            for (auto [l, s] : {std::pair<cublasLtMatrixLayout_t, long long>{la, sw}, {lb, zero}, {lc, sy}}) {
                lay = lay && ok(cublasLtMatrixLayoutSetAttribute(l, CUBLASLT_MATRIX_LAYOUT_BATCH_COUNT, &batch,
                                                                 sizeof(batch))) &&
                      ok(cublasLtMatrixLayoutSetAttribute(l, CUBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET, &s,
                                                          sizeof(s)));
            }
        LtPlan* plan = nullptr;
        for (LtPlan& p : lt_plans_)
            if (std::equal(key, key + 8, p.key)) plan = &p;
        if (lay && !plan) {
            LtPlan p{};
            std::copy(key, key + 8, p.key);
            cublasLtMatmulPreference_t pref = nullptr;
            const size_t wsb = WS_BYTES;
            cublasLtMatmulHeuristicResult_t res{};
            int nres = 0;
            p.ok = ok(cublasLtMatmulPreferenceCreate(&pref)) &&
                   ok(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &wsb,
                                                           sizeof(wsb))) &&
                   ok(cublasLtMatmulAlgoGetHeuristic(lt_, op, la, lb, lc, lc, pref, 1, &res, &nres)) && nres > 0;
            if (pref) cublasLtMatmulPreferenceDestroy(pref);
            p.algo = res.algo;
            lt_plans_.push_back(p);
            plan = &lt_plans_.back();
        }
        if (lay && plan && plan->ok)
            rc = ok(cublasLtMatmul(lt_, op, &one, w, la, x, lb, &nil, y, lc, y, lc, &plan->algo, ws_, WS_BYTES, st_))
                     ? 0
                     : failf("cublasLtMatmul failed");
    }
    if (la) cublasLtMatrixLayoutDestroy(la);
    if (lb) cublasLtMatrixLayoutDestroy(lb);
    if (lc) cublasLtMatrixLayoutDestroy(lc);
    if (op) cublasLtMatmulDescDestroy(op);
    return rc;
}

int Engine::lin_enc(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k) {
    const int r = gemm_bias(x, ldx, l.w, 0, l.b, y, ldy, 0, m, n, k, 1);
    return r == -2 ? lin(x, ldx, l, y, ldy, m, n, k) : r;
}

// model.rs:543-625
int Engine::encode_dev(const void* mel16, int gn, int slot0) {
    if (gn < 1 || gn > eg_ || slot0 < 0 || slot0 + gn > bmax_) return fail("encode: bad group");
    const int d = dm_.d, nm = dm_.n_mels, nh = dm_.nh, ff = dm_.ff, nl = dm_.dec_layers;
    const long r1 = (long)gn * NFRAMES, r2 = (long)gn * TENC_;
    const bool tc = enc_tc_ && k_->native();
    if (mel16 != mel_) CUDA_CK(cudaMemcpyAsync(mel_, mel16, (size_t)gn * nm * NFRAMES * 2, cudaMemcpyDeviceToDevice, st_));
    CK(k_->im2col1(mel_, x1_, r1 * 3 * nm, nm, st_));
    CK(lin_enc(x1_, 3 * nm, conv1_, h1_, d, r1, d, 3 * nm));
    CK(k_->gelu(h1_, r1 * d, st_));
    CK(k_->im2col2(h1_, x2_, r2 * 3 * d, d, st_));
    CK(lin_enc(x2_, 3 * d, conv2_, ex_, d, r2, d, 3 * d));
    CK(k_->gelu(ex_, r2 * d, st_));
    CK(k_->add_pos(ex_, epos_, r2, d, TENC_, st_));
    CK(k_->layernorm(ex_, enc_[0].ln1, eh_, r2, d, st_));
    for (size_t i = 0; i < enc_.size(); i++) {
        const EncLayer& l = enc_[i];
        if (tc) CK(launch_gemm_bias(eh_, d, l.qkv.w, l.qkv.b, eqkv_, 3 * d, r2, 3 * d, d, 0, 0, st_));
        else CK(lin_enc(eh_, d, l.qkv, eqkv_, 3 * d, r2, 3 * d, d));
        if (enc_unfused_) CK(enc_attn_unfused(gn));
        else CK(k_->enc_attn(eqkv_, eatt_, gn, d, nh, st_));
        CK(lin_enc(eatt_, d, l.o, eh_, d, r2, d, d));
        CK(k_->add_layernorm(ex_, eh_, l.ln2, eh_, r2, d, st_));
        if (tc) {
            CK(launch_gemm_bias(eh_, d, l.fc1.w, l.fc1.b, ef_, ff, r2, ff, d, 1, 0, st_));
        } else {
            CK(lin_enc(eh_, d, l.fc1, ef_, ff, r2, ff, d));
            CK(k_->gelu(ef_, r2 * ff, st_));
        }
        CK(lin_enc(ef_, ff, l.fc2, eh_, d, r2, d, ff));
        const Ln& next = i + 1 < enc_.size() ? enc_[i + 1].ln1 : eln_;
        CK(k_->add_layernorm(ex_, eh_, next, eh_, r2, d, st_));
    }
    // cross k/v per (layer, k|v, head) as [position][64] blocks: one batched GEMM per clip onto the bias (:614-623)
    const long xkv = (long)nl * 2 * d * TENC_;
    const int nblk = nl * 2 * nh;
    for (int c = 0; c < gn; c++) {
        void* dst = (char*)xkv_buf_ + 2 * (size_t)(slot0 + c) * xkv;
        const void* xc = (char*)eh_ + 2 * (size_t)c * TENC_ * d;
        if (tc) {
            CK(launch_gemm_bias(xc, d, xkv_.w, xkv_.b, dst, 0, TENC_, nblk * HDIM, d, 2, (long)TENC_ * HDIM, st_));
            continue;
        }
        const int r = gemm_bias(xc, d, xkv_.w, (long long)HDIM * d, xkv_.b, dst, HDIM, (long long)TENC_ * HDIM, TENC_,
                                HDIM, d, nblk);
        if (r == 0) continue;
        if (r != -2) return r;
        CK(k_->fill_bias_heads(dst, xkv_.b, xkv / 8, st_));
        CK(matmul(true, false, HDIM, TENC_, d, 1.f, xkv_.w, d, (long long)HDIM * d, xc, d, 0, 1.f, dst, HDIM,
                  (long long)TENC_ * HDIM, nblk));
    }
    return 0;
}

// The unfused encoder attention of model.rs:567-604 (--enc-attn cublas), clip by clip: scores^T = 0.125 K Q^T per head
// into the [heads][query][key] fp16 buffer esc (one strided-batched GEMM), the row softmax in place, then
// att = (V^T P^T)^T (one more), with the reference's GEMM parameters.
int Engine::enc_attn_unfused(int gn) {
    const int d = dm_.d, nh = dm_.nh;
    if (!esc_) {
        esc_ = alloc((size_t)nh * TENC_ * TENC_ * 2);
        if (!esc_) return fail("enc_attn (cublas): device memory allocation failed");
    }
    for (int c = 0; c < gn; c++) {
        const char* q = (const char*)eqkv_ + 2 * (size_t)c * TENC_ * 3 * d;
        const char* kk = q + 2 * (size_t)d;
        const char* v = q + 4 * (size_t)d;
        CK(matmul(true, false, TENC_, TENC_, HDIM, 0.125f, kk, 3 * d, HDIM, q, 3 * d, HDIM, 0.f, esc_, TENC_,
                  (long long)TENC_ * TENC_, nh));
        CK(k_->softmax_rows(esc_, (long)nh * TENC_, TENC_, st_));
        void* out = (char*)eatt_ + 2 * (size_t)c * TENC_ * d;
        CK(matmul(false, false, HDIM, TENC_, TENC_, 1.f, v, 3 * d, HDIM, esc_, TENC_, (long long)TENC_ * TENC_, 0.f,
                  out, d, HDIM, nh));
    }
    return 0;
}

int Engine::set_enc_gemm(int mode) {
    if (mode != 0 && mode != 1) return fail("set_enc_gemm: 0 (cuBLASLt) or 1 (this library's tensor-core GEMM)");
    enc_tc_ = mode == 1;
    return 0;
}

int Engine::set_enc_attn(int unfused) {
    if (unfused != 0 && unfused != 1) return fail("set_enc_attn: 0 (fused kernel) or 1 (cuBLAS scores, row softmax, cuBLAS P.V)");
    enc_unfused_ = unfused == 1;
    return 0;
}

int Engine::reset(const int* prompts, int b, int np) {
    if (b < 1 || b > bmax_ || np < 1 || np >= dm_.max_t) return fail("reset: bad batch or prompt");
    const int mt = dm_.max_t;
    std::vector<int> t((size_t)b * mt, 0);
    for (int s = 0; s < b; s++) std::memcpy(&t[(size_t)s * mt], prompts + (size_t)s * np, np * 4);
    CUDA_CK(cudaMemcpyAsync(tok_, t.data(), t.size() * 4, cudaMemcpyHostToDevice, st_));
    CUDA_CK(cudaMemsetAsync(done_, 0, (size_t)b * 4, st_));
    CUDA_CK(cudaMemsetAsync(ctr_, 0, 16, st_));
    CUDA_CK(cudaStreamSynchronize(st_));
    return 0;
}

int Engine::set_lanes(int n) {
    if (n != 1 && n != 2) return fail("set_lanes: 1 or 2");
    if (n == 2 && !st2_)
        return fail("set_lanes: two lanes need the native kernel image and an engine for at least 32 sequences");
    if (n == 2 && !lanes_ok_)
        return fail("set_lanes: cuBLAS on this GPU returns other rows for half batches; decoding stays on one lane");
    lanes_ = n;
    return 0;
}

// model.rs:665-705 for the sequences [r0, r0 + bh): every buffer of the step is [sequence][...], so a lane works on
// its rows of each (and on its own part of the cross-attention scratch)
int Engine::dec_layer(int i, int r0, int bh, cudaStream_t st, cublasHandle_t h) {
    const int d = dm_.d, ff = dm_.ff, nh = dm_.nh, nl = dm_.dec_layers, mt = dm_.max_t;
    const int na = (int)gc_.align_heads.size();
    const DecLayer& l = dec_[i];
    auto rows = [&](void* p, size_t n) { return (void*)((char*)p + 2 * (size_t)r0 * n); };  // row r0 of fp16 [.][n]
    void* kc = (char*)kc_ + 2 * ((size_t)i * bmax_ + r0) * mt * d;
    void* vc = (char*)vc_ + 2 * ((size_t)i * bmax_ + r0) * mt * d;
    void *oqkv = rows(dec_out(i, 0), 3 * d), *oo = rows(dec_out(i, 1), d), *oxq = rows(dec_out(i, 2), d),
         *oxo = rows(dec_out(i, 3), d), *ofc1 = rows(dec_out(i, 4), ff), *ofc2 = rows(dec_out(i, 5), d);
    void *x = rows(x_, d), *hb = rows(hb_, d), *att = rows(att_, d);
    const int* done = done_ + r0;
    const void* xkv = (const char*)xkv_buf_ + 2 * (size_t)r0 * nl * 2 * d * TENC_;
    void* align = (char*)align_ + 2 * (size_t)r0 * mt * na * TENC_;
    void* xs = s_;
    if (r0 > 0) {
        if (!k_->native()) return fail("dec_layer: the fatbin image decodes the whole batch on one lane");
        xs = (char*)s_ + cross_attn_scratch_bytes(r0, d);
    }
    CK(lin_onto_bias_on(hb, d, l.qkv, oqkv, 3 * d, bh, 3 * d, d, st, h));
    CK(k_->self_attn(oqkv, kc, vc, att, ctr_, done, bh, mt, d, nh, st));
    CK(lin_onto_bias_on(att, d, l.o, oo, d, bh, d, d, st, h));
    CK(k_->add_layernorm(x, oo, l.lnx, hb, bh, d, st));
    CK(lin_onto_bias_on(hb, d, l.xq, oxq, d, bh, d, d, st, h));
    CK(k_->cross_attn(oxq, xkv, xs, stat_, part_, att, align, aslot_, ctr_, done, bh, i, nl, d, nh, na, mt, st));
    CK(lin_onto_bias_on(att, d, l.xo, oxo, d, bh, d, d, st, h));
    CK(k_->add_layernorm(x, oxo, l.ln3, hb, bh, d, st));
    // up to 8 sequences the fc1 product and its GELU are one kernel where the image has it (model.rs:708-709)
    const int fg = bh <= 8 ? k_->gemv_gelu(hb, d, l.fc1.w, ofc1, ff, bh, ff, d, l.fc1.b, st) : -2;
    if (fg == -1) return -1;
    if (fg == -2) {
        CK(lin_onto_bias_on(hb, d, l.fc1, ofc1, ff, bh, ff, d, st, h));
        CK(k_->gelu(ofc1, (long)bh * ff, st));
    }
    CK(lin_onto_bias_on(ofc1, ff, l.fc2, ofc2, d, bh, d, ff, st, h));
    const Ln& next = i + 1 < nl ? dec_[i + 1].ln1 : dln_;
    return k_->add_layernorm(x, ofc2, next, hb, bh, d, st);
}

// model.rs:648-736
int Engine::step(int b, int prompt_len) {
    const int d = dm_.d, ff = dm_.ff, nl = dm_.dec_layers, mt = dm_.max_t;
    CK(k_->embed(tok_, ctr_, emb_, dpos_, x_, b, mt, d, st_));
    CK(k_->layernorm(x_, dec_[0].ln1, hb_, b, d, st_));
    // the bias images the cuBLAS products accumulate onto; up to 8 sequences the native gemv adds the bias itself and
    // overwrites every output, so the copy (and the break it makes in the chain of programmatic launches) is left out
    if (!(b <= 8 && k_->native()))
        CUDA_CK(cudaMemcpyAsync(dout_, dbias_, (size_t)2 * nl * bmax_ * (7 * d + ff), cudaMemcpyDeviceToDevice, st_));
    if (lanes_ == 2 && b == 2 * LANE_ROWS) {
        // two lanes: the first half of the sequences on the engine's stream, the second half on the other; forked
        // here, joined before the logits (also inside a graph capture, where the second stream joins the capture)
        const int b0 = LANE_ROWS;
        CUDA_CK(cudaEventRecord(fork_ev_, st_));
        CUDA_CK(cudaStreamWaitEvent(st2_, fork_ev_, 0));
        int r = 0;
        for (int i = 0; i < nl && !r; i++) {
            r = dec_layer(i, 0, b0, st_, blas_);
            if (!r) r = dec_layer(i, b0, b - b0, st2_, blas2_);
        }
        // the join is recorded even after a failure, so that a capture in progress ends with both streams joined
        CUDA_CK(cudaEventRecord(join_ev_, st2_));
        CUDA_CK(cudaStreamWaitEvent(st_, join_ev_, 0));
        if (r) return -1;
    } else {
        for (int i = 0; i < nl; i++) CK(dec_layer(i, 0, b, st_, blas_));
    }
    // logits = hb emb^T (no bias), then the greedy choice and the position counter
    const int bs1 = gc_.bs[0], bs2 = gc_.bs[1];
    const int fr = k_->logits_argmax(hb_, d, emb_, dm_.vocab, b, sup_, tok_, done_, ctr_, mt, prompt_len, gc_.eos, bs1,
                                     bs2, st_);
    if (fr != -2) return fr;  // one kernel did all three (model.rs:714-735)
    const int lr = k_->logits(hb_, d, emb_, logits_, dm_.vocab, b, d, st_);
    if (lr == -1) return -1;
    if (lr == 0) {
    } else if (b <= 8) {
        int r = k_->gemv(hb_, d, emb_, logits_, dm_.vocab, b, dm_.vocab, d, nullptr, st_);
        if (r == -1) return -1;
        if (r == -2) CK(matmul(true, false, dm_.vocab, b, d, 1.f, emb_, d, 0, hb_, d, 0, 0.f, logits_, dm_.vocab, 0, 1));
    } else {
        CK(matmul(true, false, dm_.vocab, b, d, 1.f, emb_, d, 0, hb_, d, 0, 0.f, logits_, dm_.vocab, 0, 1));
    }
    CK(k_->argmax_tok(logits_, dm_.vocab, sup_, tok_, done_, ctr_, b, mt, prompt_len, gc_.eos, bs1, bs2, st_));
    return k_->advance(ctr_, st_);
}

int Engine::capture(int b, int prompt_len) {
    if (graph_) {
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    cudaGraph_t g = nullptr;
    CUDA_CK(cudaStreamBeginCapture(st_, cudaStreamCaptureModeThreadLocal));
    const long long before = k_->launches;
    int r = step(b, prompt_len);
    step_launches_ = k_->launches - before;
    k_->launches = before;  // captured, not executed
    cudaError_t e = cudaStreamEndCapture(st_, &g);
    if (r) {
        if (g) cudaGraphDestroy(g);
        return -1;
    }
    CUDA_CK(e);
    e = cudaGraphInstantiate(&graph_, g, 0);
    cudaGraphDestroy(g);
    CUDA_CK(e);
    CUDA_CK(cudaGraphUpload(graph_, st_));
    graph_b_ = b;
    graph_np_ = prompt_len;
    return 0;
}

int Engine::replay() {
    if (!graph_) return fail("replay: no captured step");
    CUDA_CK(cudaGraphLaunch(graph_, st_));
    k_->launches += step_launches_;
    return 0;
}

// transcribe.rs:104-167
int Engine::transcribe(const float* mel, const int* frames, int n, const int* prompt, int np, int max_steps,
                       bool graph, int threads, int* tokens, int* lens, float* times, double* stage_s) {
    if (n < 1 || n > bmax_) return fail("transcribe: 1..bmax clips per call");
    const auto t0 = std::chrono::steady_clock::now();
    const size_t per = (size_t)dm_.n_mels * NFRAMES;
    if (k_->native()) {
        // fp32 log-mel to the device, rounded to fp16 there by this library's kernel
        for (int g0 = 0; g0 < n; g0 += eg_) {
            const int gn = std::min(eg_, n - g0);
            CUDA_CK(cudaMemcpyAsync(mel32_, mel + per * g0, per * gn * 4, cudaMemcpyHostToDevice, st_));
            CK(launch_f32_to_f16(mel32_, mel_, (long)(per * gn), st_));
            k_->launches++;
            CK(encode_dev(mel_, gn, g0));
        }
    } else {
        // the reference's way (model.rs:549-550, gpu.rs:160-163): each group rounded to fp16 on the host with f2h,
        // uploaded, and the stream synchronised before the host buffer is reused
        std::vector<uint16_t> host(per * (size_t)eg_);
        for (int g0 = 0; g0 < n; g0 += eg_) {
            const int gn = std::min(eg_, n - g0);
            const float* src = mel + per * g0;
            for (size_t i = 0; i < per * gn; i++) host[i] = f2h(src[i]);
            CUDA_CK(cudaMemcpyAsync(mel_, host.data(), per * gn * 2, cudaMemcpyHostToDevice, st_));
            CUDA_CK(cudaStreamSynchronize(st_));
            CK(encode_dev(mel_, gn, g0));
        }
    }
    CUDA_CK(cudaStreamSynchronize(st_));
    return decode_and_times(frames, n, prompt, np, max_steps, graph, threads, tokens, lens, times, stage_s, t0);
}

// The same pipeline from host audio: each group's samples to the device, log-mel there (logmel.cu: the host
// restatement's power spectra, log10 rounded once), then as above. frames [n] receives the 10 ms frames that hold audio.
int Engine::transcribe_audio(const float* const* ys, const long* ns, int n, const int* prompt, int np, int max_steps,
                             bool graph, int threads, int* tokens, int* lens, float* times, int* frames,
                             double* stage_s) {
    if (n < 1 || n > bmax_) return fail("transcribe_audio: 1..bmax clips per call");
    if (!k_->native()) return fail("transcribe_audio: needs the native kernel image (log-mel on the GPU)");
    const auto t0 = std::chrono::steady_clock::now();
    if (!audio_) {  // first call: device staging for one encoder group
        audio_ = (float*)alloc((size_t)eg_ * N_SAMPLES * 4);
        alens_ = (int*)alloc((size_t)eg_ * 4);
        lmw_bytes_ = log_mel_work_bytes(eg_);
        lmw_ = alloc(lmw_bytes_);
        if (!audio_ || !alens_ || !lmw_) return fail("transcribe_audio: device memory allocation failed");
    }
    std::vector<int> lens32(eg_);
    for (int g0 = 0; g0 < n; g0 += eg_) {
        const int gn = std::min(eg_, n - g0);
        for (int c = 0; c < gn; c++) {
            const long len = std::max(0L, std::min(ns[g0 + c], N_SAMPLES));
            lens32[c] = (int)len;
            if (len > 0)
                CUDA_CK(cudaMemcpyAsync(audio_ + (size_t)c * N_SAMPLES, ys[g0 + c], (size_t)len * 4,
                                        cudaMemcpyHostToDevice, st_));
        }
        CUDA_CK(cudaMemcpyAsync(alens_, lens32.data(), (size_t)gn * 4, cudaMemcpyHostToDevice, st_));
        CK(launch_log_mel(audio_, alens_, gn, dm_.n_mels, mel32_, lmw_, lmw_bytes_, st_));
        CK(launch_f32_to_f16(mel32_, mel_, (long)((size_t)dm_.n_mels * NFRAMES * gn), st_));
        CK(encode_dev(mel_, gn, g0));
        CUDA_CK(cudaStreamSynchronize(st_));  // lens32 and the staging buffers are reused by the next group
    }
    for (int s = 0; s < n; s++) frames[s] = (int)std::min((std::max(0L, std::min(ns[s], N_SAMPLES)) + HOP - 1) / HOP,
                                                          (long)NFRAMES);
    return decode_and_times(frames, n, prompt, np, max_steps, graph, threads, tokens, lens, times, stage_s, t0);
}

int Engine::decode_and_times(const int* frames, int n, const int* prompt, int np, int max_steps, bool graph,
                             int threads, int* tokens, int* lens, float* times, double* stage_s,
                             std::chrono::steady_clock::time_point t0) {
    using clk = std::chrono::steady_clock;
    const int mt = dm_.max_t, na = (int)gc_.align_heads.size();
    if (max_steps < 1 || max_steps > mt - 1) max_steps = mt - 1;
    auto t1 = clk::now();
    std::vector<int> prompts((size_t)n * np);
    for (int s = 0; s < n; s++) std::memcpy(&prompts[(size_t)s * np], prompt, np * 4);
    CK(reset(prompts.data(), n, np));
    if (graph && (graph_b_ != n || graph_np_ != np || !graph_)) CK(capture(n, np));
    // src/transcribe.rs:123-142 polls `done` every 8 steps. Here the poll reads the copy recorded 8 steps earlier, which
    // has landed while those steps were queued behind it, so the stream never drains for a poll; a batch whose
    // sequences have all finished may then run up to 8 more steps, which write only end-of-text tokens after the first
    // one and change no output.
    int steps = 0;
    bool polled = false;
    while (steps < max_steps) {
        if (graph) CK(replay());
        else CK(step(n, np));
        steps++;
        if (steps % 8 == 0 && steps >= np) {
            if (polled) {
                CUDA_CK(cudaEventSynchronize(poll_ev_));
                bool all = true;
                for (int s = 0; s < n; s++) all = all && done_host_[s] != 0;
                if (all) break;
            }
            CUDA_CK(cudaMemcpyAsync(done_host_, done_, (size_t)n * 4, cudaMemcpyDeviceToHost, st_));
            CUDA_CK(cudaEventRecord(poll_ev_, st_));
            polled = true;
        }
    }
    CUDA_CK(cudaStreamSynchronize(st_));
    graph_steps_ = steps;
    auto t2 = clk::now();
    CUDA_CK(cudaMemcpyAsync(tokens, tok_, (size_t)n * mt * 4, cudaMemcpyDeviceToHost, st_));
    CUDA_CK(cudaStreamSynchronize(st_));
    // the alignment rows of the generated tokens fed back as input; the last token takes the time of the one before
    const size_t row = (size_t)na * TENC_;
    std::vector<int> nseq(n), nrows(n);
    size_t total = 0;
    for (int s = 0; s < n; s++) {
        const int* t = tokens + (size_t)s * mt;
        int ns = std::min(steps + 1, mt);
        for (int k = np; k < mt; k++)
            if (t[k] == gc_.eos) {
                ns = std::min(k + 1, mt);
                break;
            }
        nseq[s] = ns;
        nrows[s] = std::max(0, ns - 1 - np);
        total += (size_t)nrows[s] * row;
    }
    if (threads < 1) threads = (int)std::max(1u, std::thread::hardware_concurrency());
    threads = std::min(threads, n);
    d2h_bytes_ = (size_t)n * mt * 4;
    if (k_->native()) {
        // the DTW cost and the DTW itself for every clip on the GPU (align.rs:6-106): only the times come back
        std::vector<int> rc(2 * (size_t)n);
        for (int s = 0; s < n; s++) {
            rc[s] = nrows[s];
            rc[n + s] = frames[s] / 2;
        }
        CUDA_CK(cudaMemcpyAsync(rc_, rc.data(), rc.size() * 4, cudaMemcpyHostToDevice, st_));
        CK(launch_align_cost(align_, rc_, rc_ + n, n, np, mt, na, cost_, st_));
        CK(launch_dtw_times(cost_, rc_, rc_ + n, n, mt, tms_, st_));
        k_->launches += 2;
        std::vector<float> th((size_t)n * mt);
        CUDA_CK(cudaMemcpyAsync(th.data(), tms_, th.size() * 4, cudaMemcpyDeviceToHost, st_));
        d2h_bytes_ += th.size() * 4;
        CUDA_CK(cudaStreamSynchronize(st_));
        for (int s = 0; s < n; s++) {
            float* ts = times + (size_t)s * mt;
            std::fill(ts, ts + mt, 0.f);
            lens[s] = nseq[s];
            const int rows = nrows[s];
            if (rows <= 0) continue;
            std::copy(th.data() + (size_t)s * mt, th.data() + (size_t)s * mt + rows, ts + np);
            ts[nseq[s] - 1] = ts[np + rows - 1];
        }
    } else {
        // the reference's path: every recorded probability to the host, jump_times per clip there (align.rs:8-63)
        std::vector<uint16_t> a16(total);
        size_t off = 0;
        for (int s = 0; s < n; s++) {
            if (nrows[s] > 0)
                CUDA_CK(cudaMemcpyAsync(a16.data() + off, (char*)align_ + 2 * ((size_t)s * mt + np) * row,
                                        (size_t)nrows[s] * row * 2, cudaMemcpyDeviceToHost, st_));
            off += (size_t)nrows[s] * row;
        }
        d2h_bytes_ += total * 2;
        CUDA_CK(cudaStreamSynchronize(st_));
        std::vector<size_t> starts(n);
        for (int s = 0, o = 0; s < n; s++) {
            starts[s] = o;
            o += nrows[s] * row;
        }
        auto work = [&](int w) {
            std::vector<float> wf;
            for (int s = w; s < n; s += threads) {
                float* ts = times + (size_t)s * mt;
                std::fill(ts, ts + mt, 0.f);
                lens[s] = nseq[s];
                const int rows = nrows[s];
                if (rows <= 0) continue;
                wf.resize((size_t)rows * row);
                const uint16_t* src = a16.data() + starts[s];
                for (size_t i = 0; i < wf.size(); i++) wf[i] = h2f(src[i]);
                jump_times(wf.data(), rows, na, TENC_, frames[s] / 2, 7, ts + np);
                ts[nseq[s] - 1] = ts[np + rows - 1];
            }
        };
        std::vector<std::thread> th;
        for (int w = 1; w < threads; w++) th.emplace_back(work, w);
        work(0);
        for (auto& t : th) t.join();
    }
    auto t3 = clk::now();
    if (stage_s) {
        stage_s[0] = std::chrono::duration<double>(t1 - t0).count();
        stage_s[1] = std::chrono::duration<double>(t2 - t1).count();
        stage_s[2] = std::chrono::duration<double>(t3 - t2).count();
    }
    return 0;
}

long long Engine::launches() const { return k_ ? k_->launches : 0; }

void* Engine::buffer(const std::string& name) const {
    if (name == "tok") return tok_;
    if (name == "done") return done_;
    if (name == "ctr") return ctr_;
    if (name == "align") return align_;
    if (name == "logits") return logits_;
    if (name == "eh") return eh_;
    if (name == "eqkv") return eqkv_;
    if (name == "eatt") return eatt_;
    if (name == "xkv") return xkv_buf_;
    if (name == "mel") return mel_;
    if (name == "kc") return kc_;
    if (name == "vc") return vc_;
    if (name == "x") return x_;
    if (name == "hb") return hb_;
    if (name == "att") return att_;
    if (name == "aslot") return aslot_;
    return nullptr;
}

}  // namespace mmz
