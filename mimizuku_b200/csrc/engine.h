// The Whisper engine around the attention hot path: a C++ restatement of the reference's src/model.rs (Engine: weight
// layout, buffers, encoder and decoder-step launch sequences) and src/transcribe.rs (batch driver with CUDA-graph
// replay and token timestamps), with the GPU boundary of src/gpu.rs (launch by name, cuBLAS GEMM with the beta = 1
// bias trick).
//
// The engine runs on one of two kernel images with the same buffer layouts:
//   native     the sm_100a kernels of this library (the product)
//   fatbin     any image that exports the reference's 23 kernel names with its argument lists (the reference's own
//              kernels/whisper.cu build is one), launched by name with the reference's grid geometry (model.rs)
#pragma once
#include <cublasLt.h>
#include <cublas_v2.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <chrono>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace mmz {

struct Dims {
    int d, ff, nh, enc_layers, dec_layers, n_mels, vocab, max_t;
};

struct GenCfg {
    int sot, eos, no_timestamps;
    std::vector<int> suppress;
    int bs[2];                                      // begin-suppressed tokens, -1 = none
    std::vector<std::pair<int, int>> align_heads;   // (decoder layer, head)
};

struct Lin {
    void* w;
    void* b;
};
struct Ln {
    void* w;
    void* b;
};

class Kernels;

class Engine {
   public:
    Engine(const Dims& dims, const GenCfg& gc, int bmax, int eg, const char* kernel_image, unsigned long long seed);
    ~Engine();
    bool ok() const { return err_.empty(); }
    const std::string& error() const { return err_; }

    // encoder for gn clips (fp16 log-mel on the device, [gn][n_mels][3000]); cross k/v into slots slot0..
    int encode_dev(const void* mel16, int gn, int slot0);
    // prompt tokens into each slot, all unfinished, position 0 (model.rs:627-637)
    int reset(const int* prompts, int b, int np);
    // one decoding step for b sequences (model.rs:648-736)
    int step(int b, int prompt_len);
    // captures step(b, prompt_len) as a CUDA graph (transcribe.rs:122-131) and replays it
    int capture(int b, int prompt_len);
    int replay();
    // the whole pipeline for n <= bmax clips given host fp32 log-mel [n][n_mels][3000] (transcribe.rs:104-167):
    // upload, encode in groups, greedy decoding (at most max_steps steps, stopping early when every sequence is done),
    // then token timestamps on `threads` host threads. tokens [n][max_t], lens [n], times [n][max_t];
    // stage_s = {encode, decode, timestamps} seconds
    int transcribe(const float* mel, const int* frames, int n, const int* prompt, int np, int max_steps, bool graph,
                   int threads, int* tokens, int* lens, float* times, double* stage_s);
    // the same from host audio (ys[s]: ns[s] samples at 16 kHz, the first 30 s are used): log-mel on the GPU (native
    // image only); frames [n] receives each clip's 10 ms frames that hold audio; stage_s[0] includes the features
    int transcribe_audio(const float* const* ys, const long* ns, int n, const int* prompt, int np, int max_steps,
                         bool graph, int threads, int* tokens, int* lens, float* times, int* frames, double* stage_s);

    void* buffer(const std::string& name) const;
    cudaStream_t stream() const { return st_; }
    const Dims& dims() const { return dm_; }
    int bmax() const { return bmax_; }
    int eg() const { return eg_; }
    int na() const { return (int)gc_.align_heads.size(); }
    size_t allocated() const { return allocated_; }
    int graph_steps() const { return graph_steps_; }
    // kernels of the engine's kernel image launched so far (graph replays count every kernel of the step; cuBLAS
    // GEMMs are not counted)
    long long launches() const;
    long long step_launches() const { return step_launches_; }
    size_t last_d2h_bytes() const { return d2h_bytes_; }
    // decoder-step lanes: 1 runs the step's layers for the whole batch on one stream, as src/model.rs does; 2 (the
    // native image's default) splits a batch of 32 into two halves whose layers run on two streams (one cuBLAS handle
    // and workspace each), forked after the embedding and joined before the logits, so that the latency-bound
    // launches of one half overlap the other's. Every kernel of the step works row by row, so both settings give the
    // same results where cuBLAS gives the same rows for 16 sequences as for 32, which the constructor checks
    // (lanes_rows_match; 1 lane if not); other batch sizes use one lane. The fatbin image always uses 1.
    int set_lanes(int n);
    int lanes() const { return lanes_; }
    // encoder attention: 0 the image's fused kernel (enc_flash), 1 the unfused comparison path of model.rs:567-604
    // (cuBLAS scores into a [heads][1500][1500] buffer, row softmax, cuBLAS P.V; --enc-attn cublas, main.rs:37, 179)
    int set_enc_attn(int unfused);
    int enc_attn() const { return enc_unfused_ ? 1 : 0; }
    // encoder GEMMs of the native image: 0 cuBLASLt with the bias in its epilogue for every linear layer (GELU as a
    // separate kernel, the cross k/v as strided-batched products onto the head blocks); 1 (the default) this
    // library's tensor-core GEMM (mmz_gemm_bias) for qkv, fc1 with its GELU in the epilogue and the cross k/v
    // projection stored into the head blocks, cuBLASLt for the others (o, fc2, the convolutions: faster there)
    int set_enc_gemm(int mode);
    int enc_gemm() const { return enc_tc_ ? 1 : 0; }

   private:
    int lin(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k);
    int lin_onto_bias(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k);
    // native image, encoder: y = x W^T + bias with the bias added in the GEMM's epilogue (cuBLASLt), batched over
    // `batch` weight blocks (strides sw, sy; the bias advances by n per block); -2 when no algorithm supports it
    int gemm_bias(const void* x, int ldx, const void* w, long long sw, const void* bias, void* y, int ldy,
                  long long sy, int m, int n, int k, int batch);
    int lin_enc(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k);
    int matmul(bool ta, bool tb, int m, int n, int k, float alpha, const void* a, int lda, long long sa, const void* b,
               int ldb, long long sb, float beta, void* c, int ldc, long long sc, int batch,
               cublasHandle_t h = nullptr);
    // lin_onto_bias on a given stream and cuBLAS handle (one decoder lane)
    int lin_onto_bias_on(const void* x, int ldx, const Lin& l, void* y, int ldy, int m, int n, int k, cudaStream_t st,
                         cublasHandle_t h);
    // decoder layer i (model.rs:665-705) for the sequences [r0, r0 + bh) on stream st with cuBLAS handle h
    int dec_layer(int i, int r0, int bh, cudaStream_t st, cublasHandle_t h);
    int lanes_rows_match();
    int enc_attn_unfused(int gn);
    void* alloc(size_t bytes);
    int decode_and_times(const int* frames, int n, const int* prompt, int np, int max_steps, bool graph, int threads,
                         int* tokens, int* lens, float* times, double* stage_s,
                         std::chrono::steady_clock::time_point t0);
    void* dec_out(int layer, int which) const;
    int init_weights(unsigned long long seed);

    std::string err_;
    Dims dm_;
    GenCfg gc_;
    int bmax_, eg_;
    int dev_ = 0;
    cudaStream_t st_ = nullptr;
    cublasHandle_t blas_ = nullptr;
    int lanes_ = 1;
    bool enc_unfused_ = false;
    bool enc_tc_ = true;
    void* esc_ = nullptr;  // the unfused encoder attention's scores, allocated on first use
    bool lanes_ok_ = false;          // lanes_rows_match() found the half-batch rows equal
    cudaStream_t st2_ = nullptr;     // second decoder lane
    cublasHandle_t blas2_ = nullptr;
    void* ws2_ = nullptr;
    cudaEvent_t fork_ev_ = nullptr, join_ev_ = nullptr;
    cublasLtHandle_t lt_ = nullptr;
    struct LtPlan {
        long long key[8];
        cublasLtMatmulAlgo_t algo;
        bool ok;
    };
    std::vector<LtPlan> lt_plans_;  // heuristic choice per encoder GEMM shape
    std::unique_ptr<Kernels> k_;
    std::vector<void*> allocs_;
    size_t allocated_ = 0;
    cudaGraphExec_t graph_ = nullptr;
    int graph_b_ = -1, graph_np_ = -1, graph_steps_ = 0;
    long long step_launches_ = 0;

    // weights
    struct EncLayer {
        Ln ln1;
        Lin qkv, o;
        Ln ln2;
        Lin fc1, fc2;
    };
    struct DecLayer {
        Ln ln1;
        Lin qkv, o;
        Ln lnx;
        Lin xq, xo;
        Ln ln3;
        Lin fc1, fc2;
    };
    std::vector<EncLayer> enc_;
    std::vector<DecLayer> dec_;
    Lin conv1_, conv2_, xkv_;
    void *epos_, *emb_, *dpos_;
    Ln eln_, dln_;
    // encoder scratch for eg clips, decoder state for bmax sequences (model.rs:289-321)
    void *mel_, *x1_, *h1_, *x2_, *ex_, *eh_, *eqkv_, *eatt_, *ef_;
    void *xkv_buf_, *x_, *hb_, *att_, *dout_, *dbias_, *logits_, *kc_, *vc_, *s_, *stat_, *part_, *align_;
    float* cost_ = nullptr;  // native image: the token-timestamp DTW cost [bmax][max_t][1500], reduced on the GPU
    int* rc_ = nullptr;      // native image: token rows and frame columns per clip for the cost kernel
    float* tms_ = nullptr;   // native image: the token start times [bmax][max_t] from the GPU DTW
    size_t d2h_bytes_ = 0;   // bytes the last transcribe copied device -> host
    int* done_host_ = nullptr;       // pinned copy of done for the decoding loop's poll
    float* audio_ = nullptr;         // transcribe_audio: one encoder group's samples [eg][480000]
    int* alens_ = nullptr;           // and their lengths
    void* lmw_ = nullptr;            // log-mel work space
    size_t lmw_bytes_ = 0;
    cudaEvent_t poll_ev_ = nullptr;  // recorded after that copy
    int *tok_, *done_, *ctr_, *aslot_;
    unsigned char *sup_;
    float* mel32_;
    void* ws_;
};

}  // namespace mmz
