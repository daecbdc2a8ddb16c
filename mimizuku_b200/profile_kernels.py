"""Runs one hot kernel four times at the benchmark's shapes, for an ncu capture of a single launch
(e.g. ncu --set full --clock-control none -k regex:enc_flash -s 2 -c 1 ...):

    python -m mimizuku_b200.profile_kernels enc            encoder attention, large-v3, 8 clips x 20 heads
    python -m mimizuku_b200.profile_kernels cross          cross-attention, large-v3, batch 32, one layer
    python -m mimizuku_b200.profile_kernels self [p]       self-attention, large-v3, batch 32, position p (default 223)
    python -m mimizuku_b200.profile_kernels step [n] [b]   n decoding steps (default 4) of the large-v3 engine at batch
                                                           b (default 32) from one captured graph, inside the NVTX
                                                           range "steps" (ncu --nvtx --nvtx-include "steps/" captures
                                                           only those)
    python -m mimizuku_b200.profile_kernels logits         logits fused with the greedy choice, large-v3, batch 32
    python -m mimizuku_b200.profile_kernels ln             add_layernorm at the encoder's 12000 x 1280
    python -m mimizuku_b200.profile_kernels logmel         the GPU log-mel of 32 synthetic 30 s clips (128 mel bins)
    python -m mimizuku_b200.profile_kernels align          timestamp cost and DTW of 32 clips x 223 tokens x 10 heads
    python -m mimizuku_b200.profile_kernels encode         one encoder group of the large-v3 engine (8 clips), inside the
                                                           NVTX range "encode" (after one untimed group)
    python -m mimizuku_b200.profile_kernels gemm [mode]    the encoder's qkv projection (12000 x 3840 x 1280) on the
                                                           tensor-core GEMM; mode 1: fc1 with GELU (12000 x 5120 x 1280)
    python -m mimizuku_b200.profile_kernels gemv [m] [n k] the decoder's gemv at m sequences (default 8) over the
                                                           large-v3 logits (51866 x 1280) or n x k
"""
import sys

import torch

import mimizuku_b200 as m


def main(argv):
    which = argv[0] if argv else "enc"
    m.init(0)
    torch.manual_seed(0)
    if which == "enc":
        g, d = 8, 1280
        qkv = torch.randn(g, 1500, 3 * d, device="cuda", dtype=torch.float16)
        out = torch.empty(g, 1500, d, device="cuda", dtype=torch.float16)
        for _ in range(4):
            m.enc_flash(qkv, out, d)
    elif which == "cross":
        B, d, nl, nh, mt, na = 32, 1280, 1, 20, 448, 10
        kv = torch.randn(B, nl, 2, nh, 1500, 64, device="cuda", dtype=torch.float16)
        q = torch.randn(B, d, device="cuda", dtype=torch.float16)
        aslot = torch.full((nl * nh,), -1, dtype=torch.int32, device="cuda")
        aslot[:na] = torch.arange(na, dtype=torch.int32, device="cuda")
        align = torch.zeros(B, mt, na, 1500, dtype=torch.float16, device="cuda")
        ctr = torch.tensor([100, 0, 0, 0], dtype=torch.int32, device="cuda")
        done = torch.zeros(B, dtype=torch.int32, device="cuda")
        out = torch.zeros(B, d, dtype=torch.float16, device="cuda")
        scratch = torch.zeros(m.cross_attn_scratch_bytes(B, d), dtype=torch.uint8, device="cuda")
        for _ in range(4):
            m.cross_attn(q, kv, out, align, aslot, ctr, done, 0, nl, d, na, mt, scratch)
    elif which == "self":
        B, d, mt = 32, 1280, 448
        p = int(argv[1]) if len(argv) > 1 else 223
        kc = torch.randn(B, mt, d, device="cuda", dtype=torch.float16)
        vc = torch.randn(B, mt, d, device="cuda", dtype=torch.float16)
        qkv = torch.randn(B, 3 * d, device="cuda", dtype=torch.float16)
        done = torch.zeros(B, dtype=torch.int32, device="cuda")
        out = torch.zeros(B, d, dtype=torch.float16, device="cuda")
        ctr = torch.tensor([p, 0, 0, 0], dtype=torch.int32, device="cuda")
        for _ in range(4):
            m.self_attn(qkv, kc, vc, out, ctr, done, mt, d)
    elif which == "step":
        import numpy as np
        n = int(argv[1]) if len(argv) > 1 else 4
        b = int(argv[2]) if len(argv) > 2 else 32
        cfg = m.LARGE_V3
        e = m.Engine(cfg, bmax=b, eg=8, device=0, seed=1234, suppress=[cfg.eos])
        mel16 = torch.randn(b, cfg.n_mels, 3000, device="cuda").half()
        for g0 in range(0, b, 8):
            e.encode(mel16[g0].data_ptr(), min(8, b - g0), g0)
        e.reset(np.tile(np.array(cfg.prompt, np.int32), (b, 1)))
        e.capture(b, len(cfg.prompt))
        for _ in range(len(cfg.prompt) + 8):  # past the prompt, graph captured and warm
            e.replay()
        e.sync()
        torch.cuda.nvtx.range_push("steps")
        for _ in range(n):
            e.replay()
        e.sync()
        torch.cuda.nvtx.range_pop()
        e.close()
    elif which == "encode":
        cfg = m.LARGE_V3
        e = m.Engine(cfg, bmax=8, eg=8, device=0, seed=1234, suppress=[cfg.eos])
        mel16 = torch.randn(8, cfg.n_mels, 3000, device="cuda").half()
        e.encode(mel16.data_ptr(), 8, 0)
        e.sync()
        torch.cuda.nvtx.range_push("encode")
        e.encode(mel16.data_ptr(), 8, 0)
        e.sync()
        torch.cuda.nvtx.range_pop()
        e.close()
    elif which == "logits":
        V, d, B, mt = 51866, 1280, 32, 448
        emb = (torch.randn(V, d, device="cuda") * 0.02).half()
        x = torch.randn(B, d, device="cuda").half()
        sup = torch.zeros(V, dtype=torch.uint8, device="cuda")
        tok = torch.zeros(B, mt, dtype=torch.int32, device="cuda")
        done = torch.zeros(B, dtype=torch.int32, device="cuda")
        ctr = torch.tensor([100, 0, 0, 0], dtype=torch.int32, device="cuda")
        scratch = torch.zeros(m.logits_argmax_scratch_bytes(), dtype=torch.uint8, device="cuda")
        for _ in range(4):
            m.logits_argmax(x, emb, sup, tok, done, ctr, mt, 4, 50257, scratch=scratch)
    elif which == "ln":
        R, D = 12000, 1280
        x = torch.randn(R, D, device="cuda").half()
        dx = torch.randn(R, D, device="cuda").half()
        w, b = torch.randn(D, device="cuda").half(), torch.randn(D, device="cuda").half()
        for _ in range(4):
            m.add_layernorm(x, dx, w, b, dx)
    elif which == "logmel":
        n = 32
        ys = [torch.from_numpy(m.synth_clip(1000003 * i + 17)) for i in range(n)]
        audio = torch.stack(ys).cuda()
        lens = torch.full((n,), 480000, dtype=torch.int32, device="cuda")
        out = torch.empty(n, 128, 3000, device="cuda")
        work = torch.empty(m.log_mel_gpu_work_bytes(n), dtype=torch.uint8, device="cuda")
        for _ in range(4):
            m.log_mel_gpu(audio, lens, 128, out, work=work)
    elif which == "gemm":
        mode = int(argv[1]) if len(argv) > 1 else 0
        M, N, K = (12000, 5120, 1280) if mode == 1 else (12000, 3840, 1280)
        a = torch.randn(M, K, device="cuda", dtype=torch.float16)
        w = torch.randn(N, K, device="cuda", dtype=torch.float16) * 0.03
        b = torch.randn(N, device="cuda", dtype=torch.float16)
        c = torch.empty(M, N, device="cuda", dtype=torch.float16)
        for _ in range(4):
            m.gemm_bias(a, w, b, c, mode=mode)
    elif which == "gemv":
        mm = int(argv[1]) if len(argv) > 1 else 8
        N, K = (int(argv[2]), int(argv[3])) if len(argv) > 3 else (51866, 1280)
        w = (torch.randn(N, K, device="cuda") * 0.02).half()
        x = torch.randn(mm, K, device="cuda").half()
        y = torch.empty(mm, N, device="cuda", dtype=torch.float16)
        for _ in range(4):
            m.gemv(x, w, None, y)
    elif which == "align":
        n, mt, na, np_, rows = 32, 448, 10, 4, 223
        align = torch.rand(n, mt, na, 1500, device="cuda").half()
        rc = torch.tensor([rows] * n + [1500] * n, dtype=torch.int32, device="cuda")
        cost = torch.empty(n, mt, 1500, device="cuda")
        times = torch.empty(n, mt, device="cuda")
        for _ in range(4):
            m.align_cost(align, rc[:n], rc[n:], np_, mt, na, cost, n=n)
            m.dtw_times(cost, rc[:n], rc[n:], mt, times, n=n)
    else:
        raise SystemExit(__doc__)
    torch.cuda.synchronize()
    if m.status()[0] != 0:
        raise SystemExit(f"kernel status word {m.status()}")
    print("ok", which)


if __name__ == "__main__":
    main(sys.argv[1:])
