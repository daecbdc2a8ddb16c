"""Benchmark: end-to-end Whisper large-v3 transcription throughput (clips/s) on B200, 32 synthetic 30 s clips per GPU,
random-init weights, 224 fixed greedy tokens, token timestamps by DTW; the metric's other two figures, encoder-attention
TFLOP/s and decoder-attention HBM GB/s, are reported beside it. --model large-v3-turbo runs the 4-decoder-layer model
(the multi-GPU configuration: 32 clips per GPU at 1, 2, 4 and 8 GPUs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference] [--model M] [--clips-per-gpu C]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one process per GPU, 32 clips per GPU: weak scaling)

A step is one batch of 32 clips per GPU. `value` times the GPU pipeline (encoder for 4 groups of 8 clips, then 227
decoding steps replayed from one captured CUDA graph) with the log-mel already in HBM; `e2e` times the C-ABI
transcribe call from host log-mel to host timestamps (upload, encode, decode, token and alignment download, DTW).
--impl reference runs the same host code on the reference's own kernels (the compute_80 build of kernels/whisper.cu,
JIT-compiled by the driver), the GPU implementation the reference ships.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CLIPS_PER_GPU = 32  # default; --clips-per-gpu
NEW_TOKENS = 224
REF_FATBIN = os.path.join(ROOT, "oracle", "_ref", "whisper_ref.fatbin")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, max clock, throttle reasons)."""

    def __init__(self, device):
        self.device, self.proc, self.lines = device, None, []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(5)

    def summary(self):
        sm, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = max(mx, float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_features(n_mels, first_clip, count, threads):
    """The benchmark's seeded clips and their log-mel features on the host (src/audio.rs's restatement on `threads`
    host threads, as src/transcribe.rs:25-56); also returns the clips and the host time."""
    import mimizuku_b200 as m
    ys = [m.synth_clip(1000003 * (first_clip + i) + 17) for i in range(count)]
    t0 = time.perf_counter()
    mel, frames = m.log_mel_batch(ys, n_mels, threads=threads)
    return mel, frames, ys, time.perf_counter() - t0


def features_gpu(ys, n_mels, torch):
    """The same features on the GPU from pinned host audio: host-to-device copy of the samples, then the DFT,
    filterbank and log kernels; seconds for the batch (one warm-up call first, which uploads the tables)."""
    import mimizuku_b200 as m
    count = len(ys)
    audio = torch.zeros((count, 480000), dtype=torch.float32).pin_memory()
    for i, y in enumerate(ys):
        audio[i, :len(y)] = torch.from_numpy(y[:480000])
    lens = torch.tensor([min(len(y), 480000) for y in ys], dtype=torch.int32, device="cuda")
    dev = torch.empty((count, 480000), dtype=torch.float32, device="cuda")
    out = torch.empty((count, n_mels, 3000), dtype=torch.float32, device="cuda")
    work = torch.empty(m.log_mel_gpu_work_bytes(count), dtype=torch.uint8, device="cuda")
    best = None
    for _ in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        dev.copy_(audio, non_blocking=True)
        m.log_mel_gpu(dev, lens, n_mels, out, work=work, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        t = time.perf_counter() - t0
        best = t if best is None else min(best, t)
    return best, audio.numel() * 4


def cpu_baseline(cfg, threads):
    """The oracle's multithreaded f32 CPU restatement of the path's attention (the reference has no CPU attention
    path; oracle/oracle_fast.c, AVX2/F16C/FMA), timed on whole clips of the benchmark's workload: one clip's encoder
    attention (every encoder layer, all heads, 1500 x 1500 x 64, on `threads` threads), then `threads` clips' decoder
    attention, one clip per thread (227 decoding steps x every decoder layer: kv_write, causal self-attention and the
    cross-attention over 1500 positions, with the reference kernels' fp16 rounding points). clips/s = 1 / (encoder
    seconds of one clip + decoder seconds / clips)."""
    import ctypes
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import _oracle as O
    rng = np.random.default_rng(0)
    d, nh = cfg.d, cfg.heads
    qkv = O.normal16(rng, (1, 1500, 3 * d))
    out = np.zeros((1, 1500, d), np.float16)
    t0 = time.perf_counter()
    for _ in range(cfg.enc_layers):
        O.orc.orc_cpu_enc_attn(O.u16(qkv), O.u16(out), 1, d, nh, 1500, threads)
    t_enc = time.perf_counter() - t0
    sec = ctypes.c_double()
    np_ = len(cfg.prompt)
    steps = np_ - 1 + NEW_TOKENS
    O.orc.orc_cpu_dec_attn_clips(threads, cfg.dec_layers, nh, np_, steps, cfg.max_t, ctypes.byref(sec))
    t_dec = sec.value
    per_clip = t_enc + t_dec / threads
    return {"value": round(1.0 / per_clip, 5), "unit": "clips/s", "cores": threads, "kind": "port",
            "sample": (f"attention of whole clips: 1 clip's encoder ({cfg.enc_layers} layers x {nh} heads, "
                       f"{t_enc:.2f} s on {threads} threads) + {threads} clips' decoder ({steps} steps x "
                       f"{cfg.dec_layers} layers of self- and cross-attention, one clip per thread, {t_dec:.2f} s)"),
            "enc_s_per_clip": round(t_enc, 3), "dec_s_per_clip": round(t_dec / threads, 3)}


def kernel_rooflines(e, cfg, torch, impl, B):
    """Live CUDA-event timings of the hot kernels, replayed from a CUDA graph on the engine's stream and buffers
    (inputs larger than L2):
    cross-attention (the dominant kernel of the decoding step), self-attention at the mean context, and encoder
    attention. impl "reference" times the reference's kernels (cross_scores + cross_pv + cross_combine, kv_write +
    self_attn, enc_flash) with src/model.rs's launch geometry on the same buffers."""
    import mimizuku_b200 as m
    st = torch.cuda.ExternalStream(e.stream)
    d, nl, mt, na, nh = cfg.d, cfg.dec_layers, cfg.max_t, e.na, cfg.heads
    buf = e.buffer
    ctr = torch.tensor([100, 0, 0, 0], dtype=torch.int32, device="cuda")
    done = torch.zeros(B, dtype=torch.int32, device="cuda")
    q = torch.randn(B, d, device="cuda", dtype=torch.float16)
    out = torch.empty(B, d, device="cuda", dtype=torch.float16)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    heads_per_layer = np.bincount([l for l, _ in e.heads], minlength=nl)
    L = 4 + NEW_TOKENS // 2  # mean context of a 224-token decode
    ctr_s = torch.tensor([L - 1, 0, 0, 0], dtype=torch.int32, device="cuda")
    qkv = torch.randn(B, 3 * d, device="cuda", dtype=torch.float16)
    lstride = B * mt * d * 2
    g = 8
    qkv_e = torch.randn(4, g, 1500, 3 * d, device="cuda", dtype=torch.float16)
    oute = torch.empty(g, 1500, d, device="cuda", dtype=torch.float16)

    def timed(fn, iters):
        """device time per call of `iters` consecutive calls captured in one CUDA graph (no host launch cost in
        the timed replay, as in the decoding step's own graph)"""
        with torch.cuda.stream(st):
            for i in range(3):
                fn(i)
        st.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            for i in range(iters):
                fn(i)
        with torch.cuda.stream(st):
            gr.replay()
            a.record(st)
            gr.replay()
            b.record(st)
        b.synchronize()
        del gr
        return a.elapsed_time(b) * 1e-3 / iters

    if impl == "native":
        scratch = torch.zeros(m.cross_attn_scratch_bytes(B, d), dtype=torch.uint8, device="cuda")
        cross = lambda i: m.cross_attn(q, buf("xkv"), out, buf("align"), buf("aslot"), ctr, done, i % nl, nl, d,  # noqa
                                       na, mt, scratch, batch=B, stream=e.stream)
        selfa = lambda i: m.self_attn(qkv, buf("kc") + (i % nl) * lstride, buf("vc") + (i % nl) * lstride, out,  # noqa
                                      ctr_s, done, mt, d, batch=B, stream=e.stream)
        enc = lambda i: m.enc_flash(qkv_e[i % 4], oute, d, stream=e.stream)  # noqa
    else:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import _oracle as O
        ref = O.RefKernels()
        S = torch.zeros(B * nh * 1500, dtype=torch.float32, device="cuda")
        ST = torch.zeros(B * nh * 48, dtype=torch.float32, device="cuda")
        PT = torch.zeros(B * nh * 24 * 64, dtype=torch.float32, device="cuda")
        P = lambda t: ("p", t if isinstance(t, int) else t.data_ptr())  # noqa: E731

        def cross(i):
            l = i % nl
            ref.launch("cross_scores", (B * nh, 24), 128, [P(q), P(buf("xkv")), P(S), P(ST), P(done), ("i", l),
                                                           ("i", nl), ("i", d)], stream=e.stream)
            ref.launch("cross_pv", (B * nh, 24), 128, [P(S), P(ST), P(buf("xkv")), P(PT), P(buf("align")),
                                                       P(buf("aslot")), P(ctr), P(done), ("i", l), ("i", nl),
                                                       ("i", d), ("i", na), ("i", mt)], stream=e.stream)
            ref.launch("cross_combine", (B * nh,), 64, [P(PT), P(out), P(done), ("i", d)], stream=e.stream)

        def selfa(i):
            kc, vc = buf("kc") + (i % nl) * lstride, buf("vc") + (i % nl) * lstride
            ref.launch("kv_write", (B,), 256, [P(qkv), P(kc), P(vc), P(ctr_s), ("i", mt), ("i", d)], stream=e.stream)
            ref.launch("self_attn", (B, nh), 128, [P(qkv), P(kc), P(vc), P(out), P(ctr_s), P(done), ("i", mt),
                                                   ("i", d)], stream=e.stream)

        enc = lambda i: ref.launch("enc_flash", (24, nh, g), 128, [P(qkv_e[i % 4]), P(oute), ("i", d)],  # noqa
                                   stream=e.stream)
    t_x = timed(cross, 4 * nl)
    bytes_x = B * 1500 * d * 4 + B * d * 4 + B * float(heads_per_layer.mean()) * 1500 * 2
    t_s = timed(selfa, 4 * nl)
    bytes_s = B * L * d * 4 + B * d * 8
    t_e = timed(enc, 12)
    flop_e = 4 * 1500 * 1500 * 64 * nh * g
    torch.cuda.synchronize()
    if impl == "native":
        status = m.status()
        if status[0] != 0:
            raise RuntimeError(f"kernel status word {status}")
    return {"cross": (bytes_x, t_x), "self": (bytes_s, t_s), "enc": (flop_e, t_e)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--threads", type=int, default=0, help="host threads for DTW (0 = all)")
    ap.add_argument("--model", choices=["large-v3", "large-v3-turbo"], default="large-v3")
    ap.add_argument("--clips-per-gpu", type=int, default=CLIPS_PER_GPU, help="clips per GPU (a multiple of 8, <= 32)")
    args = ap.parse_args()
    nb = args.clips_per_gpu
    if nb < 8 or nb > 32 or nb % 8:
        ap.error("--clips-per-gpu: a multiple of 8 from 8 to 32 (encoder groups of 8 clips)")
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and not os.path.exists(REF_FATBIN):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": f"{REF_FATBIN} not built (needs the reference "
                              "sources: make -C oracle ref)"}))
        return

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))

    import mimizuku_b200 as m
    m.init(local)
    cfg = m.LARGE_V3 if args.model == "large-v3" else m.LARGE_V3_TURBO
    metric = f"clips/s (30 s, {cfg.name}, batch {nb})"
    hbm_peak, tc_peak, peak_src = peaks()
    n_threads = args.threads or max(1, (os.cpu_count() or 8) // max(1, world))

    mel, frames, clips, t_feat_host = make_features(cfg.n_mels, rank * nb, nb, n_threads)
    # the end-to-end inputs live in pinned host memory (page-locked: the copies to the device run at full speed)
    mel = torch.from_numpy(mel).pin_memory().numpy()
    clips = [torch.from_numpy(y).pin_memory().numpy() for y in clips]
    kimg = REF_FATBIN if args.impl == "reference" else None
    e = m.Engine(cfg, bmax=nb, eg=8, device=local, kernel_image=kimg, seed=1234,
                 suppress=[cfg.eos])
    mel16 = torch.from_numpy(mel.astype(np.float16)).cuda()
    prompt = np.array(cfg.prompt, np.int32)
    np_ = len(prompt)
    steps_dec = np_ - 1 + NEW_TOKENS
    st = torch.cuda.ExternalStream(e.stream)

    if args.impl == "native":  # the timestamp cost and DTW run on the GPU (the reference does them on the host)
        rc_dev = torch.tensor([NEW_TOKENS - 1] * nb + [int(f) // 2 for f in frames], dtype=torch.int32,
                              device="cuda")
        cost_dev = torch.empty((nb, cfg.max_t, 1500), dtype=torch.float32, device="cuda")
        times_dev = torch.empty((nb, cfg.max_t), dtype=torch.float32, device="cuda")

    def gpu_pipeline():
        for g0 in range(0, nb, 8):
            e.encode(mel16[g0].data_ptr(), 8, g0)
        e.reset(np.tile(prompt, (nb, 1)))
        for _ in range(steps_dec):
            e.replay()
        if args.impl == "native":
            m.align_cost(e.buffer("align"), rc_dev[:nb], rc_dev[nb:], np_, cfg.max_t, e.na,
                         cost_dev, n=nb, stream=e.stream)
            m.dtw_times(cost_dev, rc_dev[:nb], rc_dev[nb:], cfg.max_t, times_dev,
                        n=nb, stream=e.stream)

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    # capture the decoding step once (outside every timed region), as transcribe.rs:122-131 does
    e.reset(np.tile(prompt, (nb, 1)))
    e.capture(nb, np_)
    for _ in range(args.warmup):
        gpu_pipeline()
    e.sync()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    launches0 = e.launches
    with Clocks(local) as clk:
        a.record(st)
        for _ in range(args.steps):
            gpu_pipeline()
        b.record(st)
        b.synchronize()
    launches = e.launches - launches0 + (2 * args.steps if args.impl == "native" else 0)  # + cost and DTW kernels
    t_dev = max_over_ranks(a.elapsed_time(b) * 1e-3)
    torch.cuda.synchronize()
    barrier()

    # end to end through the C-ABI: host log-mel in, host tokens and timestamps out
    for _ in range(max(1, args.warmup - 2)):
        r = e.transcribe(mel, frames, max_new=NEW_TOKENS, threads=n_threads)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    stages = np.zeros(3)
    for _ in range(args.steps):
        r = e.transcribe(mel, frames, max_new=NEW_TOKENS, threads=n_threads)
        stages += r["stage_s"]
    torch.cuda.synchronize()
    t_e2e = max_over_ranks(time.perf_counter() - t0)
    assert (r["lens"] == np_ + NEW_TOKENS).all()

    # the same from host audio, log-mel on the GPU (outside the metric's definition, which starts from the features)
    t_audio = None
    if args.impl == "native":
        ra = e.transcribe_audio(clips, max_new=NEW_TOKENS, threads=n_threads)  # warm: allocates the staging buffers
        assert np.array_equal(ra["frames"], frames)
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ra = e.transcribe_audio(clips, max_new=NEW_TOKENS, threads=n_threads)
        torch.cuda.synchronize()
        t_audio = max_over_ranks(time.perf_counter() - t0)

    kr = kernel_rooflines(e, cfg, torch, args.impl, nb)
    bx, tx = kr["cross"]
    bs_, ts_ = kr["self"]
    fe, te = kr["enc"]
    n_total = nb * world
    value = n_total * args.steps / t_dev
    e2e = n_total * args.steps / t_e2e
    # the log-mel crosses as fp32 for the native image (rounded on the device) and as fp16 for the reference's (rounded
    # on the host, src/model.rs:549); plus the prompt tokens
    h2d = (mel.nbytes if args.impl == "native" else mel.nbytes // 2) + 4 * nb * np_
    d2h = e.d2h_bytes  # tokens, and the recorded probabilities (reference) or the DTW cost rows (native)
    # DRAM bytes per launch of the native cross-attention kernels from an ncu capture of the large-v3 batch-32 layer
    # (profiles/cross_attn_traffic.txt); the reference's kernels and other shapes were not captured: null
    traffic = None
    if args.impl == "native" and cfg.d == 1280 and nb == 32:
        try:
            with open(os.path.join(ROOT, "profiles", "cross_attn_traffic.txt")) as f:
                for ln in f:
                    if ln.startswith("cross_attn_bytes_per_launch"):
                        traffic = int(ln.split()[1])
        except OSError:
            pass
    line = {
        "metric": metric,
        "value": round(value, 3),
        "unit": "clips/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_dev / args.steps * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded 30 s clips: 1-8 sinusoids 80-4000 Hz + noise at 10 dB SNR; random-init weights)",
        "config": {"workload": (f"e2e whisper {cfg.name} (random init, {cfg.enc_layers} encoder + {cfg.dec_layers} "
                                f"decoder layers), {nb} clips of 30 s per GPU, encoder groups of 8, {NEW_TOKENS} fixed "
                                f"greedy tokens (eos suppressed), {e.na} alignment heads, DTW timestamps"),
                   "model": cfg.name,
                   "clips_per_gpu": nb, "new_tokens": NEW_TOKENS, "decoder_lanes": e.lanes,
                   "l2": (f"inputs larger than L2: cross k/v {nb * cfg.dec_layers * 2 * cfg.d * 1500 * 2 / 1e9:.2f} GB "
                          "and the decoder weights per GPU are streamed each step")},
        "e2e": {"value": round(e2e, 3), "unit": "clips/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "stage_s_per_step": [round(x / args.steps, 4) for x in stages]},
        "roofline": {"kernel": ("cross_scores_kernel+cross_pv_kernel+cross_combine_kernel" if args.impl == "native"
                                else "cross_scores+cross_pv+cross_combine"),
                     "bound": "hbm", "achieved": round(bx / tx / 1e9, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(bx / tx / 1e9 / hbm_peak, 3), "traffic": traffic,
                     "peak_source": peak_src + " (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
                     "algorithmic_bytes_per_launch": int(bx), "avg_launch_us": round(tx * 1e6, 2)},
        "enc_attn": {"tflops": round(fe / te / 1e12, 1), "frac_of_bf16_peak": round(fe / te / 1e12 / tc_peak, 3),
                     "us_per_layer": round(te * 1e6, 1), "shape": "8 clips x 20 heads x 1500 x 64"},
        "dec_attn": {"cross_gbs": round(bx / tx / 1e9, 1), "self_gbs_at_L116": round(bs_ / ts_ / 1e9, 1),
                     "cross_us_per_layer": round(tx * 1e6, 2), "self_us_per_layer": round(ts_ * 1e6, 2),
                     "frac_of_hbm": round((bx + bs_) / (tx + ts_) / 1e9 / hbm_peak, 3)},
        "clocks": clk.summary(),
        "gpu_launches": int(launches),
    }
    if t_audio is not None:
        line["e2e_from_audio"] = {"value": round(n_total * args.steps / t_audio, 3), "unit": "clips/s",
                                  "h2d_bytes_per_step": int(sum(4 * min(len(y), 480000) for y in clips)),
                                  "what": "the C-ABI transcribe from host audio: log-mel on the GPU, then as e2e"}
    if args.impl == "native":  # log-mel is outside the clips/s metric (features are reported separately)
        t_feat_gpu, feat_h2d = features_gpu(clips, cfg.n_mels, torch)
        line["features"] = {"clips": nb, "host_s": round(t_feat_host, 4), "host_threads": n_threads,
                            "gpu_s": round(t_feat_gpu, 5), "gpu_h2d_bytes": int(feat_h2d),
                            "what": "log-mel of 30 s clips (src/audio.rs): host restatement vs the GPU kernels "
                                    "(host-to-device copy of the samples included)"}
    if args.impl == "reference":
        line["impl"] = "reference"
        line["reference_kind"] = ("the reference's own kernels (kernels/whisper.cu, compute_80 PTX JIT-compiled on "
                                  "the B200) driven by this repository's C++ restatement of its host")
    if rank == 0 and world == 1 and args.impl == "native":
        line["cpu_baseline"] = cpu_baseline(cfg, min(32, os.cpu_count() or 1))
    if rank == 0:
        print(json.dumps(line), flush=True)
    e.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
