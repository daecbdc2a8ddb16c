"""Python face of the C++ engine (src/model.rs Engine + src/transcribe.rs transcribe of the reference)."""
import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence, Tuple

import numpy as np

from . import _DP, _FP, _IP, _check, lib, mmz_dims, mmz_gencfg, MmzError


@dataclass(frozen=True)
class ModelConfig:
    """Whisper shape (config.json) plus the decoding settings the engine needs (generation_config.json)."""
    name: str
    d: int
    ff: int
    heads: int
    enc_layers: int
    dec_layers: int
    n_mels: int
    vocab: int
    max_t: int = 448
    eos: int = 50257
    prompt: Tuple[int, ...] = (50258, 50259, 50360, 50364)  # start, language, task, no timestamps
    begin_suppress: Tuple[int, int] = (220, 50257)
    n_align: Optional[int] = None  # None: every head of the second half of the decoder layers (model.rs:101)


TINY = ModelConfig("tiny", 384, 1536, 6, 4, 4, 80, 51865, prompt=(50258, 50259, 50359, 50363), n_align=2)
LARGE_V3 = ModelConfig("large-v3", 1280, 5120, 20, 32, 32, 128, 51866, n_align=10)
LARGE_V3_TURBO = ModelConfig("large-v3-turbo", 1280, 5120, 20, 32, 4, 128, 51866, n_align=6)


def align_heads(cfg: ModelConfig, n: Optional[int] = None, seed: int = 0):
    """(layer, head) pairs: every head of the second half of the decoder layers (the reference's default,
    src/model.rs:99-101), or n of them drawn with a seed."""
    pairs = [(l, h) for l in range(cfg.dec_layers // 2, cfg.dec_layers) for h in range(cfg.heads)]
    n = cfg.n_align if n is None else n
    if n is None or n >= len(pairs):
        return pairs
    rng = np.random.default_rng(seed)
    idx = sorted(rng.choice(len(pairs), size=n, replace=False).tolist())
    return [pairs[i] for i in idx]


class Engine:
    """Engine::new (src/model.rs:333-514) with seeded random-init weights. kernel_image=None runs the sm_100a kernels
    of this library; a path runs a fatbin exporting the reference's kernel names (e.g. the reference's own
    kernels/whisper.cu build) through the same host code. lanes: decoder-step lanes (None: the image's default, 2 for
    the native kernels, 1 for a fatbin)."""

    def __init__(self, cfg: ModelConfig, bmax: int, eg: int = 8, device: int = 0, kernel_image: Optional[str] = None,
                 seed: int = 0, heads: Optional[Sequence[Tuple[int, int]]] = None,
                 suppress: Optional[Sequence[int]] = None, begin_suppress: Optional[Tuple[int, int]] = None,
                 lanes: Optional[int] = None):
        self.cfg = cfg
        self.bmax, self.eg, self.device = bmax, min(eg, bmax), device
        self.heads = list(heads) if heads is not None else align_heads(cfg)
        self.suppress = list(suppress) if suppress is not None else []
        bs = begin_suppress if begin_suppress is not None else cfg.begin_suppress
        dims = mmz_dims(cfg.d, cfg.ff, cfg.heads, cfg.enc_layers, cfg.dec_layers, cfg.n_mels, cfg.vocab, cfg.max_t)
        self._sup = (ctypes.c_int * max(1, len(self.suppress)))(*self.suppress)
        flat = [v for p in self.heads for v in p]
        self._ah = (ctypes.c_int * max(1, len(flat)))(*flat)
        gc = mmz_gencfg(cfg.eos, ctypes.cast(self._sup, _IP), len(self.suppress), (ctypes.c_int * 2)(*bs),
                        ctypes.cast(self._ah, _IP), len(self.heads))
        img = kernel_image.encode() if kernel_image else None
        self._h = lib.mmz_engine_create(ctypes.byref(dims), ctypes.byref(gc), bmax, self.eg, device, img, seed)
        if not self._h:
            raise MmzError(lib.mmz_last_error().decode())
        if lanes is not None:
            self.lanes = lanes

    @property
    def na(self):
        return len(self.heads)

    def close(self):
        if self._h:
            lib.mmz_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def transcribe(self, mel, frames, prompt=None, max_new=None, graph=True, threads=0):
        """src/transcribe.rs:104-167 for n <= bmax clips of host log-mel [n][n_mels][3000] float32. max_new caps the
        generated tokens (None: up to max_t). Returns dict(tokens [n][max_t], lens [n], times [n][max_t],
        stage_s (encode, decode, timestamps))."""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        n = mel.shape[0]
        frames = np.ascontiguousarray(frames, dtype=np.int32)
        prompt = np.asarray(prompt if prompt is not None else self.cfg.prompt, dtype=np.int32)
        np_ = len(prompt)
        mt = self.cfg.max_t
        max_steps = 0 if max_new is None else min(mt - 1, np_ - 1 + max_new)
        tokens = np.zeros((n, mt), np.int32)
        lens = np.zeros(n, np.int32)
        times = np.zeros((n, mt), np.float32)
        stage = np.zeros(3, np.float64)
        _check(lib.mmz_engine_transcribe(self._h, mel.ctypes.data_as(_FP), frames.ctypes.data_as(_IP), n,
                                         prompt.ctypes.data_as(_IP), np_, max_steps, int(graph), threads,
                                         tokens.ctypes.data_as(_IP), lens.ctypes.data_as(_IP),
                                         times.ctypes.data_as(_FP), stage.ctypes.data_as(_DP)), "transcribe")
        return {"tokens": tokens, "lens": lens, "times": times, "stage_s": stage}

    def transcribe_audio(self, clips, prompt=None, max_new=None, graph=True, threads=0):
        """src/transcribe.rs:25-167 from host audio: clips is a list of float32 sample arrays at 16 kHz (n <= bmax);
        the log-mel features are computed on the GPU. Returns transcribe's dict plus frames [n]."""
        clips = [np.ascontiguousarray(c, dtype=np.float32) for c in clips]
        n = len(clips)
        prompt = np.asarray(prompt if prompt is not None else self.cfg.prompt, dtype=np.int32)
        np_ = len(prompt)
        mt = self.cfg.max_t
        max_steps = 0 if max_new is None else min(mt - 1, np_ - 1 + max_new)
        ptrs = (_FP * n)(*[c.ctypes.data_as(_FP) for c in clips])
        lens_in = (ctypes.c_long * n)(*[len(c) for c in clips])
        tokens = np.zeros((n, mt), np.int32)
        lens = np.zeros(n, np.int32)
        times = np.zeros((n, mt), np.float32)
        frames = np.zeros(n, np.int32)
        stage = np.zeros(3, np.float64)
        _check(lib.mmz_engine_transcribe_audio(self._h, ptrs, lens_in, n, prompt.ctypes.data_as(_IP), np_, max_steps,
                                               int(graph), threads, tokens.ctypes.data_as(_IP),
                                               lens.ctypes.data_as(_IP), times.ctypes.data_as(_FP),
                                               frames.ctypes.data_as(_IP), stage.ctypes.data_as(_DP)),
               "transcribe_audio")
        return {"tokens": tokens, "lens": lens, "times": times, "frames": frames, "stage_s": stage}

    def encode(self, mel16, gn, slot0=0):
        """Engine::encode (src/model.rs:545-625) of gn clips of fp16 log-mel at device address mel16."""
        _check(lib.mmz_engine_encode(self._h, mel16 if isinstance(mel16, int) else mel16.data_ptr(), gn, slot0),
               "encode")

    def reset(self, prompts):
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        _check(lib.mmz_engine_reset(self._h, p.ctypes.data_as(_IP), p.shape[0], p.shape[1]), "reset")

    def step(self, b, prompt_len):
        _check(lib.mmz_engine_step(self._h, b, prompt_len), "step")

    def capture(self, b, prompt_len):
        _check(lib.mmz_engine_capture(self._h, b, prompt_len), "capture")

    def replay(self):
        _check(lib.mmz_engine_replay(self._h), "replay")

    @property
    def lanes(self):
        """Decoder-step lanes: 1 decodes the whole batch on one stream (the reference's way), 2 (the native image's
        default) the two halves of a 32-sequence batch on two concurrent streams (other batch sizes use one lane);
        results are the same."""
        return lib.mmz_engine_lanes(self._h)

    @lanes.setter
    def lanes(self, n):
        _check(lib.mmz_engine_set_lanes(self._h, int(n)), "set_lanes")

    @property
    def enc_attn(self):
        """Encoder attention: "flash" (the default: the kernel image's fused attention) or "cublas" (the unfused
        comparison path of src/model.rs:567-604: cuBLAS scores, row softmax, cuBLAS P.V)."""
        return "cublas" if lib.mmz_engine_enc_attn(self._h) == 1 else "flash"

    @enc_attn.setter
    def enc_attn(self, mode):
        if mode not in ("flash", "cublas"):
            raise MmzError("enc_attn: 'flash' or 'cublas'")
        _check(lib.mmz_engine_set_enc_attn(self._h, 1 if mode == "cublas" else 0), "set_enc_attn")

    @property
    def enc_gemm(self):
        """Encoder GEMMs: "native" (the default: this library's tensor-core GEMM for qkv, fc1 + GELU and the cross
        k/v projection into the head blocks) or "cublaslt" (every linear layer on cuBLASLt, GELU and the cross k/v
        layout separate)."""
        return "native" if lib.mmz_engine_enc_gemm(self._h) == 1 else "cublaslt"

    @enc_gemm.setter
    def enc_gemm(self, mode):
        if mode not in ("cublaslt", "native"):
            raise MmzError("enc_gemm: 'cublaslt' or 'native'")
        _check(lib.mmz_engine_set_enc_gemm(self._h, 1 if mode == "native" else 0), "set_enc_gemm")

    def buffer(self, name):
        p = lib.mmz_engine_buffer(self._h, name.encode())
        if not p:
            raise MmzError(f"no engine buffer {name}")
        return p

    @property
    def stream(self):
        return lib.mmz_engine_stream(self._h)

    def sync(self):
        _check(lib.mmz_engine_sync(self._h), "sync")

    @property
    def allocated(self):
        return lib.mmz_engine_allocated(self._h)

    @property
    def launches(self):
        """Kernels of the engine's kernel image launched so far (graph replays included, cuBLAS not)."""
        return lib.mmz_engine_launches(self._h)

    @property
    def d2h_bytes(self):
        """Bytes the last transcribe copied device -> host."""
        return lib.mmz_engine_d2h_bytes(self._h)
