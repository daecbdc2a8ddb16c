"""mimizuku_b200: the B200-native attention hot path of the mimizuku Whisper engine.

The product is the C-ABI library ``libmimizuku_b200.so`` (declared in ``include/mimizuku_b200.h``): sm_100a kernels
for encoder flash attention (tcgen05/TMEM/TMA), decoder self-attention (TMA-streamed) and cross-attention (split-KV
streaming kernels), fused
residual-add + LayerNorm, the engine that drives them (a C++ restatement of the reference's model.rs and
transcribe.rs) and the CPU timestamp stage (align.rs). This module binds it with ctypes under the reference's names
(``enc_flash``, ``self_attn``, ``cross_attn``, ``layernorm``, ``add_layernorm``, ``jump_times``, ``dtw``, ``Engine``).

Importing fails loudly when the library has not been built (``python mimizuku_b200/build.py``): there is no CPU or
Python fallback for any of these functions.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmimizuku_b200.so")
# layernorm, add_layernorm and kv_write under the reference's names and argument lists, for a host that launches
# kernels by name (built by build.py next to the library)
DROPIN_FATBIN = os.path.join(_HERE, "dropin_sm100a.fatbin")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing; build it with `python mimizuku_b200/build.py`")

lib = ctypes.CDLL(LIB_PATH)

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_long
_LL = ctypes.c_longlong
_F = ctypes.c_float
_ULL = ctypes.c_ulonglong
_IP = ctypes.POINTER(ctypes.c_int)
_FP = ctypes.POINTER(ctypes.c_float)
_DP = ctypes.POINTER(ctypes.c_double)


class mmz_dims(ctypes.Structure):
    _fields_ = [(n, _I) for n in ("d", "ff", "heads", "enc_layers", "dec_layers", "n_mels", "vocab", "max_t")]


class mmz_gencfg(ctypes.Structure):
    _fields_ = [("eos", _I), ("suppress", _IP), ("n_suppress", _I), ("begin_suppress", _I * 2),
                ("align_heads", _IP), ("n_align", _I)]


# name -> (restype, argtypes); every symbol include/mimizuku_b200.h declares
SIGNATURES = {
    "mmz_init": (_I, [_I]),
    "mmz_last_error": (ctypes.c_char_p, []),
    "mmz_status": (_I, [_IP]),
    "mmz_set_wait_limit_ms": (_I, [_I, _I]),
    "mmz_selftest_wait": (_I, [_I, _P]),
    "mmz_h2f": (_F, [ctypes.c_uint16]),
    "mmz_f2h": (ctypes.c_uint16, [_F]),
    "mmz_rh": (_F, [_F]),
    "mmz_enc_flash": (_I, [_P, _P, _I, _I, _P]),
    "mmz_self_attn": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "mmz_kv_write": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "mmz_cross_attn": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _ULL, _P]),
    "mmz_cross_attn_scratch_bytes": (_ULL, [_I, _I]),
    "mmz_cross_attn_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "mmz_layernorm": (_I, [_P, _P, _P, _P, _I, _I, _F, _P]),
    "mmz_add_layernorm": (_I, [_P, _P, _P, _P, _P, _I, _I, _F, _P]),
    "mmz_jump_times": (_I, [_FP, _I, _I, _I, _I, _I, _FP]),
    "mmz_dtw": (_I, [_DP, _I, _I, _IP, _IP, _IP]),
    "mmz_align_cost": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "mmz_dtw_times": (_I, [_P, _P, _P, _I, _I, _P, _P]),
    "mmz_dec_linear": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "mmz_softmax_rows": (_I, [_P, _L, _I, _P]),
    "mmz_gemv": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _P]),
    "mmz_gemv_gelu": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _P]),
    "mmz_im2col1": (_I, [_P, _P, _LL, _I, _P]),
    "mmz_im2col2": (_I, [_P, _P, _LL, _I, _P]),
    "mmz_add_pos": (_I, [_P, _P, _LL, _I, _I, _P]),
    "mmz_gemm_bias": (_I, [_P, _I, _P, _P, _P, _LL, _I, _I, _I, _I, _LL, _P]),
    "mmz_logits_argmax_scratch_bytes": (_ULL, []),
    "mmz_logits_argmax": (_I, [_P, _I, _P, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _P, _ULL, _P]),
    "mmz_times_from_cost": (_I, [_FP, _I, _I, _I, _FP]),
    "mmz_log_mel": (_I, [_FP, _L, _I, _FP, _IP]),
    "mmz_log_mel_gpu_work_bytes": (_ULL, [_I]),
    "mmz_log_mel_gpu": (_I, [_P, _P, _I, _I, _P, _P, _ULL, _P]),
    "mmz_log_mel_batch": (_I, [ctypes.POINTER(_FP), ctypes.POINTER(_L), _I, _I, _I, _FP, _IP]),
    "mmz_synth_clip": (_I, [_ULL, _FP, _L]),
    "mmz_engine_create": (_P, [ctypes.POINTER(mmz_dims), ctypes.POINTER(mmz_gencfg), _I, _I, _I, ctypes.c_char_p,
                               _ULL]),
    "mmz_engine_destroy": (None, [_P]),
    "mmz_engine_transcribe": (_I, [_P, _FP, _IP, _I, _IP, _I, _I, _I, _I, _IP, _IP, _FP, _DP]),
    "mmz_engine_transcribe_audio": (_I, [_P, ctypes.POINTER(_FP), ctypes.POINTER(_L), _I, _IP, _I, _I, _I, _I, _IP,
                                         _IP, _FP, _IP, _DP]),
    "mmz_engine_encode": (_I, [_P, _P, _I, _I]),
    "mmz_engine_reset": (_I, [_P, _IP, _I, _I]),
    "mmz_engine_step": (_I, [_P, _I, _I]),
    "mmz_engine_capture": (_I, [_P, _I, _I]),
    "mmz_engine_replay": (_I, [_P]),
    "mmz_engine_set_lanes": (_I, [_P, _I]),
    "mmz_engine_lanes": (_I, [_P]),
    "mmz_engine_set_enc_attn": (_I, [_P, _I]),
    "mmz_engine_enc_attn": (_I, [_P]),
    "mmz_engine_set_enc_gemm": (_I, [_P, _I]),
    "mmz_engine_enc_gemm": (_I, [_P]),
    "mmz_engine_buffer": (_P, [_P, ctypes.c_char_p]),
    "mmz_engine_stream": (_P, [_P]),
    "mmz_engine_sync": (_I, [_P]),
    "mmz_engine_allocated": (_LL, [_P]),
    "mmz_engine_launches": (_LL, [_P]),
    "mmz_engine_d2h_bytes": (_ULL, [_P]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class MmzError(RuntimeError):
    pass


def _check(rc, what):
    if rc != 0:
        raise MmzError(f"{what}: {lib.mmz_last_error().decode()}")


def _ptr(x):
    """Device address of a torch tensor, an int address, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def init(device=0):
    _check(lib.mmz_init(device), "mmz_init")


def status():
    """Reads and clears the device status word: (code, kernel, site); code 0 = no error."""
    out = (ctypes.c_int * 3)()
    _check(lib.mmz_status(out), "mmz_status")
    return tuple(out)


def selftest_wait(limit_ms, stream=None):
    """Runs a kernel whose bounded waits run out on purpose (nothing arrives on its barrier); returns status()."""
    _check(lib.mmz_selftest_wait(limit_ms, _stream(stream)), "mmz_selftest_wait")
    return status()


def set_wait_limit_ms(device, ms):
    _check(lib.mmz_set_wait_limit_ms(device, ms), "mmz_set_wait_limit_ms")


# ------------------------------------------------------------------ fp16 helpers (src/gpu.rs:79-119)

def h2f(h):
    return lib.mmz_h2f(h)


def f2h(x):
    return lib.mmz_f2h(x)


def rh(x):
    return lib.mmz_rh(x)


# ------------------------------------------------------------------ kernels (torch CUDA tensors or raw addresses)

def enc_flash(qkv, out, d, groups=None, stream=None):
    """kernels/whisper.cu:209 enc_flash: qkv [g][1500][3d] fp16 -> out [g][1500][d] fp16."""
    g = groups if groups is not None else qkv.shape[0]
    _check(lib.mmz_enc_flash(_ptr(qkv), _ptr(out), g, d, _stream(stream)), "enc_flash")


def self_attn(qkv, kc, vc, out, ctr, done, max_t, d, batch=None, stream=None):
    """kernels/whisper.cu:310-353 kv_write + self_attn (fused): position ctr[0]."""
    b = batch if batch is not None else done.shape[0]
    _check(lib.mmz_self_attn(_ptr(qkv), _ptr(kc), _ptr(vc), _ptr(out), _ptr(ctr), _ptr(done), b, max_t, d,
                             _stream(stream)), "self_attn")


def kv_write(qkv, kc, vc, ctr, max_t, d, batch, stream=None):
    _check(lib.mmz_kv_write(_ptr(qkv), _ptr(kc), _ptr(vc), _ptr(ctr), batch, max_t, d, _stream(stream)), "kv_write")


def cross_attn_scratch_bytes(batch, d):
    """Bytes of device scratch mmz_cross_attn needs for `batch` sequences of width d."""
    return lib.mmz_cross_attn_scratch_bytes(batch, d)


def cross_attn(q, kv, out, align, aslot, ctr, done, layer, nl, d, na, max_t, scratch, batch=None, stream=None,
               scratch_bytes=None):
    """kernels/whisper.cu:368-449 cross_scores + cross_pv + cross_combine as three chained kernels. scratch: a device
    buffer (torch tensor or address) of at least cross_attn_scratch_bytes(batch, d) bytes."""
    b = batch if batch is not None else done.shape[0]
    if scratch_bytes is None:
        scratch_bytes = (scratch.numel() * scratch.element_size() if hasattr(scratch, "numel")
                         else cross_attn_scratch_bytes(b, d))
    _check(lib.mmz_cross_attn(_ptr(q), _ptr(kv), _ptr(out), _ptr(align), _ptr(aslot), _ptr(ctr), _ptr(done), b,
                              layer, nl, d, na, max_t, _ptr(scratch), scratch_bytes, _stream(stream)), "cross_attn")


def cross_attn_noalloc(q, kv, out, align, aslot, ctr, done, layer, nl, d, na, max_t, batch=None, stream=None):
    """cross_attn for callers that cannot allocate: the scratch is a static device array of the library (batch x
    heads <= 640); calls that overlap on the GPU race on it."""
    b = batch if batch is not None else done.shape[0]
    _check(lib.mmz_cross_attn_noalloc(_ptr(q), _ptr(kv), _ptr(out), _ptr(align), _ptr(aslot), _ptr(ctr), _ptr(done),
                                      b, layer, nl, d, na, max_t, _stream(stream)), "cross_attn_noalloc")


def layernorm(x, w, b, out, eps=1e-5, rows=None, stream=None):
    """kernels/whisper.cu:66 layernorm over the last dimension."""
    dim = w.shape[-1]
    r = rows if rows is not None else x.numel() // dim
    _check(lib.mmz_layernorm(_ptr(x), _ptr(w), _ptr(b), _ptr(out), r, dim, eps, _stream(stream)), "layernorm")


def add_layernorm(x, dx, w, b, out, eps=1e-5, rows=None, stream=None):
    """kernels/whisper.cu:72 add_layernorm: x = h(x + dx), out = layernorm(x)."""
    dim = w.shape[-1]
    r = rows if rows is not None else x.numel() // dim
    _check(lib.mmz_add_layernorm(_ptr(x), _ptr(dx), _ptr(w), _ptr(b), _ptr(out), r, dim, eps, _stream(stream)),
           "add_layernorm")


# ------------------------------------------------------------------ CPU stages

def _fp(a):
    return a.ctypes.data_as(_FP)


def jump_times(w, cols, width=7):
    """src/align.rs:8-63. w: float32 [rows][heads][cols_full] -> float32 [rows] start times (s)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, heads, cols_full = w.shape
    out = np.zeros(rows, np.float32)
    _check(lib.mmz_jump_times(_fp(w), rows, heads, cols_full, cols, width, _fp(out)), "jump_times")
    return out


def dec_linear(x, w, bias, y, gelu=False, m=None, stream=None):
    """y[m][n] = rh(x[m] . w[n] + bias[n]) (GELU after when gelu) on the tensor cores; x [m][k], w [n][k], y [m][n]
    fp16 device tensors, m <= 32."""
    mm = m if m is not None else x.shape[0]
    n, k = w.shape
    _check(lib.mmz_dec_linear(_ptr(x), x.stride(0), _ptr(w), _ptr(bias), _ptr(y), y.stride(0), mm, n, k,
                              1 if gelu else 0, _stream(stream)), "dec_linear")


def gemm_bias(a, w, bias, c, mode=0, blk=0, m=None, ldc=None, stream=None):
    """c = rh(a w^T + bias) on the tensor cores (mode 1: then GELU; mode 2: head-blocked store, blk elements per
    64-column block): a [m][k], w [n][k], bias [n] fp16 device tensors."""
    mm = m if m is not None else a.shape[0]
    n, k = w.shape
    ld = ldc if ldc is not None else (c.stride(0) if mode != 2 else 0)
    _check(lib.mmz_gemm_bias(_ptr(a), a.stride(0), _ptr(w), _ptr(bias), _ptr(c), ld, mm, n, k, mode, blk,
                             _stream(stream)), "gemm_bias")


def softmax_rows(s, n=None, rows=None, stream=None):
    """Row softmax in place of an fp16 device tensor [rows][n] (kernels/whisper.cu:141-166)."""
    n = n if n is not None else s.shape[-1]
    rows = rows if rows is not None else s.numel() // n
    _check(lib.mmz_softmax_rows(_ptr(s), rows, n, _stream(stream)), "softmax_rows")


def gemv(x, w, bias, y, m=None, gelu=False, stream=None):
    """y[m][n] = rh(x[m] . w[n] + bias[n]) for m <= 8 rows, bit-identical to the reference's gemv kernels; x [m][k],
    w [n][k], y [m][n] fp16 device tensors, bias [n] or None; gelu: then rh(GELU(y)), as gelu_inplace after it."""
    mm = m if m is not None else x.shape[0]
    n, k = w.shape
    fn = lib.mmz_gemv_gelu if gelu else lib.mmz_gemv
    _check(fn(_ptr(x), x.stride(0), _ptr(w), _ptr(y), y.stride(0), mm, n, k, _ptr(bias), _stream(stream)), "gemv")


def im2col1(mel, X, nm, n=None, stream=None):
    """conv1's operand from the log-mel: X [groups][3000][3 nm] from mel [groups][nm][3000] (fp16 device tensors)."""
    _check(lib.mmz_im2col1(_ptr(mel), _ptr(X), n if n is not None else X.numel(), nm, _stream(stream)), "im2col1")


def im2col2(h1, X, d, n=None, stream=None):
    """conv2's operand: X [groups][1500][3d] from conv1's output h1 [groups][3000][d] (fp16 device tensors)."""
    _check(lib.mmz_im2col2(_ptr(h1), _ptr(X), n if n is not None else X.numel(), d, _stream(stream)), "im2col2")


def add_pos(x, pos, period, n=None, rows=None, stream=None):
    """x[r] += pos[r % period] in place, x [rows][n] and pos [period][n] fp16 device tensors."""
    n = n if n is not None else x.shape[-1]
    rows = rows if rows is not None else x.numel() // n
    _check(lib.mmz_add_pos(_ptr(x), _ptr(pos), rows, n, period, _stream(stream)), "add_pos")


def logits_argmax_scratch_bytes():
    return lib.mmz_logits_argmax_scratch_bytes()


def logits_argmax(x, emb, sup, tok, done, ctr, max_t, prompt_len, eos, bs=(-1, -1), scratch=None, logits=None,
                  advance=False, m=None, stream=None):
    """The decoding step's logits x . emb^T fused with argmax_tok's greedy choice of token ctr[0] + 1 (src/model.rs:
    714-735): x [m][d] fp16, emb [vocab][d] fp16, sup [vocab] uint8, tok [m][max_t] int32, done [m] int32, ctr int32
    device tensors; scratch: a zero-filled uint8 device tensor of logits_argmax_scratch_bytes() (left zero); logits
    [m][vocab] fp16 written when given."""
    mm = m if m is not None else x.shape[0]
    V, d = emb.shape
    _check(lib.mmz_logits_argmax(_ptr(x), x.stride(0), _ptr(emb), V, d, mm, _ptr(sup), _ptr(tok), _ptr(done), _ptr(ctr),
                                 max_t, prompt_len, eos, bs[0], bs[1], _ptr(logits), 1 if advance else 0, _ptr(scratch),
                                 scratch.numel() * scratch.element_size(), _stream(stream)), "logits_argmax")


def align_cost(align, rows, cols, np_, max_t, na, cost, n=None, stream=None):
    """src/align.rs:6-43 on the GPU: align fp16 [n][max_t][na][1500] -> cost f32 [n][max_t][1500] (row i of clip s
    from position np_ + i). rows, cols: int32 device arrays [n]."""
    n = n if n is not None else rows.shape[0]
    _check(lib.mmz_align_cost(_ptr(align), _ptr(rows), _ptr(cols), n, np_, max_t, na, _ptr(cost), _stream(stream)),
           "align_cost")


def dtw_times(cost, rows, cols, max_t, times, n=None, stream=None):
    """src/align.rs:44-106 on the GPU for a batch: cost f32 [n][max_t][1500] (as align_cost writes it) -> times f32
    [n][max_t] (row i < rows[s]: start time in seconds, 0 past it). rows, cols: int32 device arrays [n]."""
    n = n if n is not None else rows.shape[0]
    _check(lib.mmz_dtw_times(_ptr(cost), _ptr(rows), _ptr(cols), n, max_t, _ptr(times), _stream(stream)),
           "dtw_times")


def times_from_cost(cost, cols):
    """src/align.rs:44-63: float32 cost [rows][ld] (DTW over -cost) -> float32 [rows] start times (s)."""
    cost = np.ascontiguousarray(cost, dtype=np.float32)
    rows, ld = cost.shape
    out = np.zeros(rows, np.float32)
    _check(lib.mmz_times_from_cost(_fp(cost), rows, cols, ld, _fp(out)), "times_from_cost")
    return out


def dtw(m):
    """src/align.rs:66-106 on a float64 cost matrix [rows][cols] -> (text, time) int arrays."""
    m = np.ascontiguousarray(m, dtype=np.float64)
    rows, cols = m.shape
    text = np.zeros(rows + cols + 1, np.int32)
    time = np.zeros(rows + cols + 1, np.int32)
    n = ctypes.c_int(0)
    _check(lib.mmz_dtw(m.ctypes.data_as(_DP), rows, cols, text.ctypes.data_as(_IP), time.ctypes.data_as(_IP),
                       ctypes.byref(n)), "dtw")
    return text[:n.value].copy(), time[:n.value].copy()


def log_mel(y, n_mels):
    """src/audio.rs:192-237: float32 samples at 16 kHz -> (log-mel [n_mels][3000], frames)."""
    y = np.ascontiguousarray(y, dtype=np.float32)
    out = np.zeros((n_mels, 3000), np.float32)
    fr = ctypes.c_int(0)
    _check(lib.mmz_log_mel(_fp(y), len(y), n_mels, _fp(out), ctypes.byref(fr)), "log_mel")
    return out, fr.value


def log_mel_batch(clips, n_mels, threads=0):
    clips = [np.ascontiguousarray(c, dtype=np.float32) for c in clips]
    n = len(clips)
    out = np.zeros((n, n_mels, 3000), np.float32)
    frames = np.zeros(n, np.int32)
    ptrs = (_FP * n)(*[_fp(c) for c in clips])
    lens = (_L * n)(*[len(c) for c in clips])
    _check(lib.mmz_log_mel_batch(ptrs, lens, n, n_mels, threads, _fp(out), frames.ctypes.data_as(_IP)),
           "log_mel_batch")
    return out, frames


def log_mel_gpu_work_bytes(count):
    """Bytes of device work space log_mel_gpu needs for `count` clips."""
    return lib.mmz_log_mel_gpu_work_bytes(count)


def log_mel_gpu(audio, lens, n_mels, out, work=None, stream=None):
    """src/audio.rs:192-237 on the GPU for a batch: audio float32 device [count][480000], lens int32 device [count]
    (samples that hold audio) -> out float32 device [count][n_mels][3000]. work: a device buffer of at least
    log_mel_gpu_work_bytes(count) bytes (allocated here when None)."""
    count = lens.shape[0]
    if work is None:
        import torch
        work = torch.empty(log_mel_gpu_work_bytes(count), dtype=torch.uint8, device=out.device)
    nbytes = work.numel() * work.element_size()
    _check(lib.mmz_log_mel_gpu(_ptr(audio), _ptr(lens), count, n_mels, _ptr(out), _ptr(work), nbytes,
                               _stream(stream)), "log_mel_gpu")


def synth_clip(seed, n=480000):
    y = np.zeros(n, np.float32)
    _check(lib.mmz_synth_clip(seed, _fp(y), n), "synth_clip")
    return y


# ------------------------------------------------------------------ engine

from .engine import Engine, ModelConfig, LARGE_V3, LARGE_V3_TURBO, TINY  # noqa: E402,F401
