"""ctypes bindings of the CPU parity oracle (oracle/, test infrastructure) and a launcher for the reference's own
kernels (oracle/_ref/whisper_ref.fatbin, compiled from the reference's kernels/whisper.cu) through the CUDA driver.
Only the tests, __graft_entry__.smoke() and bench.py's baseline legs use this module."""
import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "_build", "liboracle.so")
REF_FATBIN = os.path.join(ORACLE_DIR, "_ref", "whisper_ref.fatbin")

_U16P = ctypes.POINTER(ctypes.c_uint16)
_DP = ctypes.POINTER(ctypes.c_double)
_FP = ctypes.POINTER(ctypes.c_float)
_IP = ctypes.POINTER(ctypes.c_int)
_I = ctypes.c_int


def _load():
    if not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-C", ORACLE_DIR], check=True, capture_output=True)
    lib = ctypes.CDLL(ORACLE_SO)
    sig = {
        "orc_h2f": (ctypes.c_float, [ctypes.c_uint16]),
        "orc_f2h": (ctypes.c_uint16, [ctypes.c_float]),
        "orc_rh": (ctypes.c_float, [ctypes.c_float]),
        "orc_f2h_array": (None, [_FP, _U16P, ctypes.c_long]),
        "orc_h2f_array": (None, [_U16P, _FP, ctypes.c_long]),
        "orc_layernorm": (None, [_U16P, _U16P, _U16P, _U16P, _I, _I, ctypes.c_float]),
        "orc_add_layernorm": (None, [_U16P, _U16P, _U16P, _U16P, _U16P, _I, _I, ctypes.c_float]),
        "orc_enc_attn_f64": (None, [_U16P, _DP, _I, _I, _I, _I, _I]),
        "orc_cpu_enc_attn": (None, [_U16P, _U16P, _I, _I, _I, _I, _I]),
        "orc_cpu_cross_step": (ctypes.c_double, [_U16P, _U16P, _U16P, _I]),
        "orc_cpu_dec_attn_clips": (ctypes.c_double, [_I, _I, _I, _I, _I, _I, _DP]),
        "orc_self_attn": (None, [_U16P, _U16P, _U16P, _U16P, _I, _IP, _I, _I, _I]),
        "orc_self_attn_f64": (None, [_U16P, _U16P, _U16P, _DP, _I, _IP, _I, _I, _I]),
        "orc_cross_attn": (None, [_U16P, _U16P, _U16P, _U16P, _IP, _I, _IP, _I, _I, _I, _I, _I, _I]),
        "orc_cross_attn_f64": (None, [_U16P, _U16P, _DP, _DP, _IP, _I, _I, _I, _I]),
        "orc_dtw": (_I, [_DP, _I, _I, _IP, _IP]),
        "orc_jump_times": (None, [_FP, _I, _I, _I, _I, _I, _FP]),
        "orc_align_cost": (None, [_FP, _I, _I, _I, _I, _I, _FP]),
        "orc_times_from_cost": (None, [_FP, _I, _I, _I, _FP]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


orc = _load()


def u16(a):
    """fp16 array (numpy float16 or uint16) as a uint16 pointer."""
    a = np.ascontiguousarray(a)
    assert a.dtype in (np.float16, np.uint16)
    return a.view(np.uint16).ctypes.data_as(_U16P)


def ip(a):
    return a.ctypes.data_as(_IP)


def fp(a):
    return a.ctypes.data_as(_FP)


def dp(a):
    return a.ctypes.data_as(_DP)


# ------------------------------------------------------------------ oracle wrappers (numpy in, numpy out)

def layernorm(x, w, b, eps=1e-5):
    x = np.ascontiguousarray(x, np.float16)
    out = np.zeros_like(x)
    orc.orc_layernorm(u16(x), u16(w), u16(b), u16(out), x.shape[0], x.shape[1], eps)
    return out


def add_layernorm(x, d, w, b, eps=1e-5):
    x = np.ascontiguousarray(x, np.float16).copy()
    out = np.zeros_like(x)
    orc.orc_add_layernorm(u16(x), u16(d), u16(w), u16(b), u16(out), x.shape[0], x.shape[1], eps)
    return x, out


def enc_attn_f64(qkv, d, r0=0, nr=1500, threads=0):
    qkv = np.ascontiguousarray(qkv, np.float16)
    g = qkv.shape[0]
    out = np.zeros((g, 1500, d), np.float64)
    orc.orc_enc_attn_f64(u16(qkv), dp(out), g, d, r0, nr, threads or (os.cpu_count() or 4))
    return out


def self_attn(qkv, kc, vc, p, done, max_t, d):
    kc = np.ascontiguousarray(kc, np.float16).copy()
    vc = np.ascontiguousarray(vc, np.float16).copy()
    B = qkv.shape[0]
    out = np.zeros((B, d), np.float16)
    done = np.ascontiguousarray(done, np.int32)
    orc.orc_self_attn(u16(qkv), u16(kc), u16(vc), u16(out), p, ip(done), B, max_t, d)
    return out, kc, vc


def self_attn_f64(qkv, kc, vc, p, done, max_t, d):
    B = qkv.shape[0]
    out = np.zeros((B, d), np.float64)
    done = np.ascontiguousarray(done, np.int32)
    orc.orc_self_attn_f64(u16(qkv), u16(kc), u16(vc), dp(out), p, ip(done), B, max_t, d)
    return out


def cross_attn(q, kv, align, aslot, p, done, layer, nl, d, na, max_t):
    B = q.shape[0]
    out = np.zeros((B, d), np.float16)
    align = np.ascontiguousarray(align, np.float16).copy()
    done = np.ascontiguousarray(done, np.int32)
    aslot = np.ascontiguousarray(aslot, np.int32)
    orc.orc_cross_attn(u16(q), u16(kv), u16(out), u16(align), ip(aslot), p, ip(done), B, layer, nl, d, na, max_t)
    return out, align


def cross_attn_f64(q, kv, done, layer, nl, d):
    B = q.shape[0]
    nh = d // 64
    out = np.zeros((B, d), np.float64)
    probs = np.zeros((B, nh, 1500), np.float64)
    done = np.ascontiguousarray(done, np.int32)
    orc.orc_cross_attn_f64(u16(q), u16(kv), dp(out), dp(probs), ip(done), B, layer, nl, d)
    return out, probs


def dtw(m):
    m = np.ascontiguousarray(m, np.float64)
    rows, cols = m.shape
    text = np.zeros(rows + cols + 1, np.int32)
    time = np.zeros(rows + cols + 1, np.int32)
    n = orc.orc_dtw(dp(m), rows, cols, ip(text), ip(time))
    return text[:n].copy(), time[:n].copy()


def jump_times(w, cols, width=7):
    w = np.ascontiguousarray(w, np.float32)
    rows, heads, cols_full = w.shape
    out = np.zeros(rows, np.float32)
    orc.orc_jump_times(fp(w), rows, heads, cols_full, cols, width, fp(out))
    return out


def align_cost(w, cols, width=7):
    """w float32 [rows][heads][cols_full] -> cost float32 [rows][cols] (src/align.rs:6-43)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, heads, cols_full = w.shape
    out = np.zeros((rows, cols), np.float32)
    orc.orc_align_cost(fp(w), rows, heads, cols_full, cols, width, fp(out))
    return out


def times_from_cost(cost, cols):
    cost = np.ascontiguousarray(cost, dtype=np.float32)
    rows, ld = cost.shape
    out = np.zeros(rows, np.float32)
    orc.orc_times_from_cost(fp(cost), rows, cols, ld, fp(out))
    return out


# ------------------------------------------------------------------ raw device copies (engine buffers)

def _cudart():
    import torch  # noqa: F401  (loads the CUDA runtime)
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    return rt


def d2h(dst, src_ptr):
    """Copies dst.nbytes from device address src_ptr into the numpy array dst."""
    assert _cudart().cudaMemcpy(dst.ctypes.data, src_ptr, dst.nbytes, 2) == 0


def h2d(dst_ptr, src):
    assert _cudart().cudaMemcpy(dst_ptr, np.ascontiguousarray(src).ctypes.data, src.nbytes, 1) == 0


def d2d(dst_ptr, src_ptr, nbytes):
    """Copies nbytes between two device addresses (synchronous with respect to the host)."""
    assert _cudart().cudaMemcpy(dst_ptr, src_ptr, nbytes, 3) == 0


# ------------------------------------------------------------------ seeded inputs

def normal16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float16)


# ------------------------------------------------------------------ the reference's kernels through the driver

class RefKernels:
    """Loads oracle/_ref/whisper_ref.fatbin (the reference's kernels/whisper.cu, compute_80), or another image with
    the same names, into the current CUDA context and launches its kernels by name with explicit argument types, as the
    reference's gpu.rs does."""

    def __init__(self, path=None):
        import torch  # noqa: F401  (creates and binds the primary context)
        torch.cuda.init()
        torch.zeros(1, device="cuda")
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.cu.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
        self.cu.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
        self.cu.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 7 + [
            ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        with open(path or REF_FATBIN, "rb") as f:
            self._image = ctypes.create_string_buffer(f.read())
        self.mod = ctypes.c_void_p()
        rc = self.cu.cuModuleLoadData(ctypes.byref(self.mod), self._image)
        if rc != 0:
            raise RuntimeError(f"cuModuleLoadData failed: {rc}")
        self.fns = {}

    def fn(self, name):
        if name not in self.fns:
            f = ctypes.c_void_p()
            rc = self.cu.cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode())
            if rc != 0:
                raise RuntimeError(f"no reference kernel {name}: {rc}")
            self.fns[name] = f
        return self.fns[name]

    def launch(self, name, grid, block, args, smem=0, stream=None):
        """args: sequence of ('p', int) | ('i', int) | ('l', int) | ('f', float)."""
        import torch
        vals = []
        for kind, v in args:
            if kind == "p":
                vals.append(ctypes.c_uint64(v))
            elif kind == "i":
                vals.append(ctypes.c_int32(v))
            elif kind == "l":
                vals.append(ctypes.c_int64(v))
            elif kind == "f":
                vals.append(ctypes.c_float(v))
            else:
                raise ValueError(kind)
        arr = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in vals])
        g = tuple(grid) + (1,) * (3 - len(grid))
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        rc = self.cu.cuLaunchKernel(self.fn(name), g[0], g[1], g[2], block, 1, 1, smem, st, arr, None)
        if rc != 0:
            raise RuntimeError(f"cuLaunchKernel({name}) failed: {rc}")
