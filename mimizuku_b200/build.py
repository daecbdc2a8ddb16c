"""Builds libmimizuku_b200.so in-tree: the sm_100a kernels (nvcc, -gencode arch=compute_100a,code=sm_100a), the C++
engine and CPU stages, linked against cuBLAS with a static CUDA runtime.

    python mimizuku_b200/build.py [--force] [-j N]      (by path: importing the package needs the library)

Objects go to mimizuku_b200/_build/; a source is recompiled when it or a header changed.
"""
import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmimizuku_b200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills",
                     "--expt-relaxed-constexpr"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function", f"-I{CUDA}/include"]

CU = ["runtime.cu", "dec_attn.cu", "enc_attn.cu", "ln.cu", "misc.cu", "cross_noalloc.cu", "align.cu", "dec_linear.cu", "logmel.cu", "logits_argmax.cu", "gemm.cu", "gemv.cu"]
CPP = ["host_cpu.cpp", "engine.cpp", "capi.cpp"]
HEADERS = ["common.cuh", "launch.h", "engine.h", "host_cpu.h", "ln_row.cuh", "gemv_row.cuh"]
# kernels under the reference's own names, as an image its host loads by name (not linked into the library)
DROPIN_SRC = os.path.join(CSRC, "dropin.cu")
DROPIN = os.path.join(HERE, "dropin_sm100a.fatbin")


def _newest_header():
    paths = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(HERE, "..", "include", "mimizuku_b200.h")]
    return max(os.path.getmtime(p) for p in paths if os.path.exists(p))


def _compile(src, force, hdr_time):
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), hdr_time):
        return obj, None
    if src.endswith(".cu"):
        cmd = [NVCC] + NVCC_FLAGS + ["-c", path, "-o", obj]
    else:
        cxx = os.environ.get("CXX", "g++")
        extra = ["-ffp-contract=off"] if src == "host_cpu.cpp" else []
        cmd = [cxx] + CXX_FLAGS + extra + ["-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}{r.stderr}"
    return obj, None


def build(force=False, jobs=None, verbose=False):
    """Compiles every source and links the library; raises RuntimeError with the compiler output on failure."""
    if not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    os.makedirs(BUILD, exist_ok=True)
    hdr = _newest_header()
    srcs = CU + CPP
    with ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, hdr), srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("build failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if force or not os.path.exists(DROPIN) or os.path.getmtime(DROPIN) < max(os.path.getmtime(DROPIN_SRC), hdr):
        cmd = [NVCC] + ARCH + ["-O3", "-std=c++17", "-lineinfo", "-fatbin", DROPIN_SRC, "-o", DROPIN]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"build failed:\n{' '.join(cmd)}\n{r.stdout}{r.stderr}")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC] + ARCH + ["-shared", "-o", tmp] + objs + [
            f"-L{CUDA}/lib64", "-lcublas", "-lcublasLt", "-Xlinker", f"-rpath,{CUDA}/lib64", "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}{r.stderr}")
        shutil.move(tmp, LIB)
        if verbose:
            print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args()
    try:
        build(a.force, a.j, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
