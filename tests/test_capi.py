"""The C-ABI library loads, exports every symbol include/mimizuku_b200.h declares, and reports errors through its
return codes and mmz_last_error (no GPU compute here)."""
import ctypes
import os
import re

import numpy as np

import mimizuku_b200 as m

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mimizuku_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mmz_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported_and_bound():
    names = declared()
    assert len(names) >= 25
    for n in names:
        assert hasattr(m.lib, n), n           # exported by the .so
        assert n in m.SIGNATURES, n           # bound with argument types by the Python layer
    assert set(m.SIGNATURES) == set(names)


def test_library_is_the_in_tree_build():
    assert os.path.dirname(m.LIB_PATH) == os.path.dirname(os.path.abspath(m.__file__))
    with open("/proc/self/maps") as f:
        assert m.LIB_PATH in f.read()


def test_errors_are_reported_not_raised_in_c():
    w = np.zeros((2, 1, 10), np.float32)
    out = np.zeros(2, np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    rc = m.lib.mmz_jump_times(w.ctypes.data_as(fp), 2, 1, 10, 11, 7, out.ctypes.data_as(fp))
    assert rc != 0 and b"cols" in m.lib.mmz_last_error()
    rc = m.lib.mmz_jump_times(w.ctypes.data_as(fp), 2, 1, 10, 5, 6, out.ctypes.data_as(fp))
    assert rc != 0
    assert not m.lib.mmz_engine_create(None, None, 1, 1, 0, None, 0)
    assert b"null" in m.lib.mmz_last_error()


def test_kernel_entry_points_validate_shapes_before_touching_a_device():
    # bad shapes are rejected on the host, before any launch
    assert m.lib.mmz_enc_flash(None, None, 0, 384, None) != 0
    assert b"enc_flash" in m.lib.mmz_last_error()
    assert m.lib.mmz_cross_attn(None, None, None, None, None, None, None, 1, 3, 2, 384, 1, 448, None, 0, None) != 0
    assert b"cross_attn" in m.lib.mmz_last_error()
    assert m.lib.mmz_cross_attn_scratch_bytes(32, 1280) == 32 * 20 * (1500 * 4 + 24 * 8 + 24 * 64 * 4)
    assert m.lib.mmz_self_attn(None, None, None, None, None, None, 1, 600, 384, None) != 0
    assert m.lib.mmz_layernorm(None, None, None, None, 1, 4097, 1e-5, None) != 0
    # the tensor-core GEMM: n a multiple of 128, k of 64, mode 0-2, 16-byte aligned operands and pitches
    g = m.lib.mmz_gemm_bias
    assert g(None, 64, None, None, None, 256, 16, 100, 64, 0, 0, None) != 0  # n
    assert b"gemm_bias" in m.lib.mmz_last_error()
    assert g(None, 64, None, None, None, 256, 16, 256, 70, 0, 0, None) != 0  # k
    assert g(None, 64, None, None, None, 256, 16, 256, 64, 3, 0, None) != 0  # mode
    assert g(8, 64, 16, None, 16, 256, 16, 256, 64, 0, 0, None) != 0  # a not 16-byte aligned
    assert g(16, 36, 16, None, 16, 256, 16, 256, 64, 0, 0, None) != 0  # lda below k
    assert g(16, 64, 16, None, 16, 256, 16, 256, 64, 2, 100, None) != 0  # head blocks smaller than m x 64
    # the gemv: 1 <= m <= 8, k a multiple of 8, ldx >= k, ldy >= n
    v = m.lib.mmz_gemv
    assert v(None, 16, None, None, 16, 9, 16, 16, None, None) != 0 and b"gemv" in m.lib.mmz_last_error()
    assert v(None, 16, None, None, 16, 0, 16, 16, None, None) != 0
    assert v(None, 16, None, None, 16, 1, 16, 12, None, None) != 0
    assert v(None, 8, None, None, 16, 1, 16, 16, None, None) != 0
    assert v(8, 16, 16, None, 16, 1, 16, 16, None, None) != 0  # x not 16-byte aligned
    assert m.lib.mmz_gemv_gelu(None, 16, None, None, 16, 9, 16, 16, None, None) != 0
    assert m.lib.mmz_im2col1(None, None, 10, 0, None) != 0
    assert m.lib.mmz_add_pos(None, None, 4, 8, 0, None) != 0


def test_missing_device_is_an_error_not_a_crash():
    import torch
    if torch.cuda.is_available():
        return
    assert m.lib.mmz_init(0) != 0
    assert m.lib.mmz_last_error()
