"""The oracle pinned to the reference's own kernels: tests/golden/ref_fixtures.npz holds outputs of kernels/whisper.cu
(compute_80 build, run on a B200 by tests/golden/make_ref_fixtures.py) on seeded inputs that are regenerated here.
Layer norm and the decoder attention's rounded outputs must agree with the oracle's restatement of the same
arithmetic to within an fp16 ulp nearly everywhere; the encoder attention must sit within the 2e-3 bar of the exact
oracle."""
import os

import numpy as np
import pytest

import _oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "ref_fixtures.npz")

import importlib.util  # noqa: E402
_spec = importlib.util.spec_from_file_location("mkfix", os.path.join(HERE, "golden", "make_ref_fixtures.py"))
mkfix = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mkfix)


@pytest.fixture(scope="module")
def fx():
    return np.load(FIX)


def ulps(a, b):
    """distance in fp16 units in the last place, per element"""
    ia = a.view(np.uint16).astype(np.int32)
    ib = b.view(np.uint16).astype(np.int32)
    ia = np.where(ia & 0x8000, 0x8000 - ia, ia)
    ib = np.where(ib & 0x8000, 0x8000 - ib, ib)
    return np.abs(ia - ib)


def within_ulp(a, ref, k=1):
    """|a - ref| <= k fp16 spacings at ref, for elements whose value rounding alone can move"""
    sp = np.abs(np.spacing(ref.astype(np.float16))).astype(np.float32)
    return np.all(np.abs(a.astype(np.float32) - ref.astype(np.float32)) <= k * sp + 1e-7)


def test_layernorm(fx):
    x, dx, w, b = mkfix.inputs_ln()
    y = O.layernorm(x, w, b)
    assert ulps(y, fx["ln_y"]).max() <= 1 and np.mean(y.view(np.uint16) == fx["ln_y"].view(np.uint16)) > 0.99
    xo, yo = O.add_layernorm(x, dx, w, b)
    assert np.array_equal(xo.view(np.uint16), fx["ln_x"].view(np.uint16))  # the residual add is exact
    assert ulps(yo, fx["addln_y"]).max() <= 1


def test_cross_attention(fx):
    q, kv, aslot, c = mkfix.inputs_cross()
    done = np.zeros(c["B"], np.int32)
    align0 = np.zeros((c["B"], c["max_t"], c["na"], 1500), np.float16)
    out, align = O.cross_attn(q, kv, align0, aslot, c["p"], done, c["layer"], c["nl"], c["d"], c["na"], c["max_t"])
    # the oracle accumulates scores in double, the reference in fp32: a score that rounds to the other fp16 neighbour
    # moves its probability by ~1e-3 relative and an output by ~1e-6 absolute
    # (and a near-tie of the final rounding moves it by one fp16 spacing)
    ref = fx["cross_out"]
    allowed = np.maximum(np.abs(np.spacing(ref.astype(np.float16))).astype(np.float32), 4e-6)
    assert np.all(np.abs(out.astype(np.float32) - ref.astype(np.float32)) <= allowed)
    assert np.mean(out.view(np.uint16) == fx["cross_out"].view(np.uint16)) > 0.95
    a = align[:, c["p"]]
    assert ulps(a, fx["cross_align"]).max() <= 1
    assert np.mean(a.view(np.uint16) == fx["cross_align"].view(np.uint16)) > 0.999


def test_self_attention(fx):
    qkv, kc, vc, c = mkfix.inputs_self()
    out, _, _ = O.self_attn(qkv, kc, vc, c["p"], np.zeros(c["B"], np.int32), c["max_t"], c["d"])
    assert within_ulp(out, fx["self_out"], 1)
    assert np.mean(out.view(np.uint16) == fx["self_out"].view(np.uint16)) > 0.95


def test_encoder_attention(fx):
    qkv = mkfix.inputs_enc()
    ex = O.enc_attn_f64(qkv, 384)[0, mkfix.ENC_ROWS]
    ref = fx["enc_rows"].astype(np.float64)
    assert np.abs(ref - ex).max() < 2e-3
