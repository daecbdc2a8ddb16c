"""CPU tests: the oracle against the reference's own known answers (tests/golden/kat.json), the product's CPU stages
(fp16 helpers, timestamps, features) bit-identical to the oracle, and the oracle's attention routines against each
other (rounding restatement vs exact)."""
import json
import os

import numpy as np
import pytest

import _oracle as O
import mimizuku_b200 as m

KAT = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "kat.json")))


# ------------------------------------------------------------------ fp16 (src/gpu.rs:79-119, tests :380-397)

def test_fp16_exhaustive_round_trip():
    hs = np.arange(65536, dtype=np.uint16)
    xs = np.zeros(65536, np.float32)
    O.orc.orc_h2f_array(O.u16(hs), O.fp(xs), 65536)
    # h2f agrees with numpy's binary16 decoding on every pattern
    ref = hs.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(xs[~nan].view(np.uint32), ref[~nan].view(np.uint32)) and np.isnan(xs[nan]).all()
    back = np.zeros(65536, np.uint16)
    O.orc.orc_f2h_array(O.fp(xs), O.u16(back), 65536)
    assert np.array_equal(back[~nan], hs[~nan])
    # the product's helpers are the same functions
    for h in list(range(0, 65536, 97)) + [0x7C00, 0xFC00, 0x7E00, 0x0001, 0x8001, 0x03FF, 0x7BFF]:
        x = m.h2f(h)
        assert np.float32(x).view(np.uint32) == np.float32(O.orc.orc_h2f(h)).view(np.uint32) or (np.isnan(x))
        if not np.isnan(x):
            assert m.f2h(x) == h


def test_fp16_golden():
    for v in KAT["fp16"]:
        assert O.orc.orc_f2h(v["x"]) == v["bits"]
        assert m.f2h(v["x"]) == v["bits"]
    for v in KAT["rh"]:
        assert O.orc.orc_rh(v["x"]) == np.float32(v["y"])
        assert m.rh(v["x"]) == np.float32(v["y"])


def test_f2h_random_patterns_match_numpy():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[~np.isnan(x)]
    out = np.zeros(len(x), np.uint16)
    O.orc.orc_f2h_array(O.fp(x), O.u16(out), len(x))
    assert np.array_equal(out, x.astype(np.float16).view(np.uint16))


# ------------------------------------------------------------------ timestamps (src/align.rs, tests :108-140)

def _kat_w():
    j = KAT["jump"]
    w = np.zeros((j["rows"], j["heads"], j["cols_full"]), np.float32)
    for i, c in j["nonzero"]:
        w[i, 0, c] = j["value"]
    return w


@pytest.mark.parametrize("impl", ["oracle", "product"])
def test_dtw_kat(impl):
    k = KAT["dtw"]
    fn = O.dtw if impl == "oracle" else m.dtw
    text, time = fn(np.array(k["m"], np.float64))
    assert text.tolist() == k["text"] and time.tolist() == k["time"]


@pytest.mark.parametrize("impl", ["oracle", "product"])
def test_jump_times_kat(impl):
    j = KAT["jump"]
    fn = O.jump_times if impl == "oracle" else m.jump_times
    w = _kat_w()
    t = fn(w, j["cols"], j["width"])
    assert len(t) == j["rows"]
    assert np.all(np.abs(t - np.array(j["expect_near"], np.float32)) < j["tol"])
    assert fn(w, 0, j["width"]).tolist() == j["zero_frames"]
    assert fn(w[:1], j["cols"], j["width"]).tolist() == j["one_token"]


@pytest.mark.parametrize("rows,heads,cols_full,cols", [(1, 2, 1500, 750), (5, 3, 60, 2), (5, 3, 60, 3), (5, 3, 60, 4),
                                                       (17, 10, 1500, 1500), (224, 2, 1500, 1117), (3, 40, 100, 99)])
def test_jump_times_product_is_the_oracle_bit_for_bit(rows, heads, cols_full, cols):
    rng = np.random.default_rng(rows * 7 + heads)
    # fp16-valued probabilities as the engine records them, with ties and constant columns mixed in
    w = rng.random((rows, heads, cols_full)).astype(np.float16).astype(np.float32) * 0.01
    w[:, :, ::17] = 0.0
    w[:, 0, 5:9] = 0.25
    a = m.jump_times(w, cols)
    b = O.jump_times(w, cols)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_times_from_cost_product_is_the_oracle_and_splits_jump_times():
    rng = np.random.default_rng(5)
    for rows, heads, cols_full, cols in [(1, 2, 40, 30), (7, 3, 60, 4), (30, 10, 1500, 1500), (223, 2, 1500, 999)]:
        w = rng.random((rows, heads, cols_full)).astype(np.float16).astype(np.float32) * 0.01
        w[:, :, ::13] = 0.0
        cost = O.align_cost(w, cols)
        t_split = O.times_from_cost(cost, cols)
        assert np.array_equal(t_split.view(np.uint32), O.jump_times(w, cols).view(np.uint32))
        padded = np.zeros((rows, cols_full), np.float32)  # a row stride wider than cols, as the engine's buffer
        padded[:, :cols] = cost
        padded[:, cols:] = 1e6  # never read
        assert np.array_equal(m.times_from_cost(padded, cols).view(np.uint32), t_split.view(np.uint32))


def test_dtw_product_is_the_oracle_with_ties():
    rng = np.random.default_rng(1)
    for rows, cols in [(1, 1), (1, 9), (9, 1), (12, 40), (40, 12), (64, 300)]:
        cost = rng.integers(-2, 3, (rows, cols)).astype(np.float64)  # small integers: many ties
        ta, sa = m.dtw(cost)
        tb, sb = O.dtw(cost)
        assert np.array_equal(ta, tb) and np.array_equal(sa, sb)
        assert ta[-1] == rows - 1 and sa[-1] == cols - 1


# ------------------------------------------------------------------ features (src/audio.rs:192-237)

def test_log_mel_silence_and_frames():
    mel, frames = m.log_mel(np.zeros(16000 * 3, np.float32), 80)
    assert frames == 300
    assert np.all(mel == mel[0, 0])  # silence: every value is the floor, (-10 + 4) / 4
    assert mel[0, 0] == np.float32(-1.5)


def test_log_mel_tone_peaks_near_its_frequency():
    t = np.arange(16000 * 2) / 16000.0
    y = (0.5 * np.sin(2 * np.pi * 1000.0 * t)).astype(np.float32)
    mel, frames = m.log_mel(y, 128)
    assert frames == 200
    band = int(np.argmax(mel[:, 100]))
    # the 1 kHz tone falls in the mel bands around 1 kHz (Slaney scale: mel 15 at 1 kHz of 45 at 8 kHz)
    centres = np.array([200.0 * mm / 3 if mm < 15 else 1000.0 * np.exp(np.log(6.4) / 27 * (mm - 15))
                        for mm in np.linspace(0, 45.245640471924965, 130)[1:-1]])
    assert abs(centres[band] - 1000.0) < 60.0
    assert np.all(mel[:, 250:] == mel.min())  # frames past the audio sit at the floor


def _log_mel_numpy(y, n_mels):
    """Independent numpy statement of src/audio.rs:147-237 (rfft instead of the direct DFT, f64 throughout): reflect
    padding of 200, periodic Hann window, |X|^2, Slaney-style filterbank with area normalisation, log10 floor 1e-10,
    max - 8 clamp, (x + 4) / 4; frames past the audio at the floor."""
    sr, n_fft, hop, n_frames = 16000, 400, 160, 3000
    x = np.zeros(30 * sr, np.float64)
    n = min(len(y), 30 * sr)
    x[:n] = y[:n]
    xp = np.pad(x, (n_fft // 2, n_fft // 2), mode="reflect")
    win = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(n_fft) / n_fft)
    live = min((n + n_fft // 2 + hop - 1) // hop, n_frames)
    frames = np.stack([xp[t * hop:t * hop + n_fft] * win for t in range(live)])
    power = np.abs(np.fft.rfft(frames, axis=1)) ** 2
    logstep = 27.0 / np.log(6.4)

    def hz_to_mel(f):
        return 15.0 + np.log(f / 1000.0) * logstep if f >= 1000.0 else 3.0 * f / 200.0

    def mel_to_hz(mm):
        return 1000.0 * np.exp((mm - 15.0) / logstep) if mm >= 15.0 else 200.0 * mm / 3.0

    fft_f = np.arange(n_fft // 2 + 1) * (sr / 2.0) / (n_fft // 2)
    m0, m1 = hz_to_mel(0.0), hz_to_mel(8000.0)
    ff = np.array([mel_to_hz(m0 + (m1 - m0) * i / (n_mels + 1)) for i in range(n_mels + 2)])
    fb = np.zeros((n_mels, n_fft // 2 + 1))
    for i in range(n_mels):
        down = (fft_f - ff[i]) / (ff[i + 1] - ff[i])
        up = (ff[i + 2] - fft_f) / (ff[i + 2] - ff[i + 1])
        fb[i] = np.maximum(np.minimum(down, up), 0.0) * 2.0 / (ff[i + 2] - ff[i])
    out = np.full((n_mels, n_frames), -10.0)
    out[:, :live] = np.log10(np.maximum(fb @ power.T, 1e-10))
    return (np.maximum(out, out.max() - 8.0) + 4.0) / 4.0


@pytest.mark.parametrize("seed,n", [(5, 480000), (6, 123457), (7, 3000)])
def test_log_mel_matches_an_independent_numpy_statement(seed, n):
    y = m.synth_clip(seed, n)
    mel, frames = m.log_mel(y, 128)
    want = _log_mel_numpy(y, 128)
    assert frames == min((n + 159) // 160, 3000)
    # f32 power and filterbank sums against f64 throughout: well inside the fp16 step the encoder reads them with
    assert np.abs(mel - want).max() < 1e-4


def test_synth_clip_is_seeded():
    a, b, c = m.synth_clip(3, 16000), m.synth_clip(3, 16000), m.synth_clip(4, 16000)
    assert np.array_equal(a, b) and not np.array_equal(a, c) and np.abs(a).max() <= 1.0


# ------------------------------------------------------------------ attention oracles against each other

def test_self_attn_rounding_oracle_vs_exact():
    rng = np.random.default_rng(2)
    B, d, mt = 3, 384, 448
    qkv = O.normal16(rng, (B, 3 * d))
    kc, vc = O.normal16(rng, (B, mt, d)), O.normal16(rng, (B, mt, d))
    done = np.array([0, 1, 0], np.int32)
    for p in (0, 5, 447):
        out, kc2, vc2 = O.self_attn(qkv, kc, vc, p, done, mt, d)
        ex = O.self_attn_f64(qkv, kc, vc, p, done, mt, d)
        assert np.abs(out[[0, 2]].astype(np.float64) - ex[[0, 2]]).max() < 2e-3
        assert np.array_equal(kc2[:, p], qkv[:, d:2 * d]) and np.array_equal(vc2[:, p], qkv[:, 2 * d:])
        assert np.all(out[1] == 0)


def test_cross_attn_rounding_oracle_vs_exact():
    rng = np.random.default_rng(3)
    B, d, nl, mt, p = 2, 384, 2, 448, 7
    q = O.normal16(rng, (B, d))
    kv = O.normal16(rng, (B, nl, 2, 6, 1500, 64))
    aslot = -np.ones(nl * 6, np.int32)
    aslot[6 + 2] = 0
    done = np.zeros(B, np.int32)
    out, align = O.cross_attn(q, kv, np.zeros((B, mt, 1, 1500), np.float16), aslot, p, done, 1, nl, d, 1, mt)
    ex, probs = O.cross_attn_f64(q, kv, done, 1, nl, d)
    assert np.abs(out.astype(np.float64) - ex).max() < 2e-3
    assert np.abs(align[:, p, 0].astype(np.float64) - probs[:, 2]).max() < 2e-3
    assert abs(align[:, p, 0].astype(np.float64).sum(axis=1) - 1.0).max() < 1e-2


def test_cpu_baseline_attention_matches_exact():
    rng = np.random.default_rng(4)
    d = 128
    qkv = O.normal16(rng, (1, 1500, 3 * d))
    out = np.zeros((1, 1500, d), np.float16)
    O.orc.orc_cpu_enc_attn(O.u16(qkv), O.u16(out), 1, d, 2, 64, 2)
    ex = O.enc_attn_f64(qkv, d, 0, 64)
    assert np.abs(out[0, :64].astype(np.float64) - ex[0, :64]).max() < 2e-3
