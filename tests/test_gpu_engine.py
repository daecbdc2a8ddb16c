"""End-to-end parity of the engine on the native sm_100a kernels against the same engine on the reference's own
kernels (the compute_80 build of kernels/whisper.cu), random-init tiny Whisper, synthetic clips.

Bars (north star): greedy tokens identical except at steps where the reference's top-2 logit gap is below 1e-2
(checked in lockstep with teacher forcing, so every later step is still compared); token timestamps identical
wherever the tokens agree."""
import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu


def _clips(n, n_mels, seed=0):
    import mimizuku_b200 as m
    ys = [m.synth_clip(seed * 1000 + i, 16000 * (10 + 7 * i)) for i in range(n)]
    return m.log_mel_batch(ys, n_mels)


def _engines(cfg, b):
    import mimizuku_b200 as m
    sup = [cfg.eos]  # fixed-length decoding, as the benchmark runs it
    nat = m.Engine(cfg, bmax=b, eg=2, seed=11, suppress=sup)
    refe = m.Engine(cfg, bmax=b, eg=2, seed=11, suppress=sup, kernel_image=O.REF_FATBIN)
    return nat, refe


def _top2_gap(logits, sup, first, bs):
    v = logits.astype(np.float32).copy()
    v[sup] = -np.inf
    if first:
        v[[t for t in bs if t >= 0]] = -np.inf
    top = np.sort(v)[-2:]
    return top[1] - top[0]


def _lockstep(cfg, nat, refe, b, steps):
    """Decodes both engines step by step; where their tokens differ the reference's top-2 logit gap must be below
    1e-2, and the reference's token is fed to both (teacher forcing). Returns (diverged, compared)."""
    prompt = np.array(cfg.prompt, np.int32)
    np_ = len(prompt)
    for e in (nat, refe):
        e.reset(np.tile(prompt, (b, 1)))
    mt, V = cfg.max_t, cfg.vocab
    tok_n = np.empty(b * mt, np.int32)
    tok_r = np.empty(b * mt, np.int32)
    lg = np.empty(b * V, np.float16)
    diverged, compared = 0, 0
    for p in range(np_ - 1 + steps):  # the step feeding position p chooses p + 1
        nat.step(b, np_)
        refe.step(b, np_)
        nat.sync()
        refe.sync()
        if p + 1 < np_:
            continue
        O.d2h(tok_n, nat.buffer("tok"))
        O.d2h(tok_r, refe.buffer("tok"))
        O.d2h(lg, refe.buffer("logits"))
        fix = False
        for i in range(b):
            tn, tr = tok_n[i * mt + p + 1], tok_r[i * mt + p + 1]
            compared += 1
            if tn != tr:
                diverged += 1
                gap = _top2_gap(lg[i * V:(i + 1) * V], [cfg.eos], p + 1 == np_, cfg.begin_suppress)
                assert gap < 1e-2, f"step {p}: tokens {tn} vs {tr} with a top-2 gap of {gap}"
                tok_n[i * mt + p + 1] = tr
                fix = True
        if fix:
            O.h2d(nat.buffer("tok"), tok_n)
    return diverged, compared


def _align_rows(e, cfg, b):
    a = np.empty(b * cfg.max_t * e.na * 1500, np.float16)
    O.d2h(a, e.buffer("align"))
    return a.reshape(b, cfg.max_t, e.na, 1500).astype(np.float32)


def test_engine_lockstep_against_reference_kernels(cuda, ref):
    """Native encoder and decoder against the reference's: cross k/v within fp16 noise of each other, tokens
    identical except at near-ties, alignment probabilities within 2e-3."""
    import mimizuku_b200 as m
    torch = cuda
    cfg = m.TINY
    b, steps = 3, 40
    mel, frames = _clips(b, cfg.n_mels)
    nat, refe = _engines(cfg, b)
    mel16 = torch.from_numpy(mel.astype(np.float16)).cuda()
    for e in (nat, refe):
        e.encode(mel16[:2].data_ptr(), 2, 0)
        e.encode(mel16[2:].data_ptr(), 1, 2)
        e.sync()
    # cross k/v of every slot, written from each engine's encoder output (dev.rs:7-26 style report)
    xkv_n = b * cfg.dec_layers * 2 * cfg.d * 1500
    a = np.empty(xkv_n, np.float16)
    r = np.empty(xkv_n, np.float16)
    O.d2h(a, nat.buffer("xkv"))
    O.d2h(r, refe.buffer("xkv"))
    af, rf = a.astype(np.float32), r.astype(np.float32)
    rel = np.sqrt(((af - rf) ** 2).sum() / (rf ** 2).sum())
    assert rel < 2e-2, rel
    diverged, compared = _lockstep(cfg, nat, refe, b, steps)
    assert compared == b * steps
    assert diverged <= max(1, compared // 20), (diverged, compared)
    np_ = len(cfg.prompt)
    al_n, al_r = _align_rows(nat, cfg, b), _align_rows(refe, cfg, b)
    assert np.abs(al_n[:, np_:np_ + steps - 1] - al_r[:, np_:np_ + steps - 1]).max() < 2e-3
    nat.close()
    refe.close()


@pytest.mark.parametrize("b", [9, 5, 1])
def test_decoder_and_timestamps_against_reference_kernels(cuda, ref, b):
    """Both engines decode from the same encoder output (the reference engine's cross k/v copied into the native
    one): the decoder path alone then gives the same tokens, nearly bit-identical alignment probabilities, and token
    timestamps (median filter + DTW) identical wherever the tokens agree. Nine sequences run every decoder GEMM
    through cuBLAS in both engines; five and one run them, and the logits, through the gemv kernels (the reference's
    up to 8 rows, src/gpu.rs:211-228, this library's own in the native engine)."""
    import mimizuku_b200 as m
    torch = cuda
    cfg = m.TINY
    steps = 48
    mel, frames = _clips(b, cfg.n_mels, seed=1)
    nat, refe = _engines(cfg, b)
    mel16 = torch.from_numpy(mel.astype(np.float16)).cuda()
    for g0 in range(0, b, 2):
        refe.encode(mel16[g0].data_ptr(), min(2, b - g0), g0)
    refe.sync()
    xkv_n = b * cfg.dec_layers * 2 * cfg.d * 1500
    r = np.empty(xkv_n, np.float16)
    O.d2h(r, refe.buffer("xkv"))
    O.h2d(nat.buffer("xkv"), r)
    diverged, compared = _lockstep(cfg, nat, refe, b, steps)
    assert diverged <= 1, (diverged, compared)
    np_ = len(cfg.prompt)
    rows = steps - 1
    al_n, al_r = _align_rows(nat, cfg, b), _align_rows(refe, cfg, b)
    wn, wr = al_n[:, np_:np_ + rows], al_r[:, np_:np_ + rows]
    assert np.abs(wn - wr).max() < 2e-3
    assert np.mean(wn == wr) > 0.99, np.mean(wn == wr)
    for i in range(b):
        tn = m.jump_times(wn[i], frames[i] // 2)
        tr = m.jump_times(wr[i], frames[i] // 2)
        assert np.array_equal(tr, O.jump_times(wr[i], frames[i] // 2))  # the product DTW is the oracle's
        assert np.array_equal(tn, tr), (i, tn, tr)
    nat.close()
    refe.close()


def test_transcribe_graph_matches_eager(cuda):
    """The CUDA-graph decode (one captured step replayed, position read from device memory) produces exactly the
    tokens and times of eager stepping."""
    import mimizuku_b200 as m
    cfg = m.TINY
    b = 2
    mel, frames = _clips(b, cfg.n_mels, seed=3)
    e = m.Engine(cfg, bmax=b, eg=2, seed=5, suppress=[cfg.eos])
    g = e.transcribe(mel, frames, max_new=24, graph=True)
    x = e.transcribe(mel, frames, max_new=24, graph=False)
    assert np.array_equal(g["tokens"], x["tokens"]) and np.array_equal(g["times"], x["times"])
    assert (g["lens"] == len(cfg.prompt) + 24).all()
    e.close()


def test_transcribe_stops_once_every_sequence_has_finished(cuda):
    """With every token but end-of-text suppressed, each sequence finishes at its first generated token: the decoding
    loop stops at a poll (the steps it may run past that change nothing), graph and eager agree, and every length is
    the prompt plus one."""
    import mimizuku_b200 as m
    cfg = m.TINY
    b = 3
    mel, frames = _clips(b, cfg.n_mels, seed=4)
    sup = [t for t in range(cfg.vocab) if t != cfg.eos]
    e = m.Engine(cfg, bmax=b, eg=2, seed=6, suppress=sup)
    g = e.transcribe(mel, frames, max_new=200, graph=True)
    x = e.transcribe(mel, frames, max_new=200, graph=False)
    np_ = len(cfg.prompt)
    assert (g["lens"] == np_ + 1).all() and (x["lens"] == np_ + 1).all()
    assert (g["tokens"][:, np_] == cfg.eos).all()
    assert np.array_equal(g["tokens"], x["tokens"]) and np.array_equal(g["times"], x["times"])
    e.close()


def test_transcribe_from_audio_is_transcribe_of_the_gpu_features(cuda):
    """mmz_engine_transcribe_audio (features on the GPU, group by group) gives exactly what mmz_engine_transcribe gives
    for the features of mmz_log_mel_gpu, with the host's frame counts."""
    import mimizuku_b200 as m
    torch = cuda
    cfg = m.TINY
    b = 3
    ys = [m.synth_clip(20 + i, 16000 * (5 + 9 * i)) for i in range(b)]
    e = m.Engine(cfg, bmax=b, eg=2, seed=8, suppress=[cfg.eos])
    r = e.transcribe_audio(ys, max_new=16)
    audio = np.zeros((b, 480000), np.float32)
    for i, y in enumerate(ys):
        audio[i, :len(y)] = y
    mel = torch.empty((b, cfg.n_mels, 3000), dtype=torch.float32, device="cuda")
    m.log_mel_gpu(torch.from_numpy(audio).cuda(), torch.tensor([len(y) for y in ys], dtype=torch.int32,
                                                               device="cuda"), cfg.n_mels, mel)
    _, frames = m.log_mel_batch(ys, cfg.n_mels)
    assert np.array_equal(r["frames"], frames)
    x = e.transcribe(mel.cpu().numpy(), frames, max_new=16)
    for k in ("tokens", "lens", "times"):
        assert np.array_equal(r[k], x[k]), k
    e.close()


@pytest.mark.parametrize("name,b,new", [("TINY", 32, 24), ("LARGE_V3_TURBO", 32, 12)])
def test_two_decoder_lanes_match_one(cuda, name, b, new):
    """Two decoder lanes (the halves of a 32-sequence batch on two streams, the native image's default) give exactly
    the tokens, alignment rows and token times of one lane (the whole batch on one stream, as src/model.rs runs the
    step), in the captured graph and eagerly; the turbo case has large-v3's decoder GEMM shapes."""
    import mimizuku_b200 as m
    cfg = getattr(m, name)
    mel, frames = _clips(b, cfg.n_mels, seed=2)
    e = m.Engine(cfg, bmax=b, eg=8, seed=5, suppress=[cfg.eos])
    assert e.lanes == 2
    out = {}
    for lanes in (2, 1):
        e.lanes = lanes
        for graph in (True, False):
            r = e.transcribe(mel, frames, max_new=new, graph=graph)
            r["align"] = _align_rows(e, cfg, b)
            out[lanes, graph] = r
    for k in ("tokens", "lens", "times", "align"):
        for key in out:
            assert np.array_equal(out[key][k], out[1, True][k]), (key, k)
    assert (out[2, True]["lens"] == len(cfg.prompt) + new).all()
    e.close()


def test_fatbin_engine_decodes_on_one_lane(cuda, ref):
    """An engine on the reference's kernels keeps the reference host's single stream and refuses a second lane."""
    import mimizuku_b200 as m
    e = m.Engine(m.TINY, bmax=2, eg=2, kernel_image=O.REF_FATBIN)
    assert e.lanes == 1
    with pytest.raises(m.MmzError):
        e.lanes = 2
    e.close()


def test_engine_for_fewer_than_32_sequences_has_one_lane(cuda):
    """An engine created for fewer than 32 sequences sets up no second lane: it reports one lane and refuses two."""
    import mimizuku_b200 as m
    e = m.Engine(m.TINY, bmax=9, eg=8, seed=5, suppress=[m.TINY.eos])
    assert e.lanes == 1
    with pytest.raises(m.MmzError):
        e.lanes = 2
    e.close()


def test_lane_check_failure_falls_back_to_one_lane(cuda, monkeypatch):
    """When the creation-time check finds cuBLAS's half-batch rows different from the whole batch's (forced here by
    the library's test hook), the engine starts on one lane, refuses two, and decodes exactly as an engine that
    passed the check and was set to one lane."""
    import mimizuku_b200 as m
    cfg, b, new = m.TINY, 32, 12
    mel, frames = _clips(b, cfg.n_mels, seed=7)
    monkeypatch.setenv("MMZ_TEST_LANES_DIFFER", "1")
    e = m.Engine(cfg, bmax=b, eg=8, seed=5, suppress=[cfg.eos])
    monkeypatch.delenv("MMZ_TEST_LANES_DIFFER")
    assert e.lanes == 1
    with pytest.raises(m.MmzError):
        e.lanes = 2
    r = e.transcribe(mel, frames, max_new=new)
    e.close()
    ok = m.Engine(cfg, bmax=b, eg=8, seed=5, suppress=[cfg.eos])
    assert ok.lanes == 2
    ok.lanes = 1
    x = ok.transcribe(mel, frames, max_new=new)
    ok.close()
    for k in ("tokens", "lens", "times"):
        assert np.array_equal(r[k], x[k]), k


@pytest.mark.parametrize("b", [32, 12])
def test_fused_logits_argmax_matches_three_launches(cuda, monkeypatch, b):
    """The native step's fused logits + greedy choice + advance (one kernel) gives exactly the tokens, lengths and
    times of the logits kernel, argmax_tok and advance launched one after the other (the library's test hook keeps
    that path), in the captured graph and eagerly."""
    import mimizuku_b200 as m
    cfg = m.TINY
    mel, frames = _clips(b, cfg.n_mels, seed=9)
    out = {}
    for unfused in (False, True):
        if unfused:
            monkeypatch.setenv("MMZ_TEST_UNFUSED_LOGITS", "1")
        e = m.Engine(cfg, bmax=b, eg=8, seed=3, suppress=[cfg.eos])
        monkeypatch.delenv("MMZ_TEST_UNFUSED_LOGITS", raising=False)
        for graph in (True, False):
            out[unfused, graph] = e.transcribe(mel, frames, max_new=20, graph=graph)
        e.close()
    for key in out:
        for k in ("tokens", "lens", "times"):
            assert np.array_equal(out[key][k], out[True, True][k]), (key, k)
    assert (out[False, True]["lens"] == len(cfg.prompt) + 20).all()


@pytest.mark.parametrize("b,eos", [(1, False), (5, False), (8, False), (6, True)])
def test_one_launch_cross_attention_matches_three(cuda, monkeypatch, b, eos):
    """Up to 8 sequences the native step runs the cross-attention as one launch on clusters of 8 CTAs (no scratch);
    its tokens, times and every alignment probability equal those of the three-kernel cross-attention (the library's
    hook MMZ_CROSS_FUSED_MAX=0 keeps it), bit for bit; also when every sequence has finished and both skip it."""
    import mimizuku_b200 as m
    cfg = m.TINY
    mel, frames = _clips(b, cfg.n_mels, seed=17)
    res = {}
    for mx in ("8", "0"):
        monkeypatch.setenv("MMZ_CROSS_FUSED_MAX", mx)
        # eos: only end-of-text left, so every sequence ends at its first token and the steps run until the next
        # poll of the finished flags skip them all
        sup = [t for t in range(cfg.vocab) if t != cfg.eos] if eos else [cfg.eos]
        e = m.Engine(cfg, bmax=b, eg=min(b, 8), seed=6, suppress=sup)
        monkeypatch.delenv("MMZ_CROSS_FUSED_MAX", raising=False)
        out = e.transcribe(mel, frames, max_new=20, graph=True)
        al = np.empty(b * cfg.max_t * e.na * 1500, np.float16)
        O.d2h(al, e.buffer("align"))
        res[mx] = (out, al.view(np.uint16))
        e.close()
    for k in ("tokens", "lens", "times"):
        assert np.array_equal(res["8"][0][k], res["0"][0][k]), k
    assert np.array_equal(res["8"][1], res["0"][1])
    if eos:
        assert (res["8"][0]["lens"] == len(cfg.prompt) + 1).all(), res["8"][0]["lens"]
    assert m.status()[0] == 0
