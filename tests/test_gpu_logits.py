"""The decoding step's logits fused with the greedy token choice (mmz_logits_argmax) against this library's logits
kernel (mmz_dec_linear, bit for bit) and argmax_tok's rule restated in numpy (kernels/whisper.cu:451-493: suppressed
ids never chosen, bs1/bs2 also at the first generated position, ties to the lower id, eos for finished sequences and
for sequences with no candidate, eos sets done; nothing chosen before the prompt's end or past max_t)."""
import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu

MAX_T = 448


def _choose(lg, sup, first, bs, done, eos):
    """argmax_tok on fp16 logits lg [m][V] (host restatement)."""
    V = lg.shape[1]
    mask = sup.astype(bool).copy()
    if first:
        for t in bs:
            if 0 <= t < V:
                mask[t] = True
    out = []
    for i in range(lg.shape[0]):
        v = lg[i].astype(np.float32)
        cand = ~mask & ~np.isnan(v)
        if done[i] or not cand.any():
            out.append(eos)
            continue
        best = v[cand].max()
        out.append(int(np.flatnonzero(cand & (v == best))[0]))
    return np.array(out, np.int32)


def _case(torch, V, d, m, seed, sup_frac=0.0, ties=False):
    rng = np.random.default_rng(seed)
    x = O.normal16(rng, (m, d))
    emb = O.normal16(rng, (V, d), 0.02)
    sup = (rng.random(V) < sup_frac).astype(np.uint8)
    if ties:  # three equal rows along the sequences' common sign pattern: every sequence's maximum, tied three ways
        row = (0.05 * np.sign(x.astype(np.float32).sum(0))).astype(np.float16)
        for t in (V // 7, V // 2, V - 3):
            emb[t] = row
            sup[t] = 0
    return emb, x, sup


def _run(m_, torch, emb, x, sup, p, np_, done, bs=(-1, -1), advance=True, logits=True):
    V, d = emb.shape
    m = x.shape[0]
    E, X = torch.from_numpy(emb).cuda(), torch.from_numpy(x).cuda()
    S = torch.from_numpy(sup).cuda()
    tok = torch.full((m, MAX_T), -7, dtype=torch.int32, device="cuda")
    D = torch.from_numpy(np.array(done, np.int32)).cuda()
    ctr = torch.tensor([p, 0, 0, 0], dtype=torch.int32, device="cuda")
    scratch = torch.zeros(m_.logits_argmax_scratch_bytes(), dtype=torch.uint8, device="cuda")
    L = torch.zeros(m, V, dtype=torch.float16, device="cuda") if logits else None
    m_.logits_argmax(X, E, S, tok, D, ctr, MAX_T, np_, 50257, bs=bs, scratch=scratch, logits=L, advance=advance)
    # the same logits from the library's logits kernel
    Y = torch.zeros(m, V, dtype=torch.float16, device="cuda")
    m_.dec_linear(X, E, None, Y)
    torch.cuda.synchronize()
    assert m_.status()[0] == 0
    assert int(scratch.count_nonzero()) == 0  # left zero for the next launch
    return tok.cpu().numpy(), D.cpu().numpy(), ctr.cpu().numpy(), (L.cpu().numpy() if logits else None), Y.cpu().numpy()


@pytest.mark.parametrize("V,d,m,sup_frac,first,ties", [
    (51866, 1280, 32, 0.0, False, False),    # large-v3 vocabulary and width, the benchmark's batch
    (51866, 1280, 9, 0.1, True, False),      # suppression and the begin-suppressed ids at the first position
    (51865, 384, 3, 0.02, False, True),      # tiny width, odd vocabulary, exact ties
    (1000, 512, 1, 0.0, False, True),        # fewer tiles than SMs
])
def test_logits_argmax_matches_logits_kernel_and_argmax_rule(cuda, V, d, m, sup_frac, first, ties):
    import mimizuku_b200 as m_
    torch = cuda
    emb, x, sup, = _case(torch, V, d, m, V + d + m, sup_frac, ties)
    np_ = 4
    p = np_ - 1 if first else 57
    done = [1 if (i % 5 == 4) else 0 for i in range(m)]
    bs = (220, 50257)
    tok, D, ctr, L, Y = _run(m_, torch, emb, x, sup, p, np_, done, bs=bs)
    if V > 148 * 128:  # the logits kernel does not split K here (every Whisper vocabulary): bit for bit
        assert np.array_equal(L.view(np.uint16), Y.view(np.uint16))
    else:  # it splits K, which associates the fp32 sums differently: one fp16 rounding apart at most
        assert np.all(np.abs(L.astype(np.float32) - Y.astype(np.float32)) <= np.abs(Y.astype(np.float32)) * 2 ** -10
                      + 2 ** -24)
    want = _choose(L, sup, first, bs, done, 50257)
    assert np.array_equal(tok[:, p + 1], want), (tok[:, p + 1], want)
    assert (tok[:, :p + 1] == -7).all() and (tok[:, p + 2:] == -7).all()  # only position p + 1 is written
    assert np.array_equal(D, np.array([1 if (done[i] or want[i] == 50257) else 0 for i in range(m)], np.int32))
    assert ctr[0] == p + 1
    if ties:
        assert (want[np.array(done) == 0] == V // 7).all()  # the lowest of the tied ids


def test_logits_argmax_chooses_nothing_inside_the_prompt_or_past_max_t(cuda):
    import mimizuku_b200 as m_
    torch = cuda
    emb, x, sup = _case(torch, 4096, 384, 4, 3)
    for p, np_ in ((1, 4), (MAX_T - 1, 4)):
        tok, D, ctr, L, Y = _run(m_, torch, emb, x, sup, p, np_, [0] * 4, logits=False)
        assert (tok == -7).all() and (D == 0).all()
        assert ctr[0] == p + 1  # the position still advances


def test_logits_argmax_with_every_id_suppressed_gives_eos(cuda):
    import mimizuku_b200 as m_
    torch = cuda
    emb, x, _ = _case(torch, 700, 384, 5, 4)
    sup = np.ones(700, np.uint8)
    tok, D, ctr, L, Y = _run(m_, torch, emb, x, sup, 10, 4, [0] * 5, advance=False)
    assert (tok[:, 11] == 50257).all() and (D == 1).all() and ctr[0] == 10


def test_logits_argmax_steps_in_a_graph(cuda):
    """Consecutive steps replayed from one CUDA graph (the position read from ctr and advanced by the kernel) choose
    what eager launches choose."""
    import mimizuku_b200 as m_
    torch = cuda
    emb, x, sup = _case(torch, 51866, 1280, 32, 5, 0.01)
    E, X, S = torch.from_numpy(emb).cuda(), torch.from_numpy(x).cuda(), torch.from_numpy(sup).cuda()
    outs = []
    for graph in (False, True):
        tok = torch.zeros(32, MAX_T, dtype=torch.int32, device="cuda")
        D = torch.zeros(32, dtype=torch.int32, device="cuda")
        ctr = torch.tensor([0, 0, 0, 0], dtype=torch.int32, device="cuda")
        scratch = torch.zeros(m_.logits_argmax_scratch_bytes(), dtype=torch.uint8, device="cuda")
        st = torch.cuda.Stream()
        step = lambda: m_.logits_argmax(X, E, S, tok, D, ctr, MAX_T, 4, 50257, bs=(220, 50257),  # noqa: E731
                                        scratch=scratch, advance=True, stream=st.cuda_stream)
        if graph:
            with torch.cuda.stream(st):
                step()  # warm, outside the capture
            st.synchronize()
            tok.zero_(); D.zero_(); ctr.zero_()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=st):
                step()
            for _ in range(12):
                gr.replay()
        else:
            with torch.cuda.stream(st):
                for _ in range(12):
                    step()
        torch.cuda.synchronize()
        assert int(ctr[0]) == 12 and int(scratch.count_nonzero()) == 0
        outs.append(tok.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert (outs[0][:, 4:13] != 0).all()  # positions 4..12 were chosen
