"""Parity of the sm_100a kernels, called through the C-ABI, with the CPU oracle and with the reference's own kernels
(kernels/whisper.cu compiled from source, launched with src/model.rs's geometry) on identical seeded inputs.

Bars (from the project's north star): attention outputs and alignment-head probabilities within 2e-3 max-abs of the
exact (f64) oracle and no worse than the reference kernel; layer norm bit-identical to the reference kernel."""
import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3          # max-abs bar against the exact oracle
ULP_SLACK = 1e-4    # "no worse than the reference" allows this much on top of the reference's own error


def dev(a, torch):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def f16(t):
    return host(t).astype(np.float32)


# ------------------------------------------------------------------ layer norm

@pytest.mark.parametrize("rows,dim", [(1, 384), (3, 1280), (32, 1280), (12000, 1280), (7, 512), (5, 768),
                                      (2049, 384), (1030, 640), (1100, 1278)])
def test_layernorm_matches_reference_bit_for_bit(cuda, ref, rows, dim):
    import mimizuku_b200 as m
    torch = cuda
    rng = np.random.default_rng(rows * 131 + dim)
    x = O.normal16(rng, (rows, dim), 3.0)
    dx = O.normal16(rng, (rows, dim), 1.0)
    w = O.normal16(rng, (dim,), 0.2) + np.float16(1)
    b = O.normal16(rng, (dim,), 0.1)
    W, Bb = dev(w, torch), dev(b, torch)
    # plain layer norm
    X = dev(x, torch)
    Y = torch.empty_like(X)
    m.layernorm(X, W, Bb, Y)
    Yr = torch.empty_like(X)
    ref.launch("layernorm", (rows,), 128, [("p", X.data_ptr()), ("p", W.data_ptr()), ("p", Bb.data_ptr()),
                                           ("p", Yr.data_ptr()), ("i", dim), ("f", 1e-5)])
    torch.cuda.synchronize()
    assert np.array_equal(host(Y).view(np.uint16), host(Yr).view(np.uint16))
    yo = O.layernorm(x, w, b)
    assert np.max(np.abs(f16(Y) - yo.astype(np.float32))) <= 2 ** -8 * max(1.0, np.abs(yo).max())
    # residual add fused with layer norm, output written over the addend (model.rs:607)
    X1, X2 = dev(x, torch), dev(x, torch)
    D1, D2 = dev(dx, torch), dev(dx, torch)
    m.add_layernorm(X1, D1, W, Bb, D1)
    ref.launch("add_layernorm", (rows,), 128, [("p", X2.data_ptr()), ("p", D2.data_ptr()), ("p", W.data_ptr()),
                                               ("p", Bb.data_ptr()), ("p", D2.data_ptr()), ("i", dim), ("f", 1e-5)])
    torch.cuda.synchronize()
    assert np.array_equal(host(X1).view(np.uint16), host(X2).view(np.uint16))
    assert np.array_equal(host(D1).view(np.uint16), host(D2).view(np.uint16))
    xo, yo = O.add_layernorm(x, dx, w, b)
    assert np.array_equal(host(X1).view(np.uint16), xo.view(np.uint16))


# ------------------------------------------------------------------ cross-attention

def _cross_inputs(B, d, nl, na_heads, seed):
    rng = np.random.default_rng(seed)
    nh = d // 64
    q = O.normal16(rng, (B, d))
    kv = O.normal16(rng, (B, nl, 2, nh, 1500, 64))
    aslot = -np.ones(nl * nh, np.int32)
    slots = rng.choice(nl * nh, size=min(na_heads, nl * nh), replace=False)
    for s, idx in enumerate(sorted(slots.tolist())):
        aslot[idx] = s
    return q, kv, aslot


def _ref_cross(ref, torch, Q, KV, ALN, ASL, CTR, DONE, B, layer, nl, d, na, max_t):
    nh = d // 64
    S = torch.zeros(B * nh * 1500, dtype=torch.float32, device="cuda")
    ST = torch.zeros(B * nh * 24 * 2, dtype=torch.float32, device="cuda")
    PT = torch.zeros(B * nh * 24 * 64, dtype=torch.float32, device="cuda")
    OUT = torch.zeros(B, d, dtype=torch.float16, device="cuda")
    ref.launch("cross_scores", (B * nh, 24), 128, [("p", Q.data_ptr()), ("p", KV.data_ptr()), ("p", S.data_ptr()),
                                                   ("p", ST.data_ptr()), ("p", DONE.data_ptr()), ("i", layer),
                                                   ("i", nl), ("i", d)])
    ref.launch("cross_pv", (B * nh, 24), 128, [("p", S.data_ptr()), ("p", ST.data_ptr()), ("p", KV.data_ptr()),
                                               ("p", PT.data_ptr()), ("p", ALN.data_ptr()), ("p", ASL.data_ptr()),
                                               ("p", CTR.data_ptr()), ("p", DONE.data_ptr()), ("i", layer), ("i", nl),
                                               ("i", d), ("i", na), ("i", max_t)])
    ref.launch("cross_combine", (B * nh,), 64, [("p", PT.data_ptr()), ("p", OUT.data_ptr()), ("p", DONE.data_ptr()),
                                                ("i", d)])
    return OUT


@pytest.mark.parametrize("B,d,nl,layer,p", [(1, 384, 2, 1, 4), (3, 384, 1, 0, 0), (32, 1280, 1, 0, 17),
                                            (5, 1280, 2, 1, 447)])
def test_cross_attn(cuda, ref, B, d, nl, layer, p):
    import mimizuku_b200 as m
    torch = cuda
    max_t, nh = 448, d // 64
    q, kv, aslot = _cross_inputs(B, d, nl, 2 * nh if B <= 8 else 4, seed=B * 7 + d + p)
    na = int((aslot >= 0).sum())
    done = np.zeros(B, np.int32)
    if B > 2:
        done[1] = 1
    Q, KV, ASL, DONE = dev(q, torch), dev(kv, torch), dev(aslot, torch), dev(done, torch)
    CTR = dev(np.array([p, 0, 0, 0], np.int32), torch)
    ALN = torch.zeros(B, max_t, na, 1500, dtype=torch.float16, device="cuda")
    ALNr = torch.zeros_like(ALN)
    OUT = torch.zeros(B, d, dtype=torch.float16, device="cuda")
    scratch = torch.zeros(m.cross_attn_scratch_bytes(B, d), dtype=torch.uint8, device="cuda")
    for _ in range(2):  # twice: the scratch must be reusable without clearing
        m.cross_attn(Q, KV, OUT, ALN, ASL, CTR, DONE, layer, nl, d, na, max_t, scratch)
    OUTr = _ref_cross(ref, torch, Q, KV, ALNr, ASL, CTR, DONE, B, layer, nl, d, na, max_t)
    torch.cuda.synchronize()
    assert m.status()[0] == 0
    out, outr = f16(OUT), f16(OUTr)
    aln, alnr = f16(ALN), f16(ALNr)
    exact, probs = O.cross_attn_f64(q, kv, done, layer, nl, d)
    live = done == 0
    err = np.abs(out[live] - exact[live]).max()
    err_r = np.abs(outr[live] - exact[live]).max()
    assert err <= TOL and err <= err_r + ULP_SLACK, (err, err_r)
    # alignment probabilities: every recorded head of every live sequence at position p
    for hh in range(nh):
        s = aslot[layer * nh + hh]
        if s < 0:
            continue
        a = aln[live, p, s]
        ex = probs[live, hh]
        assert np.abs(a - ex).max() <= TOL
        assert np.abs(a - ex).max() <= np.abs(alnr[live, p, s] - ex).max() + ULP_SLACK
    # nothing written for finished sequences or other positions
    assert np.all(aln[~live] == 0) and np.all(np.delete(aln, p, axis=1) == 0)
    # the rounding oracle restates the reference's arithmetic: outputs agree to fp16 ulps
    oo, ao = O.cross_attn(q, kv, np.zeros((B, max_t, na, 1500), np.float16), aslot, p, done, layer, nl, d, na, max_t)
    assert np.abs(out[live] - oo.astype(np.float32)[live]).max() <= 2 ** -9
    # and the reference kernel's probabilities agree with ours nearly everywhere bit for bit
    same = np.mean(host(ALN).view(np.uint16) == host(ALNr).view(np.uint16))
    assert same > 0.999, same


def test_cross_attn_scratch_shared_by_different_batches(cuda):
    """One scratch buffer serves launches of different batch sizes (the engine's buffer is sized for its largest
    batch): a small launch after a large one must not see the large launch's scores where its counters are."""
    import mimizuku_b200 as m
    torch = cuda
    d, nl, layer, max_t, nh = 1280, 1, 0, 448, 20
    scratch = torch.zeros(m.cross_attn_scratch_bytes(12, d), dtype=torch.uint8, device="cuda")
    for B, seed in [(12, 1), (3, 2), (12, 3), (5, 4)]:
        q, kv, aslot = _cross_inputs(B, d, nl, 4, seed=seed)
        na = int((aslot >= 0).sum())
        done = np.zeros(B, np.int32)
        Q, KV, ASL, DONE = dev(q, torch), dev(kv, torch), dev(aslot, torch), dev(done, torch)
        CTR = dev(np.array([9, 0, 0, 0], np.int32), torch)
        ALN = torch.zeros(B, max_t, na, 1500, dtype=torch.float16, device="cuda")
        OUT = torch.zeros(B, d, dtype=torch.float16, device="cuda")
        m.cross_attn(Q, KV, OUT, ALN, ASL, CTR, DONE, layer, nl, d, na, max_t, scratch)
        torch.cuda.synchronize()
        assert m.status()[0] == 0
        oo, _ = O.cross_attn(q, kv, np.zeros((B, max_t, na, 1500), np.float16), aslot, 9, done, layer, nl, d, na,
                             max_t)
        assert np.abs(f16(OUT) - oo.astype(np.float32)).max() <= 2 ** -9, B


# ------------------------------------------------------------------ self-attention (kv_write folded in)

@pytest.mark.parametrize("B,d,p", [(1, 384, 0), (3, 384, 1), (3, 384, 62), (2, 1280, 64), (4, 1280, 127),
                                   (4, 1280, 128), (1, 1280, 199), (3, 384, 446), (32, 1280, 447)])
def test_self_attn(cuda, ref, B, d, p):
    import mimizuku_b200 as m
    torch = cuda
    max_t = 448
    rng = np.random.default_rng(B * 1000 + p)
    qkv = O.normal16(rng, (B, 3 * d))
    kc = O.normal16(rng, (B, max_t, d))
    vc = O.normal16(rng, (B, max_t, d))
    done = np.zeros(B, np.int32)
    if B > 2:
        done[2] = 1
    QKV, DONE = dev(qkv, torch), dev(done, torch)
    CTR = dev(np.array([p, 0, 0, 0], np.int32), torch)
    KC, VC, KCr, VCr = dev(kc, torch), dev(vc, torch), dev(kc, torch), dev(vc, torch)
    OUT = torch.zeros(B, d, dtype=torch.float16, device="cuda")
    OUTr = torch.zeros_like(OUT)
    m.self_attn(QKV, KC, VC, OUT, CTR, DONE, max_t, d)
    ref.launch("kv_write", (B,), 256, [("p", QKV.data_ptr()), ("p", KCr.data_ptr()), ("p", VCr.data_ptr()),
                                       ("p", CTR.data_ptr()), ("i", max_t), ("i", d)])
    ref.launch("self_attn", (B, d // 64), 128, [("p", QKV.data_ptr()), ("p", KCr.data_ptr()), ("p", VCr.data_ptr()),
                                                ("p", OUTr.data_ptr()), ("p", CTR.data_ptr()), ("p", DONE.data_ptr()),
                                                ("i", max_t), ("i", d)])
    torch.cuda.synchronize()
    assert m.status()[0] == 0
    # the caches hold the same rows afterwards (the reference writes every sequence's row p)
    assert np.array_equal(host(KC).view(np.uint16), host(KCr).view(np.uint16))
    assert np.array_equal(host(VC).view(np.uint16), host(VCr).view(np.uint16))
    live = done == 0
    out, outr = f16(OUT), f16(OUTr)
    # every sum runs in the reference's order: the outputs are the reference kernel's bit for bit
    assert np.array_equal(host(OUT).view(np.uint16)[live], host(OUTr).view(np.uint16)[live])
    exact = O.self_attn_f64(qkv, kc, vc, p, done, max_t, d)
    err = np.abs(out[live] - exact[live]).max()
    err_r = np.abs(outr[live] - exact[live]).max()
    assert err <= TOL and err <= err_r + ULP_SLACK, (err, err_r)
    oo, _, _ = O.self_attn(qkv, kc, vc, p, done, max_t, d)
    assert np.abs(out[live] - oo.astype(np.float32)[live]).max() <= 2 ** -9
    assert np.all(out[~live] == 0)


def test_kv_write_alone(cuda, ref):
    import mimizuku_b200 as m
    torch = cuda
    B, d, max_t, p = 3, 384, 448, 9
    rng = np.random.default_rng(5)
    qkv = O.normal16(rng, (B, 3 * d))
    QKV, CTR = dev(qkv, torch), dev(np.array([p, 0, 0, 0], np.int32), torch)
    KC = torch.zeros(B, max_t, d, dtype=torch.float16, device="cuda")
    VC = torch.zeros_like(KC)
    m.kv_write(QKV, KC, VC, CTR, max_t, d, B)
    torch.cuda.synchronize()
    kc = host(KC)
    assert np.array_equal(kc[:, p], qkv[:, d:2 * d]) and np.array_equal(host(VC)[:, p], qkv[:, 2 * d:])
    assert np.all(np.delete(kc, p, axis=1) == 0)


# ------------------------------------------------------------------ encoder attention (tcgen05)

def _ref_enc(ref, torch, QKV, g, d):
    OUT = torch.zeros(g, 1500, d, dtype=torch.float16, device="cuda")
    ref.launch("enc_flash", (24, d // 64, g), 128, [("p", QKV.data_ptr()), ("p", OUT.data_ptr()), ("i", d)])
    return OUT


@pytest.mark.parametrize("g,d,scale,rows", [(1, 384, 0.125, None), (1, 384, 1.0, None), (8, 1280, 1.0, (0, 96)),
                                            (8, 1280, 1.0, (1404, 96))])
def test_enc_flash(cuda, ref, g, d, scale, rows):
    import mimizuku_b200 as m
    torch = cuda
    rng = np.random.default_rng(g * 31 + d)
    qkv = O.normal16(rng, (g, 1500, 3 * d), scale)
    QKV = dev(qkv, torch)
    OUT = torch.zeros(g, 1500, d, dtype=torch.float16, device="cuda")
    m.enc_flash(QKV, OUT, d)
    OUTr = _ref_enc(ref, torch, QKV, g, d)
    torch.cuda.synchronize()
    assert m.status()[0] == 0
    r0, nr = rows if rows else (0, 1500)
    exact = O.enc_attn_f64(qkv, d, r0, nr)[:, r0:r0 + nr]
    out = f16(OUT)[:, r0:r0 + nr]
    outr = f16(OUTr)[:, r0:r0 + nr]
    err = np.abs(out - exact).max()
    err_r = np.abs(outr - exact).max()
    assert err <= TOL and err <= err_r + ULP_SLACK, (err, err_r)
    # every row of every clip and head is written (rows past the checked window included)
    assert np.isfinite(f16(OUT)).all() and (np.abs(f16(OUT)).sum(axis=2) > 0).all()


def test_enc_flash_graph_and_repeat(cuda):
    """Two launches give identical results, also when replayed from a CUDA graph."""
    import mimizuku_b200 as m
    torch = cuda
    g, d = 2, 512
    qkv = O.normal16(np.random.default_rng(3), (g, 1500, 3 * d))
    QKV = dev(qkv, torch)
    A = torch.zeros(g, 1500, d, dtype=torch.float16, device="cuda")
    Bt = torch.zeros_like(A)
    C = torch.zeros_like(A)
    m.enc_flash(QKV, A, d)
    m.enc_flash(QKV, Bt, d)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s):
            m.enc_flash(QKV, C, d, stream=s)
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(A, Bt) and torch.equal(A, C)
