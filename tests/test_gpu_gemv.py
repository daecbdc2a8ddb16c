"""The decoder's linear layers at m <= 8 sequences: this library's gemv (mmz_gemv, and the name-compatible gemv_1/2/4/8
of the drop-in image) against the reference's gemv kernels (kernels/whisper.cu:501-567) launched as src/gpu.rs:211-228
launches them, on the same inputs: equal bit for bit, at every decoder shape of tiny and large-v3 (the logits
included), at ragged n, padded rows and without a bias."""
import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu

# (n, k): qkv, o / xq / xo, fc1, fc2, logits of tiny (d 384) and large-v3 (d 1280); then ragged and short shapes
SHAPES = [(1152, 384), (384, 384), (1536, 384), (384, 1536), (51865, 384),
          (3840, 1280), (1280, 1280), (5120, 1280), (1280, 5120), (51866, 1280),
          (37, 264), (33, 8), (100, 2056), (40, 16384)]


def _ref_geometry(m):
    """(name, mr, kc) of src/gpu.rs:213-218."""
    if m == 1:
        return "gemv_1", 1, 2048
    if m == 2:
        return "gemv_2", 2, 2048
    if m <= 4:
        return "gemv_4", 4, 1024
    return "gemv_8", 8, 1024


def _launch_by_name(k, m, n, kk, X, ldx, W, Y, ldy, B):
    name, mr, kc = _ref_geometry(m)
    k.launch(name, ((n + 31) // 32,), 256,
             [("p", X.data_ptr()), ("i", ldx), ("p", W.data_ptr()), ("p", Y.data_ptr()), ("i", ldy), ("i", m),
              ("i", n), ("i", kk), ("p", B.data_ptr() if B is not None else 0)], smem=mr * kc * 2)


def _weights(torch, n, k, seed):
    rng = np.random.default_rng(seed)
    w = O.normal16(rng, (n, k), 0.05)
    b = O.normal16(rng, (n,), 0.2)
    return torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda()


def _rows(torch, m, ldx, seed):
    return torch.from_numpy(O.normal16(np.random.default_rng(seed), (m, ldx), 1.0)).cuda()


@pytest.fixture(scope="module")
def dropin(cuda):
    import mimizuku_b200 as m
    return O.RefKernels(m.DROPIN_FATBIN)


@pytest.fixture(params=["chosen", "rows"])
def form(request, monkeypatch):
    """The library's own choice (the shared-memory ring for every large-model shape, the register form with two
    CTAs per SM for the tiny vocabulary's k = 384 rows) and the register form with one CTA per SM, which the library
    falls back to when x and two 256-value stages per warp do not fit a CTA's shared memory (m k > 99 328:
    (40, 16384) at m >= 7 takes it without the hook)."""
    if request.param == "rows":
        monkeypatch.setenv("MMZ_TEST_GEMV_ROWS", "1")
    return request.param


@pytest.mark.parametrize("n,k", SHAPES)
def test_gemv_matches_reference(cuda, ref, form, n, k):
    import mimizuku_b200 as mm
    torch = cuda
    W, B = _weights(torch, n, k, n * 10 + k)
    for m in range(1, 9):
        X = _rows(torch, m, k, m)
        bias = B if n != 51865 and n != 51866 else None  # the logits have no bias
        Y = torch.full((m, n), 7.0, dtype=torch.float16, device="cuda")
        Yr = torch.full((m, n), 7.0, dtype=torch.float16, device="cuda")
        mm.gemv(X, W, bias, Y)
        _launch_by_name(ref, m, n, k, X, k, W, Yr, n, bias)
        torch.cuda.synchronize()
        assert mm.status()[0] == 0
        assert torch.equal(Y.view(torch.int16), Yr.view(torch.int16)), (m, n, k)


@pytest.mark.parametrize("m", [1, 3, 8])
def test_gemv_padded_rows_and_no_bias(cuda, ref, form, m):
    """x rows wider than k, y rows wider than n (the engine's [sequence][3d] buffers), no bias: the padding of y is
    left alone."""
    import mimizuku_b200 as mm
    torch = cuda
    n, k, ldx, ldy = 1152, 384, 1152, 1160
    W, _ = _weights(torch, n, k, 5)
    X = _rows(torch, m, ldx, m)
    Y = torch.full((m, ldy), 7.0, dtype=torch.float16, device="cuda")
    Yr = torch.full((m, ldy), 7.0, dtype=torch.float16, device="cuda")
    mm.gemv(X, W, None, Y[:, :n])
    _launch_by_name(ref, m, n, k, X, ldx, W, Yr, ldy, None)
    torch.cuda.synchronize()
    assert mm.status()[0] == 0
    assert torch.equal(Y.view(torch.int16), Yr.view(torch.int16))
    assert (Y[:, n:] == 7.0).all()
    exact = X[:, :k].double() @ W.double().T
    assert torch.allclose(Y.double(), torch.cat([exact, Y[:, n:].double()], 1), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("n,k", [(1280, 5120), (51866, 1280), (37, 264)])
def test_gemv_by_name_matches_reference(cuda, ref, dropin, n, k):
    """gemv_1/2/4/8 of the drop-in image, launched by name with the reference's geometry and shared memory."""
    torch = cuda
    W, B = _weights(torch, n, k, n + k)
    for m in (1, 2, 3, 4, 5, 8):
        X = _rows(torch, m, k, m)
        outs = []
        for kern in (dropin, ref):
            Y = torch.full((m, n), 7.0, dtype=torch.float16, device="cuda")
            _launch_by_name(kern, m, n, k, X, k, W, Y, n, B)
            outs.append(Y)
        torch.cuda.synchronize()
        assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16)), (m, n, k)


@pytest.mark.parametrize("n,k", [(5120, 1280), (1536, 384), (1000, 264)])
def test_gemv_gelu_matches_reference_gemv_then_gelu(cuda, ref, form, n, k):
    """The decoder's fc1 product and its GELU in one launch (mmz_gemv_gelu) against the reference's gemv kernel
    followed by its gelu_inplace over the b x ff values (src/model.rs:708-709): equal bit for bit."""
    import mimizuku_b200 as mm
    torch = cuda
    W, B = _weights(torch, n, k, n + 3 * k)
    for m in (1, 2, 3, 5, 8):
        X = _rows(torch, m, k, 10 + m)
        Y = torch.full((m, n), 7.0, dtype=torch.float16, device="cuda")
        Yr = torch.full((m, n), 7.0, dtype=torch.float16, device="cuda")
        mm.gemv(X, W, B, Y, gelu=True)
        _launch_by_name(ref, m, n, k, X, k, W, Yr, n, B)
        n2 = m * n // 2
        ref.launch("gelu_inplace", ((n2 + 255) // 256,), 256, [("p", Yr.data_ptr()), ("l", n2)])
        torch.cuda.synchronize()
        assert mm.status()[0] == 0
        assert torch.equal(Y.view(torch.int16), Yr.view(torch.int16)), (m, n, k)
