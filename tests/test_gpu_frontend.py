"""The encoder front end's data movement (kernels/whisper.cu:115-139 im2col1 / im2col2 / add_pos, launched at
src/model.rs:553-559) against the reference's own kernels on the same inputs: equal bit for bit, at the engine's
shapes (the wide-access kernels) and at shapes only the element-wise kernels take."""
import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu

NFR, TENC = 3000, 1500


def _ref1(ref, name, n, args):
    ref.launch(name, ((n + 255) // 256,), 256, args)


@pytest.mark.parametrize("groups,nm", [(2, 128), (1, 80), (3, 81)])
def test_im2col1_matches_reference(cuda, ref, groups, nm):
    import mimizuku_b200 as m
    torch = cuda
    rng = np.random.default_rng(groups * 1000 + nm)
    mel = torch.from_numpy(O.normal16(rng, (groups, nm, NFR))).cuda()
    n = groups * NFR * 3 * nm
    X = torch.full((n,), 9.0, dtype=torch.float16, device="cuda")
    Xr = torch.full((n,), 9.0, dtype=torch.float16, device="cuda")
    m.im2col1(mel, X, nm)
    _ref1(ref, "im2col1", n, [("p", mel.data_ptr()), ("p", Xr.data_ptr()), ("l", n), ("i", nm)])
    torch.cuda.synchronize()
    assert m.status()[0] == 0
    assert torch.equal(X.view(torch.int16), Xr.view(torch.int16))


@pytest.mark.parametrize("groups,d", [(2, 1280), (1, 384), (1, 36)])
def test_im2col2_matches_reference(cuda, ref, groups, d):
    import mimizuku_b200 as m
    torch = cuda
    rng = np.random.default_rng(groups * 100 + d)
    h1 = torch.from_numpy(O.normal16(rng, (groups, NFR, d))).cuda()
    n = groups * TENC * 3 * d
    X = torch.full((n,), 9.0, dtype=torch.float16, device="cuda")
    Xr = torch.full((n,), 9.0, dtype=torch.float16, device="cuda")
    m.im2col2(h1, X, d)
    _ref1(ref, "im2col2", n, [("p", h1.data_ptr()), ("p", Xr.data_ptr()), ("l", n), ("i", d)])
    torch.cuda.synchronize()
    assert m.status()[0] == 0
    assert torch.equal(X.view(torch.int16), Xr.view(torch.int16))


@pytest.mark.parametrize("rows,n,period", [(2 * TENC, 1280, TENC), (TENC, 384, TENC), (301, 37, 100)])
def test_add_pos_matches_reference(cuda, ref, rows, n, period):
    import mimizuku_b200 as m
    torch = cuda
    rng = np.random.default_rng(rows + n)
    x = O.normal16(rng, (rows, n), 4.0)
    pos = O.normal16(rng, (period, n), 1.0)
    P = torch.from_numpy(pos).cuda()
    X = torch.from_numpy(x).cuda()
    Xr = torch.from_numpy(x).cuda()
    m.add_pos(X, P, period)
    _ref1(ref, "add_pos", rows * n, [("p", Xr.data_ptr()), ("p", P.data_ptr()), ("l", rows), ("i", n),
                                     ("i", period)])
    torch.cuda.synchronize()
    assert m.status()[0] == 0
    assert torch.equal(X.view(torch.int16), Xr.view(torch.int16))
