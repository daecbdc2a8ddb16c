"""The name-compatible image (mimizuku_b200/dropin_sm100a.fatbin): layernorm, add_layernorm and kv_write under the
reference's names and argument lists, launched by name with src/model.rs's geometry (rows x 128 threads; B x 256), as
the reference's gpu.rs would launch them, against the reference's own kernels: equal bit for bit."""
import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dropin(cuda):
    import mimizuku_b200 as m
    return O.RefKernels(m.DROPIN_FATBIN)


@pytest.mark.parametrize("rows,dim", [(1, 384), (32, 1280), (12000, 1280), (7, 512), (5, 768), (3, 1278)])
def test_layernorm_by_name(cuda, ref, dropin, rows, dim):
    torch = cuda
    rng = np.random.default_rng(rows + dim)
    x = O.normal16(rng, (rows, dim), 3.0)
    dx = O.normal16(rng, (rows, dim), 1.0)
    w = O.normal16(rng, (dim,), 0.2) + np.float16(1)
    b = O.normal16(rng, (dim,), 0.1)
    W, Bb = torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda()
    outs = []
    for k in (dropin, ref):
        X = torch.from_numpy(x).cuda()
        Y = torch.empty_like(X)
        k.launch("layernorm", (rows,), 128, [("p", X.data_ptr()), ("p", W.data_ptr()), ("p", Bb.data_ptr()),
                                             ("p", Y.data_ptr()), ("i", dim), ("f", 1e-5)])
        X2 = torch.from_numpy(x).cuda()
        D2 = torch.from_numpy(dx).cuda()
        k.launch("add_layernorm", (rows,), 128, [("p", X2.data_ptr()), ("p", D2.data_ptr()), ("p", W.data_ptr()),
                                                 ("p", Bb.data_ptr()), ("p", D2.data_ptr()), ("i", dim), ("f", 1e-5)])
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy().view(np.uint16) for t in (Y, X2, D2)])
    for a, r in zip(*outs):
        assert np.array_equal(a, r)


@pytest.mark.parametrize("B,d,p", [(32, 1280, 0), (5, 384, 447), (3, 36, 9)])
def test_kv_write_by_name(cuda, ref, dropin, B, d, p):
    torch = cuda
    rng = np.random.default_rng(B * d + p)
    mt = 448
    qkv = torch.from_numpy(O.normal16(rng, (B, 3 * d))).cuda()
    ctr = torch.tensor([p, 0, 0, 0], dtype=torch.int32, device="cuda")
    res = []
    for k in (dropin, ref):
        kc = torch.zeros(B, mt, d, dtype=torch.float16, device="cuda")
        vc = torch.zeros(B, mt, d, dtype=torch.float16, device="cuda")
        k.launch("kv_write", (B,), 256, [("p", qkv.data_ptr()), ("p", kc.data_ptr()), ("p", vc.data_ptr()),
                                         ("p", ctr.data_ptr()), ("i", mt), ("i", d)])
        torch.cuda.synchronize()
        res.append((kc.cpu().numpy().view(np.uint16), vc.cpu().numpy().view(np.uint16)))
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][1], res[1][1])
    assert np.array_equal(res[0][0][:, p], qkv.cpu().numpy()[:, d:2 * d].view(np.uint16))
