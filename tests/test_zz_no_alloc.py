"""mmz_cross_attn_noalloc, the cross-attention entry point for callers that cannot allocate device memory (its
scratch is a static device array of the library), called through the C-ABI: two calls in a row must give what
mmz_cross_attn gives with a caller-provided scratch buffer, within the kernel tests' tolerance. This file is collected
last, so a run that stops at the first failure has run every other test before it; it also passes alone."""
import ctypes

import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(torch, B, d, nl, layer, p):
    """Seeded inputs of one cross-attention call (one finished sequence, two alignment heads)."""
    max_t, nh = 448, d // 64
    rng = np.random.default_rng(B + d + p)
    q = torch.from_numpy(O.normal16(rng, (B, d))).cuda()
    kv = torch.from_numpy(O.normal16(rng, (B, nl, 2, nh, 1500, 64))).cuda()
    aslot = -np.ones(nl * nh, np.int32)
    aslot[layer * nh + 1], aslot[layer * nh + nh - 1] = 0, 1
    aslot = torch.from_numpy(aslot).cuda()
    done = torch.zeros(B, dtype=torch.int32, device="cuda")
    done[B // 2] = 1
    ctr = torch.tensor([p, 0, 0, 0], dtype=torch.int32, device="cuda")
    return dict(q=q, kv=kv, aslot=aslot, done=done, ctr=ctr, B=B, d=d, nl=nl, layer=layer, max_t=max_t)


def _call(m, torch, c, noalloc, stream):
    """One call through the C-ABI: the allocation-free entry point, or mmz_cross_attn with a fresh caller scratch."""
    B, d = c["B"], c["d"]
    out = torch.zeros(B, d, dtype=torch.float16, device="cuda")
    al = torch.zeros(B, c["max_t"], 2, 1500, dtype=torch.float16, device="cuda")
    args = (_p(c["q"]), _p(c["kv"]), _p(out), _p(al), _p(c["aslot"]), _p(c["ctr"]), _p(c["done"]), B, c["layer"],
            c["nl"], d, 2, c["max_t"])
    if noalloc:
        rc = m.lib.mmz_cross_attn_noalloc(*args, stream)
    else:
        nbytes = m.cross_attn_scratch_bytes(B, d)
        scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        rc = m.lib.mmz_cross_attn(*args, _p(scratch), nbytes, stream)
    assert rc == 0, m.lib.mmz_last_error()
    return out, al


def test_noalloc_large_then_small_call(cuda):
    """A large call (32 sequences, d 1280) fills most of the shared array; a small call after it on the same stream
    (3 sequences, d 384) still gives what mmz_cross_attn gives with a fresh scratch buffer: no value a call reads is
    left over from the call before."""
    import mimizuku_b200 as m
    torch = cuda
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    big, small = _case(torch, 32, 1280, 1, 0, 11), _case(torch, 3, 384, 2, 1, 447)
    ref_big, ref_small = _call(m, torch, big, False, stream), _call(m, torch, small, False, stream)
    got_big = _call(m, torch, big, True, stream)
    got_small = _call(m, torch, small, True, stream)
    torch.cuda.synchronize()
    assert m.status()[0] == 0
    for got, ref in ((got_big, ref_big), (got_small, ref_small)):
        for a, r in zip(got, ref):
            assert np.abs(a.float().cpu().numpy() - r.float().cpu().numpy()).max() <= 2e-3
            assert torch.equal(a, r)


@pytest.mark.parametrize("B,d,nl,layer,p", [(32, 1280, 1, 0, 11), (3, 384, 2, 1, 447)])
def test_noalloc_matches_the_caller_scratch_entry_point(cuda, B, d, nl, layer, p):
    import mimizuku_b200 as m
    torch = cuda
    max_t, nh = 448, d // 64
    rng = np.random.default_rng(B + d + p)
    q = torch.from_numpy(O.normal16(rng, (B, d))).cuda()
    kv = torch.from_numpy(O.normal16(rng, (B, nl, 2, nh, 1500, 64))).cuda()
    aslot = -np.ones(nl * nh, np.int32)
    aslot[layer * nh + 1], aslot[layer * nh + nh - 1] = 0, 1
    aslot = torch.from_numpy(aslot).cuda()
    done = torch.zeros(B, dtype=torch.int32, device="cuda")
    done[B // 2] = 1
    ctr = torch.tensor([p, 0, 0, 0], dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the existing entry point, with its own scratch
    out_ref = torch.zeros(B, d, dtype=torch.float16, device="cuda")
    al_ref = torch.zeros(B, max_t, 2, 1500, dtype=torch.float16, device="cuda")
    nbytes = m.cross_attn_scratch_bytes(B, d)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    rc = m.lib.mmz_cross_attn(_p(q), _p(kv), _p(out_ref), _p(al_ref), _p(aslot), _p(ctr), _p(done), B, layer, nl, d,
                              2, max_t, _p(scratch), nbytes, stream)
    assert rc == 0, m.lib.mmz_last_error()
    for call in range(2):  # two calls in a row on the shared static scratch
        out = torch.zeros(B, d, dtype=torch.float16, device="cuda")
        al = torch.zeros(B, max_t, 2, 1500, dtype=torch.float16, device="cuda")
        rc = m.lib.mmz_cross_attn_noalloc(_p(q), _p(kv), _p(out), _p(al), _p(aslot), _p(ctr), _p(done), B, layer, nl,
                                          d, 2, max_t, stream)
        assert rc == 0, m.lib.mmz_last_error()
        torch.cuda.synchronize()
        assert m.status()[0] == 0
        a, r = out.float().cpu().numpy(), out_ref.float().cpu().numpy()
        assert np.abs(a - r).max() <= 2e-3, (call, np.abs(a - r).max())
        assert np.abs(al.float().cpu().numpy() - al_ref.float().cpu().numpy()).max() <= 2e-3
        assert torch.equal(out, out_ref) and torch.equal(al, al_ref)  # the same kernels: identical in fact


def test_noalloc_rejects_batches_beyond_its_static_scratch(cuda):
    import mimizuku_b200 as m
    rc = m.lib.mmz_cross_attn_noalloc(None, None, None, None, None, None, None, 33, 0, 1, 1280, 1, 448, None)
    assert rc != 0 and b"static scratch" in m.lib.mmz_last_error()
