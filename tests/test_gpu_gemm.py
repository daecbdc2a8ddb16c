"""The encoder's tensor-core GEMM with fused epilogues (mmz_gemm_bias) against an fp32 torch product of the same fp16
operands: c = rh(a w^T + b), GELU after the rounding (mode 1), and the head-contiguous cross k/v store (mode 2).
Tolerance: the fp32 sums associate differently from torch's, so a value may differ by a few fp16 units."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref(torch, a, w, b, mode):
    y = (a.float() @ w.float().t() + b.float()).half()
    if mode == 1:
        v = y.float()
        y = (0.5 * v * (1.0 + torch.erf(v * 0.70710678118654752))).half()
    return y.float()


def _close(got, want):
    err = (got - want).abs()
    tol = 4e-3 * want.abs() + 2e-3
    return bool((err <= tol).all()), float(err.max())


@pytest.mark.parametrize("impl", ["pair", "single"])
@pytest.mark.parametrize("M,N,K,mode", [(12000, 3840, 1280, 0), (12000, 1280, 1280, 0), (3000, 5120, 1280, 1),
                                        (24000, 1280, 384, 1), (12000, 1280, 5120, 0), (100, 256, 64, 0),
                                        (1500, 10240, 1280, 2), (1500, 2560, 384, 2), (1100, 512, 256, 0),
                                        (300, 768, 128, 1), (13300, 512, 128, 0), (13300, 512, 128, 2),
                                        (600, 512, 64, 0), (200, 256, 1280, 1)])
def test_gemm_bias(cuda, monkeypatch, impl, M, N, K, mode):
    """Both kernels: pairs of CTAs on 256 x 256 tiles (the default where N is a multiple of 256 and M > 128; the last
    row tile of 1100 rows leaves the second CTA of its pair wholly past the rows; K = 64 is one stage per tile; 200
    rows are one row tile) and one CTA per 128-row tile."""
    import mimizuku_b200 as m
    torch = cuda
    if impl == "single":
        monkeypatch.setenv("MMZ_TEST_GEMM_1SM", "1")
    g = torch.Generator(device="cuda").manual_seed(M + N + K + mode)
    a = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).half()
    b = (torch.randn(N, device="cuda", generator=g) * 0.1).half()
    want = _ref(torch, a, w, b, mode)
    if mode == 2:
        rows = max(M, 1500)  # a block holds 1500 rows (the encoder length), more when M is larger
        blk = rows * 64
        c = torch.full((N // 64, rows, 64), 7.0, dtype=torch.float16, device="cuda")
        m.gemm_bias(a, w, b, c, mode=2, blk=blk)
        torch.cuda.synchronize()
        got = c[:, :M, :].permute(1, 0, 2).reshape(M, N).float()
        assert (c[:, M:, :] == 7.0).all()  # nothing written past the rows
    else:
        c = torch.full((M, N), 7.0, dtype=torch.float16, device="cuda")
        m.gemm_bias(a, w, b, c, mode=mode)
        torch.cuda.synchronize()
        got = c.float()
    assert m.status()[0] == 0
    ok, err = _close(got, want)
    assert ok, err


def test_gemm_bias_rejects_bad_shapes(cuda):
    import mimizuku_b200 as m
    torch = cuda
    a = torch.zeros(16, 64, dtype=torch.float16, device="cuda")
    w = torch.zeros(100, 64, dtype=torch.float16, device="cuda")
    c = torch.zeros(16, 100, dtype=torch.float16, device="cuda")
    with pytest.raises(m.MmzError):
        m.gemm_bias(a, w, None, c)  # N not a multiple of 128
