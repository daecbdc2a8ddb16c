"""Decoder linear layers on the tensor cores (mmz_dec_linear) against an exact (float64) product: every output within
one fp16 rounding step of the correctly rounded value plus the fp32 accumulation error bound (which only shows where
the sum cancels), GELU applied after the fp16 rounding as the reference's separate gelu_inplace kernel does
(kernels/whisper.cu:107-112)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ulp(v):
    import torch
    return torch.clamp(v.abs(), min=2.0 ** -14) * 2.0 ** -10  # one fp16 step at |v|


def _gelu(v):
    import torch
    return 0.5 * v * (1.0 + torch.erf(v * 0.70710678118654752))


def _ref(x, w, b, gelu):
    """The correctly rounded output and its error bound: one fp16 step at the pre-activation plus the fp32
    accumulation error (which only shows where the sum cancels), carried through GELU's slope."""
    import math
    import torch
    pre = (x.double() @ w.double().T + b.double()).half().float()  # rh(acc + b) with an exact acc
    bound = _ulp(pre) * 1.01 + 2e-6 * (x.float().abs() @ w.float().abs().T + b.float().abs())
    if not gelu:
        return pre, bound
    y = _gelu(pre).half().float()
    slope = 0.5 * (1.0 + torch.erf(pre * 0.70710678118654752)) + pre * torch.exp(-0.5 * pre * pre) / math.sqrt(
        2 * math.pi)
    return y, _ulp(y) * 1.01 + (slope.abs() + 0.01) * bound


@pytest.mark.parametrize("m,n,k,gelu,ldx_pad", [
    (32, 1280, 1280, False, 0), (32, 3840, 1280, False, 0), (32, 5120, 1280, True, 0), (32, 1280, 5120, False, 0),
    (7, 1000, 640, False, 64), (1, 333, 64, True, 0), (32, 51866, 1280, False, 0), (20, 1280, 1280, False, 0),
    (32, 51866, 1280, None, 0),
])
def test_dec_linear_matches_exact_product(cuda, m, n, k, gelu, ldx_pad):
    import torch
    import mimizuku_b200 as mm
    g = torch.Generator(device="cuda").manual_seed(m * 1000 + n)
    xs = torch.randn(m, k + ldx_pad, device="cuda", generator=g).half()
    x = xs[:, :k]
    w = (torch.randn(n, k, device="cuda", generator=g) * (1.0 / k ** 0.5)).half()
    b = (torch.randn(n, device="cuda", generator=g) * 0.1).half()
    if gelu is None:  # no bias (the logits product)
        gelu, b = False, None
        bz = torch.zeros(n, device="cuda", dtype=torch.float16)
    y = torch.full((m, n), 7.0, device="cuda", dtype=torch.float16)
    mm.dec_linear(x, w, b, y, gelu=gelu)
    torch.cuda.synchronize()
    assert mm.status()[0] == 0
    if b is None:
        b = bz
    ref, bound = _ref(x, w, b, gelu)
    got = y.float()
    err = (got - ref).abs()
    assert torch.all(err <= bound), float((err / bound).max())
    assert (err <= _ulp(ref) * 1.01).float().mean().item() > (0.995 if gelu else 0.999)
    # agreement with cuBLAS (fp32 accumulation in another order): nearly every element identical
    cub = (x.float() @ w.float().T + b.float()).half().float()
    if gelu:
        cub = _gelu(cub).half().float()
    assert (cub == got).float().mean().item() > 0.98
