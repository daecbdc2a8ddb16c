"""Failure detection on the GPU without faulting it: a kernel waits on a barrier nothing arrives on; its bounded waits
give up after the limit, the device status word records (timeout, kernel, site), and the context keeps working."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ST_TIMEOUT, K_SELFTEST = 1, 6


def test_bounded_wait_reports_and_context_survives(cuda):
    import torch
    import mimizuku_b200 as m
    assert m.status()[0] == 0
    t0 = time.perf_counter()
    code = m.selftest_wait(200)
    dt = time.perf_counter() - t0
    assert code[0] == ST_TIMEOUT and code[1] == K_SELFTEST and code[2] in (1, 2), code
    assert 0.15 < dt < 5.0
    assert m.status() == (0, 0, 0)  # read and cleared
    # the context is usable: a layernorm right after matches a float64 restatement to fp16 rounding
    x = torch.randn(4, 384, device="cuda").half()
    w = torch.ones(384, device="cuda").half()
    b = torch.zeros(384, device="cuda").half()
    out = torch.empty_like(x)
    m.layernorm(x, w, b, out, 1e-5)
    torch.cuda.synchronize()
    xd = x.double()
    ref = ((xd - xd.mean(1, keepdim=True)) / torch.sqrt(xd.var(1, unbiased=False, keepdim=True) + 1e-5)).float()
    assert float((out.float() - ref).abs().max()) < 4e-3
    assert m.status() == (0, 0, 0)
