"""The token-timestamp cost (src/align.rs:6-43) and the DTW with the start times (src/align.rs:44-106) on the GPU
against the oracle's restatement, bit for bit, for batches of clips with different token and frame counts."""
import numpy as np
import pytest

import _oracle as O

pytestmark = pytest.mark.gpu


def _weights(rng, n, mt, na):
    w = rng.random((n, mt, na, 1500)).astype(np.float16) * np.float16(0.01)
    w[:, :, :, ::17] = 0  # ties and constant columns, as recorded probabilities have
    w[:, :, 0, 5:9] = np.float16(0.25)
    return w


@pytest.mark.parametrize("na,np_,mt,rows,cols", [
    (10, 4, 448, [223, 1, 40, 5], [1500, 750, 2, 4]),
    (2, 3, 64, [60, 7, 3], [1117, 3, 1500]),
    (16, 1, 32, [31, 0, 12], [1500, 1500, 6]),
])
def test_align_cost_is_the_oracle_bit_for_bit(cuda, na, np_, mt, rows, cols):
    import torch
    import mimizuku_b200 as m
    rng = np.random.default_rng(na * 100 + mt)
    n = len(rows)
    w = _weights(rng, n, mt, na)
    dev = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    cost = torch.full((n, mt, 1500), -7.0, dtype=torch.float32, device="cuda")  # untouched where no row exists
    r = torch.tensor(rows, dtype=torch.int32, device="cuda")
    c = torch.tensor(cols, dtype=torch.int32, device="cuda")
    m.align_cost(dev, r, c, np_, mt, na, cost)
    got = cost.cpu().numpy()
    assert m.status()[0] == 0
    for s in range(n):
        if rows[s] == 0:
            assert np.all(got[s] == -7.0)
            continue
        ws = w[s, np_:np_ + rows[s]].astype(np.float32)
        want = O.align_cost(ws, cols[s])
        assert np.array_equal(got[s, :rows[s], :cols[s]].view(np.uint32), want.view(np.uint32)), s
        assert np.all(got[s, rows[s]:] == -7.0)
        t = m.times_from_cost(got[s, :rows[s]], cols[s])
        assert np.array_equal(t.view(np.uint32), O.jump_times(ws, cols[s]).view(np.uint32))


def _dtw_case(rng, n, mt, rows, cols, kind):
    cost = np.full((n, mt, 1500), np.nan, dtype=np.float32)  # never read past a clip's rows and columns
    for s in range(n):
        r, c = rows[s], cols[s]
        if kind == "ties":  # few distinct values: many equal costs, so the tie-breaking decides the path
            v = rng.integers(-2, 3, size=(r, c)).astype(np.float32)
        elif kind == "wide":  # magnitudes far apart: the f32 sums round
            v = (rng.standard_normal((r, c)) * 10.0 ** rng.integers(-6, 7, size=(r, c))).astype(np.float32)
        else:
            v = rng.standard_normal((r, c)).astype(np.float32)
        cost[s, :r, :c] = v
    return cost


@pytest.mark.parametrize("kind,mt,rows,cols", [
    ("normal", 448, [223, 1, 40, 5, 447], [1500, 750, 2, 1, 1500]),
    ("ties", 448, [100, 3, 17, 446], [1500, 1, 333, 1499]),
    ("wide", 64, [63, 2, 31], [1500, 1500, 7]),
    ("normal", 512, [512, 0, 9], [1500, 1500, 0]),
])
def test_dtw_times_is_the_oracle_bit_for_bit(cuda, kind, mt, rows, cols):
    import torch
    import mimizuku_b200 as m
    rng = np.random.default_rng(len(rows) * 1000 + mt + len(kind))
    n = len(rows)
    cost = _dtw_case(rng, n, mt, rows, cols, kind)
    dev = torch.from_numpy(cost).cuda()
    times = torch.full((n, mt), -7.0, dtype=torch.float32, device="cuda")
    r = torch.tensor(rows, dtype=torch.int32, device="cuda")
    c = torch.tensor(cols, dtype=torch.int32, device="cuda")
    m.dtw_times(dev, r, c, mt, times)
    got = times.cpu().numpy()
    assert m.status()[0] == 0
    for s in range(n):
        want = np.zeros(mt, np.float32)
        if rows[s] > 0:
            want[:rows[s]] = O.times_from_cost(cost[s, :rows[s], :max(cols[s], 1)].copy(), cols[s])
        assert np.array_equal(got[s].view(np.uint32), want.view(np.uint32)), (s, rows[s], cols[s])


def test_cost_then_dtw_on_the_gpu_is_jump_times(cuda):
    import torch
    import mimizuku_b200 as m
    rng = np.random.default_rng(7)
    na, np_, mt, rows, cols = 10, 4, 448, [223, 60, 1], [1500, 640, 9]
    n = len(rows)
    w = _weights(rng, n, mt, na)
    dev = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    cost = torch.zeros((n, mt, 1500), dtype=torch.float32, device="cuda")
    times = torch.zeros((n, mt), dtype=torch.float32, device="cuda")
    r = torch.tensor(rows, dtype=torch.int32, device="cuda")
    c = torch.tensor(cols, dtype=torch.int32, device="cuda")
    m.align_cost(dev, r, c, np_, mt, na, cost)
    m.dtw_times(cost, r, c, mt, times)
    got = times.cpu().numpy()
    for s in range(n):
        want = O.jump_times(w[s, np_:np_ + rows[s]].astype(np.float32), cols[s])
        assert np.array_equal(got[s, :rows[s]].view(np.uint32), want.view(np.uint32)), s


def test_dtw_times_rejects_long_clips(cuda):
    import torch
    import mimizuku_b200 as m
    z = torch.zeros((1, 513, 1500), dtype=torch.float32, device="cuda")
    r = torch.ones(1, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError):
        m.dtw_times(z, r, r, 513, torch.zeros((1, 513), dtype=torch.float32, device="cuda"))
