"""The token-timestamp cost on the GPU (src/align.rs:6-43) against the oracle's restatement, bit for bit, for a batch
of clips with different token and frame counts, and the start times through the host DTW."""
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
