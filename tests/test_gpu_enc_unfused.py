"""The unfused encoder attention (src/model.rs:567-604, --enc-attn cublas): this library's row softmax against the f64
softmax and the reference's softmax_rows kernel (kernels/whisper.cu:141-166), and the engine in that mode against the
reference-kernel engine in the same mode and against the fused encoder kernel."""
import numpy as np
import pytest

import _oracle as O
from test_gpu_engine import _clips, _lockstep

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,n,scale", [(20 * 1500, 1500, 1.0), (300, 2048, 4.0), (37, 1024, 0.1), (1, 7, 1.0),
                                          (64, 1500, 30.0)])
def test_softmax_rows(cuda, ref, rows, n, scale):
    import mimizuku_b200 as m
    torch = cuda
    rng = np.random.default_rng(rows + n)
    s = O.normal16(rng, (rows, n), scale)
    if rows > 2:
        s[1, ::3] = -np.inf  # masked entries
    S = torch.from_numpy(s).cuda()
    m.softmax_rows(S)
    R = torch.from_numpy(s).cuda()
    ref.launch("softmax_rows", (rows,), 256, [("p", R.data_ptr()), ("i", n)])
    torch.cuda.synchronize()
    out = S.cpu().numpy().astype(np.float64)
    outr = R.cpu().numpy().astype(np.float64)
    x = s.astype(np.float64)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    exact = e / e.sum(axis=1, keepdims=True)
    ulp = np.maximum(np.abs(exact), 2.0 ** -14) * 2.0 ** -10  # one fp16 unit (subnormals: the smallest normal's)
    assert np.all(np.abs(out - exact) <= ulp), np.abs(out - exact).max()
    assert np.abs(out - exact).max() <= np.abs(outr - exact).max() + 2.0 ** -11
    assert np.all(np.abs(out - outr) <= ulp)  # the reference kernel's, to the last fp16 bit


def test_engine_unfused_encoder_against_reference_and_fused(cuda, ref):
    """The engine's --enc-attn cublas mode: cross k/v within fp16 noise of the reference-kernel engine in the same mode
    and of the fused encoder kernel; greedy tokens in lockstep with the reference engine (near-ties only)."""
    import mimizuku_b200 as m
    torch = cuda
    cfg = m.TINY
    b = 3
    mel, frames = _clips(b, cfg.n_mels, seed=5)
    sup = [cfg.eos]
    nat = m.Engine(cfg, bmax=b, eg=2, seed=11, suppress=sup)
    fused = m.Engine(cfg, bmax=b, eg=2, seed=11, suppress=sup)
    refe = m.Engine(cfg, bmax=b, eg=2, seed=11, suppress=sup, kernel_image=O.REF_FATBIN)
    nat.enc_attn = "cublas"
    refe.enc_attn = "cublas"
    assert nat.enc_attn == "cublas" and fused.enc_attn == "flash"
    mel16 = torch.from_numpy(mel.astype(np.float16)).cuda()
    for e in (nat, fused, refe):
        e.encode(mel16[:2].data_ptr(), 2, 0)
        e.encode(mel16[2:].data_ptr(), 1, 2)
        e.sync()
    n = b * cfg.dec_layers * 2 * cfg.d * 1500
    xkv = {}
    for name, e in (("nat", nat), ("fused", fused), ("ref", refe)):
        a = np.empty(n, np.float16)
        O.d2h(a, e.buffer("xkv"))
        xkv[name] = a.astype(np.float32)
    rel = lambda a, r: float(np.sqrt(((a - r) ** 2).sum() / (r ** 2).sum()))  # noqa: E731
    assert rel(xkv["nat"], xkv["ref"]) < 2e-2, rel(xkv["nat"], xkv["ref"])
    assert rel(xkv["nat"], xkv["fused"]) < 2e-2, rel(xkv["nat"], xkv["fused"])
    diverged, compared = _lockstep(cfg, nat, refe, b, 24)
    assert diverged <= max(1, compared // 20), (diverged, compared)
    assert m.status()[0] == 0
    for e in (nat, fused, refe):
        e.close()
