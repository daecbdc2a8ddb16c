"""Generates ref_fixtures.npz: outputs of the reference's own kernels (kernels/whisper.cu, compute_80 build in
oracle/_ref/, launched with src/model.rs's geometry) on small seeded inputs, run on a B200. The inputs are not
stored: they are regenerated from the seeds below with numpy's PCG64, which is stable across machines. The CPU
tests pin the oracle to these outputs (tests/test_golden_ref.py).

    python tests/golden/make_ref_fixtures.py [out.npz]      (needs a GPU and oracle/_ref/whisper_ref.fatbin)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import _oracle as O  # noqa: E402

SEEDS = {"ln": 101, "cross": 202, "self": 303, "enc": 404}


def inputs_ln():
    rng = np.random.default_rng(SEEDS["ln"])
    x = O.normal16(rng, (8, 384), 3.0)
    dx = O.normal16(rng, (8, 384), 1.0)
    w = O.normal16(rng, (384,), 0.2) + np.float16(1)
    b = O.normal16(rng, (384,), 0.1)
    return x, dx, w, b


def inputs_cross():
    rng = np.random.default_rng(SEEDS["cross"])
    B, nl, d = 2, 1, 384
    q = O.normal16(rng, (B, d))
    kv = O.normal16(rng, (B, nl, 2, d // 64, 1500, 64))
    aslot = -np.ones(nl * (d // 64), np.int32)
    aslot[1], aslot[4] = 0, 1
    return q, kv, aslot, dict(B=B, nl=nl, d=d, na=2, p=3, max_t=448, layer=0)


def inputs_self():
    rng = np.random.default_rng(SEEDS["self"])
    B, d, mt = 2, 384, 448
    qkv = O.normal16(rng, (B, 3 * d))
    kc = O.normal16(rng, (B, mt, d))
    vc = O.normal16(rng, (B, mt, d))
    return qkv, kc, vc, dict(B=B, d=d, max_t=mt, p=9)


def inputs_enc():
    rng = np.random.default_rng(SEEDS["enc"])
    return O.normal16(rng, (1, 1500, 3 * 384), 0.125)


ENC_ROWS = np.r_[0:64, 1436:1500]


def main(out_path):
    import torch
    ref = O.RefKernels()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    res = {}
    x, dx, w, b = inputs_ln()
    X, D, W, Bb = dev(x), dev(dx), dev(w), dev(b)
    Y = torch.empty_like(X)
    ref.launch("layernorm", (8,), 128, [("p", X.data_ptr()), ("p", W.data_ptr()), ("p", Bb.data_ptr()),
                                        ("p", Y.data_ptr()), ("i", 384), ("f", 1e-5)])
    ref.launch("add_layernorm", (8,), 128, [("p", X.data_ptr()), ("p", D.data_ptr()), ("p", W.data_ptr()),
                                            ("p", Bb.data_ptr()), ("p", D.data_ptr()), ("i", 384), ("f", 1e-5)])
    torch.cuda.synchronize()
    res["ln_y"], res["ln_x"], res["addln_y"] = Y.cpu().numpy(), X.cpu().numpy(), D.cpu().numpy()

    q, kv, aslot, c = inputs_cross()
    B, d, nh = c["B"], c["d"], c["d"] // 64
    Q, KV, ASL = dev(q), dev(kv), dev(aslot)
    DONE = torch.zeros(B, dtype=torch.int32, device="cuda")
    CTR = torch.tensor([c["p"], 0, 0, 0], dtype=torch.int32, device="cuda")
    S = torch.zeros(B * nh * 1500, dtype=torch.float32, device="cuda")
    ST = torch.zeros(B * nh * 48, dtype=torch.float32, device="cuda")
    PT = torch.zeros(B * nh * 24 * 64, dtype=torch.float32, device="cuda")
    OUT = torch.zeros(B, d, dtype=torch.float16, device="cuda")
    ALN = torch.zeros(B, c["max_t"], c["na"], 1500, dtype=torch.float16, device="cuda")
    ref.launch("cross_scores", (B * nh, 24), 128, [("p", Q.data_ptr()), ("p", KV.data_ptr()), ("p", S.data_ptr()),
                                                   ("p", ST.data_ptr()), ("p", DONE.data_ptr()), ("i", 0), ("i", 1),
                                                   ("i", d)])
    ref.launch("cross_pv", (B * nh, 24), 128, [("p", S.data_ptr()), ("p", ST.data_ptr()), ("p", KV.data_ptr()),
                                               ("p", PT.data_ptr()), ("p", ALN.data_ptr()), ("p", ASL.data_ptr()),
                                               ("p", CTR.data_ptr()), ("p", DONE.data_ptr()), ("i", 0), ("i", 1),
                                               ("i", d), ("i", c["na"]), ("i", c["max_t"])])
    ref.launch("cross_combine", (B * nh,), 64, [("p", PT.data_ptr()), ("p", OUT.data_ptr()), ("p", DONE.data_ptr()),
                                                ("i", d)])
    torch.cuda.synchronize()
    res["cross_out"] = OUT.cpu().numpy()
    res["cross_align"] = ALN.cpu().numpy()[:, c["p"]]
    res["cross_scores"] = S.cpu().numpy().reshape(B, nh, 1500)

    qkv, kc, vc, c = inputs_self()
    B, d = c["B"], c["d"]
    QKV, KC, VC = dev(qkv), dev(kc), dev(vc)
    CTR = torch.tensor([c["p"], 0, 0, 0], dtype=torch.int32, device="cuda")
    DONE = torch.zeros(B, dtype=torch.int32, device="cuda")
    OUT = torch.zeros(B, d, dtype=torch.float16, device="cuda")
    ref.launch("kv_write", (B,), 256, [("p", QKV.data_ptr()), ("p", KC.data_ptr()), ("p", VC.data_ptr()),
                                       ("p", CTR.data_ptr()), ("i", c["max_t"]), ("i", d)])
    ref.launch("self_attn", (B, d // 64), 128, [("p", QKV.data_ptr()), ("p", KC.data_ptr()), ("p", VC.data_ptr()),
                                                ("p", OUT.data_ptr()), ("p", CTR.data_ptr()), ("p", DONE.data_ptr()),
                                                ("i", c["max_t"]), ("i", d)])
    torch.cuda.synchronize()
    res["self_out"] = OUT.cpu().numpy()

    qkv = inputs_enc()
    QKV = dev(qkv)
    OUT = torch.zeros(1, 1500, 384, dtype=torch.float16, device="cuda")
    ref.launch("enc_flash", (24, 6, 1), 128, [("p", QKV.data_ptr()), ("p", OUT.data_ptr()), ("i", 384)])
    torch.cuda.synchronize()
    o = OUT.cpu().numpy()
    res["enc_rows"] = o[0, ENC_ROWS]
    res["enc_sum"] = np.array([o.astype(np.float64).sum(), np.abs(o.astype(np.float64)).sum()])
    np.savez_compressed(out_path, **res)
    print("wrote", out_path, {k: v.shape for k, v in res.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ref_fixtures.npz"))
