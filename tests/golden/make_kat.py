"""Writes kat.json: the known-answer vectors of the reference's own unit tests, restated as data.

  fp16   src/gpu.rs:380-397   (ties to even, overflow, subnormal ties, 0.1)
  dtw    src/align.rs:112-120 (3 x 6 cost with a cheap diagonal band)
  jump   src/align.rs:122-139 (4 tokens on 40 of 60 frames, 0 frames, 1 token)

    python tests/golden/make_kat.py
"""
import json
import os

kat = {
    "fp16": [
        {"x": 1.0 + 1.0 / 2048.0, "bits": 0x3C00},
        {"x": 1.0 + 3.0 / 2048.0, "bits": 0x3C02},
        {"x": 65520.0, "bits": 0x7C00},
        {"x": 65519.0, "bits": 0x7BFF},
        {"x": 2.0 ** -25, "bits": 0},
        {"x": 3.0 * 2.0 ** -25, "bits": 2},
    ],
    "rh": [{"x": 0.1, "y": 1638.0 / 16384.0}],
    "dtw": {
        "rows": 3, "cols": 6,
        "m": [[-1.0 if (k % 6) // 2 == k // 6 else 1.0 for k in range(r * 6, r * 6 + 6)] for r in range(3)],
        "text": [0, 0, 1, 1, 2, 2],
        "time": [0, 1, 2, 3, 4, 5],
    },
    "jump": {
        "rows": 4, "heads": 1, "cols_full": 60, "cols": 40, "width": 7,
        "nonzero": [[i, j] for i in range(4) for j in range(10 * i, 10 * i + 10)], "value": 0.1,
        "expect_near": [0.0, 0.2, 0.4, 0.6], "tol": 0.03,
        "zero_frames": [0.0, 0.0, 0.0, 0.0],
        "one_token": [0.0],
    },
}
with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat.json"), "w") as f:
    json.dump(kat, f, indent=1)
