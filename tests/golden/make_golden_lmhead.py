"""Generates tests/golden/lmhead_cases.npz.

    python tests/golden/make_golden_lmhead.py

Small seeded cases of the output projection (matmul, model.nim:179-189 in
the reference repository) for every restated weight type (F32, F16, Q4_0,
Q8_0, Q6_K): 9 rows of 512 values, one activation matrix of 5 rows, batch
sizes 1 and 5 (the two sides of the Q8_0 switch at nb = 4, model.nim:185)
and both paths (int8 activations, and exactMatmul). Expected logits come
from oracle/translit.py, the line-by-line Python transliteration (it shares
no code with the C oracle, which the tests check against these fixtures).
The reference itself cannot run here (no Nim toolchain), so these vectors
pin the restatements to each other and the GPU kernels to both.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import translit  # noqa: E402

TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q6_k": 14}
ROWS, COLS, NB = 9, 512, 5


def weights(t: int, rng: np.random.Generator) -> np.ndarray:
    """[ROWS, rowBytes] uint8 in the ggml layout of type t (quant.nim)."""
    if t == 0:
        return (rng.standard_normal((ROWS, COLS)) * 0.05).astype("<f4").view(np.uint8)
    if t == 1:
        return (rng.standard_normal((ROWS, COLS)) * 0.05).astype("<f2").view(np.uint8)
    bv, bb, off = {2: (32, 18, 0), 8: (32, 34, 0), 14: (256, 210, 208)}[t]
    nblk = COLS // bv
    w = rng.integers(0, 256, size=(ROWS, nblk, bb), dtype=np.uint8)
    if t == 14:
        w[:, :, 192:208] = rng.integers(-40, 40, size=(ROWS, nblk, 16), dtype=np.int8).view(np.uint8)
    d = (rng.uniform(0.5, 1.5, size=(ROWS, nblk)) * {2: 0.01, 8: 0.0007, 14: 0.00004}[t]).astype("<f2")
    d[0, 0] = 0.0                      # a zero scale
    d[1, 0] = -d[1, 0]                 # a negative one
    w[:, :, off:off + 2] = d.view(np.uint8).reshape(ROWS, nblk, 2)
    return w.reshape(ROWS, nblk * bb)


def main() -> None:
    rng = np.random.default_rng(20261202)
    x = rng.standard_normal((NB, COLS)).astype(np.float32)
    x[0, :32] = 0.0                    # an all-zero activation block
    out = {"x": x}
    for name, t in TYPES.items():
        w = weights(t, rng)
        out[f"w_{name}"] = w
        for nb in (1, NB):
            for exact in (0, 1):
                y = translit.lm_head(w.reshape(-1), t, ROWS, COLS, x[:nb], exact_matmul=bool(exact))
                out[f"y_{name}_{nb}_{exact}"] = np.array(y, dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "lmhead_cases.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
