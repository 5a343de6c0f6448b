"""Generates tests/golden/sampler_cases.npz.

    python tests/golden/make_golden.py

Small seeded cases (vocab 1..400) covering every branch of
src/nimllm/sampler.nim (reference repository): penalties with every window
rule, out-of-range ids, bias (including -Inf), greedy, the heap path with
ties, the full stable sort, top-p / min-p on and off, uniforms at 0 and near 1.
Expected outputs come from oracle/translit.py, the line-by-line Python
transliteration (it does not share code with the C oracle, which the tests
check against these fixtures). The reference itself cannot run here (no Nim
toolchain), so these vectors pin the restatements to each other, not to Nim.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import translit  # noqa: E402

PARAMS_DTYPE = np.dtype([
    ("temperature", "<f8"), ("top_p", "<f8"), ("min_p", "<f8"),
    ("repeat_penalty", "<f8"), ("presence_penalty", "<f8"),
    ("frequency_penalty", "<f8"), ("top_k", "<i8"), ("repeat_last_n", "<i8"),
])


def gen_cases(n_cases: int = 480, seed: int = 20261201):
    rng = np.random.default_rng(seed)
    cases = []
    for c in range(n_cases):
        V = int(rng.choice([1, 2, 3, 4, 7, 16, 33, 64, 100, 257, 400]))
        kind = rng.random()
        x = rng.normal(0.0, float(rng.choice([0.5, 2.0, 4.0])), V).astype(np.float32)
        if kind < 0.25:
            x = np.round(x).astype(np.float32)             # many exact ties
        elif kind < 0.35:
            x = np.round(x * 2).astype(np.float32) * np.float32(0.5)
        if rng.random() < 0.15:
            x[rng.integers(0, V, max(1, V // 10))] = -np.inf
        if rng.random() < 0.05:
            x[:] = np.float32(1.5)                          # all equal
        if rng.random() < 0.05:
            x[rng.integers(0, V)] = np.float32(-0.0)
        T = float(rng.choice([0.0, 0.0, 0.3, 0.7, 1.0, 1.5]))
        k = int(rng.choice([0, 1, 2, 3, 5, 40, V - 1 if V > 1 else 0, V, V + 5, -1]))
        topP = float(rng.choice([0.0, 0.5, 0.8, 0.95, 1.0, -0.5]))
        minP = float(rng.choice([0.0, 0.0, 0.05, 0.3]))
        rep = float(rng.choice([1.0, 1.1, 0.8, 1.5]))
        lastN = int(rng.choice([0, -1, 3, 64]))
        pres = float(rng.choice([0.0, 0.2, -0.5]))
        freq = float(rng.choice([0.0, 0.2, 0.7]))
        hlen = int(rng.choice([0, 1, 5, 20]))
        hist = [int(v) for v in rng.integers(-3, V + 3, hlen)]
        nb = int(rng.choice([0, 0, 1, 3]))
        bias = {}
        for tok in rng.integers(-2, V + 2, nb):
            bias[int(tok)] = float(rng.choice([-5.0, 5.0, 0.25, -np.inf]))
        u = float(rng.choice([rng.random(), 0.0, 0.9999999, 1.0 - 2.0 ** -40]))
        p = translit.SamplerParams(temperature=T, topK=k, topP=topP, minP=minP,
                                   repeatPenalty=rep, repeatLastN=lastN,
                                   presencePenalty=pres, frequencyPenalty=freq,
                                   logitBias=bias)
        d: dict = {}
        with np.errstate(all="ignore"):
            ref = translit.sample(p, hist, x, u, d)
        cases.append(dict(V=V, x=x, prm=(T, topP, minP, rep, pres, freq, k, lastN),
                          hist=hist, bias=bias, u=u, id=ref,
                          prob=d.get("prob", 1.0), n=d.get("n", 1), pos=d.get("pos", 0)))
    return cases


def pack(cases):
    n = len(cases)
    Vs = np.array([c["V"] for c in cases], np.int64)
    loff = np.zeros(n + 1, np.int64)
    loff[1:] = np.cumsum(Vs)
    logits = np.concatenate([c["x"] for c in cases]).astype(np.float32)
    params = np.zeros(n, PARAMS_DTYPE)
    for i, c in enumerate(cases):
        params[i] = c["prm"]
    hoff = np.zeros(n + 1, np.int64)
    hoff[1:] = np.cumsum([len(c["hist"]) for c in cases])
    hist = np.array([t for c in cases for t in c["hist"]], np.int64)
    boff = np.zeros(n + 1, np.int64)
    boff[1:] = np.cumsum([len(c["bias"]) for c in cases])
    bids = np.array([t for c in cases for t in c["bias"].keys()], np.int64)
    bvals = np.array([b for c in cases for b in c["bias"].values()], np.float64)
    return dict(V=Vs, logit_off=loff, logits=logits, params=params, hist_off=hoff, hist=hist,
                bias_off=boff, bias_ids=bids, bias_vals=bvals,
                uniforms=np.array([c["u"] for c in cases], np.float64),
                ids=np.array([c["id"] for c in cases], np.int64),
                probs=np.array([c["prob"] for c in cases], np.float32),
                n=np.array([c["n"] for c in cases], np.int64),
                pos=np.array([c["pos"] for c in cases], np.int64))


def main():
    cases = gen_cases()
    out = os.path.join(HERE, "sampler_cases.npz")
    np.savez_compressed(out, **pack(cases))
    print(out, os.path.getsize(out), "bytes,", len(cases), "cases")


if __name__ == "__main__":
    main()
