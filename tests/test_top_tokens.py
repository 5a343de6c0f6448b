"""topTokens (sampler.nim:123-130) on the GPU against the CPU oracle: ids
equal and probabilities bitwise equal (the GPU replays the index-order fp32
sum exactly and computes glibc's expf), including ties at the n-th
probability."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def check(engine, oracle_mod, x, n):
    ids, probs = engine.top_tokens(x, n)
    for r in range(x.shape[0]):
        ref = oracle_mod.top_tokens(x[r], n)
        m = len(ref)
        assert [int(i) for i in ids[r, :m]] == [i for i, _ in ref], f"row {r} n={n}"
        want = np.array([p for _, p in ref], np.float32)
        got = probs[r, :m].astype(np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
            f"row {r} n={n}: probs differ at {np.nonzero(got != want)[0][:5].tolist()}"
        assert np.all(ids[r, m:] == -1)


def test_random_rows(engine, oracle_mod):
    rng = np.random.default_rng(5)
    for V, n in [(1, 5), (3, 5), (7, 7), (2000, 5), (2000, 40), (128256, 5), (151936, 256)]:
        x = (rng.standard_normal((3, V)) * rng.choice([0.5, 2.0, 8.0])).astype(np.float32)
        check(engine, oracle_mod, x, n)


def test_ties_and_degenerate_rows(engine, oracle_mod):
    V = 5000
    rows = [np.zeros(V, np.float32),                               # all equal: lowest indices
            np.repeat(np.arange(50, dtype=np.float32), V // 50),   # many equal groups
            np.full(V, -200.0, np.float32)]                        # one large, the rest underflow to 0
    rows[2][1234] = 0.0
    x = np.stack(rows)
    x[1, ::7] = -np.inf
    for n in (1, 5, 64, 256):
        check(engine, oracle_mod, x, n)


def test_nan_row_is_an_error(engine):
    x = np.zeros((2, 100), np.float32)
    x[1, 3] = np.nan
    with pytest.raises(Exception):
        engine.top_tokens(x, 5)


def test_python_mirror(pkg, oracle_mod):
    rng = np.random.default_rng(9)
    x = rng.standard_normal(3000).astype(np.float32)
    assert pkg.topTokens(x, 6) == oracle_mod.top_tokens(x, 6)
