"""Perplexity's per-position term (model.nim:570-589): nls_token_nll against
the CPU oracle.

CPU: the C restatement (oracle/ref_sampler.c) equals the line-by-line Python
transliteration (oracle/translit.py) bit for bit, and both sit within float64
rounding of an exactly rounded sum (math.fsum) of the same terms.

GPU: the library sums the float64 terms in a tree order instead of the
reference's index order, so the bar is a float64 tolerance: each term within
NLL_RTOL = 1e-12 relative (absolute for terms below 1) of the oracle's. NaN
rows, non-finite maxima and out-of-range targets give NaN and an error
status; a target whose logit is -inf gives +inf, as in the reference.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

NLL_RTOL = 1e-12


def _rows(rng, V, n, scale):
    return (rng.standard_normal((n, V)) * scale).astype(np.float32)


def test_oracle_matches_transliteration(oracle_mod):
    from oracle import translit
    rng = np.random.default_rng(1)
    for V, scale in [(1, 1.0), (7, 3.0), (300, 0.5), (2000, 2.0)]:
        x = _rows(rng, V, 3, scale)
        t = rng.integers(0, V, 3)
        got = oracle_mod.token_nll(x, t)
        want = [translit.token_nll(list(x[r]), int(t[r])) for r in range(3)]
        assert got.tolist() == want


def test_oracle_against_exact_sum(oracle_mod):
    rng = np.random.default_rng(2)
    x = _rows(rng, 5000, 4, 2.5)
    t = rng.integers(0, 5000, 4)
    got = oracle_mod.token_nll(x, t)
    for r in range(4):
        mx = np.float32(x[r].max())
        d = (x[r] - mx).astype(np.float32)             # fp32 difference, as the reference
        s = math.fsum(math.exp(float(v)) for v in d)
        want = -(float(d[t[r]]) - math.log(s))
        assert abs(got[r] - want) <= 1e-12 * max(1.0, abs(want))


def _check(engine, oracle_mod, x, t):
    got, st = engine.token_nll(x, t)
    assert st == 0
    want = oracle_mod.token_nll(x, t)
    err = np.abs(got - want) / np.maximum(np.abs(want), 1.0)
    assert np.all(err <= NLL_RTOL), f"max rel err {err.max()}"


@pytest.mark.gpu
def test_random_rows(engine, oracle_mod):
    rng = np.random.default_rng(3)
    for V, scale in [(1, 1.0), (5, 2.0), (2000, 2.0), (2001, 0.3), (128256, 3.0), (151936, 1.0)]:
        x = _rows(rng, V, 8, scale)
        t = rng.integers(0, V, 8)
        t[0] = int(np.argmax(x[0]))  # the most probable token
        _check(engine, oracle_mod, x, t)


@pytest.mark.gpu
def test_strided_rows_and_many_positions(engine, oracle_mod):
    """A chunk of 511 positions (nCtx 512, model.nim:572) read from a wider
    buffer (ld > V: the float4 path is off for most rows)."""
    rng = np.random.default_rng(4)
    full = _rows(rng, 20003, 511, 2.0)
    x = full[:, :20000]
    t = rng.integers(0, 20000, 511)
    assert x.strides[0] == 4 * 20003
    got, st = engine.token_nll(x, t)
    assert st == 0
    want = oracle_mod.token_nll(x, t)
    assert np.all(np.abs(got - want) / np.maximum(np.abs(want), 1.0) <= NLL_RTOL)


@pytest.mark.gpu
def test_edge_rows(engine, oracle_mod):
    V = 3000
    x = np.zeros((3, V), np.float32)
    x[1, ::2] = -np.inf          # -inf logits contribute exp(-inf) = 0
    x[2, :] = -100.0
    x[2, 17] = 50.0
    t = np.array([5, 0, 16])     # row 1: a -inf target -> +inf
    got, st = engine.token_nll(x, t)
    assert st == 0
    want = oracle_mod.token_nll(x, t)
    assert got[1] == np.inf and want[1] == np.inf
    assert np.all(np.abs(got[[0, 2]] - want[[0, 2]]) <= NLL_RTOL * np.maximum(np.abs(want[[0, 2]]), 1.0))
    # the -inf logits of row 1 drop out of its sum: the others give ln(1500)
    got1, _ = engine.token_nll(x[1:2], [1])
    assert got1[0] == pytest.approx(math.log(1500.0), rel=1e-12)


@pytest.mark.gpu
def test_bad_rows_report_errors(engine):
    x = np.zeros((3, 100), np.float32)
    x[1, 3] = np.nan
    got, st = engine.token_nll(x, [0, 0, 0], check=False)
    assert st == 5 and np.isnan(got[1]) and not np.isnan(got[0]) and not np.isnan(got[2])
    got, st = engine.token_nll(np.zeros((2, 100), np.float32), [0, 100], check=False)
    assert st == 1 and np.isnan(got[1]) and got[0] == pytest.approx(math.log(100.0), rel=1e-12)


@pytest.mark.gpu
def test_perplexity_mirror(pkg, engine, oracle_mod):
    rng = np.random.default_rng(6)
    T, V = 64, 4096
    x = _rows(rng, V, T, 2.0)
    tok = rng.integers(0, V, T)
    ppl = pkg.perplexity_from_logits(x, tok, engine=engine)
    nll = oracle_mod.token_nll(x[:T - 1], tok[1:])
    total = 0.0
    for v in nll:  # model.nim:584, position order
        total += float(v)
    assert ppl == pytest.approx(math.exp(total / (T - 1)), rel=1e-12)
    assert pkg.perplexity_from_logits(x[:1], tok[:1], engine=engine) == 1.0
