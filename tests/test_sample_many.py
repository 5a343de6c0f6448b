"""Many independent samplers in one batched call (separate Chats sharing one
model, examples/ex11_bas_niveau.nim:57-62 run together): batch_inputs /
sample_many / decode_step_many against each sampler run alone.

CPU: the batch's CSR histories and bias lists are each sampler's own, and
every RNG draws exactly as it would alone (a uniform only for temperature
> 0, sampler.nim:77-78, :117).
GPU: sample_many returns the ids of each sampler's own sample() on the same
logits, and decode_step_many (output projection + sampling with rows
independent) the ids of one-row projections sampled one by one.
"""
from __future__ import annotations

import copy

import numpy as np
import pytest


def _samplers(pkg, n, V, seed=3):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        p = pkg.defaultSampling() if i % 3 else pkg.greedySampling()
        p.seed = 1000 + i
        if i % 3:
            p.temperature = float(rng.uniform(0.5, 1.2))
            p.topK = int(rng.choice([0, 20, 40, 300]))
            p.topP = float(rng.uniform(0.8, 1.0))
            p.minP = float(rng.choice([0.0, 0.05]))
            p.repeatPenalty, p.presencePenalty, p.frequencyPenalty = 1.1, 0.2, 0.1
            p.logitBias = {int(k): float(rng.normal(0, 3)) for k in rng.integers(0, V, 3)}
        s = pkg.newSampler(p)
        for t in rng.integers(0, V, int(rng.integers(0, 40))):
            s.accept(int(t))
        out.append(s)
    return out


def test_batch_inputs_layout(pkg):
    V = 500
    ss = _samplers(pkg, 7, V)
    alone = copy.deepcopy(ss)
    a = pkg.batch_inputs(ss)
    for i, s in enumerate(ss):
        h = a["hist_ids"][a["hist_off"][i]:a["hist_off"][i + 1]]
        assert h.tolist() == s.history
        b = a["bias_ids"][a["bias_off"][i]:a["bias_off"][i + 1]]
        assert b.tolist() == list(s.params.logitBias.keys())
        # the RNG drew once for a sampling row, never for a greedy one
        want = alone[i].rng.rand(1.0) if s.params.temperature > 0 else 0.0
        assert a["uniforms"][i] == want
        assert s.rng.rand(1.0) == alone[i].rng.rand(1.0)


@pytest.mark.gpu
def test_sample_many_equals_one_by_one(pkg, engine):
    V = 4000
    ss = _samplers(pkg, 12, V, seed=5)
    alone = copy.deepcopy(ss)
    for s in ss + alone:
        s.engine = engine
    logits = (np.random.default_rng(6).standard_normal((12, V)) * 3).astype(np.float32)
    for step in range(3):
        got = pkg.sample_many(ss, logits, engine=engine)
        want = [s.sample(logits[i]) for i, s in enumerate(alone)]
        assert got == want, f"step {step}"
        for s, t in zip(ss, got):
            s.accept(t)
        for s, t in zip(alone, want):
            s.accept(t)
        logits = np.roll(logits, 17, axis=1)


@pytest.mark.gpu
def test_decode_step_many_rows_independent(pkg, engine, oracle_mod):
    """Q8_0 weights and 6 Chats: each row's logits are a one-row matmul's
    (int8 path), not the float path a 6-row matmul would take."""
    import torch
    t, V, cols = pkg.workloads.LM_TYPES["q8_0"], 3000, 1024
    w = pkg.workloads.lm_weights(t, V, cols, seed=12, sigma=0.08)
    dw = torch.from_numpy(w).cuda()
    x = np.random.default_rng(13).standard_normal((6, cols)).astype(np.float32)
    y_ind = engine.lm_head(dw, t, V, cols, x, independent=True)
    y_one = np.concatenate([oracle_mod.lm_head(w, t, V, cols, x[i:i + 1]) for i in range(6)])
    assert np.array_equal(y_ind.view(np.uint32), y_one.view(np.uint32))
    y_all = oracle_mod.lm_head(w, t, V, cols, x)   # one 6-row matmul: the float path
    assert not np.array_equal(y_all.view(np.uint32), y_one.view(np.uint32))
    ss = _samplers(pkg, 6, V, seed=14)
    alone = copy.deepcopy(ss)
    got = pkg.decode_step_many(ss, engine, dw, t, V, cols, x)
    want = [int(oracle_mod.sample_batch(y_one[i:i + 1],
                                        np.array([pkg.params_record(s.params)], dtype=pkg.ROW_PARAMS_DTYPE),
                                        np.asarray(s.history, np.int64),
                                        np.array([0, len(s.history)], np.int64),
                                        np.fromiter(s.params.logitBias.keys(), np.int64),
                                        np.fromiter(s.params.logitBias.values(), np.float64),
                                        np.array([0, len(s.params.logitBias)], np.int64),
                                        np.array([s.rng.rand(1.0) if s.params.temperature > 0 else 0.0]))[0])
            for i, s in enumerate(alone)]
    assert got == want
