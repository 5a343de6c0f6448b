"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on
CPU. GPU fixtures fail (not skip) without a usable device: a GPU test must
never pass on a fallback."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__ as g
    g._load_build_module().build()
    return g.load_package()


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def golden():
    z = np.load(os.path.join(TESTS, "golden", "sampler_cases.npz"))
    return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def engine(pkg):
    eng = pkg.Engine(0, max_rows=512, max_vocab=1 << 18)
    yield eng
    eng.close()


def case_arrays(g, i):
    """Inputs of golden case i as single-row arrays."""
    lo, hi = g["logit_off"][i], g["logit_off"][i + 1]
    x = g["logits"][lo:hi][None, :]
    h0, h1 = g["hist_off"][i], g["hist_off"][i + 1]
    b0, b1 = g["bias_off"][i], g["bias_off"][i + 1]
    return dict(logits=x, params=g["params"][i:i + 1],
                hist_ids=g["hist"][h0:h1], hist_off=np.array([0, h1 - h0], np.int64),
                bias_ids=g["bias_ids"][b0:b1], bias_vals=g["bias_vals"][b0:b1],
                bias_off=np.array([0, b1 - b0], np.int64),
                uniforms=g["uniforms"][i:i + 1])


def kat_arrays(case):
    """Inputs of a known-answer case (tests/kat_cases.py) as single-row arrays."""
    name, logits, prm, hist, bias, u, expected = case
    from oracle.oracle import PARAMS_DTYPE
    P = np.zeros(1, PARAMS_DTYPE)
    P[0] = prm
    return dict(logits=np.array([logits], np.float32), params=P,
                hist_ids=np.array(hist, np.int64), hist_off=np.array([0, len(hist)], np.int64),
                bias_ids=np.array(list(bias.keys()), np.int64),
                bias_vals=np.array(list(bias.values()), np.float64),
                bias_off=np.array([0, len(bias)], np.int64),
                uniforms=np.array([u], np.float64)), expected
