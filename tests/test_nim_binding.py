"""The library as Nim's {.importc, dynlib.} declarations bind it.

tests/nim_abi_harness.c dlopen()s libnimllm_sample.so, dlsym()s every name
the binding module imports, with the C types Nim's code
generator gives those declarations, and runs the generation loop of
chat.nim:204-208 (`sample` with the unchanged signature of sampler.nim:59,
then `accept`, then the next logits) for a sampling Sampler and, interleaved,
a greedy one that must draw no uniform. The same loop is replayed here with
the CPU oracle, feeding each step's id back into the history, so a single
wrong token would change every later step.

CPU: the harness compiles and every imported name resolves.
GPU: 64 + 16 steps at the config-2 vocabulary (V = 128256), ids equal to the
oracle's, the same number of uniforms consumed, and the reference's
behaviour on an empty logitsIn.
"""
from __future__ import annotations

import os
import struct
import subprocess

import numpy as np
import pytest

TESTS = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def harness(pkg, tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("nimabi") / "nim_abi_harness")
    subprocess.run(["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-o", exe,
                    os.path.join(TESTS, "nim_abi_harness.c"), "-ldl"], check=True)
    return exe


def test_every_imported_name_resolves(pkg, harness):
    out = subprocess.run([harness, pkg.LIB_PATH, "--resolve-only"], capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0, out.stderr
    assert "sm_100a" in out.stdout


def oracle_loop(oracle_mod, pa, pb, hist0, bias, unif, la, lb):
    """chat.nim:204-208 with the oracle: the same interleaving as the harness."""
    used = 0
    ha, hb = list(hist0), []
    ids_a, ids_b = [], []
    bids = np.array(list(bias.keys()), np.int64)
    bvals = np.array(list(bias.values()), np.float64)
    ib = 0

    def one(x, prm, hist, with_bias, u):
        h = np.array(hist, np.int64)
        return int(oracle_mod.sample_batch(
            x[None, :], prm, h if h.size else None, np.array([0, h.size], np.int64) if h.size else None,
            bids if with_bias else None, bvals if with_bias else None,
            np.array([0, bids.size], np.int64) if with_bias else None, np.array([u]))[0])

    for t in range(la.shape[0]):
        u = unif[used] if pa["temperature"][0] > 0 else 0.0
        used += int(pa["temperature"][0] > 0)
        i = one(la[t], pa, ha, True, u)
        ids_a.append(i)
        ha.append(i)
        if t % 4 == 3 and ib < lb.shape[0]:
            g = one(lb[ib], pb, hb, False, 0.0)
            ids_b.append(g)
            hb.append(g)
            ib += 1
    used += 1  # the empty sampling call draws before it raises (min-p off)
    return ids_a, ids_b, used


@pytest.mark.gpu
def test_generation_loop_through_the_nim_binding(pkg, oracle_mod, harness, tmp_path):
    from oracle.oracle import PARAMS_DTYPE
    steps_a, steps_b = 64, 16
    w = pkg.workloads.make("c2_llama3_b1", seed=1234, rows=np.arange(steps_a))
    g = pkg.workloads.make("c2_llama3_b1_greedy", seed=99, rows=np.arange(steps_b))
    V = w.V
    pa = np.zeros(1, PARAMS_DTYPE)
    pa[0] = (0.7, 0.9, 0.0, 1.1, 0.1, 0.05, 40, 64)   # min-p off: the empty call draws first
    pb = np.zeros(1, PARAMS_DTYPE)
    pb[0] = (0.0, 1.0, 0.0, 1.3, 0.0, 0.0, 0, 16)      # greedy with a repeat penalty
    hist0 = w.hist_ids[:64]
    bias = {3: float("-inf"), 17: 2.5, int(V) + 5: 1.0, int(np.argmax(w.logits[0])): -30.0}
    unif = np.random.default_rng(5).random(200)
    la = np.ascontiguousarray(w.logits)
    lb = np.ascontiguousarray(g.logits)
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as f:
        f.write(struct.pack("<6q", V, steps_a, steps_b, hist0.size, len(bias), unif.size))
        f.write(pa.tobytes())
        f.write(pb.tobytes())
        f.write(np.asarray(hist0, np.int64).tobytes())
        f.write(np.array(list(bias.keys()), np.int64).tobytes())
        f.write(np.array(list(bias.values()), np.float64).tobytes())
        f.write(unif.tobytes())
        f.write(la.tobytes())
        f.write(lb.tobytes())
    outp = tmp_path / "out.bin"
    r = subprocess.run([harness, pkg.LIB_PATH, str(inp), str(outp)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(outp, np.int64)
    ids_a, ids_b = got[:steps_a], got[steps_a:steps_a + steps_b]
    used, probe_greedy, probe_raised = got[steps_a + steps_b:]
    ref_a, ref_b, ref_used = oracle_loop(oracle_mod, pa, pb, hist0, bias, unif, la, lb)
    assert ids_a.tolist() == ref_a
    assert ids_b.tolist() == ref_b
    assert used == ref_used == steps_a + 1   # greedy calls drew nothing
    assert probe_greedy == 0 and probe_raised == 1
    assert 3 not in ids_a                     # -inf bias is never sampled
