"""Failure detection, in forms that fault, trap or hang no GPU.

1 GPU: the streaming kernel's waits for its bulk copies are bounded; a
handle whose wait limit is 0 gives up on every such wait, so each streaming
row fails with NLS_ERR_TIMEOUT (id -1) after the kernel has drained the
copies it has in flight under the normal limit. The full-sort rows of the
same call are unaffected, and once the limit is restored the same handle
and stream give the oracle's results again (the context stays usable).

2 GPUs: vocab-sharded calls over a non-blocking NCCL communicator. Both
ranks make one call; then rank 1 stops taking part (it stays alive, with
nothing of its own in flight) and rank 0 makes a second call with a 3 s
deadline: its collectives cannot finish, the library aborts the
communicator and returns NLS_ERR_TIMEOUT within the deadline. NVLS is off
(NCCL_NVLS_ENABLE=0) and no kernel of this library waits on another rank.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
@pytest.mark.parametrize("B", [3, 12])  # the sequential and the concurrent launch paths
def test_wait_limit_zero_times_out_then_recovers(pkg, oracle_mod, B):
    import torch
    w = pkg.workloads.make("c3_batched_hetero", seed=61, rows=np.arange(B), V=50000)
    P = w.params.copy()
    P["top_k"][::3] = 0                 # some full-sort rows
    P["temperature"][1] = 0.0           # a greedy row (streaming kernel)
    a = dict(logits=w.logits, params=P, hist_ids=w.hist_ids, hist_off=w.hist_off,
             bias_ids=w.bias_ids, bias_vals=w.bias_vals, bias_off=w.bias_off, uniforms=w.uniforms)
    ref = oracle_mod.sample_batch(**a, threads=8)
    full = (P["temperature"] > 0) & (P["top_k"] == 0)
    eng = pkg.Engine(0, max_rows=64, max_vocab=50000)
    try:
        eng.set_wait_limit(0)
        ids, _, st = eng.sample_batch(**a, check=False)
        assert st == pkg._abi.NLS_ERR_TIMEOUT
        assert np.all(ids[~full] == -1)
        assert np.array_equal(ids[full], ref[full])
        # the device-output path reports the same through nls_stream_status
        dev = torch.device("cuda:0")
        t = lambda x: None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to(dev)
        out = torch.empty(B, dtype=torch.int64, device=dev)
        eng.sample_batch(t(w.logits), torch.from_numpy(P.view(np.uint8).copy()).to(dev), t(w.hist_ids),
                         t(w.hist_off), t(w.bias_ids), t(w.bias_vals), t(w.bias_off), t(w.uniforms),
                         out_ids=out, check=False)
        assert eng._lib.nls_stream_status(eng._h, None) == pkg._abi.NLS_ERR_TIMEOUT
        # restored: the same handle and stream sample correctly again
        eng.set_wait_limit(200 * 1000 * 1000)
        for _ in range(2):
            ids, _, st = eng.sample_batch(**a, check=False)
            assert st == 0 and np.array_equal(ids, ref)
    finally:
        eng.close()


def _rank_main(rank: int, nranks: int, uid: bytes, out_dir: str) -> None:
    sys.path.insert(0, ROOT)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    import __graft_entry__ as g
    pkg = g.load_package()
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    comm = pkg.Comm(uid, nranks, rank, rank)
    eng = pkg.Engine(rank, max_rows=16, max_vocab=40000)
    w = pkg.workloads.make("c5_full_vocab_nucleus", seed=3, rows=np.arange(6), V=40000)
    lo, hi = pkg.vocab_shard(w.V, nranks, rank)
    shard = torch.from_numpy(np.ascontiguousarray(w.logits[:, lo:hi])).to(dev)
    params = torch.from_numpy(w.params.view(np.uint8).copy()).to(dev)
    unif = torch.from_numpy(w.uniforms).to(dev)
    ids = torch.empty(w.B, dtype=torch.int64, device=dev)
    eng.sample_batch_vocab_sharded(comm, shard, w.V, params, uniforms=unif, out_ids=ids)
    first_ok = int(ids.cpu().numpy().min() >= 0)
    torch.cuda.synchronize(dev)
    res = {"first_ok": first_ok}
    if rank == 0:
        comm.set_timeout(3000)
        t0 = time.time()
        st = eng._lib.nls_sample_batch_vocab_sharded(
            eng._h, comm._c, shard.data_ptr(), shard.stride(0), w.B, w.V, params.data_ptr(), None,
            None, None, None, None, unif.data_ptr(), ids.data_ptr(), None, None)
        res.update(status=int(st), seconds=time.time() - t0,
                   again=int(eng._lib.nls_sample_batch_vocab_sharded(
                       eng._h, comm._c, shard.data_ptr(), shard.stride(0), w.B, w.V, params.data_ptr(),
                       None, None, None, None, None, unif.data_ptr(), ids.data_ptr(), None, None)))
        open(os.path.join(out_dir, "rank0.done"), "w").close()
    else:
        # leave between steps: nothing in flight; wait (bounded) until rank 0
        # has given up, then abort this rank's side too
        deadline = time.time() + 120
        while not os.path.exists(os.path.join(out_dir, "rank0.done")) and time.time() < deadline:
            time.sleep(0.05)
        comm.abort()
    comm.close()
    eng.close()
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([res.get("first_ok", 0), res.get("status", 0),
                                                             res.get("seconds", 0.0), res.get("again", 0)]))


@pytest.mark.gpu
def test_rank_that_stops_taking_part_ends_in_timeout(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import __graft_entry__ as g
    pkg = g.load_package()
    uid = pkg.comm_unique_id()
    ctx = mp.start_processes(_rank_main, args=(2, uid, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 240
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            pytest.fail("ranks did not finish within 240 s")
    r0 = np.load(tmp_path / "r0.npy")
    r1 = np.load(tmp_path / "r1.npy")
    assert r0[0] == 1 and r1[0] == 1               # the first call worked on both ranks
    assert int(r0[1]) == pkg._abi.NLS_ERR_TIMEOUT  # the second ended in the deadline
    assert 2.5 <= r0[2] <= 20.0
    assert int(r0[3]) == pkg._abi.NLS_ERR_NCCL     # the aborted communicator refuses more calls


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q6_k", "q4_0"])
def test_lm_head_tensor_core_wait_limit_zero(pkg, oracle_mod, name):
    """The tensor-core output projection's pipeline waits are bounded too: at
    a wait limit of 0 every wait gives up at once, the call returns
    NLS_ERR_TIMEOUT after the kernel has let its copies in flight land, and
    once the limit is restored the same handle gives the oracle's logits."""
    import ctypes
    import torch
    t = {"q6_k": 14, "q4_0": 2}[name]
    rows, cols, nb = 1000, 1024, 9
    w = pkg.workloads.lm_weights(t, rows, cols, seed=71)
    x = np.random.default_rng(72).standard_normal((nb, cols)).astype(np.float32)
    want = oracle_mod.lm_head(w, t, rows, cols, x, threads=8)
    dw = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    eng = pkg.Engine(0, max_rows=16, max_vocab=rows)
    try:
        y = np.empty((nb, rows), np.float32)
        eng.set_wait_limit(0)
        st = eng._lib.nls_lm_head(eng._h, ctypes.c_void_p(dw.data_ptr()), t, rows, cols,
                                  ctypes.c_void_p(x.ctypes.data), nb, ctypes.c_void_p(y.ctypes.data), 0,
                                  ctypes.c_void_p(0))
        assert st == pkg._abi.NLS_ERR_TIMEOUT
        eng.set_wait_limit(200 * 1000 * 1000)
        for _ in range(2):
            got = eng.lm_head(dw, t, rows, cols, x)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        eng.close()
