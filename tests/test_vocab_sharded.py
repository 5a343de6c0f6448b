"""Vocab-sharded mode (nls_sample_batch_vocab_sharded).

CPU: the column and row partitions cover the vocabulary and the batch once.
GPU (2 devices): two ranks, each holding its columns of every row, sample
through the library's NCCL transpose; every rank's results must equal the CPU
oracle on the whole rows bit for bit (the bar of the single-GPU parity tests). The
NCCL id is made in this process and handed to the ranks; each rank writes its
results to a file and exits.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NRANKS = 2


def test_partitions_cover_vocab_and_rows():
    import __graft_entry__ as g
    pkg = g.load_package()
    for V in (2, 7, 2000, 128256, 151936):
        for P in (1, 2, 3, 4, 8):
            if V < P or pkg.vocab_shard(V, P, P - 1)[1] - pkg.vocab_shard(V, P, P - 1)[0] < 1:
                continue
            cols = [pkg.vocab_shard(V, P, r) for r in range(P)]
            assert cols[0][0] == 0 and cols[-1][1] == V
            assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
    for B in (1, 5, 64, 256):
        for P in (1, 2, 3, 8):
            rows = [pkg.row_owner_range(B, P, r) for r in range(P)]
            assert rows[0][0] == 0 and rows[-1][1] == B
            assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))


def _rank_main(rank: int, nranks: int, uid: bytes, out_dir: str, cases: list) -> None:
    sys.path.insert(0, ROOT)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch

    import __graft_entry__ as g
    pkg = g.load_package()
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    comm = pkg.Comm(uid, nranks, rank, rank)
    eng = pkg.Engine(rank, max_rows=256, max_vocab=1 << 18)

    def t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    for name, rows, V in cases:
        w = pkg.workloads.make(name, seed=1234, rows=np.arange(rows), V=V)
        lo, hi = pkg.vocab_shard(V, nranks, rank)
        shard = t(w.logits[:, lo:hi])
        params = torch.from_numpy(w.params.view(np.uint8).copy()).to(dev)
        ids = torch.empty(rows, dtype=torch.int64, device=dev)
        probs = torch.empty(rows, dtype=torch.float32, device=dev)
        eng.sample_batch_vocab_sharded(comm, shard, V, params, t(w.hist_ids), t(w.hist_off),
                                       t(w.bias_ids), t(w.bias_vals), t(w.bias_off), t(w.uniforms),
                                       out_ids=ids, out_probs=probs)
        np.savez(os.path.join(out_dir, f"{name}_{rank}.npz"), ids=ids.cpu().numpy(),
                 probs=probs.cpu().numpy())
    eng.close()
    comm.close()


CASES = [("c3_batched_hetero", 24, 20000), ("c5_full_vocab_nucleus", 6, 30000),
         ("c5_full_vocab_greedy", 5, 30001), ("c4_qwen2_sharded", 7, 151936)]


@pytest.mark.gpu
def test_two_rank_vocab_sharded(tmp_path, oracle_mod):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < NRANKS:
        pytest.skip(f"needs {NRANKS} GPUs")
    import __graft_entry__ as g
    pkg = g.load_package()
    uid = pkg.comm_unique_id()
    ctx = mp.start_processes(_rank_main, args=(NRANKS, uid, str(tmp_path), CASES), nprocs=NRANKS,
                             join=False, start_method="spawn")
    deadline = time.time() + 300
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail("vocab-sharded ranks did not finish within 300 s")
    for name, rows, V in CASES:
        w = pkg.workloads.make(name, seed=1234, rows=np.arange(rows), V=V)
        ref, dg = oracle_mod.sample_batch(w.logits, w.params, w.hist_ids, w.hist_off, w.bias_ids,
                                          w.bias_vals, w.bias_off, w.uniforms, diag=True)
        for r in range(NRANKS):
            z = np.load(tmp_path / f"{name}_{r}.npz")
            bad = np.nonzero(z["ids"] != ref)[0].tolist()
            assert not bad, f"{name} rank {r}: rows {bad} differ from the oracle"
            samp = w.params["temperature"] > 0
            got = z["probs"][samp].astype(np.float32)
            want = dg["prob"][samp].astype(np.float32)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
                f"{name} rank {r}: probs differ from the oracle"
