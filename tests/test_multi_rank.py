"""Batch-sharded mode across ranks, world size 2 over gloo on CPU.

The multi-GPU mode splits the batch into contiguous row shards with no
collective on the data path: each rank regenerates its own rows from
(seed, global row) and samples them, and the bench takes the max of the
per-rank step times. These tests run that host logic with two CPU ranks:
the shards cover the batch exactly once, each rank's regenerated rows equal
the same rows of the whole batch, per-rank results (the oracle stands in for
the GPU here) gathered in rank order equal the whole batch's results, and the
bench's max-over-ranks reduction returns the slowest rank's time.
"""
from __future__ import annotations

import os
import socket
import sys
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORLD = 2
CFG, B, V = "c3_batched_hetero", 10, 4096


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist

    import __graft_entry__ as g
    import bench
    from oracle import oracle

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        pkg = g.load_package()
        rows = pkg.workloads.shard_rows(B, rank, world)
        w = pkg.workloads.make(CFG, seed=1234, rows=rows, V=V)
        ids = oracle.sample_batch(w.logits, w.params, w.hist_ids, w.hist_off, w.bias_ids,
                                  w.bias_vals, w.bias_off, w.uniforms)
        # results gathered in rank order (padded to the largest shard)
        n = torch.tensor([len(rows)], dtype=torch.int64)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, n)
        cap = int(max(int(s.item()) for s in sizes))
        buf = torch.full((cap,), -7, dtype=torch.int64)
        buf[: len(rows)] = torch.from_numpy(ids)
        outs = [torch.empty(cap, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(outs, buf)
        # the bench's step time: the max over ranks
        t = bench.reduce_max(dist, 1.0 + rank, torch.device("cpu"))
        if rank == 0:
            got = np.concatenate([o[: int(s.item())].numpy() for o, s in zip(outs, sizes)])
            np.savez(os.path.join(out_dir, "rank0.npz"), ids=got, tmax=np.float64(t),
                     rows=np.concatenate([pkg.workloads.shard_rows(B, r, world) for r in range(world)]))
        np.save(os.path.join(out_dir, f"logits{rank}.npy"), w.logits)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_shards_cover_batch():
    import __graft_entry__ as g
    pkg = g.load_package()
    for Btot in (1, 7, 256, 8192):
        for world in (1, 2, 3, 4, 8):
            parts = [pkg.workloads.shard_rows(Btot, r, world) for r in range(world)]
            allr = np.concatenate(parts)
            assert np.array_equal(allr, np.arange(Btot))
            sizes = [p.size for p in parts]
            assert max(sizes) - min(sizes) <= 1


def test_two_ranks_gloo(tmp_path, oracle_mod):
    import torch.multiprocessing as mp

    port = _free_port()
    ctx = mp.start_processes(_rank_main, args=(WORLD, port, str(tmp_path)), nprocs=WORLD,
                             join=False, start_method="spawn")
    deadline = time.time() + 240
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail("gloo ranks did not finish within 240 s")

    import __graft_entry__ as g
    pkg = g.load_package()
    res = np.load(tmp_path / "rank0.npz")
    assert np.array_equal(res["rows"], np.arange(B))
    assert float(res["tmax"]) == float(WORLD)  # slowest rank's time
    whole = pkg.workloads.make(CFG, seed=1234, rows=np.arange(B), V=V)
    # each rank regenerated exactly its rows of the whole batch
    for r in range(WORLD):
        rows = pkg.workloads.shard_rows(B, r, WORLD)
        assert np.array_equal(np.load(tmp_path / f"logits{r}.npy"), whole.logits[rows])
    ref = oracle_mod.sample_batch(whole.logits, whole.params, whole.hist_ids, whole.hist_off,
                                  whole.bias_ids, whole.bias_vals, whole.bias_off, whole.uniforms)
    assert np.array_equal(res["ids"], ref)
