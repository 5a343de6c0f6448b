"""Seeded synthetic sampler workloads (the five BASELINE configurations).

No public dataset is involved: every input is generated from a seed with the
shapes and distributions the configurations name. Row r of a workload is
generated from numpy's PCG64 seeded with (seed, config id, r), so any subset
of rows can be regenerated on its own -- a GPU rank regenerates only its
shard, and the CPU baseline only its sample -- with identical values.

Workload fields (host numpy arrays, the layout of include/nimllm_sample.h):
  logits   float32 [B, V]
  params   ROW_PARAMS_DTYPE [B]
  hist_ids int64, hist_off int64 [B+1]   (CSR; None when the config has none)
  bias_ids int64, bias_vals float64, bias_off int64 [B+1] (CSR; None if none)
  uniforms float64 [B]                   (stand-in for Nim's rng.rand(1.0))
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np

from ._abi import ROW_PARAMS_DTYPE

CONFIGS = {
    # name: (config index in BASELINE.json, B, V)
    "c1_tiny": (0, 1, 2000),
    "c2_llama3_b1": (1, 1, 128256),
    "c2_llama3_b1_greedy": (1, 1, 128256),
    "c3_batched_hetero": (2, 256, 128256),
    "c4_qwen2_sharded": (3, 8192, 151936),
    "c5_full_vocab_nucleus": (4, 64, 151936),
    "c5_full_vocab_greedy": (4, 64, 151936),
}


@dataclasses.dataclass
class Workload:
    name: str
    logits: np.ndarray
    params: np.ndarray
    hist_ids: Optional[np.ndarray]
    hist_off: Optional[np.ndarray]
    bias_ids: Optional[np.ndarray]
    bias_vals: Optional[np.ndarray]
    bias_off: Optional[np.ndarray]
    uniforms: np.ndarray
    rows: np.ndarray  # global row ids of this workload's rows

    @property
    def B(self) -> int:
        return self.logits.shape[0]

    @property
    def V(self) -> int:
        return self.logits.shape[1]

    def algorithmic_bytes(self) -> int:
        """Bytes one pass must move: logits once, history and bias lists,
        params, uniforms and the outputs (id int64 + prob fp32)."""
        n = self.logits.size * 4 + self.params.nbytes + self.uniforms.nbytes + self.B * 12
        if self.hist_ids is not None:
            n += self.hist_ids.nbytes + self.hist_off.nbytes
        if self.bias_ids is not None:
            n += self.bias_ids.nbytes + self.bias_vals.nbytes + self.bias_off.nbytes
        return int(n)


def _rng(seed: int, cfg: int, row: int) -> np.random.Generator:
    return np.random.default_rng([seed, cfg, row])


def _row(name: str, seed: int, r: int, V: int):
    """Generate one row: (logits, params tuple, history, bias ids, bias vals, uniform)."""
    cfg = CONFIGS[name][0]
    g = _rng(seed, cfg, r)
    hist = np.zeros(0, np.int64)
    bids = np.zeros(0, np.int64)
    bvals = np.zeros(0, np.float64)
    if name == "c1_tiny":
        x = g.standard_normal(V, dtype=np.float32) * np.float32(2.0)
        prm = (0.8, 0.95, 0.05, 1.1, 0.0, 0.0, 40, 64)
        hist = g.integers(0, V, 64).astype(np.int64)
    elif name.startswith("c2_llama3_b1"):
        x = g.standard_normal(V, dtype=np.float32) * np.float32(2.5)
        boost = g.choice(V, 20, replace=False)
        x[boost] += np.float32(8.0)
        hist = g.integers(0, V, 64).astype(np.int64)
        if name.endswith("greedy"):
            prm = (0.0, 0.9, 0.05, 1.1, 0.0, 0.0, 40, 64)
        else:
            prm = (0.7, 0.9, 0.05, 1.1, 0.0, 0.0, 40, 64)
    elif name == "c3_batched_hetero":
        x = g.standard_normal(V, dtype=np.float32) * np.float32(3.0)
        T = float(g.uniform(0.5, 1.2))
        k = int(g.choice([0, 20, 50, 100]))
        p = float(g.uniform(0.8, 1.0))
        mp = float(g.choice([0.0, 0.05]))
        prm = (T, p, mp, 1.1, 0.2, 0.2, k, 256)
        hist = g.integers(0, V, 256).astype(np.int64)
        bids = g.choice(V, 16, replace=False).astype(np.int64)
        bvals = g.choice([-5.0, 5.0], 16).astype(np.float64)
    elif name == "c4_qwen2_sharded":
        x = g.standard_normal(V, dtype=np.float32) * np.float32(3.0)
        heavy = g.random(V) < 0.01
        nh = int(heavy.sum())
        x[heavy] = (g.standard_t(3.0, nh) * 3.0).astype(np.float32)
        prm = (1.0, 0.95, 0.02, 1.0, 0.2, 0.2, 50, 512)
        hist = g.integers(0, V, 512).astype(np.int64)
    elif name.startswith("c5_full_vocab"):
        x = g.standard_normal(V, dtype=np.float32)
        if name.endswith("greedy"):
            prm = (0.0, 0.99, 0.0, 1.0, 0.0, 0.0, 0, 64)
        else:
            prm = (1.0, 0.99, 0.0, 1.0, 0.0, 0.0, 0, 64)
    else:
        raise KeyError(name)
    u = float(g.random())
    return x, prm, hist, bids, bvals, u


def make(name: str, seed: int = 1234, rows: Optional[np.ndarray] = None,
         V: Optional[int] = None) -> Workload:
    """Build workload `name` (all rows, or the given global row ids).
    `V` overrides the vocabulary size (parity tests at reduced size)."""
    _, B, V0 = CONFIGS[name]
    V = V0 if V is None else int(V)
    rows = np.arange(B) if rows is None else np.asarray(rows, dtype=np.int64)
    n = rows.size
    logits = np.empty((n, V), np.float32)
    params = np.zeros(n, ROW_PARAMS_DTYPE)
    hists, bidl, bvl = [], [], []
    uni = np.empty(n, np.float64)
    for i, r in enumerate(rows):
        x, prm, h, bi, bv, u = _row(name, seed, int(r), V)
        logits[i] = x
        params[i] = prm
        hists.append(h)
        bidl.append(bi)
        bvl.append(bv)
        uni[i] = u
    hist_off = np.zeros(n + 1, np.int64)
    hist_off[1:] = np.cumsum([h.size for h in hists])
    bias_off = np.zeros(n + 1, np.int64)
    bias_off[1:] = np.cumsum([b.size for b in bidl])
    hist_ids = np.concatenate(hists) if hist_off[-1] > 0 else None
    bias_ids = np.concatenate(bidl) if bias_off[-1] > 0 else None
    bias_vals = np.concatenate(bvl) if bias_off[-1] > 0 else None
    return Workload(name, logits, params, hist_ids, hist_off if hist_ids is not None else None,
                    bias_ids, bias_vals, bias_off if bias_ids is not None else None, uni, rows)


def shard_rows(B: int, rank: int, world: int) -> np.ndarray:
    """Contiguous batch shard of rank `rank` of `world` (rows are independent,
    so the batch-sharded mode needs no collective)."""
    lo = (B * rank) // world
    hi = (B * (rank + 1)) // world
    return np.arange(lo, hi, dtype=np.int64)
