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


def make_parallel(name: str, seed: int = 1234, rows: Optional[np.ndarray] = None,
                  V: Optional[int] = None, threads: int = 0, block: int = 64) -> Workload:
    """`make` with the rows generated in blocks on a thread pool (numpy's
    generators release the GIL while they fill arrays); identical values."""
    import concurrent.futures
    import os
    _, B, _ = CONFIGS[name]
    rows = np.arange(B) if rows is None else np.asarray(rows, dtype=np.int64)
    threads = threads or (os.cpu_count() or 1)
    if threads <= 1 or rows.size <= block:
        return make(name, seed, rows, V)
    parts = [rows[i:i + block] for i in range(0, rows.size, block)]
    with concurrent.futures.ThreadPoolExecutor(max_workers=threads) as ex:
        ws = list(ex.map(lambda r: make(name, seed, r, V), parts))
    logits = np.concatenate([w.logits for w in ws])
    params = np.concatenate([w.params for w in ws])
    uni = np.concatenate([w.uniforms for w in ws])

    def csr(ids_of, off_of, vals_of=None):
        if ids_of(ws[0]) is None:
            return None, None, None
        ids = np.concatenate([ids_of(w) for w in ws])
        counts = np.concatenate([np.diff(off_of(w)) for w in ws])
        off = np.zeros(rows.size + 1, np.int64)
        off[1:] = np.cumsum(counts)
        vals = np.concatenate([vals_of(w) for w in ws]) if vals_of else None
        return ids, off, vals

    hid, hoff, _ = csr(lambda w: w.hist_ids, lambda w: w.hist_off)
    bid, boff, bval = csr(lambda w: w.bias_ids, lambda w: w.bias_off, lambda w: w.bias_vals)
    return Workload(name, logits, params, hid, hoff, bid, bval, boff, uni, rows)


def shard_rows(B: int, rank: int, world: int) -> np.ndarray:
    """Contiguous batch shard of rank `rank` of `world` (rows are independent,
    so the batch-sharded mode needs no collective)."""
    lo = (B * rank) // world
    hi = (B * (rank + 1)) // world
    return np.arange(lo, hi, dtype=np.int64)


# ---- output-projection weights (ggml layout) ---------------------------------
# Synthetic weights for nls_lm_head: seeded bytes in the block layout of each
# ggml type (quant.nim:160-202, 303-321). Values are drawn directly as the
# stored integers and fp16 scales (no float weights are quantised), scaled so
# that logits of a unit-normal hidden state have a standard deviation near
# 1-2, like a trained output layer's.

LM_TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q6_k": 14}
_BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 14: (256, 210)}


def lm_row_bytes(wtype: int, cols: int) -> int:
    bv, bb = _BLOCK[wtype]
    if cols % bv:
        raise ValueError(f"cols={cols} is not a whole number of {bv}-value blocks")
    return cols // bv * bb


def _f16_bytes(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a.astype("<f2")).view(np.uint8)


def lm_weights(wtype: int, rows: int, cols: int, seed: int = 7, sigma: float = 0.02) -> np.ndarray:
    """[rows, rowBytes] uint8 weights of `wtype`, seeded."""
    rng = np.random.default_rng([seed, wtype, rows, cols])
    if wtype == 0:
        return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma)).view(np.uint8)
    if wtype == 1:
        return _f16_bytes(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma)).reshape(rows, -1)
    bv, bb = _BLOCK[wtype]
    nblk = cols // bv
    out = np.empty((rows, nblk, bb), dtype=np.uint8)
    u = rng.uniform(0.5, 1.5, size=(rows, nblk)).astype(np.float32)
    if wtype == 8:
        out[:, :, 0:2] = _f16_bytes(u * np.float32(sigma / 73.0)).reshape(rows, nblk, 2)
        out[:, :, 2:] = rng.integers(-128, 128, size=(rows, nblk, 32), dtype=np.int8).view(np.uint8)
    elif wtype == 2:
        out[:, :, 0:2] = _f16_bytes(u * np.float32(sigma / 4.6)).reshape(rows, nblk, 2)
        out[:, :, 2:] = rng.integers(0, 256, size=(rows, nblk, 16), dtype=np.uint8)
    else:  # Q6_K: ql[128] qh[64] int8 scales[16] d
        out[:, :, 0:192] = rng.integers(0, 256, size=(rows, nblk, 192), dtype=np.uint8)
        out[:, :, 192:208] = rng.integers(-64, 64, size=(rows, nblk, 16), dtype=np.int8).view(np.uint8)
        out[:, :, 208:210] = _f16_bytes(u * np.float32(sigma / (18.5 * 37.0))).reshape(rows, nblk, 2)
    return out.reshape(rows, nblk * bb)


def lm_weights_device(wtype: int, rows: int, cols: int, seed: int = 7, sigma: float = 0.02,
                      device: str = "cuda"):
    """The same kind of weights generated on the GPU with torch (for
    full-size benchmarks, where host generation and a copy would take long);
    not bit-identical to lm_weights."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) * 1000003 + int(wtype) * 7919 + rows * 31 + cols)
    if wtype in (0, 1):
        w = torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32) * sigma
        w = w if wtype == 0 else w.to(torch.float16)
        return w.view(torch.uint8).reshape(rows, -1)
    bv, bb = _BLOCK[wtype]
    nblk = cols // bv
    out = torch.empty((rows, nblk, bb), dtype=torch.uint8, device=device)
    u = torch.rand((rows, nblk), generator=g, device=device) + 0.5
    scale = {8: sigma / 73.0, 2: sigma / 4.6, 14: sigma / (18.5 * 37.0)}[wtype]
    d = (u * scale).to(torch.float16).view(torch.uint8).reshape(rows, nblk, 2)
    if wtype == 8:
        out[:, :, 0:2] = d
        out[:, :, 2:] = torch.randint(0, 256, (rows, nblk, 32), generator=g, device=device,
                                      dtype=torch.uint8)
    elif wtype == 2:
        out[:, :, 0:2] = d
        out[:, :, 2:] = torch.randint(0, 256, (rows, nblk, 16), generator=g, device=device,
                                      dtype=torch.uint8)
    else:
        out[:, :, 0:192] = torch.randint(0, 256, (rows, nblk, 192), generator=g, device=device,
                                         dtype=torch.uint8)
        out[:, :, 192:208] = (torch.randint(-64, 64, (rows, nblk, 16), generator=g, device=device,
                                            dtype=torch.int16) & 0xFF).to(torch.uint8)
        out[:, :, 208:210] = d
    return out.reshape(rows, nblk * bb)
