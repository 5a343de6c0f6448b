#!/usr/bin/env python
"""Benchmark of the B200 token sampler (BASELINE metric: sampled rows/s at
B=256, V=128256 fp32; HBM GB/s vs peak; p50 us at B=1).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

One step = one nls_sample_batch call over one batch of the heterogeneous
configuration (B=256 rows per GPU, V=128256, per-row
temperature/top-k/top-p/min-p, penalties over a 256-token history, 16 bias
entries per row). Inputs are seeded synthetic data of that shape. With N GPUs
(torchrun) every rank samples the same 256-row batch (batch-sharded, no
collective; weak scaling with identical per-GPU work); rows are generated
from (seed, row). Config 4 (8192 rows of V = 151936) is split over the ranks
(strong scaling); at N > 1 config 5 is also run vocab-sharded, with its ids
and probabilities checked against one GPU.

`value` is whole-job rows/s with every input already in HBM, timed with CUDA
events on the launch stream, L2 flushed between steps. `e2e` is the same
metric through the public host API (pinned host logits, host params/history/
bias/uniforms, host outputs): H2D and D2H are inside its timed region.
`--impl reference` times the reference sampler's CPU restatement (oracle/) on
this host's cores over the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled rows/s at B=256,V=128256 fp32; HBM GB/s vs peak; p50 us at B=1"
WORKLOAD = "c3_batched_hetero"
SEED = 1234
L2_FLUSH_BYTES = 256 << 20


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback (6.65 TB/s, earlier pool measurement)"


def ncu_traffic():
    """Per-launch DRAM bytes of each kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


_POLL_SRC = r"""
import select, sys, time
import pynvml as nv
nv.nvmlInit()
key = sys.argv[1]
h = nv.nvmlDeviceGetHandleByUUID(key) if key.startswith("GPU-") else nv.nvmlDeviceGetHandleByPciBusId(key)
print("max", nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM), flush=True)
while True:
    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
    print("%.6f %d %d" % (time.time(), sm, rs), flush=True)
    if select.select([sys.stdin], [], [], 0.0005)[0]:
        break
"""


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of one GPU, polled through
    NVML (read-only queries) every ~0.5 ms by a separate process, so that the
    polling neither competes with the timed loop for the interpreter lock nor
    misses the short timed region. start() returns once the poller runs;
    stop() keeps the samples taken between the two calls."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake", 0x80))

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.smax = None
        self.err = None
        self.t0 = self.t1 = None

    def start(self):
        import subprocess
        import torch
        try:
            props = torch.cuda.get_device_properties(self.device)
            key = "GPU-" + str(props.uuid)
            self.proc = subprocess.Popen([sys.executable, "-c", _POLL_SRC, key], stdin=subprocess.PIPE,
                                         stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            first = self.proc.stdout.readline().split()
            if len(first) != 2 or first[0] != "max":
                raise RuntimeError("poller did not start: " + self.proc.stderr.read()[-300:])
            self.smax = int(first[1])
        except Exception as e:
            self.err = f"NVML poller unavailable: {e!r}"
            self.proc = None
        self.t0 = time.time()

    def stop(self):
        self.t1 = time.time()
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"]}
        try:
            out, _ = self.proc.communicate(input="x\n", timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        samples = []
        for line in out.splitlines():
            f = line.split()
            if len(f) == 3:
                samples.append((float(f[0]), int(f[1]), int(f[2])))
        inside = [x for x in samples if self.t0 <= x[0] <= self.t1]
        reasons = set()
        for _, _, rs in inside:
            for name, bit in self.REASONS:
                if rs & bit:
                    reasons.add(name)
        sm = [c for _, c, _ in inside]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.smax,
                "reasons": sorted(reasons), "samples": len(sm),
                "window_ms": round((self.t1 - self.t0) * 1e3, 3),
                "source": "NVML, polled every ~0.5 ms by a separate process during the timed region"}


def row_is_full(params, V):
    """The library's row split (nls_common.cuh row_mode): greedy and top-k
    rows with k <= 256 go to the streaming kernel, the rest to the full-sort
    kernel."""
    k = np.where(params["top_k"] > 0, np.minimum(params["top_k"], V), V)
    samp = params["temperature"] > 0
    return samp & ~((k < V) & (k <= 256))


def row_bytes(w):
    per = np.full(w.B, w.V * 4 + 64 + 8 + 12, dtype=np.int64)
    if w.hist_ids is not None:
        per += np.diff(w.hist_off) * 8 + 8
    if w.bias_ids is not None:
        per += np.diff(w.bias_off) * 16 + 8
    return per


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local, dist


def reduce_max(dist, value: float, device) -> float:
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_sample(oracle, w, rows: int, threads: int):
    """Time the oracle (reference sampler restatement) on `rows` rows."""
    sel = slice(0, rows)
    hoff = w.hist_off[: rows + 1] if w.hist_off is not None else None
    boff = w.bias_off[: rows + 1] if w.bias_off is not None else None
    t0 = time.perf_counter()
    ids = oracle.sample_batch(w.logits[sel], w.params[sel], w.hist_ids, hoff, w.bias_ids,
                              w.bias_vals, boff, w.uniforms[sel], threads=threads)
    return time.perf_counter() - t0, ids


def run_reference(args, world, rank, dist):
    """--impl reference: the reference sampler's CPU restatement on host cores."""
    if rank != 0:
        return 0
    from oracle import oracle
    import __graft_entry__ as g
    pkg = g.load_package()
    oracle.build()
    threads = os.cpu_count() or 1
    w = pkg.workloads.make(WORKLOAD, seed=SEED)
    for _ in range(args.warmup):
        cpu_sample(oracle, w, w.B, threads)
    times = []
    for _ in range(args.steps):
        dt, _ = cpu_sample(oracle, w, w.B, threads)
        times.append(dt)
    ms = 1e3 * statistics.mean(times)
    value = w.B / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy PCG64 per row, BASELINE config 3 shapes and "
                "distributions); uniforms: numpy PCG64, not Nim std/random",
        "config": config_dict(world),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"the full {w.B}-row batch per step, rows spread over "
                                   f"{threads} threads (C restatement of sampler.nim)"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def vocab_sharded_bench(pkg, dist, world, rank, local, dev, args):
    """Config 5 vocab-sharded over the `world` ranks: rows/s of the
    collective nls_sample_batch_vocab_sharded call (inputs resident)."""
    import torch
    name = "c5_full_vocab_nucleus"
    w = pkg.workloads.make(name, seed=SEED)
    B, V = w.B, w.V
    lo, hi = pkg.vocab_shard(V, world, rank)
    shard = torch.from_numpy(np.ascontiguousarray(w.logits[:, lo:hi])).to(dev)
    params = torch.from_numpy(w.params.view(np.uint8).copy()).to(dev)
    unif = torch.from_numpy(w.uniforms).to(dev)
    ids = torch.empty(B, dtype=torch.int64, device=dev)
    probs = torch.empty(B, dtype=torch.float32, device=dev)
    box = [pkg.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    comm = pkg.Comm(box[0], world, rank, local)
    eng = pkg.Engine(local, max_rows=B, max_vocab=V)
    stream = torch.cuda.current_stream(dev)

    def step():
        eng.sample_batch_vocab_sharded(comm, shard, V, params, uniforms=unif, out_ids=ids,
                                       out_probs=probs, stream=stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    dist.barrier()
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(args.steps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    torch.cuda.synchronize(dev)
    dist.barrier()
    ms = reduce_max(dist, statistics.mean(times), dev)
    # parity: the sharded call's ids and probabilities (all rows, on every
    # rank) against one-GPU nls_sample_batch over the whole rows on this GPU
    full = torch.from_numpy(w.logits).to(dev)
    ids1 = torch.empty(B, dtype=torch.int64, device=dev)
    probs1 = torch.empty(B, dtype=torch.float32, device=dev)
    eng.sample_batch(full, params, None, None, None, None, None, unif, out_ids=ids1, out_probs=probs1,
                     stream=stream.cuda_stream)
    torch.cuda.synchronize(dev)
    ok = float(np.array_equal(ids.cpu().numpy(), ids1.cpu().numpy()) and
               _bits_equal(probs.cpu().numpy(), probs1.cpu().numpy()))
    flag = torch.tensor([ok], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    eng.close()
    comm.close()
    return {"config": f"{name}: B={B} rows of V={V} fp32, top-k 0, top-p 0.99, T 1.0; "
                      f"the vocabulary split over {world} ranks (columns [r*Vs, (r+1)*Vs))",
            "value": B / (ms / 1e3), "unit": "rows/s", "ms_per_step": ms,
            "parity_ok": bool(flag.item() == 1.0),
            "parity": "ids and probabilities of all rows on every rank bitwise equal to one-GPU "
                      "nls_sample_batch over the whole rows",
            "method": "NCCL send/recv transpose to row owners, batch kernels, all-gather of ids"}


def b1_latency(pkg, eng, dev, stream, iters: int):
    """B=1 latency (BASELINE config 2 shape: one row, V=128256), device
    inputs: device time of a call (the library's own events from the call's
    first operation to its last kernel) and host wall-clock of a call through
    the Python binding with a stream sync."""
    import torch
    sptr = stream.cuda_stream

    def t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    w1 = pkg.workloads.make("c2_llama3_b1", seed=SEED)
    d1 = dict(logits=t(w1.logits), params=torch.from_numpy(w1.params.view(np.uint8).copy()).to(dev),
              hist_ids=t(w1.hist_ids), hist_off=t(w1.hist_off), uniforms=t(w1.uniforms))
    o1 = torch.empty(1, dtype=torch.int64, device=dev)
    p1 = torch.empty(1, dtype=torch.float32, device=dev)
    eng.set_profiling(True)
    lat, host_lat = [], []
    for i in range(iters + 10):
        t0 = time.perf_counter()
        eng.sample_batch(d1["logits"], d1["params"], d1["hist_ids"], d1["hist_off"], None, None,
                         None, d1["uniforms"], out_ids=o1, out_probs=p1, stream=sptr, check=False)
        stream.synchronize()
        t1 = time.perf_counter()
        if i >= 10:
            lat.append(eng.last_kernel_ms()[2] * 1e3)
            host_lat.append((t1 - t0) * 1e6)
    eng.set_profiling(False)
    lat.sort()
    host_lat.sort()
    return {"p50_us": lat[len(lat) // 2], "p99_us": lat[int(len(lat) * 0.99) - 1],
            "host_p50_us": host_lat[len(host_lat) // 2],
            "host_p99_us": host_lat[int(len(host_lat) * 0.99) - 1],
            "config": "c2_llama3_b1: B=1, V=128256, top-k 40, device inputs; p50/p99 = device "
                      "time of the call (library CUDA events), host_* = wall clock of the call "
                      "through the Python binding with a stream sync"}


def _dev_inputs(w, dev):
    import torch

    def t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return dict(logits=t(w.logits), params=torch.from_numpy(w.params.view(np.uint8).copy()).to(dev),
                hist_ids=t(w.hist_ids), hist_off=t(w.hist_off), bias_ids=t(w.bias_ids),
                bias_vals=t(w.bias_vals), bias_off=t(w.bias_off), uniforms=t(w.uniforms))


def _timed_calls(call, stream, steps, warmup, flush=None):
    """CUDA-event device time (ms) of each of `steps` calls after `warmup`."""
    import torch
    for _ in range(warmup):
        if flush is not None:
            flush.zero_()
        call()
    torch.cuda.synchronize()
    ms = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        call()
        e1.record(stream)
        e1.synchronize()
        ms.append(e0.elapsed_time(e1))
    return ms


def _bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


def c4_bench(pkg, dist, world, rank, local, dev, stream, args, peak):
    """BASELINE config 4 (Qwen2 vocabulary, B = 8192 rows of V = 151936, top-k
    50, min-p 0.02, frequency/presence penalties over 512 ids): the 8192 rows
    split evenly over the ranks (strong scaling, no collective). Device time
    per call, max over ranks; the streaming kernel's own time from the
    library's events; every rank checks 8 of its rows against the oracle."""
    import torch
    name = "c4_qwen2_sharded"
    B = args.c4_rows
    rows = pkg.workloads.shard_rows(B, rank, world)
    w = pkg.workloads.make_parallel(name, seed=SEED, rows=rows)
    d = _dev_inputs(w, dev)
    nb, V = w.B, w.V
    eng = pkg.Engine(local, max_rows=nb, max_vocab=V)
    ids = torch.empty(nb, dtype=torch.int64, device=dev)
    probs = torch.empty(nb, dtype=torch.float32, device=dev)
    kl = []

    def call():
        eng.sample_batch(d["logits"], d["params"], d["hist_ids"], d["hist_off"], None, None, None,
                         d["uniforms"], out_ids=ids, out_probs=probs, stream=stream.cuda_stream,
                         check=False)
    eng.set_profiling(True)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms = []
    for _ in range(args.steps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        call()
        e1.record(stream)
        kl.append(eng.last_kernel_ms()[0])
        e1.synchronize()
        ms.append(e0.elapsed_time(e1))
    st = eng._lib.nls_stream_status(eng._h, None)
    eng.set_profiling(False)
    # parity on 8 rows of this rank's shard
    from oracle import oracle
    oracle.build()
    sel = np.linspace(0, nb - 1, 8).astype(np.int64)
    sub = pkg.workloads.make(name, seed=SEED, rows=rows[sel])
    ref, dg = oracle.sample_batch(sub.logits, sub.params, sub.hist_ids, sub.hist_off, None, None, None,
                                  sub.uniforms, diag=True, threads=8)
    got_ids = ids.cpu().numpy()[sel]
    got_p = probs.cpu().numpy()[sel]
    ok = int(st == 0 and np.array_equal(got_ids, ref) and _bits_equal(got_p, dg["prob"]))
    mean_ms = statistics.mean(ms)
    light_ms = statistics.mean(kl)
    per = {"rank": rank, "rows": int(nb), "ms": mean_ms, "light_ms": light_ms}
    eng.close()
    del d
    if dist is not None:
        t = torch.tensor([float(ok)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = int(t.item())
        allp = [None] * world
        dist.all_gather_object(allp, per)
    else:
        allp = [per]
    ms_max = reduce_max(dist, mean_ms, dev)
    light_max = reduce_max(dist, light_ms, dev)
    algo = int(nb) * (V * 4 + 64 + 8 + 12 + 512 * 8 + 8)  # per rank: logits, params, uniform, out, history
    per1024 = ncu_traffic().get("light_kernel_c4_per_1024_rows")
    traffic = int(per1024 * nb / 1024) if per1024 else None
    ach = algo / (light_max / 1e3) / 1e9
    return {"config": f"{name}: B={B} rows of V={V} fp32 (N(0,3) with a Student-t(3) mixture on 1% "
                      f"of entries), T 1.0, top-k 50, top-p 0.95, min-p 0.02, freq/pres 0.2/0.2 over "
                      f"512 ids; rows split evenly over {world} rank(s) (strong scaling); inputs "
                      f"{V * 4 * int(nb) / 1e9:.2f} GB per rank (larger than the L2: no flush)",
            "value": B / (ms_max / 1e3), "unit": "rows/s", "ms_per_step": ms_max, "n_gpus": world,
            "scaling": "strong",
            "roofline": {"bound": "hbm", "kernel": "light_kernel", "achieved": ach, "peak": peak,
                         "unit": "GB/s", "frac": ach / peak, "algorithmic_bytes_per_rank": algo,
                         "ms": light_max, "traffic": traffic,
                         "traffic_source": "ncu capture of 1024 rows (profiles/light_kernel_c4.md), "
                                           "scaled by the rank's rows / 1024"},
            "parity_ok": bool(ok), "parity_rows_checked": 8 * world, "per_rank": allp}


def c5_single_gpu(pkg, local, dev, stream, args, flush):
    """BASELINE config 5 on one GPU (64 rows of V = 151936, flat N(0,1),
    top-k 0, top-p 0.99: every row takes the full sort) and its greedy
    variant; L2 flushed between calls. Returns the timings and the ids/probs
    of the sampling variant (the vocab-sharded mode's reference)."""
    import torch
    out = {}
    res = {}
    for name in ("c5_full_vocab_nucleus", "c5_full_vocab_greedy"):
        w = pkg.workloads.make(name, seed=SEED)
        d = _dev_inputs(w, dev)
        eng = pkg.Engine(local, max_rows=w.B, max_vocab=w.V)
        ids = torch.empty(w.B, dtype=torch.int64, device=dev)
        probs = torch.empty(w.B, dtype=torch.float32, device=dev)

        def call():
            eng.sample_batch(d["logits"], d["params"], None, None, None, None, None, d["uniforms"],
                             out_ids=ids, out_probs=probs, stream=stream.cuda_stream, check=False)
        ms = _timed_calls(call, stream, args.steps, args.warmup, flush)
        st = eng._lib.nls_stream_status(eng._h, None)
        eng.close()
        m = statistics.mean(ms)
        out[name] = {"value": w.B / (m / 1e3), "unit": "rows/s", "ms_per_step": m, "status": st,
                     "gb_per_s_algorithmic": w.algorithmic_bytes() / (m / 1e3) / 1e9}
        res[name] = (ids.cpu().numpy(), probs.cpu().numpy())
    out["config"] = ("c5_full_vocab_nucleus / _greedy on one GPU: B=64 rows of V=151936 fp32, N(0,1), "
                     "T 1.0, top-k 0, top-p 0.99 (greedy: T 0); L2 flushed between calls")
    return out, res


def c1_c2_extra(pkg, local, dev, stream, args, with_cpu):
    """Config 1 (V = 2000, 1000 draws from one row) as one batch of 1000 rows
    and as 1000 one-row calls; config 2's greedy variant at B = 1; and the
    oracle's time for one config-2 call and for config 1's 1000 draws on one
    host thread (the reference samples one row per call on the caller's
    thread)."""
    import torch
    sptr = stream.cuda_stream
    out = {}
    w1 = pkg.workloads.make("c1_tiny", seed=42)
    rng = np.random.default_rng(42)
    n = 1000
    uni = rng.random(n)
    logits = np.repeat(w1.logits, n, axis=0)
    params = np.repeat(w1.params, n)
    hist = np.tile(w1.hist_ids, n)
    hoff = np.arange(0, w1.hist_ids.size * n + 1, w1.hist_ids.size, dtype=np.int64)
    eng = pkg.Engine(local, max_rows=n, max_vocab=128256)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dl, dp, dh, dho, du = t(logits), t(params.view(np.uint8)), t(hist), t(hoff), t(uni)
    ids = torch.empty(n, dtype=torch.int64, device=dev)
    ms = _timed_calls(lambda: eng.sample_batch(dl, dp, dh, dho, None, None, None, du, out_ids=ids,
                                               stream=sptr, check=False), stream, args.steps, args.warmup)
    mb = statistics.mean(ms)
    # 1000 one-row calls, as the reference draws (device time of each call)
    eng.set_profiling(True)
    one = []
    o1 = torch.empty(1, dtype=torch.int64, device=dev)
    for i in range(n + 20):
        eng.sample_batch(dl[i % n:i % n + 1], dp[(i % n) * 64:(i % n + 1) * 64], dh[:64], dho[:2], None,
                         None, None, du[i % n:i % n + 1], out_ids=o1, stream=sptr, check=False)
        stream.synchronize()
        if i >= 20:
            one.append(eng.last_kernel_ms()[2] * 1e3)
    eng.set_profiling(False)
    one.sort()
    out["c1_tiny"] = {"config": "c1_tiny: one row of V=2000 N(0,2), T 0.8, top-k 40, top-p 0.95, min-p "
                                "0.05, rep 1.1 over 64 ids; 1000 draws (fresh uniforms)",
                      "batched_1000_rows": {"ms": mb, "draws_per_s": n / (mb / 1e3)},
                      "one_row_calls": {"p50_us": one[len(one) // 2], "p99_us": one[int(len(one) * 0.99) - 1]}}
    # config 2 greedy variant at B = 1
    g = pkg.workloads.make("c2_llama3_b1_greedy", seed=SEED)
    gl, gp, gh, gho = t(g.logits), t(g.params.view(np.uint8)), t(g.hist_ids), t(g.hist_off)
    eng.set_profiling(True)
    lat = []
    for i in range(args.latency_iters + 10):
        eng.sample_batch(gl, gp, gh, gho, None, None, None, None, out_ids=o1, stream=sptr, check=False)
        stream.synchronize()
        if i >= 10:
            lat.append(eng.last_kernel_ms()[2] * 1e3)
    eng.set_profiling(False)
    lat.sort()
    out["c2_greedy_b1"] = {"p50_us": lat[len(lat) // 2], "p99_us": lat[int(len(lat) * 0.99) - 1],
                           "config": "c2_llama3_b1_greedy: B=1, V=128256, T 0 (argmax after the "
                                     "repeat penalty), device inputs; device time of a call"}
    eng.close()
    if with_cpu:
        from oracle import oracle
        oracle.build()
        w2 = pkg.workloads.make("c2_llama3_b1", seed=SEED)
        cl = []
        for i in range(25):
            t0 = time.perf_counter()
            oracle.sample_batch(w2.logits, w2.params, w2.hist_ids, w2.hist_off, None, None, None,
                                w2.uniforms, threads=1)
            if i >= 5:
                cl.append((time.perf_counter() - t0) * 1e6)
        cl.sort()
        t0 = time.perf_counter()
        for i in range(n):
            oracle.sample_batch(w1.logits, w1.params, w1.hist_ids, w1.hist_off, None, None, None,
                                uni[i:i + 1], threads=1)
        c1s = time.perf_counter() - t0
        out["cpu"] = {"kind": "port", "cores": 1,
                      "c2_one_call_p50_us": cl[len(cl) // 2],
                      "c1_1000_draws_ms": c1s * 1e3,
                      "sample": "C restatement of sampler.nim (oracle/) on one host thread: 20 "
                                "config-2 calls, and config 1's 1000 draws one call each"}
    return out



def lm_head_bench(pkg, local, dev, stream, peak, with_cpu: bool):
    """The output projection that feeds the sampler (nls_lm_head, model.nim:
    466-470 -> matmul :179-189) on the Llama-3 output layer, 128256 x 4096,
    weights resident in HBM: device time of one call (CUDA events on the
    call's stream; the weights, 431-1051 MB, are 3-8x the 126 MB L2, so no
    flush between calls: a flush by writing would leave L2 full of dirty
    lines whose write-back the timed call would pay), the weight bytes it streams,
    and the fused projection + sampling call at B = 1. With with_cpu, the
    oracle's matmul (all host threads) on the same weights, one call."""
    import torch
    rows, cols = 128256, 4096
    sptr = stream.cuda_stream
    eng = pkg.Engine(local, max_rows=8, max_vocab=rows)
    L = eng._lib
    W = pkg.workloads
    out = {"config": "nls_lm_head: rows=128256 (vocab) x cols=4096 (Llama-3 8B output layer), "
                     "ggml-layout synthetic weights resident on the device (Q8_0 at 1-4 rows or rows "
                     "that are separate sequences, Q6_K, Q4_0: int8 path, on the tensor cores from 8 "
                     "rows; Q8_0 above 4 rows of one sequence, F16: float path), fp32 activations on "
                     "the device; weights 3-8x the L2, no flush between calls",
           "peak_gbs": peak}
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED)
    for name in ("q8_0", "q6_k", "q4_0", "f16"):
        t = W.LM_TYPES[name]
        wd = W.lm_weights_device(t, rows, cols, seed=SEED, device=dev)
        wbytes = rows * W.lm_row_bytes(t, cols)
        res = {"weight_bytes": wbytes}
        # (Q6_K and Q4_0 at 8 and 16 batch rows, and Q8_0 rows that are
        # separate sequences ("_independent", NLS_ROWS_INDEPENDENT): the
        # tensor-core path; Q8_0 above 4 rows of one sequence and F16: the
        # float path, tiled across batch rows above 1)
        legs = {"q8_0": ((1, 0), (4, 0), (8, 0), (16, 0), (8, 8), (16, 8)),
                "q6_k": ((1, 0), (4, 0), (8, 0), (16, 0)),
                "q4_0": ((1, 0), (8, 0), (16, 0)),
                "f16": ((1, 0), (4, 0), (16, 0))}[name]
        for nb, fl in legs:
            x = torch.randn((nb, cols), generator=gen, device=dev)
            y = torch.empty((nb, rows), dtype=torch.float32, device=dev)

            def call():
                return L.nls_lm_head(eng._h, ctypes.c_void_p(wd.data_ptr()), t, rows, cols,
                                     ctypes.c_void_p(x.data_ptr()), nb, ctypes.c_void_p(y.data_ptr()),
                                     3 | fl, ctypes.c_void_p(sptr))
            for _ in range(3):
                if call() != 0:
                    raise RuntimeError("nls_lm_head failed")
            ms = []
            for _ in range(10):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                call()
                e1.record(stream)
                e1.synchronize()
                ms.append(e0.elapsed_time(e1))
            if L.nls_stream_status(eng._h, ctypes.c_void_p(sptr)) != 0:
                raise RuntimeError("nls_lm_head status")
            ms.sort()
            m = ms[len(ms) // 2]
            # algorithmic bytes: the weights once, the activations, the logits
            algo = wbytes + nb * cols * 4 + nb * rows * 4
            gbs = algo / (m / 1e3) / 1e9
            res[f"nb{nb}" + ("_independent" if fl else "")] = {
                "ms": m, "algorithmic_bytes": algo, "achieved_gbs": gbs, "frac": gbs / peak}
            if name == "q8_0" and nb == 1:
                tr = ncu_traffic().get("lmh_kernel_q8_0_nb1")
                out["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                   "frac": gbs / peak, "traffic": tr, "kernel": "lmh_kernel",
                                   "case": "q8_0 nb=1"}
        if name == "q8_0":
            # projection + sampling of one decode row (config 2's sampling
            # parameters: T 0.7, top-k 40, top-p 0.9, min-p 0.05, rep 1.1)
            s = pkg.workloads.make("c2_llama3_b1", seed=SEED)
            prm = torch.from_numpy(s.params.view(np.uint8).copy()).to(dev)
            hid = torch.from_numpy(s.hist_ids).to(dev)
            hof = torch.from_numpy(s.hist_off).to(dev)
            uni = torch.from_numpy(s.uniforms).to(dev)
            x1 = torch.randn((1, cols), generator=gen, device=dev)
            oid = torch.empty(1, dtype=torch.int64, device=dev)

            def fused():
                return L.nls_lm_head_sample(
                    eng._h, ctypes.c_void_p(wd.data_ptr()), t, rows, cols, ctypes.c_void_p(x1.data_ptr()), 1,
                    ctypes.c_void_p(prm.data_ptr()), ctypes.c_void_p(hid.data_ptr()),
                    ctypes.c_void_p(hof.data_ptr()), None, None, None, ctypes.c_void_p(uni.data_ptr()),
                    ctypes.c_void_p(oid.data_ptr()), None, 3, ctypes.c_void_p(sptr))
            for _ in range(3):
                if fused() != 0:
                    raise RuntimeError("nls_lm_head_sample failed")
            ms = []
            for _ in range(20):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fused()
                e1.record(stream)
                e1.synchronize()
                ms.append(e0.elapsed_time(e1))
            if L.nls_stream_status(eng._h, ctypes.c_void_p(sptr)) != 0:
                raise RuntimeError("nls_lm_head_sample status")
            ms.sort()
            res["with_sampling_b1_ms"] = ms[len(ms) // 2]
        if with_cpu and name in ("q8_0", "q6_k"):
            from oracle import oracle
            oracle.build()
            threads = os.cpu_count() or 1
            wh = wd.cpu().numpy()
            xh = np.random.default_rng(SEED).standard_normal((1, cols)).astype(np.float32)
            oracle.lm_head(wh[:1024], t, 1024, cols, xh, threads=threads)  # warm
            t0 = time.perf_counter()
            oracle.lm_head(wh, t, rows, cols, xh, threads=threads)
            dt = time.perf_counter() - t0
            res["cpu"] = {"ms": dt * 1e3, "threads": threads, "kind": "port",
                          "sample": "one call, nb=1 (C restatement of matmul, oracle/ref_lmhead.c)"}
            del wh
        out[name] = res
        del wd
    eng.close()
    return out


def config_dict(world):
    return {"workload": f"{WORKLOAD}: B=256 rows per GPU, V=128256 fp32, per-row T~U[0.5,1.2], "
                        "top-k in {0,20,50,100}, top-p~U[0.8,1], min-p in {0,0.05}, "
                        "rep/freq/pres 1.1/0.2/0.2 over 256 ids, 16 bias entries",
            "rows_per_gpu": 256, "vocab": 128256,
            "parallelism": f"batch-sharded x{world} (no collective); every rank samples the same "
                           "256-row batch (identical per-GPU work)",
            "l2": "flushed between steps (256 MiB write, outside the step events)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)  # (a timed region of ~0.1 s: clock samples)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-lm-head", action="store_true",
                    help="skip the output-projection timing (nls_lm_head)")
    ap.add_argument("--latency-only", action="store_true",
                    help="run only the B=1 latency loop and print it")
    ap.add_argument("--lm-head-only", action="store_true",
                    help="run only the output-projection timing and print it")
    ap.add_argument("--latency-iters", type=int, default=200)
    ap.add_argument("--no-vocab-sharded", action="store_true",
                    help="skip the vocab-sharded (config 5) measurement at N > 1")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the config 1/2-greedy/4/5 legs")
    ap.add_argument("--c4-only", action="store_true",
                    help="run only the config-4 leg (rows split over the ranks) and print it")
    ap.add_argument("--c4-rows", type=int, default=8192,
                    help="config-4 rows in total (8192 is the configuration; fewer for ncu captures)")
    ap.add_argument("--kernels-only", action="store_true",
                    help="only the device-resident steps (for ncu captures); prints a short line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world, rank, local, dist = dist_setup(args)
    if args.impl == "reference":
        rc = run_reference(args, world, rank, dist)
        if dist is not None:
            dist.destroy_process_group()
        return rc

    import torch
    import __graft_entry__ as g
    pkg = g.load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    if args.latency_only:
        # only the B=1 latency loop (a short command for profiling)
        if rank == 0:
            eng1 = pkg.Engine(local, max_rows=8, max_vocab=128256)
            print(json.dumps({"latency_b1": b1_latency(pkg, eng1, dev, stream, args.latency_iters)}),
                  flush=True)
            eng1.close()
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    if args.c4_only:
        peak, _ = peaks()
        c4 = c4_bench(pkg, dist, world, rank, local, dev, stream, args, peak)
        if rank == 0:
            print(json.dumps({"c4_qwen2_sharded": c4}), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    if args.lm_head_only:
        # only the output-projection timing (a short command for profiling)
        if rank == 0:
            peak, _ = peaks()
            print(json.dumps({"lm_head": lm_head_bench(pkg, local, dev, stream, peak,
                                                       with_cpu=not args.no_cpu_baseline)}),
                  flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # Weak scaling: every rank samples the same 256-row batch (rows 0..255 of
    # the configuration), so per-GPU work is identical as N grows and the
    # max over ranks measures the system rather than which rank drew the
    # slowest full-sort row.
    B = 256
    rows = np.arange(B, dtype=np.int64)
    w = pkg.workloads.make(WORKLOAD, seed=SEED, rows=rows)
    eng = pkg.Engine(local, max_rows=B, max_vocab=w.V)

    def t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    d = dict(logits=t(w.logits), params=torch.from_numpy(w.params.view(np.uint8).copy()).to(dev),
             hist_ids=t(w.hist_ids), hist_off=t(w.hist_off), bias_ids=t(w.bias_ids),
             bias_vals=t(w.bias_vals), bias_off=t(w.bias_off), uniforms=t(w.uniforms))
    out_ids = torch.empty(B, dtype=torch.int64, device=dev)
    out_probs = torch.empty(B, dtype=torch.float32, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step():
        eng.sample_batch(d["logits"], d["params"], d["hist_ids"], d["hist_off"], d["bias_ids"],
                         d["bias_vals"], d["bias_off"], d["uniforms"], out_ids=out_ids,
                         out_probs=out_probs, stream=sptr, check=False)

    eng.set_profiling(True)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    st = eng._lib.nls_stream_status(eng._h, None)
    if st != 0:
        raise RuntimeError(f"warm-up status {st}")

    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    step_ms, k_light, k_full, host_us = [], [], [], []
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h0 = time.perf_counter()
        step()
        host_us.append((time.perf_counter() - h0) * 1e6)
        e1.record(stream)
        kl, kf, _ = eng.last_kernel_ms()
        e1.synchronize()
        step_ms.append(e0.elapsed_time(e1))
        k_light.append(kl)
        k_full.append(kf)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    clk = clocks.stop()
    st = eng._lib.nls_stream_status(eng._h, None)
    if st != 0:
        raise RuntimeError(f"timed-run status {st}")

    ms = reduce_max(dist, statistics.mean(step_ms), dev)
    value = B * world / (ms / 1e3)
    # per-rank diagnostics: each rank's own step, kernel and host launch times
    mine = {"rank": rank, "ms_mean": statistics.mean(step_ms), "ms_max": max(step_ms),
            "light_ms": statistics.mean(k_light), "full_ms": statistics.mean(k_full),
            "host_launch_us": statistics.median(host_us),
            "full_rows": int(row_is_full(w.params, w.V).sum())}
    if dist is not None:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine)
    else:
        per_rank = [mine]
    if args.kernels_only:
        if rank == 0:
            print(json.dumps({"kernels_only": True, "ms_per_step": ms, "value": value,
                              "light_ms": statistics.mean(k_light), "full_ms": statistics.mean(k_full)}))
        eng.close()
        if dist is not None:
            dist.destroy_process_group()
        return 0

    # roofline of each kernel: algorithmic bytes of the rows it serves / its time
    peak, peak_src = peaks()
    full_rows = row_is_full(w.params, w.V)
    rb = row_bytes(w)
    traffic = ncu_traffic()
    kern = {
        "light_kernel": (int(rb[~full_rows].sum()), statistics.mean(k_light), int((~full_rows).sum())),
        "full_kernel": (int(rb[full_rows].sum()), statistics.mean(k_full), int(full_rows.sum())),
    }
    roof = {}
    for name, (nbytes, kms, nrows) in kern.items():
        ach = nbytes / (kms / 1e3) / 1e9 if kms > 0 else 0.0
        tr = traffic.get(name)
        roof[name] = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                      "frac": ach / peak, "traffic": tr, "rows": nrows, "ms": kms,
                      "algorithmic_bytes": nbytes, "peak_source": peak_src}
    dominant = max(roof, key=lambda n: roof[n]["ms"])
    step_bytes = int(rb.sum())
    step_roof = {"achieved": step_bytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                 "frac": step_bytes / (ms / 1e3) / 1e9 / peak, "algorithmic_bytes": step_bytes}

    # e2e through the host API: pinned host logits, host outputs, synchronous call
    pinned = torch.empty((B, w.V), dtype=torch.float32, pin_memory=True)
    pinned.numpy()[:] = w.logits
    host_logits = pinned.numpy()
    e2e_times = []
    for i in range(args.e2e_steps + 1):
        t0 = time.perf_counter()
        ids_h, probs_h, st = eng.sample_batch(host_logits, w.params, w.hist_ids, w.hist_off,
                                              w.bias_ids, w.bias_vals, w.bias_off, w.uniforms,
                                              want_probs=True)
        dt = time.perf_counter() - t0
        if i > 0:
            e2e_times.append(dt)
    e2e_s = reduce_max(dist, statistics.mean(e2e_times), dev)
    h2d = w.logits.nbytes + w.params.nbytes + w.uniforms.nbytes + \
        (w.hist_ids.nbytes + w.hist_off.nbytes if w.hist_ids is not None else 0) + \
        (w.bias_ids.nbytes + w.bias_vals.nbytes + w.bias_off.nbytes if w.bias_ids is not None else 0)
    d2h = ids_h.nbytes + probs_h.nbytes + 4
    # device and host paths must agree
    assert np.array_equal(ids_h, out_ids.cpu().numpy()), "host and device paths differ"

    latency = b1_latency(pkg, eng, dev, stream, args.latency_iters)

    # perplexity's per-position term over one nCtx-512 chunk (511 positions,
    # V = 128256), device inputs and outputs: device time of a call
    nll = None
    if rank == 0:
        T1 = 511
        gen = torch.Generator(device=dev)
        gen.manual_seed(SEED)
        xl = torch.randn((T1, w.V), generator=gen, device=dev) * 3.0
        tg = torch.randint(0, w.V, (T1,), generator=gen, device=dev)
        on = torch.empty(T1, dtype=torch.float64, device=dev)
        eng_n = pkg.Engine(local, max_rows=T1, max_vocab=w.V)
        L = eng_n._lib

        def nll_call():
            return L.nls_token_nll(eng_n._h, ctypes.c_void_p(xl.data_ptr()), w.V, T1, w.V,
                                   ctypes.c_void_p(tg.data_ptr()), ctypes.c_void_p(on.data_ptr()),
                                   3, ctypes.c_void_p(sptr))
        for _ in range(3):
            nll_call()
        nms = []
        for _ in range(10):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            nll_call()
            e1.record(stream)
            e1.synchronize()
            nms.append(e0.elapsed_time(e1))
        if L.nls_stream_status(eng_n._h, ctypes.c_void_p(sptr)) != 0:
            raise RuntimeError("token_nll status")
        eng_n.close()
        nms.sort()
        nbytes = T1 * w.V * 4 + T1 * 16
        nll = {"ms": nms[len(nms) // 2], "positions_per_s": T1 / (nms[len(nms) // 2] / 1e3),
               "achieved_gbs": nbytes / (nms[len(nms) // 2] / 1e3) / 1e9, "peak_gbs": peak,
               "config": "nls_token_nll (perplexity's per-position term, model.nim:580-584): "
                         "511 positions x V=128256 fp32, device inputs, L2 flushed before each call"}

    # the output projection feeding the sampler (the next row of the path):
    # a one-GPU kernel timing, so only in the N = 1 run
    lmh = None
    if rank == 0 and world == 1 and not args.no_lm_head:
        lmh = lm_head_bench(pkg, local, dev, stream, peak,
                            with_cpu=(world == 1 and not args.no_cpu_baseline))

    # Vocab-sharded mode (BASELINE config 5 over the N ranks: B = 64 rows of
    # V = 151936, each rank holding its columns of every row): device time of
    # one collective call, max over ranks.
    vsh = None
    if world > 1 and not args.no_vocab_sharded:
        vsh = vocab_sharded_bench(pkg, dist, world, rank, local, dev, args)

    # the other BASELINE configurations
    c4 = c5 = extra = None
    if not args.no_configs:
        c4 = c4_bench(pkg, dist, world, rank, local, dev, stream, args, peak)
        if rank == 0 and world == 1:
            c5, _ = c5_single_gpu(pkg, local, dev, stream, args, flush)
            extra = c1_c2_extra(pkg, local, dev, stream, args, with_cpu=not args.no_cpu_baseline)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        oracle.build()
        threads = os.cpu_count() or 1
        cpu_sample(oracle, w, 32, threads)  # warm
        # the whole batch, repeated until about 10 s of CPU time (threads x wall)
        dt, ref_ids = cpu_sample(oracle, w, B, threads)
        reps, total = 1, dt
        while total * threads < 10.0 and reps < 64:
            total += cpu_sample(oracle, w, B, threads)[0]
            reps += 1
        cpu = {"value": B * reps / total, "unit": "rows/s", "cores": threads, "kind": "port",
               "sample": f"the same {B}-row batch {reps} times ({total:.1f} s wall, rows spread "
                         f"over {threads} threads; C restatement of sampler.nim, oracle/)"}
        cpu["matches_gpu_rows"] = int((ref_ids == ids_h).sum())

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy PCG64 per row, BASELINE config 3 shapes and "
                    "distributions); uniforms: numpy PCG64, not Nim std/random",
            "config": config_dict(world),
            "roofline": dict(roof[dominant], kernel=dominant),
            "roofline_kernels": roof,
            "step_roofline": step_roof,
            "cpu_baseline": cpu,
            "e2e": {"value": B * world / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_s * 1e3},
            "gpu_launches": 3 * args.steps,
            "latency_b1": latency,
            "clocks": clk,
            "vocab_sharded": vsh,
            "per_rank": per_rank,
            "step_ms_median_over_ranks": statistics.median([r["ms_mean"] for r in per_rank]),
            "configs": {"c4_qwen2_sharded": c4, "c5_single_gpu": c5,
                        "c1_c2": extra},
            "token_nll": nll,
            "lm_head": lmh,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
