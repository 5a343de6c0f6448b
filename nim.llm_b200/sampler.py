"""Host-side mirror of nimllm's sampler API over the C ABI.

Mirrors src/nimllm/sampler.nim (reference repository): the same names,
argument meaning and state -- `SamplerParams` (:11-21), `Sampler` with
`params`, `rng` and `history` (:23-26), `defaultSampling` (:28-31),
`greedySampling` (:33-35), `newSampler` (:37-39), `accept` (:41-43),
`argmax` (:45-49) and `sample` (:59-121). Every sampling decision is made by
libnimllm_sample.so on the GPU; this module only keeps the host state the
Nim `Sampler` keeps (params, history, RNG) and marshals one call.

`Engine` is the batched entry (one call samples B independent rows), used
by the bench and the parity tests; it accepts numpy arrays (host memory) or
torch CUDA tensors (device memory, NLS_DEVICE_INPUTS).
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Optional

import numpy as np

from . import _abi
from ._abi import NlsError, ROW_PARAMS_DTYPE


# ---------------------------------------------------------------------------
# SamplerParams and presets (sampler.nim:11-35)
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class SamplerParams:
    temperature: float = 0.0
    topK: int = 0
    topP: float = 0.0
    minP: float = 0.0
    repeatPenalty: float = 0.0
    repeatLastN: int = 0
    presencePenalty: float = 0.0
    frequencyPenalty: float = 0.0
    seed: int = 0
    logitBias: dict = dataclasses.field(default_factory=dict)


def defaultSampling() -> SamplerParams:
    return SamplerParams(temperature=0.7, topK=40, topP=0.95, minP=0.05,
                         repeatPenalty=1.1, repeatLastN=64, seed=-1)


def greedySampling() -> SamplerParams:
    return SamplerParams(temperature=0.0, topK=0, topP=1.0, repeatPenalty=1.0, seed=0)


def params_record(p: SamplerParams) -> np.void:
    """The 64-byte nls_row_params record of a SamplerParams."""
    rec = np.zeros(1, ROW_PARAMS_DTYPE)
    rec[0] = (p.temperature, p.topP, p.minP, p.repeatPenalty, p.presencePenalty,
              p.frequencyPenalty, p.topK, p.repeatLastN)
    return rec[0]


class Rand:
    """Uniform source for `Sampler.rng`: `rand(1.0)` returns a float in [0, 1).

    The reference draws with Nim's std/random; its stream cannot be produced
    without Nim, so this default is numpy's PCG64 seeded from `seed` (seed < 0:
    OS entropy). Any object with a `rand(max)` method can replace it, e.g. one
    replaying uniforms recorded from a Nim program."""

    def __init__(self, seed: int | None = None):
        self._g = np.random.default_rng(None if seed is None or seed < 0 else seed)

    def rand(self, maxv: float = 1.0) -> float:
        return float(self._g.random()) * maxv


# ---------------------------------------------------------------------------
# Engine: one handle of the C library
# ---------------------------------------------------------------------------
def _host_ptr(a: Optional[np.ndarray]):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


class Engine:
    """Owns one nls_handle (device staging and scratch) on `device`."""

    def __init__(self, device: int = 0, max_rows: int = 256, max_vocab: int = 131072):
        self._lib = _abi.load()
        h = ctypes.c_void_p()
        st = self._lib.nls_create(ctypes.byref(h), int(device), int(max_rows), int(max_vocab))
        if st != 0:
            raise NlsError(st, "nls_create")
        self._h = h
        self.device = device
        self.max_rows = max_rows
        self.max_vocab = max_vocab

    def close(self):
        if getattr(self, "_h", None):
            self._lib.nls_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self) -> str:
        return self._lib.nls_last_error(self._h).decode()

    def _check(self, st: int, what: str):
        if st != 0:
            raise NlsError(st, f"{what}: {self.last_error()}" if st == _abi.NLS_ERR_CUDA else what)

    # -- batched sampling ---------------------------------------------------
    def sample_batch(self, logits, params, hist_ids=None, hist_off=None, bias_ids=None,
                     bias_vals=None, bias_off=None, uniforms=None, want_probs: bool = False,
                     out_ids=None, out_probs=None, stream: int = 0, check: bool = True):
        """Sample one token per row.

        Host path: numpy arrays (logits [B, V] fp32, params ROW_PARAMS_DTYPE
        [B], CSR int64 histories and bias lists, float64 uniforms); returns
        (ids int64[B], probs float32[B] or None) and the status.
        Device path: torch CUDA tensors for every input (params as an int8/uint8
        tensor of B*64 bytes or a float64 [B, 8] view); outputs must be given
        as CUDA tensors; the call is stream-ordered (check=False returns the
        status without waiting)."""
        if _is_torch(logits):
            return self._sample_batch_device(logits, params, hist_ids, hist_off, bias_ids, bias_vals,
                                             bias_off, uniforms, out_ids, out_probs, stream, check)
        logits = np.asarray(logits, dtype=np.float32)
        if logits.ndim == 1:
            logits = logits[None, :]
        B, V = logits.shape
        if logits.strides[1] != 4 or (B > 1 and (logits.strides[0] % 4 or logits.strides[0] < 4 * V)):
            logits = np.ascontiguousarray(logits)
        ld = V if B == 1 else logits.strides[0] // 4
        params = np.ascontiguousarray(params, dtype=ROW_PARAMS_DTYPE)
        assert params.shape == (B,)
        if hist_ids is not None:
            hist_ids = np.ascontiguousarray(hist_ids, dtype=np.int64)
            hist_off = np.ascontiguousarray(hist_off, dtype=np.int64)
        if bias_ids is not None:
            bias_ids = np.ascontiguousarray(bias_ids, dtype=np.int64)
            bias_vals = np.ascontiguousarray(bias_vals, dtype=np.float64)
            bias_off = np.ascontiguousarray(bias_off, dtype=np.int64)
        if uniforms is not None:
            uniforms = np.ascontiguousarray(uniforms, dtype=np.float64)
        ids = np.empty(B, dtype=np.int64)
        probs = np.empty(B, dtype=np.float32) if want_probs else None
        st = self._lib.nls_sample_batch(
            self._h, _host_ptr(logits), ld, B, V, _host_ptr(params), _host_ptr(hist_ids),
            _host_ptr(hist_off), _host_ptr(bias_ids), _host_ptr(bias_vals), _host_ptr(bias_off),
            _host_ptr(uniforms), _host_ptr(ids), _host_ptr(probs), 0, ctypes.c_void_p(stream))
        if check:
            self._check(st, "nls_sample_batch")
        return ids, probs, st

    def _sample_batch_device(self, logits, params, hist_ids, hist_off, bias_ids, bias_vals, bias_off,
                             uniforms, out_ids, out_probs, stream, check):
        def dp(t):
            return None if t is None else ctypes.c_void_p(t.data_ptr())
        B, V = logits.shape
        ld = logits.stride(0)
        assert logits.stride(1) == 1
        st = self._lib.nls_sample_batch(
            self._h, dp(logits), ld, B, V, dp(params), dp(hist_ids), dp(hist_off), dp(bias_ids),
            dp(bias_vals), dp(bias_off), dp(uniforms), dp(out_ids), dp(out_probs),
            _abi.NLS_DEVICE_INPUTS | _abi.NLS_DEVICE_OUTPUTS, ctypes.c_void_p(stream))
        if check:
            self._check(st, "nls_sample_batch")
            st = self._lib.nls_stream_status(self._h, ctypes.c_void_p(stream))
            self._check(st, "nls_sample_batch (kernel status)")
        return out_ids, out_probs, st

    def sample_batch_vocab_sharded(self, comm: "Comm", logits_shard, vocab: int, params,
                                   hist_ids=None, hist_off=None, bias_ids=None, bias_vals=None,
                                   bias_off=None, uniforms=None, out_ids=None, out_probs=None,
                                   stream: int = 0):
        """Vocab-sharded sampling (collective over `comm`): `logits_shard` is
        this rank's columns [rank*Vs, ...) of every row as a CUDA tensor
        [B, >= its column count]; every other input is the same on every rank
        (CUDA tensors, global token ids). out_ids (and out_probs) receive all
        rows on every rank. Synchronous; raises on any rank's error."""
        def dp(t):
            return None if t is None else ctypes.c_void_p(t.data_ptr())
        B = logits_shard.shape[0]
        assert logits_shard.stride(1) == 1
        st = self._lib.nls_sample_batch_vocab_sharded(
            self._h, comm._c, dp(logits_shard), logits_shard.stride(0), B, int(vocab), dp(params),
            dp(hist_ids), dp(hist_off), dp(bias_ids), dp(bias_vals), dp(bias_off), dp(uniforms),
            dp(out_ids), dp(out_probs), ctypes.c_void_p(stream))
        self._check(st, "nls_sample_batch_vocab_sharded")
        return out_ids, out_probs

    def set_wait_limit(self, ns: int) -> None:
        """Limit of the streaming kernel's bulk-copy waits, in ns (default
        200 ms); 0 makes every such wait give up (nls_set_wait_limit)."""
        self._check(self._lib.nls_set_wait_limit(self._h, int(ns)), "nls_set_wait_limit")

    def set_profiling(self, on: bool = True) -> None:
        self._check(self._lib.nls_set_profiling(self._h, 1 if on else 0), "nls_set_profiling")

    def last_kernel_ms(self) -> tuple[float, float, float]:
        """Device ms of the last profiled call, each from the call's start: to
        the end of the streaming kernel, of the (concurrent) full-sort kernel,
        and of the call's last kernel."""
        out = (ctypes.c_float * 3)()
        self._check(self._lib.nls_last_kernel_ms(self._h, out, 3), "nls_last_kernel_ms")
        return float(out[0]), float(out[1]), float(out[2])

    def top_tokens(self, logits, n: int = 5):
        """topTokens per row (host numpy [B, V] or [V]): returns (ids int64
        [B, n], probs float32 [B, n]); entries past min(n, V) are -1 / 0."""
        logits = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
        if logits.ndim == 1:
            logits = logits[None, :]
        B, V = logits.shape
        ids = np.empty((B, n), dtype=np.int64)
        probs = np.empty((B, n), dtype=np.float32)
        st = self._lib.nls_top_tokens(self._h, _host_ptr(logits), V, B, V, int(n), _host_ptr(ids),
                                      _host_ptr(probs), 0, ctypes.c_void_p(0))
        self._check(st, "nls_top_tokens")
        return ids, probs

    def token_nll(self, logits, targets, check: bool = True):
        """Perplexity's per-position term (model.nim:581-584) for each row of
        host numpy logits [B, V] and its target token: returns (float64 [B],
        status). A row with a NaN or non-finite maximum, or a target outside
        [0, V), gets NaN and a non-zero status (raised unless check=False)."""
        logits = np.asarray(logits, dtype=np.float32)
        if logits.ndim == 1:
            logits = logits[None, :]
        if logits.strides[1] != 4 or logits.strides[0] % 4 != 0:
            logits = np.ascontiguousarray(logits)  # rows may be strided (ld > V)
        B, V = logits.shape
        ld = logits.strides[0] // 4 if B > 1 else V
        targets = np.ascontiguousarray(np.asarray(targets, dtype=np.int64).reshape(-1))
        if targets.size != B:
            raise ValueError("one target per row")
        out = np.empty(B, dtype=np.float64)
        st = self._lib.nls_token_nll(self._h, _host_ptr(logits), ld, B, V, _host_ptr(targets),
                                     _host_ptr(out), 0, ctypes.c_void_p(0))
        if check:
            self._check(st, "nls_token_nll")
        return out, st

    def upload(self, host) -> int:
        """Copy a host array to a new device buffer (nls_device_upload);
        returns its device address, to free with free_device()."""
        host = np.ascontiguousarray(host)
        d = ctypes.c_void_p()
        st = self._lib.nls_device_upload(self._h, ctypes.c_void_p(host.ctypes.data), host.nbytes,
                                         ctypes.byref(d))
        self._check(st, "nls_device_upload")
        return int(d.value)

    def free_device(self, dev: int) -> None:
        self._lib.nls_device_free(self._h, ctypes.c_void_p(dev))

    @staticmethod
    def _weights_ptr(weights):
        """Device address of ggml-layout weights: a CUDA tensor or an int."""
        if isinstance(weights, int):
            return ctypes.c_void_p(weights)
        if not _is_torch(weights) or not weights.is_cuda:
            raise TypeError("weights must be device memory (a CUDA tensor or a device address)")
        return ctypes.c_void_p(weights.data_ptr())

    def lm_head(self, weights, wtype: int, rows: int, cols: int, x, exact: bool = False,
                out=None, stream: int = 0, check: bool = True, independent: bool = False):
        """matmul(m.output, x, y, nb) (model.nim:179-189): logits [nb, rows] fp32.
        x: host numpy [nb, cols] (returns numpy) or a CUDA tensor (returns a
        CUDA tensor, or fills `out`, stream-ordered on `stream`). independent:
        the rows are separate sequences (path chosen as for nb = 1)."""
        flags = (_abi.NLS_EXACT_MATMUL if exact else 0) | (_abi.NLS_ROWS_INDEPENDENT if independent else 0)
        if _is_torch(x):
            import torch
            if x.dim() == 1:
                x = x[None, :]
            x = x.contiguous()
            nb = x.shape[0]
            y = out if out is not None else torch.empty((nb, rows), dtype=torch.float32, device=x.device)
            st = self._lib.nls_lm_head(self._h, self._weights_ptr(weights), int(wtype), int(rows),
                                       int(cols), ctypes.c_void_p(x.data_ptr()), nb,
                                       ctypes.c_void_p(y.data_ptr()),
                                       flags | _abi.NLS_DEVICE_INPUTS | _abi.NLS_DEVICE_OUTPUTS,
                                       ctypes.c_void_p(stream))
            if check:
                self._check(st, "nls_lm_head")
                st = self._lib.nls_stream_status(self._h, ctypes.c_void_p(stream))
                self._check(st, "nls_lm_head (kernel status)")
            return y
        x = np.ascontiguousarray(np.atleast_2d(np.asarray(x, dtype=np.float32)))
        nb = x.shape[0]
        y = np.empty((nb, rows), dtype=np.float32)
        st = self._lib.nls_lm_head(self._h, self._weights_ptr(weights), int(wtype), int(rows), int(cols),
                                   _host_ptr(x), nb, _host_ptr(y), flags, ctypes.c_void_p(stream))
        if check:
            self._check(st, "nls_lm_head")
        return y

    def lm_head_sample(self, weights, wtype: int, vocab: int, cols: int, x, params, hist_ids=None,
                       hist_off=None, bias_ids=None, bias_vals=None, bias_off=None, uniforms=None,
                       want_probs: bool = False, exact: bool = False, check: bool = True,
                       independent: bool = False):
        """Output projection then sampling of each row (model.nim:466-470, then
        sampler.nim:59-121), host numpy inputs: returns (ids, probs or None,
        status). The logits never leave the GPU."""
        x = np.ascontiguousarray(np.atleast_2d(np.asarray(x, dtype=np.float32)))
        B = x.shape[0]
        params = np.ascontiguousarray(params, dtype=ROW_PARAMS_DTYPE)
        conv = {}
        for name, arr, dt in (("hist_ids", hist_ids, np.int64), ("hist_off", hist_off, np.int64),
                              ("bias_ids", bias_ids, np.int64), ("bias_vals", bias_vals, np.float64),
                              ("bias_off", bias_off, np.int64), ("uniforms", uniforms, np.float64)):
            conv[name] = None if arr is None else np.ascontiguousarray(arr, dtype=dt)
        ids = np.empty(B, dtype=np.int64)
        probs = np.empty(B, dtype=np.float32) if want_probs else None
        st = self._lib.nls_lm_head_sample(
            self._h, self._weights_ptr(weights), int(wtype), int(vocab), int(cols), _host_ptr(x), B,
            _host_ptr(params), _host_ptr(conv["hist_ids"]), _host_ptr(conv["hist_off"]),
            _host_ptr(conv["bias_ids"]), _host_ptr(conv["bias_vals"]), _host_ptr(conv["bias_off"]),
            _host_ptr(conv["uniforms"]), _host_ptr(ids), _host_ptr(probs),
            (_abi.NLS_EXACT_MATMUL if exact else 0) | (_abi.NLS_ROWS_INDEPENDENT if independent else 0),
            ctypes.c_void_p(0))
        if check:
            self._check(st, "nls_lm_head_sample")
        return ids, probs, st

    def argmax_batch(self, logits) -> np.ndarray:
        logits = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
        if logits.ndim == 1:
            logits = logits[None, :]
        B, V = logits.shape
        ids = np.empty(B, dtype=np.int64)
        st = self._lib.nls_argmax_batch(self._h, _host_ptr(logits), V, B, V, _host_ptr(ids), 0,
                                        ctypes.c_void_p(0))
        self._check(st, "nls_argmax_batch")
        return ids


_default_engine: Optional[Engine] = None


def default_engine() -> Engine:
    global _default_engine
    if _default_engine is None:
        _default_engine = Engine(0, max_rows=256, max_vocab=1 << 18)
    return _default_engine


# ---------------------------------------------------------------------------
# Sampler (sampler.nim:23-121)
# ---------------------------------------------------------------------------
class Sampler:
    def __init__(self, params: SamplerParams, engine: Optional[Engine] = None):
        self.params = params
        self.rng = Rand(params.seed)
        self.history: list[int] = []
        self.engine = engine

    def accept(self, tok: int) -> None:                       # sampler.nim:41-43
        self.history.append(int(tok))

    def sample(self, logitsIn) -> int:                        # sampler.nim:59-121
        """Choose a token; `logitsIn` is not modified. Draws one uniform from
        `rng` only when temperature > 0, as the reference does."""
        p = self.params
        logits = np.ascontiguousarray(np.asarray(logitsIn, dtype=np.float32))
        hist = np.asarray(self.history, dtype=np.int64)
        bias_ids = np.fromiter(p.logitBias.keys(), dtype=np.int64, count=len(p.logitBias))
        bias_vals = np.fromiter(p.logitBias.values(), dtype=np.float64, count=len(p.logitBias))
        u = np.array([self.rng.rand(1.0) if p.temperature > 0 else 0.0], dtype=np.float64)
        eng = self.engine or default_engine()
        ids, _, _ = eng.sample_batch(
            logits[None, :], np.array([params_record(p)], dtype=ROW_PARAMS_DTYPE),
            hist, np.array([0, hist.size], dtype=np.int64),
            bias_ids, bias_vals, np.array([0, bias_ids.size], dtype=np.int64), u)
        return int(ids[0])


def batch_inputs(samplers: list) -> dict:
    """The sampling inputs of several independent samplers as one batch (the
    C ABI's layout): one params record per sampler, their histories and
    logit biases as CSR lists, and one uniform each, drawn from the
    sampler's own RNG only when its temperature is above 0 (sampler.nim:77-78,
    :117), so every RNG advances exactly as if the samplers ran one by one."""
    params = np.array([params_record(s.params) for s in samplers], dtype=ROW_PARAMS_DTYPE)
    hist = [np.asarray(s.history, dtype=np.int64) for s in samplers]
    hist_off = np.zeros(len(samplers) + 1, dtype=np.int64)
    hist_off[1:] = np.cumsum([h.size for h in hist])
    bias_ids = [np.fromiter(s.params.logitBias.keys(), dtype=np.int64, count=len(s.params.logitBias))
                for s in samplers]
    bias_vals = [np.fromiter(s.params.logitBias.values(), dtype=np.float64, count=len(s.params.logitBias))
                 for s in samplers]
    bias_off = np.zeros(len(samplers) + 1, dtype=np.int64)
    bias_off[1:] = np.cumsum([b.size for b in bias_ids])
    uniforms = np.array([s.rng.rand(1.0) if s.params.temperature > 0 else 0.0 for s in samplers],
                        dtype=np.float64)
    cat = lambda parts, dt: np.concatenate(parts).astype(dt) if parts else np.zeros(0, dt)  # noqa: E731
    return dict(params=params, hist_ids=cat(hist, np.int64), hist_off=hist_off,
                bias_ids=cat(bias_ids, np.int64), bias_vals=cat(bias_vals, np.float64),
                bias_off=bias_off, uniforms=uniforms)


def sample_many(samplers: list, logits_rows, engine: Optional[Engine] = None) -> list:
    """One sampling step of many independent samplers (separate Chats sharing
    one model) in one batched call: row i of `logits_rows` is sampled with
    samplers[i]'s params, history, bias and RNG. The ids equal what each
    sampler's own sample() returns; accept() stays with the caller."""
    logits = np.ascontiguousarray(np.atleast_2d(np.asarray(logits_rows, dtype=np.float32)))
    if logits.shape[0] != len(samplers):
        raise ValueError("one logits row per sampler")
    a = batch_inputs(samplers)
    eng = engine or default_engine()
    ids, _, _ = eng.sample_batch(logits, a["params"], a["hist_ids"], a["hist_off"], a["bias_ids"],
                                 a["bias_vals"], a["bias_off"], a["uniforms"])
    return [int(i) for i in ids]


def decode_step_many(samplers: list, engine: Engine, weights, wtype: int, vocab: int, cols: int,
                     hidden_rows) -> list:
    """The tail of one decode step of many independent Chats sharing one
    model: the output projection of each one's normalised hidden state
    (model.nim:470, as a one-row matmul each) and sampling with each one's
    sampler, in two kernels' worth of GPU work and no logits on the host."""
    a = batch_inputs(samplers)
    ids, _, _ = engine.lm_head_sample(weights, wtype, vocab, cols, hidden_rows, a["params"],
                                      a["hist_ids"], a["hist_off"], a["bias_ids"], a["bias_vals"],
                                      a["bias_off"], a["uniforms"], independent=True)
    return [int(i) for i in ids]


def newSampler(p: Optional[SamplerParams] = None, engine: Optional[Engine] = None) -> Sampler:
    return Sampler(p if p is not None else defaultSampling(), engine)


def accept(s: Sampler, tok: int) -> None:
    s.accept(tok)


def sample(s: Sampler, logitsIn) -> int:
    return s.sample(logitsIn)


def argmax(logits, engine: Optional[Engine] = None) -> int:    # sampler.nim:45-49
    eng = engine or default_engine()
    return int(eng.argmax_batch(logits)[0])


def topTokens(logits, n: int = 5, engine: Optional[Engine] = None) -> list:  # sampler.nim:123-130
    """The `n` most probable tokens of one row as [(id, prob)], like the Nim
    proc (min(n, V) entries)."""
    eng = engine or default_engine()
    x = np.asarray(logits, dtype=np.float32).reshape(-1)
    ids, probs = eng.top_tokens(x, n)
    m = min(n, x.size)
    return [(int(ids[0, i]), float(probs[0, i])) for i in range(m)]


def perplexity_from_logits(logits, tokens, engine: Optional[Engine] = None) -> float:
    """The perplexity of one chunk (model.nim:570-589) from its logits
    [T, V] (row t predicts tokens[t+1]) and its T tokens: the per-position
    terms come from the GPU, their float64 sum runs in position order as in
    the reference loop, then exp(total / max(1, count))."""
    eng = engine or default_engine()
    x = np.asarray(logits, dtype=np.float32)
    tok = np.asarray(tokens, dtype=np.int64).reshape(-1)
    n = tok.size - 1
    if n <= 0:
        return 1.0  # exp(0 / 1): the reference's loop body never runs
    nll, _ = eng.token_nll(x[:n], tok[1:n + 1])
    total = 0.0
    for v in nll:
        total += float(v)
    return float(np.exp(total / max(1, n)))


__all__ = ["SamplerParams", "defaultSampling", "greedySampling", "params_record", "Rand",
           "Engine", "Sampler", "newSampler", "accept", "sample", "argmax", "topTokens",
           "perplexity_from_logits", "default_engine", "NlsError", "ROW_PARAMS_DTYPE"]


# ---------------------------------------------------------------------------
# Vocab-sharded mode: an NCCL communicator of the C library
# ---------------------------------------------------------------------------
def vocab_shard(vocab: int, nranks: int, rank: int) -> tuple[int, int]:
    """Columns [lo, hi) of rank `rank` when `vocab` is split over `nranks`
    ranks (Vs = ceil(vocab / nranks) columns each, the last ones fewer)."""
    vs = -(-vocab // nranks)
    lo = min(vocab, rank * vs)
    return lo, min(vocab, lo + vs)


def row_owner_range(rows: int, nranks: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) that rank `rank` samples in the vocab-sharded call."""
    return rows * rank // nranks, rows * (rank + 1) // nranks


def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for Comm()."""
    lib = _abi.load()
    buf = ctypes.create_string_buffer(128)
    st = lib.nls_comm_unique_id(buf)
    if st != 0:
        raise NlsError(st, "nls_comm_unique_id")
    return buf.raw


class Comm:
    """nls_comm: this rank's place in an NCCL communicator (collective to
    create). `uid` is comm_unique_id() from one rank, sent to all others."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        self._lib = _abi.load()
        c = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        st = self._lib.nls_comm_create(ctypes.byref(c), buf, int(nranks), int(rank), int(device))
        if st != 0:
            raise NlsError(st, "nls_comm_create")
        self._c = c
        self.nranks, self.rank, self.device = nranks, rank, device

    def set_timeout(self, ms: int) -> None:
        """Host deadline of each later vocab-sharded call (nls_comm_set_timeout)."""
        st = self._lib.nls_comm_set_timeout(self._c, int(ms))
        if st != 0:
            raise NlsError(st, "nls_comm_set_timeout")

    def abort(self) -> None:
        """End the communicator at once (nls_comm_abort)."""
        st = self._lib.nls_comm_abort(self._c)
        if st != 0:
            raise NlsError(st, "nls_comm_abort")

    def close(self):
        if getattr(self, "_c", None):
            self._lib.nls_comm_destroy(self._c)
            self._c = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
