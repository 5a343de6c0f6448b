"""Line-by-line Python transliteration of nimllm's sampler (TEST INFRASTRUCTURE).

Only tests/ (and tests/golden/make_golden.py) use this module. It is a second,
independent restatement of src/nimllm/sampler.nim (reference repository) used
to cross-check the C oracle (oracle/ref_sampler.c). It is slow (pure Python
loops) and meant for small vocabularies.

Parity status: UNPINNED against the reference itself (no Nim toolchain exists
here). Each statement below mirrors one line of sampler.nim:
  - Nim float32 arithmetic  -> numpy.float32 scalar arithmetic (IEEE single)
  - Nim `x.float32`         -> numpy.float32(x) (round to nearest)
  - Nim exp(float32)        -> libm expf through ctypes (C expf, as Nim emits)
  - std/heapqueue           -> heapq (the same published binary-heap algorithm;
                               tuple `<` is lexicographic in both languages)
  - algorithm.sort          -> sorted() with the same comparator (both stable)
"""
from __future__ import annotations

import ctypes
import ctypes.util
import functools
import heapq
from collections import Counter

import numpy as np

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
_libm.exp.restype = ctypes.c_double
_libm.exp.argtypes = [ctypes.c_double]
_libm.log.restype = ctypes.c_double
_libm.log.argtypes = [ctypes.c_double]

f32 = np.float32


def expf(x) -> np.float32:
    return f32(_libm.expf(ctypes.c_float(float(x))))


def nim_cmp(x, y) -> int:
    # system.cmp: 0 when ==, -1 when <, else 1
    if x == y:
        return 0
    if x < y:
        return -1
    return 1


def argmax(logits) -> int:                                   # sampler.nim:45-49
    best = 0
    for i in range(1, len(logits)):
        if logits[i] > logits[best]:
            best = i
    return best


def softmax_inplace(x: list) -> None:                        # sampler.nim:51-57
    mx = f32(-np.inf)
    for v in x:
        mx = v if mx <= v else mx
    s = f32(0.0)
    for i in range(len(x)):
        x[i] = expf(f32(x[i] - mx))
        s = f32(s + x[i])
    for i in range(len(x)):
        x[i] = f32(x[i] / s)


class SamplerParams:                                         # sampler.nim:11-21
    def __init__(self, temperature=0.7, topK=40, topP=0.95, minP=0.05,
                 repeatPenalty=1.1, repeatLastN=64, presencePenalty=0.0,
                 frequencyPenalty=0.0, seed=-1, logitBias=None):
        self.temperature = float(temperature)
        self.topK = int(topK)
        self.topP = float(topP)
        self.minP = float(minP)
        self.repeatPenalty = float(repeatPenalty)
        self.repeatLastN = int(repeatLastN)
        self.presencePenalty = float(presencePenalty)
        self.frequencyPenalty = float(frequencyPenalty)
        self.seed = int(seed)
        self.logitBias = dict(logitBias or {})


def sample(p: SamplerParams, history: list, logitsIn, u: float, diag: dict | None = None) -> int:
    """Sampler.sample (sampler.nim:59-121); `u` stands for s.rng.rand(1.0)."""
    logits = [f32(v) for v in logitsIn]                                  # :62
    if len(history) > 0 and (p.repeatPenalty != 1.0 or p.presencePenalty != 0
                             or p.frequencyPenalty != 0):                # :64-65
        start = max(0, len(history) - p.repeatLastN) if p.repeatLastN > 0 else 0  # :67
        counts = Counter(history[start:])                                # :66,68
        for tok, cnt in counts.items():                                  # :69
            if tok < 0 or tok >= len(logits):                            # :70
                continue
            if p.repeatPenalty != 1.0:                                   # :71
                if logits[tok] > 0:
                    logits[tok] = f32(logits[tok] / f32(p.repeatPenalty))  # :72
                else:
                    logits[tok] = f32(logits[tok] * f32(p.repeatPenalty))  # :73
            logits[tok] = f32(logits[tok] - f32(float(cnt) * p.frequencyPenalty
                                                + p.presencePenalty))    # :74
    for tok, b in p.logitBias.items():                                   # :75
        if 0 <= tok < len(logits):
            logits[tok] = f32(logits[tok] + f32(b))                      # :76
    if p.temperature <= 0:                                               # :77
        return argmax(logits)                                            # :78
    invT = f32(1.0 / p.temperature)                                      # :80
    logits = [f32(v * invT) for v in logits]                             # :81
    idx = list(range(len(logits)))                                       # :83-84
    k = min(p.topK, len(logits)) if p.topK > 0 else len(logits)          # :85
    if k < len(logits):                                                  # :86
        h: list = []                                                     # :88
        for i in range(len(logits)):                                     # :89
            if len(h) < k:
                heapq.heappush(h, (logits[i], i))                        # :90
            elif logits[i] > h[0][0]:                                    # :91
                heapq.heapreplace(h, (logits[i], i))                     # :92
        idx = []                                                         # :93
        while len(h) > 0:
            idx.append(heapq.heappop(h)[1])                              # :94
        idx.reverse()                                                    # :95
    else:
        idx = sorted(idx, key=functools.cmp_to_key(
            lambda a, b: nim_cmp(logits[b], logits[a])))                 # :97
    probs = [logits[i] for i in idx]                                     # :98-99
    softmax_inplace(probs)                                               # :100
    n = len(probs)                                                       # :101
    if p.topP > 0 and p.topP < 1:                                        # :103
        cum = f32(0.0)
        for i in range(n):
            cum = f32(cum + probs[i])                                    # :106
            if float(cum) >= p.topP:                                     # :107
                n = i + 1
                break
    if p.minP > 0:                                                       # :110
        thr = f32(probs[0] * f32(p.minP))                                # :111
        m = 1
        while m < n and probs[m] >= thr:                                 # :113
            m += 1
        n = m                                                            # :114
    total = f32(0.0)
    for i in range(n):
        total = f32(total + probs[i])                                    # :116
    r = f32(f32(u) * total)                                              # :117
    result = idx[n - 1]                                                  # :121
    pos = n - 1
    for i in range(n):
        r = f32(r - probs[i])                                            # :119
        if r <= 0:                                                       # :120
            result = idx[i]
            pos = i
            break
    if diag is not None:
        diag.update(n=n, pos=pos, prob=float(probs[pos]), ncand=len(idx), total=float(total))
    return result


def token_nll(logits, target):                              # model.nim:580-584
    """One position of perplexity: Nim `float` is float64, so exp/ln are
    C's exp/log on float64; `logits[..] - mx` is a float32 subtraction."""
    mx = f32(float("-inf"))
    for v in logits:                                          # :581
        mx = max(mx, f32(v))
    s = 0.0
    for v in logits:                                          # :582-583
        s += _libm.exp(float(f32(f32(v) - mx)))
    return -(float(f32(f32(logits[target]) - mx)) - _libm.log(s))   # :584


def top_tokens(logits, n=5):                                 # sampler.nim:123-130
    probs = [f32(v) for v in logits]
    softmax_inplace(probs)
    idx = sorted(range(len(probs)), key=functools.cmp_to_key(
        lambda a, b: nim_cmp(probs[b], probs[a])))
    return [(idx[i], float(probs[idx[i]])) for i in range(min(n, len(idx)))]
