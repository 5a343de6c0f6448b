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


# ---- the output projection (model.nim:144-189, quant.nim) -------------------
# Mirrors ref_lmhead.c by a separate route: numpy float32 scalars for every
# float32 operation, Python ints for the integer dot products, numpy's own
# float16 -> float32 conversion for rdHalf.

def _rd_half(b, o) -> np.float32:                            # quant.nim:144-147
    return f32(np.frombuffer(bytes(b[o:o + 2]), dtype="<f2")[0])


def _i8(v) -> int:
    return v - 256 if v >= 128 else v


def quantize_act(x, bl):                                     # quant.nim:646-662
    x = [f32(v) for v in x]
    d_out, qs = [], []
    for b in range(len(x) // bl):
        amax = f32(0)
        for i in range(bl):
            amax = max(amax, abs(x[b * bl + i]))
        d = f32(amax / f32(127))
        idv = f32(f32(1) / d) if d > 0 else f32(0)
        d_out.append(d)
        for i in range(bl):
            v = f32(x[b * bl + i] * idv)
            qs.append(int(f32(v + f32(0.5))) if v >= 0 else -int(f32(-v + f32(0.5))))
    return d_out, qs


def _dot_f32(a, b):                                          # quant.nim:362-374
    s = [f32(0)] * 8
    n, i = len(a), 0
    while i + 8 <= n:
        for k in range(8):
            s[k] = f32(s[k] + f32(a[i + k] * b[i + k]))
        i += 8
    while i < n:
        s[0] = f32(s[0] + f32(a[i] * b[i]))
        i += 1
    t = f32(s[0] + s[1])
    t = f32(t + f32(s[2] + s[3]))
    t = f32(t + f32(s[4] + s[5]))
    return f32(t + f32(s[6] + s[7]))


def _dequant_row(t, s, n):                                   # quant.nim:160-202,303-352
    y = [f32(0)] * n
    if t == 0:
        return [f32(v) for v in np.frombuffer(bytes(s[:4 * n]), dtype="<f4")]
    if t == 1:
        return [_rd_half(s, 2 * i) for i in range(n)]
    if t == 8:
        for ib in range(n // 32):
            b = s[ib * 34:(ib + 1) * 34]
            d = _rd_half(b, 0)
            for j in range(32):
                y[ib * 32 + j] = f32(f32(_i8(b[2 + j])) * d)
        return y
    if t == 2:
        for ib in range(n // 32):
            b = s[ib * 18:(ib + 1) * 18]
            d = _rd_half(b, 0)
            for j in range(16):
                q = b[2 + j]
                y[ib * 32 + j] = f32(f32((q & 0xF) - 8) * d)
                y[ib * 32 + j + 16] = f32(f32((q >> 4) - 8) * d)
        return y
    if t == 14:
        for ib in range(n // 256):
            b = s[ib * 210:(ib + 1) * 210]
            d = _rd_half(b, 208)
            qlo, qho, sco, yo = 0, 128, 192, ib * 256
            for _ in range(2):
                for l in range(32):
                    isc = l // 16
                    qh = b[qho + l]
                    q1 = ((b[qlo + l] & 0xF) | ((qh & 3) << 4)) - 32
                    q2 = ((b[qlo + l + 32] & 0xF) | (((qh >> 2) & 3) << 4)) - 32
                    q3 = ((b[qlo + l] >> 4) | (((qh >> 4) & 3) << 4)) - 32
                    q4 = ((b[qlo + l + 32] >> 4) | (((qh >> 6) & 3) << 4)) - 32
                    y[yo + l] = f32(f32(d * f32(_i8(b[sco + isc]))) * f32(q1))
                    y[yo + l + 32] = f32(f32(d * f32(_i8(b[sco + isc + 2]))) * f32(q2))
                    y[yo + l + 64] = f32(f32(d * f32(_i8(b[sco + isc + 4]))) * f32(q3))
                    y[yo + l + 96] = f32(f32(d * f32(_i8(b[sco + isc + 6]))) * f32(q4))
                yo += 128
                qlo += 64
                qho += 32
                sco += 8
        return y
    raise ValueError(t)


def _dot_act(t, w, ad, aq, off, n):                         # quant.nim:731-786
    acc = f32(0)
    if t in (8, 2):
        for ib in range(n // 32):
            ab = off // 32 + ib
            q8 = aq[ab * 32:(ab + 1) * 32]
            if t == 8:
                o = ib * 34
                s = sum(_i8(w[o + 2 + l]) * q8[l] for l in range(32))
            else:
                o = ib * 18
                s = sum(((w[o + 2 + l] & 0xF) - 8) * q8[l] + ((w[o + 2 + l] >> 4) - 8) * q8[l + 16]
                        for l in range(16))
            acc = f32(acc + f32(f32(_rd_half(w, o) * ad[ab]) * f32(s)))
        return acc
    for ib in range(n // 256):                               # Q6_K
        b = w[ib * 210:(ib + 1) * 210]
        ab = off // 256 + ib
        q8 = aq[ab * 256:(ab + 1) * 256]
        d = _rd_half(b, 208)
        sumi = 0
        for h in range(2):
            ql, qh = 64 * h, 128 + 32 * h
            for half in range(2):
                s = [0, 0, 0, 0]
                for l in range(16 * half, 16 * half + 16):
                    hb = b[qh + l]
                    q = [((b[ql + l] & 0xF) | ((hb & 3) << 4)) - 32,
                         ((b[ql + l + 32] & 0xF) | (((hb >> 2) & 3) << 4)) - 32,
                         ((b[ql + l] >> 4) | (((hb >> 4) & 3) << 4)) - 32,
                         ((b[ql + l + 32] >> 4) | (((hb >> 6) & 3) << 4)) - 32]
                    for k in range(4):
                        s[k] += q[k] * q8[128 * h + l + 32 * k]
                so = 8 * h + half
                sumi += sum(_i8(b[192 + so + 2 * k]) * s[k] for k in range(4))
        acc = f32(acc + f32(f32(ad[ab] * d) * f32(sumi)))
    return acc


def lm_head(w, t, rows, cols, x, exact_matmul=False):        # model.nim:144-189
    """[nb][rows] float32 logits; w is the ggml-layout row bytes."""
    bs = {0: 1, 1: 1, 2: 32, 8: 32, 14: 256}[t]
    rb = cols // bs * {0: 4, 1: 2, 2: 18, 8: 34, 14: 210}[t]
    x = [[f32(v) for v in row] for row in x]
    nb = len(x)
    bl = {2: 32, 8: 32, 14: 256}.get(t, 0)
    y = [[f32(0)] * rows for _ in range(nb)]
    w = bytes(w)
    if not exact_matmul and bl > 0 and cols % bl == 0 and (nb <= 4 or t != 8):
        flat = [v for row in x for v in row]
        ad, aq = quantize_act(flat, bl)
        for r in range(rows):
            for b in range(nb):
                y[b][r] = _dot_act(t, w[r * rb:(r + 1) * rb], ad, aq, b * cols, cols)
        return y
    for r in range(rows):
        rowp = _dequant_row(t, w[r * rb:(r + 1) * rb], cols)
        for b in range(nb):
            y[b][r] = _dot_f32(rowp, x[b])
    return y
