"""ctypes binding of the C oracle (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may import this.
`build()` compiles oracle/ref_sampler.c into oracle/build/libnls_oracle.so.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libnls_oracle.so")


class NloParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_double),
        ("top_p", ctypes.c_double),
        ("min_p", ctypes.c_double),
        ("repeat_penalty", ctypes.c_double),
        ("presence_penalty", ctypes.c_double),
        ("frequency_penalty", ctypes.c_double),
        ("top_k", ctypes.c_int64),
        ("repeat_last_n", ctypes.c_int64),
    ]


class NloDiag(ctypes.Structure):
    _fields_ = [
        ("prob", ctypes.c_float),
        ("ncand", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("pos", ctypes.c_int64),
        ("margin", ctypes.c_double),
        ("total", ctypes.c_float),
        ("denom", ctypes.c_float),
    ]


# numpy mirror of NloParams / the product's nls_row_params (same 64-byte layout)
PARAMS_DTYPE = np.dtype([
    ("temperature", "<f8"), ("top_p", "<f8"), ("min_p", "<f8"),
    ("repeat_penalty", "<f8"), ("presence_penalty", "<f8"),
    ("frequency_penalty", "<f8"), ("top_k", "<i8"), ("repeat_last_n", "<i8"),
])
DIAG_DTYPE = np.dtype({"names": ["prob", "ncand", "n", "pos", "margin", "total", "denom"],
                       "formats": ["<f4", "<i8", "<i8", "<i8", "<f8", "<f4", "<f4"],
                       "offsets": [0, 8, 16, 24, 32, 40, 44], "itemsize": 48})

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        L.nlo_argmax.restype = ctypes.c_int64
        L.nlo_argmax.argtypes = [P(ctypes.c_float), ctypes.c_int64]
        L.nlo_softmax_inplace.restype = None
        L.nlo_softmax_inplace.argtypes = [P(ctypes.c_float), ctypes.c_int64]
        L.nlo_sample.restype = ctypes.c_int64
        L.nlo_sample.argtypes = [P(NloParams), P(ctypes.c_int64), ctypes.c_int64,
                                 P(ctypes.c_int64), P(ctypes.c_double), ctypes.c_int64,
                                 P(ctypes.c_float), ctypes.c_int64, ctypes.c_double,
                                 P(NloDiag)]
        L.nlo_token_nll.restype = ctypes.c_double
        L.nlo_token_nll.argtypes = [P(ctypes.c_float), ctypes.c_int64, ctypes.c_int64]
        L.nlo_top_tokens.restype = ctypes.c_int64
        L.nlo_top_tokens.argtypes = [P(ctypes.c_float), ctypes.c_int64, ctypes.c_int64,
                                     P(ctypes.c_int64), P(ctypes.c_float)]
        L.nlo_row_bytes.restype = ctypes.c_int64
        L.nlo_row_bytes.argtypes = [ctypes.c_int32, ctypes.c_int64]
        L.nlo_quantize_act.restype = None
        L.nlo_quantize_act.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_void_p, ctypes.c_void_p]
        L.nlo_lm_head.restype = ctypes.c_int
        L.nlo_lm_head.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32,
                                  ctypes.c_int32]
        L.nlo_sample_batch.restype = None
        L.nlo_sample_batch.argtypes = [ctypes.c_void_p] * 1 + [ctypes.c_int64] * 3 + \
            [ctypes.c_void_p] * 9 + [ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def sample_batch(logits: np.ndarray, params: np.ndarray, hist_ids=None, hist_off=None,
                 bias_ids=None, bias_vals=None, bias_off=None, uniforms=None,
                 threads: int = 1, diag: bool = False):
    """Run the oracle over a [B, V] fp32 batch. Arrays follow the product's
    C-ABI layout (CSR histories and bias lists, one params record per row)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = logits.shape
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    assert params.shape == (B,)
    if hist_ids is not None:
        hist_ids = np.ascontiguousarray(hist_ids, dtype=np.int64)
        hist_off = np.ascontiguousarray(hist_off, dtype=np.int64)
    if bias_ids is not None:
        bias_ids = np.ascontiguousarray(bias_ids, dtype=np.int64)
        bias_vals = np.ascontiguousarray(bias_vals, dtype=np.float64)
        bias_off = np.ascontiguousarray(bias_off, dtype=np.int64)
    uniforms = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float64)
    out = np.empty(B, dtype=np.int64)
    dg = np.zeros(B, dtype=DIAG_DTYPE) if diag else None
    lib().nlo_sample_batch(_ptr(logits), V, B, V, _ptr(params), _ptr(hist_ids), _ptr(hist_off),
                           _ptr(bias_ids), _ptr(bias_vals), _ptr(bias_off), _ptr(uniforms),
                           _ptr(out), _ptr(dg), int(threads))
    return (out, dg) if diag else out


def argmax(x: np.ndarray) -> int:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return int(lib().nlo_argmax(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), x.size))


def softmax_inplace(x: np.ndarray) -> np.ndarray:
    x = np.array(x, dtype=np.float32, copy=True)
    lib().nlo_softmax_inplace(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), x.size)
    return x


def token_nll(logits: np.ndarray, targets) -> np.ndarray:
    """perplexity's per-position term (model.nim:580-584) for each row."""
    x = np.ascontiguousarray(np.atleast_2d(logits), dtype=np.float32)
    t = np.asarray(targets, dtype=np.int64).reshape(-1)
    P = ctypes.POINTER(ctypes.c_float)
    return np.array([lib().nlo_token_nll(x[r].ctypes.data_as(P), x.shape[1], int(t[r]))
                     for r in range(x.shape[0])], dtype=np.float64)


def top_tokens(x: np.ndarray, n: int = 5):
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.zeros(max(n, 1), dtype=np.int64)
    pr = np.zeros(max(n, 1), dtype=np.float32)
    m = lib().nlo_top_tokens(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), x.size, n,
                             ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                             pr.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return [(int(ids[i]), float(pr[i])) for i in range(m)]


# ggml weight type codes (quant.nim:14-19) restated by ref_lmhead.c
WTYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q6_k": 14}


def row_bytes(wtype: int, cols: int) -> int:
    return int(lib().nlo_row_bytes(int(wtype), int(cols)))


def quantize_act(x: np.ndarray, block_len: int):
    """quantizeAct (quant.nim:646-662): per-block scales and int8 values."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    d = np.empty(x.size // block_len, dtype=np.float32)
    q = np.empty(x.size, dtype=np.int8)
    lib().nlo_quantize_act(_ptr(x), x.size, block_len, _ptr(d), _ptr(q))
    return d, q


def lm_head(w: np.ndarray, wtype: int, rows: int, cols: int, x: np.ndarray,
            exact_matmul: bool = False, threads: int = 1) -> np.ndarray:
    """matmul(m.output, x, y, nb) (model.nim:179-189): [nb, rows] fp32 logits
    from ggml-layout weight bytes `w` and activations x [nb, cols]."""
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    nb = x.shape[0]
    assert x.shape[1] == cols and w.size >= rows * row_bytes(wtype, cols)
    y = np.empty((nb, rows), dtype=np.float32)
    rc = lib().nlo_lm_head(_ptr(w), int(wtype), rows, cols, _ptr(x), nb, _ptr(y),
                           int(bool(exact_matmul)), int(threads))
    if rc != 0:
        raise ValueError(f"unsupported weight type {wtype} or shape cols={cols}")
    return y
