"""nls_sample_batch_noalloc: sampling for callers that cannot allocate GPU
memory -- a serving process whose own pool holds nearly all of the GPU's
memory, a host that forbids allocating after start-up, or a decode loop
that cannot afford the device-wide synchronisation of cudaMalloc/cudaFree --
and so cannot create a handle. Its scratch is one fixed array inside the
library, shared by every call, so each test makes two calls in a row.

It must give the same tokens and probabilities as nls_sample_batch and as
the CPU oracle, bit for bit (the bar of the other parity tests): configs 3
and 5 at their full vocabularies, a few rows of a large vocabulary and rows
of a small one (both choices of CTAs per row), NaN rows, and the status word
that nls_noalloc_status reads back. This file is collected last, so that a
failure here does not hide the other tests; it passes alone in a fresh
process as well.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b)))


class NoAlloc:
    """Device copies of one batch and calls of the allocation-free entry."""

    def __init__(self, pkg, logits, params, hist=None, hoff=None, bids=None, bvals=None, boff=None,
                 uniforms=None):
        import torch
        self.lib = pkg.load()
        self.dev = torch.device("cuda:0")
        t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(self.dev)
        self.B, self.V = logits.shape
        self.args = (t(logits), t(params.view(np.uint8)), t(hist), t(hoff), t(bids), t(bvals), t(boff),
                     t(uniforms))
        self.out_ids = torch.empty(self.B, dtype=torch.int64, device=self.dev)
        self.out_probs = torch.empty(self.B, dtype=torch.float32, device=self.dev)
        self.stream = torch.cuda.current_stream(self.dev)

    def call(self):
        import torch
        self.out_ids.fill_(-7)
        self.out_probs.fill_(-1.0)
        x, p, h, ho, bi, bv, bo, u = self.args
        st = self.lib.nls_sample_batch_noalloc(_dp(x), self.V, self.B, self.V, _dp(p), _dp(h), _dp(ho),
                                               _dp(bi), _dp(bv), _dp(bo), _dp(u), _dp(self.out_ids),
                                               _dp(self.out_probs), ctypes.c_void_p(self.stream.cuda_stream))
        assert st == 0, f"launch status {st}"
        torch.cuda.synchronize(self.dev)
        return self.out_ids.cpu().numpy(), self.out_probs.cpu().numpy()

    def status(self, device_out=False):
        import torch
        if device_out:
            d = torch.full((1,), -1, dtype=torch.int32, device=self.dev)
            assert self.lib.nls_noalloc_status(_dp(d), 2, ctypes.c_void_p(self.stream.cuda_stream)) == 0
            return int(d.cpu()[0])
        v = ctypes.c_int32(-1)
        assert self.lib.nls_noalloc_status(ctypes.byref(v), 0, ctypes.c_void_p(self.stream.cuda_stream)) == 0
        return v.value


def test_noalloc_matches_sample_batch_twice(pkg):
    V = 60000
    w = pkg.workloads.make("c3_batched_hetero", seed=77, rows=np.arange(48), V=V)
    # the batch must reach the full-sort kernel, the one that uses scratch
    assert np.any(w.params["top_k"] == 0) and np.any(w.params["top_k"] > 0)
    eng = pkg.Engine(0, max_rows=64, max_vocab=V)
    ids_ref, probs_ref, st = eng.sample_batch(w.logits, w.params, w.hist_ids, w.hist_off,
                                              w.bias_ids, w.bias_vals, w.bias_off, w.uniforms,
                                              want_probs=True)
    eng.close()
    assert st == 0
    na = NoAlloc(pkg, w.logits, w.params, w.hist_ids, w.hist_off, w.bias_ids, w.bias_vals,
                 w.bias_off, w.uniforms)
    for call in range(2):
        ids, probs = na.call()
        assert np.array_equal(ids, ids_ref), f"call {call}: ids differ"
        assert _bits_equal(probs, probs_ref), f"call {call}: probs differ"
        assert na.status() == 0


@pytest.mark.parametrize("name", ["c3_batched_hetero", "c5_full_vocab_nucleus"])
def test_noalloc_matches_the_oracle_at_full_size(pkg, oracle_mod, name):
    w = pkg.workloads.make(name, seed=1234)
    ref, dg = oracle_mod.sample_batch(w.logits, w.params, w.hist_ids, w.hist_off, w.bias_ids,
                                      w.bias_vals, w.bias_off, w.uniforms, diag=True, threads=16)
    na = NoAlloc(pkg, w.logits, w.params, w.hist_ids, w.hist_off, w.bias_ids, w.bias_vals,
                 w.bias_off, w.uniforms)
    samp = w.params["temperature"] > 0
    for call in range(2):
        ids, probs = na.call()
        assert np.array_equal(ids, ref), f"{name} call {call}: rows {np.nonzero(ids != ref)[0][:10]}"
        assert _bits_equal(probs[samp], dg["prob"][samp]), f"{name} call {call}: probs differ"
        assert na.status(device_out=(call == 1)) == 0


@pytest.mark.parametrize("B,V", [(1, 128256), (3, 128256), (8, 151936), (5, 6000), (40, 3000)])
def test_noalloc_small_batches_and_small_vocab(pkg, oracle_mod, B, V):
    """Few rows of a large vocabulary (up to 8 CTAs per row, the streaming
    kernel then the full-sort kernel over the rows it hands over) and rows of
    a vocabulary too small to split; every other row a full sort."""
    w = pkg.workloads.make("c3_batched_hetero", seed=90 + B, rows=np.arange(B), V=V)
    P = w.params.copy()
    P["top_k"][::2] = 0
    ref, dg = oracle_mod.sample_batch(w.logits, P, w.hist_ids, w.hist_off, w.bias_ids,
                                      w.bias_vals, w.bias_off, w.uniforms, diag=True)
    na = NoAlloc(pkg, w.logits, P, w.hist_ids, w.hist_off, w.bias_ids, w.bias_vals, w.bias_off,
                 w.uniforms)
    samp = P["temperature"] > 0
    for call in range(2):
        ids, probs = na.call()
        assert np.array_equal(ids, ref), f"B={B} V={V} call {call}"
        assert _bits_equal(probs[samp], dg["prob"][samp]), f"B={B} V={V} call {call}: probs"


def test_noalloc_nan_rows_and_status(pkg, oracle_mod):
    """A top-k row with a NaN among its first k positions returns the
    reference's answer (probability NaN); a full-sort row with a NaN fails
    alone with id -1, and nls_noalloc_status reports NLS_ERR_NAN_LOGITS until
    a clean call clears it."""
    V = 20000
    w = pkg.workloads.make("c3_batched_hetero", seed=5, rows=np.arange(12), V=V)
    P = w.params.copy()
    P["top_k"][:] = 40
    P["top_k"][5] = 0
    x = w.logits.copy()
    x[2, 10] = np.nan      # top-k row, NaN in the first k: the heap keeps it
    x[3, 15000] = np.nan   # top-k row, NaN past the first k: left out
    na_clean = NoAlloc(pkg, w.logits, P, w.hist_ids, w.hist_off, w.bias_ids, w.bias_vals,
                       w.bias_off, w.uniforms)
    with np.errstate(all="ignore"):
        ref, dg = oracle_mod.sample_batch(x, P, w.hist_ids, w.hist_off, w.bias_ids, w.bias_vals,
                                          w.bias_off, w.uniforms, diag=True)
    keep = np.arange(12) != 5
    for call in range(2):
        x_bad = x.copy()
        x_bad[5, 123] = np.nan  # full-sort row
        na = NoAlloc(pkg, x_bad, P, w.hist_ids, w.hist_off, w.bias_ids, w.bias_vals, w.bias_off,
                     w.uniforms)
        ids, probs = na.call()
        assert ids[5] == -1
        assert np.array_equal(ids[keep], ref[keep]), f"call {call}"
        assert np.isnan(probs[2]) and not np.isnan(probs[3])
        samp = keep & (P["temperature"] > 0)
        assert _bits_equal(probs[samp], dg["prob"][samp])
        assert na.status() == pkg._abi.NLS_ERR_NAN_LOGITS
        assert na.status(device_out=True) == pkg._abi.NLS_ERR_NAN_LOGITS
        na_clean.call()
        assert na_clean.status() == 0


def test_noalloc_rejects_sizes_beyond_its_limits(pkg):
    lib = pkg.load()
    one = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    assert lib.nls_sample_batch_noalloc(one, 10, 4097, 10, one, None, None, None, None, None, one,
                                        one, None, None) == pkg._abi.NLS_ERR_CAPACITY
    assert lib.nls_sample_batch_noalloc(one, 1 << 19, 1, (1 << 18) + 1, one, None, None, None,
                                        None, None, one, one, None, None) == pkg._abi.NLS_ERR_CAPACITY
    assert lib.nls_noalloc_status(None, 0, None) == pkg._abi.NLS_ERR_INVALID_ARG
