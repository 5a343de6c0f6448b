"""nls_sample_batch_noalloc: the entry point for callers that cannot
allocate GPU memory (graph capture, allocator-less hosts, hot serving loops),
so cannot create a handle. It must give the same tokens and probabilities as
nls_sample_batch on the same inputs -- ids identical, probabilities within
1e-5 relative (the tolerance of the other parity tests) -- on two calls in a
row, since every call reuses one fixed scratch array in the library. This
file is collected last so a failure here does not hide the other tests."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_sample_batch_twice(pkg):
    import torch
    lib = pkg.load()
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
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    logits, hist, hoff = t(w.logits), t(w.hist_ids), t(w.hist_off)
    bids, bvals, boff, uni = t(w.bias_ids), t(w.bias_vals), t(w.bias_off), t(w.uniforms)
    params = torch.from_numpy(w.params.view(np.uint8).copy()).to(dev)
    out_ids = torch.empty(w.B, dtype=torch.int64, device=dev)
    out_probs = torch.empty(w.B, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for call in range(2):
        out_ids.fill_(-7)
        out_probs.fill_(-1.0)
        st = lib.nls_sample_batch_noalloc(_dp(logits), V, w.B, V, _dp(params), _dp(hist), _dp(hoff),
                                          _dp(bids), _dp(bvals), _dp(boff), _dp(uni), _dp(out_ids),
                                          _dp(out_probs), ctypes.c_void_p(stream.cuda_stream))
        assert st == 0, f"call {call}: status {st}"
        torch.cuda.synchronize(dev)
        got_ids = out_ids.cpu().numpy()
        got_probs = out_probs.cpu().numpy().astype(np.float64)
        assert np.array_equal(got_ids, ids_ref), f"call {call}: ids differ"
        rel = np.abs(got_probs - probs_ref) / np.maximum(np.abs(probs_ref.astype(np.float64)), 1e-30)
        assert np.all(rel <= 1e-5), f"call {call}: probs rel err {rel.max()}"


def test_noalloc_rejects_sizes_beyond_its_limits(pkg):
    lib = pkg.load()
    one = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    assert lib.nls_sample_batch_noalloc(one, 10, 4097, 10, one, None, None, None, None, None, one,
                                        one, None, None) == pkg._abi.NLS_ERR_CAPACITY
    assert lib.nls_sample_batch_noalloc(one, 1 << 19, 1, (1 << 18) + 1, one, None, None, None,
                                        None, None, one, one, None, None) == pkg._abi.NLS_ERR_CAPACITY
