"""The reference's exponential, bit for bit.

The reference's softmax computes exp(float32) (sampler.nim:56), which Nim
maps to the C library's expf; on the reference's x86-64 Linux builds that is
glibc's expf, which is not correctly rounded. These tests pin
  - on the CPU: how many floats in [-104, 0] glibc's expf rounds differently
    from the correctly rounded exponential (so that a device function built
    on double-precision exp would not match), and that the C restatement of
    glibc's published method (tests/host_expf.c) matches glibc's expf on
    every float of the sampler's domain and of the positive range;
  - on the GPU: that the device function every sampling kernel uses
    (ref_expf, reached through nls_ref_expf_range) equals glibc's expf on
    every float in [-104, 0], and that the cheaper estimate the full-sort
    kernel uses for rounding-unit decisions stays within its bracket
    (2^-20 relative wherever it is at least 2^-120).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import pytest

TESTS = os.path.dirname(os.path.abspath(__file__))
NEG_FIRST = 0x80000000           # -0.0
NEG_LAST = 0xC2D00000            # -104.0
POS_LAST = 0x42B17218            # 88.7228..., the largest float whose expf is finite


@pytest.fixture(scope="module")
def hx(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("hx") / "libhost_expf.so")
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-pthread", "-o", out,
                    os.path.join(TESTS, "host_expf.c"), "-lm"], check=True)
    L = ctypes.CDLL(out)
    L.nhx_count.restype = ctypes.c_int64
    L.nhx_count.argtypes = [ctypes.c_int, ctypes.c_uint32, ctypes.c_int64, ctypes.c_void_p,
                            ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
    L.method_expf.restype = ctypes.c_float
    L.method_expf.argtypes = [ctypes.c_float]
    return L


def threads():
    return max(1, min(64, os.cpu_count() or 1))


def count(L, what, first, n, dev=None):
    fb = ctypes.c_int64(-1)
    c = L.nhx_count(what, first, n, dev, threads(), ctypes.byref(fb))
    return c, fb.value


def test_glibc_expf_is_not_the_rounded_double_exp(hx):
    """97,052 floats in [-104, 0] with glibc 2.39 (the count depends on the
    C library; what matters is that it is not zero)."""
    n, first_bad = count(hx, 0, NEG_FIRST, NEG_LAST - NEG_FIRST + 1)
    print(f"glibc expf vs (float)exp((double)x) on [-104, 0]: {n} mismatches")
    assert n > 0 and first_bad >= 0


def test_method_restatement_matches_glibc_everywhere(hx):
    n, first_bad = count(hx, 1, NEG_FIRST, NEG_LAST - NEG_FIRST + 1)
    assert n == 0, f"first mismatch at bits {NEG_FIRST + first_bad:#x}"
    n, first_bad = count(hx, 1, 0, POS_LAST + 1)
    assert n == 0, f"first mismatch at bits {first_bad:#x}"
    # special values and the ends of the domain
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    for x in (0.0, -0.0, -103.97, -103.98, -104.0, -200.0, float("-inf"), 88.72, 88.73,
              float("inf")):
        assert np.float32(hx.method_expf(x)).tobytes() == np.float32(libm.expf(x)).tobytes(), x
    assert np.isnan(hx.method_expf(float("nan")))


@pytest.mark.gpu
def test_device_expf_matches_glibc_on_the_softmax_domain(pkg, hx):
    import torch
    lib = pkg.load()
    dev = torch.device("cuda", 0)
    chunk = 1 << 26
    out = torch.empty(chunk, dtype=torch.float32, device=dev)
    est = torch.empty(chunk, dtype=torch.float32, device=dev)
    host = torch.empty(chunk, dtype=torch.float32, pin_memory=True)
    host_est = torch.empty(chunk, dtype=torch.float32, pin_memory=True)
    total = NEG_LAST - NEG_FIRST + 1
    mism = 0
    worst = 0.0
    stream = torch.cuda.current_stream(dev)
    for start in range(0, total, chunk):
        n = min(chunk, total - start)
        st = lib.nls_ref_expf_range(NEG_FIRST + start, n, out.data_ptr(), est.data_ptr(),
                                    ctypes.c_void_p(stream.cuda_stream))
        assert st == 0
        host[:n].copy_(out[:n])
        host_est[:n].copy_(est[:n])
        torch.cuda.synchronize(dev)
        c, fb = count(hx, 2, NEG_FIRST + start, n, host.data_ptr())
        assert c == 0, f"device expf differs from glibc at bits {NEG_FIRST + start + fb:#x}"
        mism += c
        r = host[:n].numpy().astype(np.float64)
        e = host_est[:n].numpy().astype(np.float64)
        sel = e >= 2.0 ** -120
        if sel.any():
            rel = np.abs(e[sel] - r[sel]) / r[sel]
            worst = max(worst, float(rel.max()))
    print(f"device ref_expf vs glibc on [-104, 0]: {mism} mismatches; estimate bracket "
          f"max rel {worst:.3g}")
    assert worst <= 2.0 ** -20
