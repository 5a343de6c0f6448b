"""CPU checks of the C-ABI boundary: the library loads, exports exactly the
entry points include/nimllm_sample.h declares, the params record has the C
layout, and argument errors come back as status codes (no GPU needed)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nimllm_sample.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"NLS_API\s+[\w\s\*]*?\b(nls_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load()
    names = declared_functions()
    assert names == sorted(pkg.EXPORTS)
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted(set(re.findall(r" T (nls_\w+)", out)))
    assert exported == names


def test_version_and_status_strings(pkg):
    lib = pkg.load()
    assert b"sm_100a" in lib.nls_version()
    assert lib.nls_status_str(0) == b"ok"
    assert lib.nls_status_str(5).startswith(b"NaN")
    assert lib.nls_status_str(999) == b"unknown status"


def test_null_handle_and_bad_args_return_status(pkg):
    lib = pkg.load()
    x = np.zeros(4, np.float32)
    ids = np.zeros(1, np.int64)
    st = lib.nls_sample_batch(None, x.ctypes.data, 4, 1, 4, None, None, None, None, None, None,
                              None, ids.ctypes.data, None, 0, None)
    assert st == pkg._abi.NLS_ERR_INVALID_ARG
    assert lib.nls_argmax_batch(None, x.ctypes.data, 4, 1, 4, ids.ctypes.data, 0, None) == 1
    h = ctypes.c_void_p()
    assert lib.nls_create(ctypes.byref(h), 0, 0, 10) == pkg._abi.NLS_ERR_INVALID_ARG
    assert lib.nls_create(ctypes.byref(h), 0, 1, (1 << 18) + 1) == pkg._abi.NLS_ERR_INVALID_ARG
    assert lib.nls_create(None, 0, 1, 10) == pkg._abi.NLS_ERR_INVALID_ARG
    lib.nls_destroy(None)


def test_create_without_device_fails_cleanly(pkg):
    """On a machine without a GPU the handle is not created (no fallback)."""
    lib = pkg.load()
    h = ctypes.c_void_p()
    st = lib.nls_create(ctypes.byref(h), 0, 4, 100)
    if st == 0:  # a GPU is present: this check belongs to the CPU-only run
        lib.nls_destroy(h)
        return
    assert st in (pkg._abi.NLS_ERR_NO_DEVICE, pkg._abi.NLS_ERR_CUDA)
    assert not h.value


def test_row_params_layout_matches_c(pkg):
    prog = r'''
    #include <stdio.h>
    #include <stddef.h>
    #include "nimllm_sample.h"
    int main(void) {
      printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(nls_row_params),
        offsetof(nls_row_params, temperature), offsetof(nls_row_params, top_p),
        offsetof(nls_row_params, min_p), offsetof(nls_row_params, repeat_penalty),
        offsetof(nls_row_params, presence_penalty), offsetof(nls_row_params, frequency_penalty),
        offsetof(nls_row_params, top_k), offsetof(nls_row_params, repeat_last_n));
      return 0; }
    '''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(prog)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        vals = [int(v) for v in subprocess.run([exe], capture_output=True, text=True,
                                               check=True).stdout.split()]
    dt = pkg.ROW_PARAMS_DTYPE
    assert vals[0] == dt.itemsize
    assert vals[1:] == [dt.fields[n][1] for n in dt.names]
