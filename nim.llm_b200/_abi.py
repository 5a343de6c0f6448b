"""ctypes binding of libnimllm_sample.so (include/nimllm_sample.h).

The library is the product; this module only declares its C entry points.
Loading fails loudly when the library is missing or was built without a GPU
path -- there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libnimllm_sample.so")

NLS_OK = 0
NLS_ERR_INVALID_ARG = 1
NLS_ERR_CUDA = 2
NLS_ERR_NCCL = 3
NLS_ERR_TIMEOUT = 4
NLS_ERR_NAN_LOGITS = 5
NLS_ERR_CAPACITY = 6
NLS_ERR_NO_DEVICE = 7

NLS_DEVICE_INPUTS = 1
NLS_DEVICE_OUTPUTS = 2

# Entry points the header declares; tests check the library exports each one.
EXPORTS = (
    "nls_create", "nls_destroy", "nls_sample_batch", "nls_argmax_batch",
    "nls_stream_status", "nls_status_str", "nls_last_error", "nls_version",
    "nls_set_profiling", "nls_last_kernel_ms", "nls_sample_batch_noalloc",
    "nls_comm_unique_id", "nls_comm_create", "nls_comm_destroy", "nls_sample_batch_vocab_sharded",
    "nls_top_tokens", "nls_token_nll", "nls_lm_head", "nls_lm_head_sample",
    "nls_device_upload", "nls_device_free", "nls_ref_expf_range", "nls_noalloc_status",
    "nls_set_wait_limit", "nls_comm_set_timeout", "nls_comm_abort",
)

# ggml weight types of nls_lm_head (GgmlType codes, quant.nim:14-19)
NLS_WT = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q6_k": 14}
NLS_EXACT_MATMUL = 4
NLS_ROWS_INDEPENDENT = 8

# nls_row_params: 6 doubles + 2 int64, 64 bytes, no padding.
ROW_PARAMS_DTYPE = np.dtype([
    ("temperature", "<f8"), ("top_p", "<f8"), ("min_p", "<f8"),
    ("repeat_penalty", "<f8"), ("presence_penalty", "<f8"),
    ("frequency_penalty", "<f8"), ("top_k", "<i8"), ("repeat_last_n", "<i8"),
])
assert ROW_PARAMS_DTYPE.itemsize == 64

_lib = None


def load(path: str | None = None):
    """Load the library once; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python nim.llm_b200/build.py`")
    L = ctypes.CDLL(path)
    vp, i32, i64, u32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32
    L.nls_create.restype = i32
    L.nls_create.argtypes = [ctypes.POINTER(vp), i32, i32, i32]
    L.nls_destroy.restype = None
    L.nls_destroy.argtypes = [vp]
    L.nls_sample_batch.restype = i32
    L.nls_sample_batch.argtypes = [vp, vp, i64, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, u32, vp]
    L.nls_argmax_batch.restype = i32
    L.nls_argmax_batch.argtypes = [vp, vp, i64, i32, i32, vp, u32, vp]
    L.nls_stream_status.restype = i32
    L.nls_stream_status.argtypes = [vp, vp]
    L.nls_status_str.restype = ctypes.c_char_p
    L.nls_status_str.argtypes = [i32]
    L.nls_last_error.restype = ctypes.c_char_p
    L.nls_last_error.argtypes = [vp]
    L.nls_version.restype = ctypes.c_char_p
    L.nls_version.argtypes = []
    L.nls_set_profiling.restype = i32
    L.nls_set_profiling.argtypes = [vp, i32]
    L.nls_last_kernel_ms.restype = i32
    L.nls_last_kernel_ms.argtypes = [vp, ctypes.POINTER(ctypes.c_float), i32]
    L.nls_sample_batch_noalloc.restype = i32
    L.nls_sample_batch_noalloc.argtypes = [vp, i64, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.nls_comm_unique_id.restype = i32
    L.nls_comm_unique_id.argtypes = [vp]
    L.nls_comm_create.restype = i32
    L.nls_comm_create.argtypes = [ctypes.POINTER(vp), vp, i32, i32, i32]
    L.nls_comm_destroy.restype = None
    L.nls_comm_destroy.argtypes = [vp]
    L.nls_sample_batch_vocab_sharded.restype = i32
    L.nls_sample_batch_vocab_sharded.argtypes = [vp, vp, vp, i64, i32, i32, vp, vp, vp, vp, vp, vp, vp,
                                                 vp, vp, vp]
    L.nls_top_tokens.restype = i32
    L.nls_top_tokens.argtypes = [vp, vp, i64, i32, i32, i32, vp, vp, u32, vp]
    L.nls_token_nll.restype = i32
    L.nls_token_nll.argtypes = [vp, vp, i64, i32, i32, vp, vp, u32, vp]
    L.nls_device_upload.restype = i32
    L.nls_device_upload.argtypes = [vp, vp, ctypes.c_uint64, ctypes.POINTER(vp)]
    L.nls_device_free.restype = None
    L.nls_device_free.argtypes = [vp, vp]
    L.nls_lm_head.restype = i32
    L.nls_lm_head.argtypes = [vp, vp, i32, i32, i32, vp, i32, vp, u32, vp]
    L.nls_lm_head_sample.restype = i32
    L.nls_lm_head_sample.argtypes = [vp, vp, i32, i32, i32, vp, i32, vp, vp, vp, vp, vp, vp, vp, vp,
                                     vp, u32, vp]
    L.nls_comm_set_timeout.restype = i32
    L.nls_comm_set_timeout.argtypes = [vp, ctypes.c_uint64]
    L.nls_comm_abort.restype = i32
    L.nls_comm_abort.argtypes = [vp]
    L.nls_set_wait_limit.restype = i32
    L.nls_set_wait_limit.argtypes = [vp, ctypes.c_uint64]
    L.nls_noalloc_status.restype = i32
    L.nls_noalloc_status.argtypes = [vp, u32, vp]
    L.nls_ref_expf_range.restype = i32
    L.nls_ref_expf_range.argtypes = [u32, i64, vp, vp, vp]
    _lib = L
    return L


class NlsError(RuntimeError):
    """A non-zero nls_status (the Nim side raises CatchableError on these)."""

    def __init__(self, status: int, detail: str = ""):
        self.status = int(status)
        msg = load().nls_status_str(self.status).decode()
        super().__init__(f"nls status {self.status} ({msg}){': ' + detail if detail else ''}")
