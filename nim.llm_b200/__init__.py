"""nimllm-sample-b200: B200-native replacement of nimllm's logits->token path.

The product is libnimllm_sample.so (CUDA for sm_100a behind the C ABI in
include/nimllm_sample.h). This package holds its sources (csrc/), its build
script (build.py), a ctypes binding (_abi.py) and a host-side mirror of the
reference's Nim sampler API (sampler.py).

The directory name carries a dot, so import it through `load_package()` in
__graft_entry__.py (or register it yourself with importlib under the module
name `nimllm_b200`).
"""
from . import workloads
from ._abi import EXPORTS, LIB_PATH, NlsError, ROW_PARAMS_DTYPE, load
from .sampler import (Comm, Engine, Rand, Sampler, SamplerParams, accept, argmax, batch_inputs,
                      comm_unique_id, decode_step_many, default_engine, defaultSampling,
                      greedySampling, newSampler, params_record, perplexity_from_logits,
                      row_owner_range, sample, sample_many, topTokens, vocab_shard)

__version__ = "0.1.0"
