"""doe_b200 -- B200-native (sm_100a) attention / KV-cache backend for Doe.

The compute lives in libdoe_cuda.so (doe_b200/csrc, C ABI in
include/doe_cuda.h).  This package holds its build script and thin Python
views of its two surfaces:

  doe_b200.backend  -- the handle / kernel_dispatch backend (Doe's BackendIface)
  doe_b200.ops      -- direct operator launches on torch device tensors
  doe_b200.kv       -- the KV page pool and the device paged cache
  doe_b200.ort_ep   -- the ORT plugin EP's basic f32 operators (execute(kind, ...))
  doe_b200.decoder  -- a Llama-style decoder step on the library's kernels
  doe_b200.tp       -- peer buffers for its tensor-parallel reduction
"""
from ._abi import DoeError, lib  # noqa: F401

__all__ = ["DoeError", "lib"]
