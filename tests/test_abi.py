"""The C-ABI library: loads, exports every declared symbol, host-side logic (no GPU)."""
from __future__ import annotations

import ctypes as C
import re
import subprocess

import numpy as np
import pytest

from doe_b200 import _abi as abi
from doe_b200.kv import KvPool

from .conftest import ROOT

HEADER = ROOT / "include" / "doe_cuda.h"


def _declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(doe_[a-z0-9_]+)\s*\(", text))


def test_header_and_bindings_agree():
    declared = _declared_functions()
    assert declared == set(abi.SIGNATURES), declared ^ set(abi.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = abi.lib()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(abi.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (doe_[a-z0-9_]+)$", out, flags=re.M))
    assert _declared_functions() <= exported


def test_abi_version_and_kernel_table():
    lib = abi.lib()
    assert lib.doe_cuda_abi_version() == 1
    for k in ("attention-decode.wgsl", "attention-prefill.wgsl", "attention_head256_f16kv.wgsl",
              "attention_head512_f16kv.wgsl", "attention", "attention_sliding", "attention_prefill",
              "attention_prefill_kv_axis_sharded", "kv_write", "kv_write_shared", "kv_read", "rope", "rope.wgsl",
              "attention_paged_decode", "kv_append_paged", "attention_stitch"):
        assert lib.doe_cuda_kernel_supported(k.encode()) == 1, k
    for k in ("matmul", "rmsnorm", "attention_linear", "", "attention-decode"):
        assert lib.doe_cuda_kernel_supported(k.encode()) == 0, k


def _has_gpu() -> bool:
    n = C.c_int()
    return abi.lib().doe_cuda_device_count(C.byref(n)) == abi.DOE_OK and n.value > 0


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device error path")
def test_open_without_device_reports_no_device():
    h = C.c_void_p()
    rc = abi.lib().doe_cuda_open(0, C.byref(h))
    assert rc == abi.DOE_NO_DEVICE
    assert not h.value
    assert "device" in abi.op_error()


def test_operator_validation_precedes_any_launch():
    lib = abi.lib()
    fake = C.c_void_p(0x1000)  # never dereferenced: every call below fails validation first
    kv = abi.PagedKV(fake, fake, None, None, abi.DOE_KV_F16, 10, 16, 8, 128, 4, fake)
    # heads not a multiple of kv heads
    assert lib.doe_paged_decode(C.byref(kv), 2, 12, fake, fake, None, None, 1.0, fake, 0, None) == \
        abi.DOE_INVALID_ARGUMENT
    # new_k without new_v
    assert lib.doe_paged_decode(C.byref(kv), 2, 32, fake, fake, fake, None, 1.0, fake, 0, None) == \
        abi.DOE_INVALID_ARGUMENT
    # page size not a multiple of 16
    bad = abi.PagedKV(fake, fake, None, None, abi.DOE_KV_F16, 10, 24, 8, 128, 4, fake)
    assert lib.doe_paged_decode(C.byref(bad), 2, 32, fake, fake, None, None, 1.0, fake, 0, None) == \
        abi.DOE_INVALID_ARGUMENT
    # int8 without scales
    i8 = abi.PagedKV(fake, fake, None, None, abi.DOE_KV_INT8, 10, 16, 8, 128, 4, fake)
    assert lib.doe_paged_append(C.byref(i8), 1, 1, fake, fake, fake, None) == abi.DOE_INVALID_ARGUMENT
    # head_dim the tensor-core kernel does not cover: explicit UNSUPPORTED, no fallback
    d64 = abi.PagedKV(fake, fake, None, None, abi.DOE_KV_F16, 10, 16, 8, 64, 4, fake)
    assert lib.doe_paged_decode(C.byref(d64), 2, 32, fake, fake, None, None, 1.0, fake, 0, None) == \
        abi.DOE_UNSUPPORTED
    assert "head_dim" in abi.op_error()
    # null pointers
    assert lib.doe_attention_decode_f32(None, fake, fake, fake, 8, 64, 512, 0.125, None) == \
        abi.DOE_INVALID_ARGUMENT
    assert lib.doe_attention_stitch_f32(fake, 1, 0, 8, fake, None) == abi.DOE_INVALID_ARGUMENT
    assert lib.doe_kv_read_dense(fake, fake, fake, fake, 1, 10, 10, 16, 8, 4, None) == abi.DOE_OUT_OF_RANGE
    assert lib.doe_kv_write_dense(fake, fake, fake, fake, fake, 3, 2, 16, 8, 4, None) == \
        abi.DOE_INVALID_ARGUMENT


def test_workspace_queries_are_host_side():
    lib = abi.lib()
    fake = C.c_void_p(0x1000)
    kv = abi.PagedKV(fake, fake, None, None, abi.DOE_KV_F16, 19369, 16, 8, 128, 513, fake)
    ws = lib.doe_paged_decode_workspace_bytes(C.byref(kv), 64, 32, 0)
    # 64 seqs x 8 kv heads x 9 splits (513 pages / 64-tile splits) x 4 heads x (128 + 2)
    # floats of partials, then one arrival counter per (sequence, kv head)
    parts = 64 * 8 * 9 * 4 * 130 * 4
    assert ws == (parts + 255) // 256 * 256 + 64 * 8 * 4
    # 8 heads x 16 splits (32-token steps: 4 warps x 8 tokens) x (64 + 2) floats
    assert lib.doe_attention_decode_f32_workspace_bytes(8, 64, 512) == 8 * 16 * 66 * 4


def test_kv_pool_allocation_and_block_table():
    pool = KvPool(num_pages=10, page_size=16, max_seqs=3, max_pages_per_seq=4)
    assert pool.free_pages() == 10
    pool.reserve(0, 1)
    pool.reserve(1, 33)  # 3 pages
    pool.reserve(0, 17)  # grows seq 0 to 2 pages
    assert pool.seq_pages(0) == 2 and pool.seq_pages(1) == 3
    bt = pool.block_table()
    assert bt.shape == (3, 4)
    used = bt[bt >= 0]
    assert len(used) == 5 and len(set(used.tolist())) == 5
    assert (bt[2] == -1).all()
    with pytest.raises(abi.DoeError) as e:
        pool.reserve(2, 5 * 16)  # beyond max_pages_per_seq
    assert e.value.rc == abi.DOE_OUT_OF_RANGE
    pool.reserve(2, 4 * 16)
    pool.reserve(1, 4 * 16)  # takes the last free page
    assert pool.free_pages() == 0
    with pytest.raises(abi.DoeError) as e:
        pool.reserve(0, 3 * 16)  # pool exhausted
    assert e.value.rc == abi.DOE_OUT_OF_RANGE
    pool.release(1)
    assert pool.free_pages() == 4
    with pytest.raises(abi.DoeError):
        pool.reserve(7, 1)
    pool.close()


def test_zig_shim_binds_only_declared_symbols():
    """zig/backend/cuda/mod.zig (the backend shim, not compiled here: no Zig
    toolchain) calls only functions include/doe_cuda.h declares and the
    library exports, and fills all eleven BackendVTable slots
    (runtime/zig/src/backend/backend_iface.zig:13-31)."""
    src = (ROOT / "zig" / "backend" / "cuda" / "mod.zig").read_text()
    used = set(re.findall(r'extern "doe_cuda" fn (\w+)\(', src))
    assert used and used <= _declared_functions(), used - _declared_functions()
    lib = abi.lib()
    for name in used:
        assert hasattr(lib, name), name
    slots = ("deinit", "execute_command", "execute_buffer_write_bytes", "set_upload_behavior",
             "set_queue_wait_mode", "set_queue_sync_mode", "set_gpu_timestamp_mode", "flush_queue",
             "prewarm_upload_path", "prewarm_kernel_dispatch", "capture_buffer")
    table = src[src.index("const VTABLE = backend_iface.BackendVTable{"):]
    for s in slots:
        assert f".{s} = " in table, s
