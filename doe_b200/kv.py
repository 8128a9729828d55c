"""KV-cache manager: the host page pool and the device-resident paged cache.

`KvPool` wraps the C pool in libdoe_cuda.so (physical page free list plus
per-sequence block-table rows).  `PagedKVCache` owns the device pools in the
layout the kernels read -- [num_pages * page_size, num_kv_heads, head_dim]
f16 or int8, int8 scales [num_pages, num_kv_heads, page_size] f16 -- and a
device copy of the block table.  This is the per-sequence generalisation of
the reference's single page_table binding
(attention_head256_f16kv.wgsl:38, get_kv_pos :51-63).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _abi as abi


class KvPool:
    """Host page allocator (doe_kv_pool_*)."""

    def __init__(self, num_pages: int, page_size: int, max_seqs: int, max_pages_per_seq: int):
        self._lib = abi.lib()
        h = C.c_void_p()
        abi.check("doe_kv_pool_create",
                  self._lib.doe_kv_pool_create(num_pages, page_size, max_seqs, max_pages_per_seq,
                                               C.byref(h)))
        self._h = h
        self.num_pages, self.page_size = num_pages, page_size
        self.max_seqs, self.max_pages_per_seq = max_seqs, max_pages_per_seq

    def close(self) -> None:
        if self._h:
            self._lib.doe_kv_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reserve(self, seq: int, tokens: int) -> None:
        abi.check("doe_kv_pool_reserve", self._lib.doe_kv_pool_reserve(self._h, seq, tokens))

    def release(self, seq: int) -> None:
        abi.check("doe_kv_pool_release", self._lib.doe_kv_pool_release(self._h, seq))

    def free_pages(self) -> int:
        v = C.c_uint32()
        abi.check("doe_kv_pool_free_pages", self._lib.doe_kv_pool_free_pages(self._h, C.byref(v)))
        return v.value

    def seq_pages(self, seq: int) -> int:
        v = C.c_uint32()
        abi.check("doe_kv_pool_seq_pages", self._lib.doe_kv_pool_seq_pages(self._h, seq, C.byref(v)))
        return v.value

    def block_table(self) -> np.ndarray:
        out = np.empty((self.max_seqs, self.max_pages_per_seq), np.int32)
        abi.check("doe_kv_pool_block_table",
                  self._lib.doe_kv_pool_block_table(self._h, out.ctypes.data, out.size))
        return out


class PagedKVCache:
    """Device pools + block table for the paged kernels (torch tensors on one GPU)."""

    def __init__(self, *, num_pages: int, page_size: int, num_kv_heads: int, head_dim: int,
                 block_table, kv_dtype: str = "f16", device="cuda"):
        import torch

        if kv_dtype not in ("f16", "int8"):
            raise ValueError("kv_dtype must be 'f16' or 'int8'")
        self.num_pages, self.page_size = num_pages, page_size
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self.kv_dtype = kv_dtype
        rows = num_pages * page_size
        tdt = torch.float16 if kv_dtype == "f16" else torch.int8
        self.k_pool = torch.zeros((rows, num_kv_heads, head_dim), dtype=tdt, device=device)
        self.v_pool = torch.zeros_like(self.k_pool)
        if kv_dtype == "int8":
            self.k_scale = torch.zeros((num_pages, num_kv_heads, page_size), dtype=torch.float16,
                                       device=device)
            self.v_scale = torch.zeros_like(self.k_scale)
        else:
            self.k_scale = self.v_scale = None
        self.set_block_table(block_table)

    def set_block_table(self, block_table) -> None:
        import torch

        bt = torch.as_tensor(np.ascontiguousarray(block_table, dtype=np.int32))
        self.block_table = bt.to(self.k_pool.device)
        self.max_pages_per_seq = int(bt.shape[1])

    def struct(self) -> abi.PagedKV:
        return abi.PagedKV(
            self.k_pool.data_ptr(), self.v_pool.data_ptr(),
            self.k_scale.data_ptr() if self.k_scale is not None else None,
            self.v_scale.data_ptr() if self.v_scale is not None else None,
            abi.DOE_KV_INT8 if self.kv_dtype == "int8" else abi.DOE_KV_F16,
            self.num_pages, self.page_size, self.num_kv_heads, self.head_dim,
            self.max_pages_per_seq, self.block_table.data_ptr())

    def nbytes(self) -> int:
        n = self.k_pool.numel() * self.k_pool.element_size() * 2
        if self.k_scale is not None:
            n += self.k_scale.numel() * 2 * 2
        return n
