"""The paged decode's automatic split rule (host logic, no GPU): the split
count read back from doe_paged_decode_workspace_bytes, whose partials area is
num_seqs x Hkv x splits x group x (D + 2) floats (rounded up to 256 bytes)
plus one counter per (sequence, kv head).

- config 5's decoder at tp1 (256 uniform (sequence, kv head) rows of 257
  tiles): one split per row, one wave of CTAs;
- its tensor-parallel ranks (128 / 64 rows): as few splits as keep about two
  CTAs per SM busy (3 / 5);
- config 4's int8 batch and its shards over 2, 4 and 8 ranks (ragged lengths
  up to 2049 tiles): splits of at most 128 tiles, which balance as CTAs finish.
"""
from __future__ import annotations

import ctypes as C

import pytest

from doe_b200 import _abi as abi

# never dereferenced: the size query only plans the launch
_P = C.c_void_p(0x100000)


def _splits(num_seqs, num_heads, num_kv_heads, max_pages, int8=False, page_size=16):
    kv = abi.PagedKV(_P, _P, _P if int8 else None, _P if int8 else None, 1 if int8 else 0, 1 << 20,
                     page_size, num_kv_heads, 128, max_pages, _P)
    ws = abi.lib().doe_paged_decode_workspace_bytes(C.byref(kv), num_seqs, num_heads, 0)
    assert ws > 0, abi.op_error()
    rows, group = num_seqs * num_kv_heads, num_heads // num_kv_heads
    for s in range(1, 1 << 12):
        part = rows * s * group * 130 * 4
        if (part + 255) // 256 * 256 + rows * 4 == ws:
            return s
    raise AssertionError(f"workspace of {ws} bytes matches no split count")


@pytest.mark.parametrize("heads,kv_heads,expect", [(32, 8, 1), (16, 4, 3), (8, 2, 5)])
def test_decoder_rows(heads, kv_heads, expect):
    assert _splits(32, heads, kv_heads, 258) == expect


@pytest.mark.parametrize("num_seqs", [32, 16, 8, 4])
def test_int8_config4_shards_keep_short_splits(num_seqs):
    s = _splits(num_seqs, 32, 8, 2049, int8=True)
    assert -(-2049 // s) <= 128, f"{s} splits of {-(-2049 // s)} tiles"
