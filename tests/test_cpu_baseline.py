"""The timed CPU baseline (oracle/cpu_baseline.c) computes what the parity
oracle computes, bit for bit: f16 and int8 pools, GQA groups 1 to 8, ragged
lengths, sliding windows and softcaps.  bench.py times it as the CPU leg."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from doe_b200 import workloads

pytestmark = pytest.mark.skipif(not oracle.fast_decode_available(), reason="needs AVX2 + F16C")


def _pools(w, seed):
    g = np.random.default_rng(seed)
    rows = w.num_pages * w.page_size
    shape = (rows, w.num_kv_heads, w.head_dim)
    x = g.standard_normal((2,) + shape, dtype=np.float32).astype(np.float16)
    if w.kv_dtype == "f16":
        return x[0].view(np.uint16), x[1].view(np.uint16), None, None
    qk, sk = oracle.quantize_rows_int8(x[0].view(np.uint16).reshape(-1, w.head_dim))
    qv, sv = oracle.quantize_rows_int8(x[1].view(np.uint16).reshape(-1, w.head_dim))
    # scales [rows, Hkv] -> page-blocked [pages, Hkv, page]
    blk = lambda s: s.reshape(w.num_pages, w.page_size, w.num_kv_heads).transpose(0, 2, 1).copy()
    return qk.reshape(shape), qv.reshape(shape), blk(sk), blk(sv)


@pytest.mark.parametrize("kv_dtype", ["f16", "int8"])
@pytest.mark.parametrize("H,Hkv", [(32, 8), (8, 8), (16, 2)])
@pytest.mark.parametrize("window,softcap", [(0, 0.0), (100, 0.0), (0, 30.0)])
def test_bit_identical_to_oracle(kv_dtype, H, Hkv, window, softcap):
    w = workloads.small_paged(H + Hkv, [0, 1, 31, 32, 300, 1000], num_heads=H, num_kv_heads=Hkv,
                              kv_dtype=kv_dtype)
    kp, vp, ks, vs = _pools(w, 5)
    args = (w.q.view(np.uint16), kp, vp, w.block_table, w.seq_lens, w.scale)
    kw = dict(page_size=w.page_size, k_scale=ks, v_scale=vs, sliding_window=window, softcap=softcap)
    ref = oracle.paged_decode(*args, **kw)
    got = oracle.cpu_paged_decode(*args, **kw)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
