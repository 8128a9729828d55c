"""GPU parity: RoPE fused into the paged append and the paged decode.

The oracle composes the reference's own pieces: rope.wgsl (oracle.rope, f32)
on the f16 rows at their absolute positions, rounding to f16, then the paged
append / decode restatements.  Cache bytes must match bit for bit; attention
outputs within 2e-3: |o - ref| <= 2e-3 * max(|ref|, 1).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from doe_b200 import ops, workloads
from doe_b200._abi import DOE_DEVICE_ERR_POSITION
from doe_b200.kv import PagedKVCache

from .gpu_util import within

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

F16_TOL = 2e-3


def rope_table(positions: int, head_dim: int = 128, theta: float = 10000.0) -> np.ndarray:
    """[positions, D/2, {cos, sin}] f32 with angle pos * theta^(-2i/D)."""
    inv = theta ** (-np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    ang = np.arange(positions, dtype=np.float64)[:, None] * inv[None, :]
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def rotate_f16(x: np.ndarray, table: np.ndarray, first_pos: int) -> np.ndarray:
    """x [S, H, D] f16 rotated at positions first_pos + s, rounded to f16."""
    return oracle.rope(x.astype(np.float32), table, position_offset=first_pos).astype(np.float16)


def _cache(w, seed=11):
    c = PagedKVCache(num_pages=w.num_pages, page_size=w.page_size, num_kv_heads=w.num_kv_heads,
                     head_dim=w.head_dim, block_table=w.block_table, kv_dtype=w.kv_dtype)
    workloads.fill_pools(c, seed)
    return c


def _host(c):
    if c.kv_dtype == "f16":
        return (c.k_pool.cpu().numpy().view(np.uint16).copy(), c.v_pool.cpu().numpy().view(np.uint16).copy(),
                None, None)
    return (c.k_pool.cpu().numpy().copy(), c.v_pool.cpu().numpy().copy(),
            c.k_scale.cpu().numpy().view(np.uint16).copy(), c.v_scale.cpu().numpy().view(np.uint16).copy())


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("kv_dtype", ["f16", "int8"])
@pytest.mark.parametrize("Hkv", [8, 2, 1])
def test_chunk_append_rope_bit_exact(kv_dtype, Hkv):
    w = workloads.small_paged(51, [0, 37, 300], num_heads=Hkv * 4, num_kv_heads=Hkv, kv_dtype=kv_dtype,
                              extra_tokens=64)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    g = np.random.default_rng(7)
    T = 40
    nk = g.standard_normal((w.num_seqs, T, Hkv, 128), dtype=np.float32).astype(np.float16)
    nv = g.standard_normal((w.num_seqs, T, Hkv, 128), dtype=np.float32).astype(np.float16)
    pos = w.ctx.astype(np.int32)
    table = rope_table(1024)
    rk = np.stack([rotate_f16(nk[b], table, int(pos[b])) for b in range(w.num_seqs)])
    oracle.paged_append(rk.view(np.uint16), nv.view(np.uint16), kp, vp, w.block_table, pos,
                        page_size=w.page_size, k_scale=ks, v_scale=vs)
    status = ops.status_word()
    ops.paged_append(c, _dev(nk), _dev(nv), _dev(pos), status=status, freq_cis=_dev(table))
    gk, gv, gks, gvs = _host(c)
    assert int(status.item()) == 0
    assert np.array_equal(gk, kp), "rotated K rows differ"
    assert np.array_equal(gv, vp), "V rows differ"
    if ks is not None:
        assert np.array_equal(gks, ks) and np.array_equal(gvs, vs)


@pytest.mark.parametrize("kv_dtype", ["f16", "int8"])
@pytest.mark.parametrize("H,Hkv", [(32, 8), (16, 2)])
def test_paged_decode_rope_fused_append(kv_dtype, H, Hkv):
    w = workloads.small_paged(57, [0, 1, 16, 300, 1000], num_heads=H, num_kv_heads=Hkv, kv_dtype=kv_dtype)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    table = rope_table(2048)
    p = w.ctx.astype(np.int64)  # the new token's (and the query's) position = seq_len - 1
    rq = np.stack([rotate_f16(w.q[b][None], table, int(p[b]))[0] for b in range(w.num_seqs)])
    rk = np.stack([rotate_f16(w.new_k[b][None], table, int(p[b]))[0] for b in range(w.num_seqs)])
    oracle.paged_append(rk[:, None].view(np.uint16), w.new_v[:, None].view(np.uint16), kp, vp, w.block_table,
                        w.ctx.astype(np.int32), page_size=w.page_size, k_scale=ks, v_scale=vs)
    ref = oracle.paged_decode(rq.view(np.uint16), kp, vp, w.block_table, w.seq_lens, w.scale,
                              page_size=w.page_size, k_scale=ks, v_scale=vs)
    status = ops.status_word()
    out = ops.paged_decode(c, _dev(w.q), _dev(w.seq_lens), w.scale, new_k=_dev(w.new_k), new_v=_dev(w.new_v),
                           status=status, freq_cis=_dev(table))
    torch.cuda.synchronize()
    gk, gv, gks, gvs = _host(c)
    assert int(status.item()) == 0
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp), "fused rope append wrote different bytes"
    if ks is not None:
        assert np.array_equal(gks, ks) and np.array_equal(gvs, vs)
    within(out.cpu().numpy(), ref, F16_TOL)


def test_rope_position_beyond_table_is_reported():
    w = workloads.small_paged(61, [30, 5], num_heads=8, num_kv_heads=2)
    c = _cache(w)
    table = rope_table(20)  # sequence 0 appends at 30..33: off the table
    g = np.random.default_rng(2)
    nk = g.standard_normal((2, 4, 2, 128), dtype=np.float32).astype(np.float16)
    status = ops.status_word()
    ops.paged_append(c, _dev(nk), _dev(nk), _dev(w.ctx.astype(np.int32)), status=status, freq_cis=_dev(table))
    torch.cuda.synchronize()
    assert int(status.item()) & DOE_DEVICE_ERR_POSITION
    status.zero_()
    ops.paged_decode(c, _dev(w.q), _dev(w.seq_lens), w.scale, status=status, freq_cis=_dev(table))
    torch.cuda.synchronize()
    assert int(status.item()) & DOE_DEVICE_ERR_POSITION


# ---- sliding window and softcap (attention_head256_f16kv.wgsl:129-135, 197-199)
@pytest.mark.parametrize("kv_dtype", ["f16", "int8"])
@pytest.mark.parametrize("window,softcap", [(1, 0.0), (16, 0.0), (100, 0.0), (5000, 0.0), (0, 30.0),
                                            (0, 5.0), (300, 50.0)])
def test_paged_decode_window_softcap(kv_dtype, window, softcap):
    w = workloads.small_paged(71, [0, 15, 16, 257, 1000, 2049], num_heads=32, num_kv_heads=8, kv_dtype=kv_dtype)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    oracle.paged_append(w.new_k[:, None].view(np.uint16), w.new_v[:, None].view(np.uint16), kp, vp,
                        w.block_table, w.ctx.astype(np.int32), page_size=w.page_size, k_scale=ks, v_scale=vs)
    ref = oracle.paged_decode(w.q.view(np.uint16), kp, vp, w.block_table, w.seq_lens, w.scale,
                              page_size=w.page_size, k_scale=ks, v_scale=vs, sliding_window=window,
                              softcap=softcap)
    status = ops.status_word()
    for split_pages in (0, 2):
        out = ops.paged_decode(c, _dev(w.q), _dev(w.seq_lens), w.scale,
                               new_k=_dev(w.new_k) if split_pages == 0 else None,
                               new_v=_dev(w.new_v) if split_pages == 0 else None,
                               status=status, split_pages=split_pages, sliding_window=window, softcap=softcap)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        within(out.cpu().numpy(), ref, F16_TOL)
    gk, gv, _, _ = _host(c)
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp)


def test_paged_decode_window_softcap_and_rope_together():
    w = workloads.small_paged(73, [3, 400, 1500], num_heads=16, num_kv_heads=2)
    c = _cache(w)
    kp, vp, _, _ = _host(c)
    table = rope_table(2048)
    p = w.ctx.astype(np.int64)
    rq = np.stack([rotate_f16(w.q[b][None], table, int(p[b]))[0] for b in range(w.num_seqs)])
    rk = np.stack([rotate_f16(w.new_k[b][None], table, int(p[b]))[0] for b in range(w.num_seqs)])
    oracle.paged_append(rk[:, None].view(np.uint16), w.new_v[:, None].view(np.uint16), kp, vp, w.block_table,
                        w.ctx.astype(np.int32), page_size=w.page_size)
    ref = oracle.paged_decode(rq.view(np.uint16), kp, vp, w.block_table, w.seq_lens, w.scale,
                              page_size=w.page_size, sliding_window=512, softcap=20.0)
    status = ops.status_word()
    out = ops.paged_decode(c, _dev(w.q), _dev(w.seq_lens), w.scale, new_k=_dev(w.new_k), new_v=_dev(w.new_v),
                           status=status, freq_cis=_dev(table), sliding_window=512, softcap=20.0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    within(out.cpu().numpy(), ref, F16_TOL)


@pytest.mark.parametrize("split_pages", [0, 2])
def test_paged_decode_bf16_output_is_the_rounded_f32_output(split_pages):
    w = workloads.small_paged(79, [0, 33, 700], num_heads=32, num_kv_heads=8)
    c = _cache(w)
    table = rope_table(1024)
    args = dict(seq_lens=_dev(w.seq_lens), scale=w.scale, split_pages=split_pages, freq_cis=_dev(table))
    f32 = ops.paged_decode(c, _dev(w.q), **args)
    status = ops.status_word()
    b16 = ops.paged_decode(c, _dev(w.q), **args, status=status, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(b16, f32.to(torch.bfloat16))
