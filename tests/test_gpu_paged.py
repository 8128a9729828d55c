"""GPU parity: paged GQA decode (configs 3, 4), fused append, chunk append, gather.

Cache writes (append, quantise, gather) must be bit-exact against the
oracle; attention outputs within 2e-3 relative (f16 / int8 KV, f32 accumulate):
|o - ref| <= 2e-3 * max(|ref|, 1).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from doe_b200 import ops, workloads
from doe_b200._abi import DOE_DEVICE_ERR_LENGTH, DOE_DEVICE_ERR_PAGE
from doe_b200.kv import PagedKVCache

from .gpu_util import max_rel, within

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

F16_TOL = 2e-3


def _cache(w: workloads.PagedWorkload, seed: int = 11) -> PagedKVCache:
    c = PagedKVCache(num_pages=w.num_pages, page_size=w.page_size, num_kv_heads=w.num_kv_heads,
                     head_dim=w.head_dim, block_table=w.block_table, kv_dtype=w.kv_dtype)
    workloads.fill_pools(c, seed)
    return c


def _host(c: PagedKVCache):
    kp = c.k_pool.cpu().numpy()
    vp = c.v_pool.cpu().numpy()
    if c.kv_dtype == "f16":
        return kp.view(np.uint16).copy(), vp.view(np.uint16).copy(), None, None
    return kp.copy(), vp.copy(), c.k_scale.cpu().numpy().view(np.uint16).copy(), \
        c.v_scale.cpu().numpy().view(np.uint16).copy()


def _oracle_step(w, kp, vp, ks, vs, rows=None):
    """Oracle: append the new token at ctx, then decode over ctx + 1 tokens."""
    sel = np.arange(w.num_seqs) if rows is None else np.asarray(rows)
    oracle.paged_append(w.new_k[sel][:, None].view(np.uint16), w.new_v[sel][:, None].view(np.uint16),
                        kp, vp, w.block_table[sel], w.ctx[sel].astype(np.int32),
                        page_size=w.page_size, k_scale=ks, v_scale=vs)
    return oracle.paged_decode(w.q[sel].view(np.uint16), kp, vp, w.block_table[sel],
                               w.seq_lens[sel], w.scale, page_size=w.page_size, k_scale=ks,
                               v_scale=vs)


def _gpu_step(w, c, split_pages=0, status=None):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = ops.paged_decode(c, t(w.q), t(w.seq_lens), w.scale, new_k=t(w.new_k), new_v=t(w.new_v),
                           split_pages=split_pages, status=status)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("kv_dtype", ["f16", "int8"])
@pytest.mark.parametrize("H,Hkv", [(32, 8), (8, 8), (16, 2), (8, 1)])
def test_paged_decode_fused_append_small(kv_dtype, H, Hkv):
    w = workloads.small_paged(5, [0, 1, 15, 16, 17, 300, 1000, 2049], num_heads=H, num_kv_heads=Hkv,
                              kv_dtype=kv_dtype)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    ref = _oracle_step(w, kp, vp, ks, vs)
    status = ops.status_word()
    out = _gpu_step(w, c, status=status)
    gk, gv, gks, gvs = _host(c)
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp), "append wrote different cache bytes"
    if ks is not None:
        assert np.array_equal(gks, ks) and np.array_equal(gvs, vs), "append wrote different scales"
    assert int(status.item()) == 0
    within(out, ref, F16_TOL)


@pytest.mark.parametrize("split_pages", [1, 2, 3, 64])
@pytest.mark.parametrize("page_size", [16, 32, 64])
def test_paged_decode_split_and_page_sizes(split_pages, page_size):
    w = workloads.small_paged(9, [5, 90, 257, 700], page_size=page_size)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    ref = _oracle_step(w, kp, vp, ks, vs)
    within(_gpu_step(w, c, split_pages=split_pages), ref, F16_TOL)


@pytest.mark.parametrize("split_pages", [1, 3, 0, 400])
def test_paged_decode_inputs_stable_and_long_splits(split_pages):
    """DOE_DECODE_INPUTS_STABLE issues each warp's first copy before the
    append and the query work, except the copy of the tile that receives the
    new row (split_pages 1: that tile is the only one of the last split;
    3: the first tile of warp 2 there).  split_pages 400 gives splits of 400
    tiles, so a warp walks up to 100 tiles and reads page ids from every
    register of its prefetch (tiles 0-31, 32-63, 64-95, 96-127)."""
    w = workloads.small_paged(17, [0, 15, 16, 33, 300, 2049, 6000, 6399])
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    ref = _oracle_step(w, kp, vp, ks, vs)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    status = ops.status_word()
    out = ops.paged_decode(c, t(w.q), t(w.seq_lens), w.scale, new_k=t(w.new_k), new_v=t(w.new_v),
                           split_pages=split_pages, status=status, inputs_stable=True)
    torch.cuda.synchronize()
    gk, gv, _, _ = _host(c)
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp), "append wrote different cache bytes"
    assert int(status.item()) == 0
    within(out.cpu().numpy(), ref, F16_TOL)


def test_paged_decode_without_append_reads_cache_only():
    w = workloads.small_paged(13, [40, 3, 129])
    c = _cache(w)
    kp, vp, _, _ = _host(c)
    lens = (w.ctx + 1).astype(np.int32)
    ref = oracle.paged_decode(w.q.view(np.uint16), kp, vp, w.block_table, lens, w.scale,
                              page_size=w.page_size)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = ops.paged_decode(c, t(w.q), t(lens), w.scale).cpu().numpy()
    within(out, ref, F16_TOL)
    assert np.array_equal(c.k_pool.cpu().numpy().view(np.uint16), kp)  # nothing written


@pytest.mark.parametrize("kv_dtype,Hkv,page_size", [("f16", 8, 16), ("int8", 8, 16), ("int8", 4, 48),
                                                    ("int8", 2, 32), ("int8", 1, 16), ("int8", 8, 80)])
def test_chunk_append_bit_exact(kv_dtype, Hkv, page_size):
    w = workloads.small_paged(21, [0, 37, 100], num_heads=4 * Hkv, num_kv_heads=Hkv, page_size=page_size,
                              kv_dtype=kv_dtype, extra_tokens=64)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    g = np.random.default_rng(3)
    T = 45
    nk = g.standard_normal((w.num_seqs, T, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    nv = g.standard_normal((w.num_seqs, T, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    nk[0, 3] = 0  # an all-zero row quantises to scale 0
    nv[1, 4, 0] *= np.float16(1e-6)  # subnormal scale: the clamped path
    nv[2, 5, -1, 7] = np.float16(60000.0)  # a large row maximum
    nk[1, 6, 0, :] = np.float16(2.0 ** -24)  # every element the smallest subnormal
    pos = w.ctx.astype(np.int32)
    oracle.paged_append(nk.view(np.uint16), nv.view(np.uint16), kp, vp, w.block_table, pos,
                        page_size=w.page_size, k_scale=ks, v_scale=vs)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    status = ops.status_word()
    ops.paged_append(c, t(nk), t(nv), t(pos), status=status)
    gk, gv, gks, gvs = _host(c)
    assert int(status.item()) == 0
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp)
    if ks is not None:
        assert np.array_equal(gks, ks) and np.array_equal(gvs, vs)


@pytest.mark.parametrize("kv_dtype", ["f16", "int8"])
def test_chunk_append_bad_page_reports_and_skips_those_tokens(kv_dtype):
    """A table entry outside the pool: the tokens that land on it are not
    written and DOE_DEVICE_ERR_PAGE is set; every other token is."""
    w = workloads.small_paged(23, [5, 40], kv_dtype=kv_dtype, extra_tokens=48)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    bt = w.block_table.copy()
    bad_seq, bad_idx = 1, (40 + 20) // w.page_size  # a page in the middle of seq 1's chunk
    bt[bad_seq, bad_idx] = w.num_pages + 3
    c.set_block_table(bt)
    g = np.random.default_rng(5)
    T = 40
    nk = g.standard_normal((w.num_seqs, T, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    nv = g.standard_normal((w.num_seqs, T, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    pos = w.ctx.astype(np.int32)
    keep = np.ones((w.num_seqs, T), bool)
    for t in range(T):
        keep[bad_seq, t] = (int(pos[bad_seq]) + t) // w.page_size != bad_idx
    for b in range(w.num_seqs):  # the oracle appends the kept tokens one at a time
        for t in np.nonzero(keep[b])[0]:
            oracle.paged_append(nk[b:b + 1, t:t + 1].view(np.uint16), nv[b:b + 1, t:t + 1].view(np.uint16),
                                kp, vp, w.block_table[b:b + 1], np.array([pos[b] + t], np.int32),
                                page_size=w.page_size, k_scale=ks, v_scale=vs)
    t_ = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    status = ops.status_word()
    ops.paged_append(c, t_(nk), t_(nv), t_(pos), status=status)
    gk, gv, gks, gvs = _host(c)
    assert int(status.item()) & DOE_DEVICE_ERR_PAGE
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp)
    if ks is not None:
        assert np.array_equal(gks, ks) and np.array_equal(gvs, vs)


@pytest.mark.parametrize("kv_dtype", ["f16", "int8"])
def test_gather_bit_exact(kv_dtype):
    w = workloads.small_paged(31, [50, 300], kv_dtype=kv_dtype)
    c = _cache(w)
    kp, vp, ks, vs = _host(c)
    for seq, start, length in ((0, 0, 51), (1, 17, 200), (1, 0, 1)):
        res = ops.paged_gather(c, seq, start, length)
        full_k = oracle.paged_gather(kp if kv_dtype == "f16" else kp, w.block_table[seq],
                                     start + length, page_size=w.page_size)[start:]
        full_v = oracle.paged_gather(vp, w.block_table[seq], start + length, page_size=w.page_size)[start:]
        gk = res[0].cpu().numpy()
        gv = res[1].cpu().numpy()
        if kv_dtype == "f16":
            gk, gv = gk.view(np.uint16), gv.view(np.uint16)
        assert np.array_equal(gk, full_k) and np.array_equal(gv, full_v)
        if kv_dtype == "int8":
            rows = np.array([w.block_table[seq][p // w.page_size] for p in range(start, start + length)])
            inp = np.array([p % w.page_size for p in range(start, start + length)])
            assert np.array_equal(res[2].cpu().numpy().view(np.uint16), ks[rows, :, inp])


def test_bad_block_table_sets_status_and_skips():
    w = workloads.small_paged(41, [20, 20])
    c = _cache(w)
    bt = w.block_table.copy()
    bt[1, 0] = w.num_pages + 5  # outside the pool
    c.set_block_table(bt)
    status = ops.status_word()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = ops.paged_decode(c, t(w.q), t(w.seq_lens), w.scale, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & DOE_DEVICE_ERR_PAGE
    assert np.isfinite(out.cpu().numpy()).all()
    # a length beyond the block table is clamped and reported
    c.set_block_table(w.block_table)
    status.zero_()
    lens = w.seq_lens.copy()
    lens[0] = w.block_table.shape[1] * w.page_size + 100
    ops.paged_decode(c, t(w.q), t(lens), w.scale, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & DOE_DEVICE_ERR_LENGTH


def _full_size(w, seed):
    """Every sequence of a full-size config: the fused append's pool bytes
    (and int8 scales) bit-exact over the whole pool, every output row within
    the f16 bound."""
    c = _cache(w, seed)
    kp, vp, ks, vs = _host(c)
    out = _gpu_step(w, c)
    assert np.isfinite(out).all()
    ref = _oracle_step(w, kp, vp, ks, vs)
    gk, gv, gks, gvs = _host(c)
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp), "fused append wrote different pool bytes"
    if ks is not None:
        assert np.array_equal(gks, ks) and np.array_equal(gvs, vs), "fused append wrote different scales"
    within(out, ref, F16_TOL)
    return c, kp, vp, ks, vs, out, ref


def test_config3_full_size_parity():
    w = workloads.paged_f16()
    assert int(w.ctx.sum()) == 309371 and w.num_pages == 19369
    _full_size(w, seed=2)


def test_config4_full_size_parity():
    w = workloads.paged_int8()
    assert int(w.ctx.sum()) == 623873
    _full_size(w, seed=3)


def test_config4_chunk_append_full_size_bit_exact():
    """Config 4b: 512 tokens per sequence quantised into the full-size pool
    (after the decode token), pool bytes and scales compared bit for bit."""
    w = workloads.paged_int8()
    c = _cache(w, 3)
    kp, vp, ks, vs = _host(c)
    g = np.random.default_rng(w.seed + 100)
    T = 512
    nk = g.standard_normal((w.num_seqs, T, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    nv = g.standard_normal((w.num_seqs, T, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    pos = (w.ctx + 1).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    status = ops.status_word()
    ops.paged_append(c, t(nk), t(nv), t(pos), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    oracle.paged_append(nk.view(np.uint16), nv.view(np.uint16), kp, vp, w.block_table, pos,
                        page_size=w.page_size, k_scale=ks, v_scale=vs)
    gk, gv, gks, gvs = _host(c)
    assert np.array_equal(gk, kp) and np.array_equal(gv, vp)
    assert np.array_equal(gks, ks) and np.array_equal(gvs, vs)


def _shard_cache(w, full, shard):
    """The cache one rank holds for `shard` (a workloads.subset of w): the
    shard's pages copied out of the full pool in the subset's renumbering."""
    rows = w.block_table[shard.meta["global_index"]]
    used = torch.from_numpy(np.unique(rows[rows >= 0]).astype(np.int64)).cuda()
    c = PagedKVCache(num_pages=shard.num_pages, page_size=w.page_size, num_kv_heads=w.num_kv_heads,
                     head_dim=w.head_dim, block_table=shard.block_table, kv_dtype=w.kv_dtype)
    P = w.page_size
    for dst, src in ((c.k_pool, full.k_pool), (c.v_pool, full.v_pool)):
        dst.view(shard.num_pages, P, *dst.shape[1:]).copy_(src.view(w.num_pages, P, *src.shape[1:])[used])
    if w.kv_dtype == "int8":
        c.k_scale.copy_(full.k_scale[used])
        c.v_scale.copy_(full.v_scale[used])
    return c, used.cpu().numpy()


@pytest.fixture(scope="module")
def config4_reference():
    """Config 4 at full size: the filled device cache (before any append) and
    the oracle's fused append + decode of every sequence."""
    w = workloads.paged_int8()
    full = _cache(w, 3)
    kp, vp, ks, vs = _host(full)
    ref = _oracle_step(w, kp, vp, ks, vs)
    yield w, full, (kp, vp, ks, vs), ref
    del full
    torch.cuda.empty_cache()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config4_sequence_shards_match_oracle(world, config4_reference):
    """Config 4 split by sequence over `world` GPUs (LPT on tokens, the split
    bench.py runs under torchrun), one shard after another on this GPU: each
    rank's outputs equal the oracle's rows for its sequences, and its pages
    equal the oracle's appended pages."""
    from doe_b200 import shard as shard_mod

    w, full, (kp, vp, ks, vs), ref = config4_reference
    shards = shard_mod.lpt_assign(w.seq_lens, world)
    assert sorted(np.concatenate(shards).tolist()) == list(range(w.num_seqs))
    P = w.page_size
    for idx in shards:
        sw = workloads.subset(w, idx)
        c, used = _shard_cache(w, full, sw)
        out = _gpu_step(sw, c)
        within(out, ref[idx], F16_TOL)
        gk, gv, gks, gvs = _host(c)
        assert np.array_equal(gk.reshape(len(used), P, -1), kp.reshape(w.num_pages, P, -1)[used])
        assert np.array_equal(gv.reshape(len(used), P, -1), vp.reshape(w.num_pages, P, -1)[used])
        assert np.array_equal(gks, ks[used]) and np.array_equal(gvs, vs[used])
        del c
