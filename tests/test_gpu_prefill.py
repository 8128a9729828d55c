"""GPU parity: tcgen05 causal prefill (config 2) and its fused KV-cache write.

Attention rows are checked against the oracle's head256 online softmax
(f16 Q/K/V, f32 accumulate) within 2e-3: |o - ref| <= 2e-3 * max(|ref|, 1).
The cache rows the kernel writes must equal the prompt's K/V bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from doe_b200 import ops, workloads
from doe_b200.kv import PagedKVCache

from .gpu_util import within

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 2e-3


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _oracle_rows(q, k, v, rows, causal, scale):
    S, H, D = q.shape
    Hkv = k.shape[1]
    kb, vb = k.view(np.uint16), v.view(np.uint16)
    out = []
    for r in rows:
        u = dict(num_heads=H, num_kv_heads=Hkv, head_dim=D, seq_len=S, query_len=1, scale=scale,
                 is_causal=int(causal), start_pos=int(r), attn_softcap=0.0, sliding_window=0,
                 kv_len_source=0, kv_start=0, page_size=16, kv_layout=0)
        out.append(oracle.attention_online_f16kv(u, q[r:r + 1].astype(np.float32), kb, vb)[0])
    return np.stack(out)


def _case(S, H, Hkv, seed):
    g = np.random.default_rng(seed)
    mk = lambda h: (g.standard_normal((S, h, 128), dtype=np.float32) * np.float32(0.5)).astype(np.float16)
    return mk(H), mk(Hkv), mk(Hkv)


@pytest.mark.parametrize("S,H,Hkv", [(128, 2, 2), (256, 4, 4), (200, 2, 1), (64, 1, 1), (130, 2, 2),
                                     (1000, 4, 2)])
def test_prefill_matches_oracle(S, H, Hkv):
    q, k, v = _case(S, H, Hkv, S + H)
    scale = 1.0 / np.sqrt(128)
    status = ops.status_word()
    out = ops.attention_prefill_f16(_t(q), _t(k), _t(v), scale, status=status).cpu().numpy()
    assert int(status.item()) == 0
    rows = np.arange(S) if S <= 256 else np.unique(np.r_[0, 1, 127, 128, 129, S - 1,
                                                          np.random.default_rng(0).integers(0, S, 24)])
    within(out[rows], _oracle_rows(q, k, v, rows, True, scale), TOL)


def test_prefill_noncausal_matches_oracle():
    S, H = 200, 2
    q, k, v = _case(S, H, H, 3)
    scale = 0.1
    out = ops.attention_prefill_f16(_t(q), _t(k), _t(v), scale, causal=False).cpu().numpy()
    within(out, _oracle_rows(q, k, v, np.arange(S), False, scale), TOL)


@pytest.mark.parametrize("cache_start", [0, 32])
def test_prefill_writes_paged_cache_bit_exact(cache_start):
    S, H, Hkv, page = 256, 4, 2, 16
    q, k, v = _case(S, H, Hkv, 9)
    g = np.random.default_rng(1)
    pages = (cache_start + S) // page + 2
    table = np.full((2, pages + 1), -1, np.int32)
    table[1, :pages] = g.permutation(pages).astype(np.int32)
    cache = PagedKVCache(num_pages=pages, page_size=page, num_kv_heads=Hkv, head_dim=128,
                         block_table=table)
    status = ops.status_word()
    out = ops.attention_prefill_f16(_t(q), _t(k), _t(v), 1 / np.sqrt(128), cache=cache, cache_seq=1,
                                    cache_start=cache_start, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    kp = cache.k_pool.cpu().numpy().view(np.uint16)
    vp = cache.v_pool.cpu().numpy().view(np.uint16)
    gk = oracle.paged_gather(kp, table[1], cache_start + S, page_size=page)[cache_start:]
    gv = oracle.paged_gather(vp, table[1], cache_start + S, page_size=page)[cache_start:]
    assert np.array_equal(gk, k.view(np.uint16)) and np.array_equal(gv, v.view(np.uint16))
    # nothing else in the pools was written
    written = np.zeros(kp.shape[0], bool)
    for p in range(cache_start, cache_start + S):
        written[table[1, p // page] * page + p % page] = True
    assert not kp[~written].any() and not vp[~written].any()
    rows = np.array([0, 5, 255])
    within(out.cpu().numpy()[rows], _oracle_rows(q, k, v, rows, True, 1 / np.sqrt(128)), TOL)


@pytest.fixture(scope="module")
def config2_reference():
    """Config 2 at full size and the oracle's causal head256 online softmax
    over every query row of every head (query_len = S, start_pos 0)."""
    w = workloads.prefill_f16()
    S, H, D = w.q.shape
    u = dict(num_heads=H, num_kv_heads=w.k.shape[1], head_dim=D, seq_len=S, query_len=S,
             scale=w.scale, is_causal=1, start_pos=0, attn_softcap=0.0, sliding_window=0,
             kv_len_source=0, kv_start=0, page_size=16, kv_layout=0)
    ref = oracle.attention_online_f16kv(u, w.q.astype(np.float32), w.k.view(np.uint16),
                                        w.v.view(np.uint16))
    return w, ref


def test_config2_full_size_parity_and_cache(config2_reference):
    """Every one of the 2048 x 32 output rows within 2e-3 of the oracle, and
    the fused cache write equal to the prompt's K and V bit for bit."""
    w, ref = config2_reference
    S, H, _ = w.q.shape
    table = np.arange(S // 16, dtype=np.int32)[None, ::-1].copy()  # reversed pages
    cache = PagedKVCache(num_pages=S // 16, page_size=16, num_kv_heads=w.k.shape[1], head_dim=128,
                         block_table=table)
    status = ops.status_word()
    out = ops.attention_prefill_f16(_t(w.q), _t(w.k), _t(w.v), w.scale, cache=cache, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    o = out.cpu().numpy()
    within(o, ref, TOL)
    # spot rows against the per-row form of the oracle (query_len 1 at start_pos r)
    rows = np.array([0, 1, 127, 128, 129, 1000, 1023, 1024, 2046, 2047])
    within(o[rows], _oracle_rows(w.q, w.k, w.v, rows, True, w.scale), TOL)
    kp = cache.k_pool.cpu().numpy().view(np.uint16)
    vp = cache.v_pool.cpu().numpy().view(np.uint16)
    assert np.array_equal(oracle.paged_gather(kp, table[0], S, page_size=16), w.k.view(np.uint16))
    assert np.array_equal(oracle.paged_gather(vp, table[0], S, page_size=16), w.v.view(np.uint16))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config2_kv_head_shards_match_oracle(world, config2_reference):
    """Config 2 sharded by KV head over `world` GPUs (each rank: Hkv / world
    KV heads and their query heads, the slicing bench.py runs under torchrun),
    run rank after rank on this GPU: every rank's output equals the oracle's
    heads of that rank, and its cache holds its heads' K/V bit for bit."""
    w, ref = config2_reference
    S, H, _ = w.q.shape
    Hkv = w.k.shape[1]
    kvh, qh = Hkv // world, H // world
    for rank in range(world):
        q = w.q[:, rank * qh:(rank + 1) * qh]
        k = w.k[:, rank * kvh:(rank + 1) * kvh]
        v = w.v[:, rank * kvh:(rank + 1) * kvh]
        cache = PagedKVCache(num_pages=S // 16, page_size=16, num_kv_heads=kvh, head_dim=128,
                             block_table=np.arange(S // 16, dtype=np.int32)[None])
        status = ops.status_word()
        out = ops.attention_prefill_f16(_t(q), _t(k), _t(v), w.scale, cache=cache, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        within(out.cpu().numpy(), ref[:, rank * qh:(rank + 1) * qh], TOL)
        assert np.array_equal(cache.k_pool.cpu().numpy().view(np.uint16), k.view(np.uint16))
        assert np.array_equal(cache.v_pool.cpu().numpy().view(np.uint16), v.view(np.uint16))
