"""Tensor-parallel decoder host logic on CPU: 2 gloo ranks.

Each rank shards a small model's layers with doe_b200.decoder.shard_layer
(KV-head split, packed q|k|v and gate|up), holds its KV heads' slice of the
paged cache, and runs the numpy restatement (oracle/decoder.py) for its shard
with the partial o_proj / down_proj products summed by a gloo all-reduce and
the residual added on rank 0 alone -- the decoder's schedule.  The result
must match the unsharded model within 2e-3 * max(|ref|, 1): the shards sum
their partial products in another order, which can flip a bf16 rounding; a
wrong shard or packing is off by O(1).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from doe_b200 import decoder

CFG = decoder.DecoderConfig(hidden=512, heads=4, kv_heads=2, ffn=1024, layers=2, batch=4, ctx=40)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(cfg, seed=4):
    """Full layers (bf16 tensors on CPU), full caches (f16 bits), block table, x0."""
    layers = [decoder.init_layer(cfg, seed, l, "cpu") for l in range(cfg.layers)]
    table = decoder.block_table(cfg, seed)
    rows = table.size * cfg.page_size
    g = np.random.default_rng(seed)
    caches = []
    for _ in range(cfg.layers):
        kp = g.standard_normal((rows, cfg.kv_heads, cfg.head_dim), dtype=np.float32).astype(np.float16)
        vp = g.standard_normal((rows, cfg.kv_heads, cfg.head_dim), dtype=np.float32).astype(np.float16)
        caches.append((kp.view(np.uint16), vp.view(np.uint16)))
    x0 = g.standard_normal((cfg.batch, cfg.hidden), dtype=np.float32)
    return layers, caches, table, x0


def _run(cfg, rank, world, all_reduce):
    from oracle import decoder as odec

    layers, caches, table, x0 = _model(cfg)
    kvh, qh = cfg.kv_heads // world, cfg.heads // world
    freq = decoder.rope_table(cfg.ctx + 1, cfg.head_dim, cfg.rope_theta)
    seq_lens = np.full(cfg.batch, cfg.ctx + 1, dtype=np.int32)
    x = x0
    for full, (kp, vp) in zip(layers, caches):
        shard = {k: v.float().numpy() for k, v in decoder.shard_layer(full, cfg, rank, world).items()}
        c = {"k": np.ascontiguousarray(kp[:, rank * kvh:(rank + 1) * kvh]),
             "v": np.ascontiguousarray(vp[:, rank * kvh:(rank + 1) * kvh]), "table": table,
             "page_size": cfg.page_size}
        x = odec.layer_partials(x, shard, c, qh=qh, kvh=kvh, head_dim=cfg.head_dim, eps=cfg.eps,
                                scale=1.0 / np.sqrt(cfg.head_dim), freq_cis=freq, seq_lens=seq_lens,
                                add_residual=rank == 0, all_reduce=all_reduce)
    return x


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def all_reduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
            dist.all_reduce(t)
            return t.numpy()

        x = _run(CFG, rank, world, all_reduce)
        if rank == 0:
            q.put(x)
    finally:
        dist.destroy_process_group()


def test_two_rank_kv_head_tensor_parallel_matches_one_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    tp = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = _run(CFG, 0, 1, lambda a: a)
    err = np.abs(tp - ref) / np.maximum(np.abs(ref), 1.0)
    assert float(err.max()) <= 2e-3, float(err.max())


def test_shard_layout_rejects_uneven_splits():
    with pytest.raises(ValueError):
        decoder.DecoderConfig(hidden=512, heads=4, kv_heads=2, ffn=1024).check(4)
    with pytest.raises(ValueError):
        decoder.DecoderConfig(hidden=512, heads=4, kv_heads=2, ffn=1000).check(2)


def test_pack_gate_up_blocks():
    f, e = 128, 8
    gate = torch.arange(f * e, dtype=torch.float32).reshape(f, e)
    up = -gate
    w = decoder.pack_gate_up(gate, up)
    assert torch.equal(w[0:64], gate[0:64]) and torch.equal(w[64:128], up[0:64])
    assert torch.equal(w[128:192], gate[64:128]) and torch.equal(w[192:256], up[64:128])


def test_tp_timeout_status_poisons_the_peers():
    """A reduction that reports DOE_DEVICE_ERR_TIMEOUT makes check_status raise
    and every later reduce_rmsnorm refuse to run (no GPU: the check is host
    logic on the status word's value)."""
    import pytest

    from doe_b200 import _abi as abi
    from doe_b200.tp import TpPeers, TpTimeoutError

    peers = TpPeers.__new__(TpPeers)
    peers.rank = 1
    peers.check_status(0)
    peers.check_status(abi.DOE_DEVICE_ERR_PAGE)  # not a reduction failure
    assert not peers.failed
    with pytest.raises(TpTimeoutError):
        peers.check_status(abi.DOE_DEVICE_ERR_TIMEOUT | abi.DOE_DEVICE_ERR_PAGE)
    assert peers.failed
    with pytest.raises(TpTimeoutError):
        peers.reduce_rmsnorm(0, None)
