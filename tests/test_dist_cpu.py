"""Multi-rank host logic on CPU: 2 gloo ranks shard a decode batch by sequence.

Each rank takes its LPT shard of the global batch, compacts its pages, runs
the oracle decode on that shard (standing in for its GPU), and the outputs
are gathered; the reassembled result must equal the unsharded computation
bit for bit, and the max-over-ranks reduction used for timing must hold.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from doe_b200 import shard, workloads


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _global_batch():
    parts = [workloads.small_paged(40 + r, [3, 200, 17, 90, 600, 1, 45, 333], num_heads=8,
                                   num_kv_heads=2, head_dim=32) for r in range(2)]
    return workloads.concat(parts)


def _pools(w, seed):
    g = np.random.default_rng(seed)
    rows = w.num_pages * w.page_size
    kp = g.standard_normal((rows, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    vp = g.standard_normal((rows, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    return kp.view(np.uint16), vp.view(np.uint16)


def _decode(w, kp, vp):
    import oracle

    return oracle.paged_decode(w.q.view(np.uint16), kp, vp, w.block_table, w.seq_lens, w.scale,
                               page_size=w.page_size, threads=1)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _global_batch()
        kp, vp = _pools(w, 5)
        mine = shard.lpt_assign(w.seq_lens, world)[rank]
        local = workloads.subset(w, mine)
        # copy this shard's pages into its own compact pools (its GPU's cache)
        rows = w.block_table[mine]
        used = np.unique(rows[rows >= 0])
        P = w.page_size
        src = (used[:, None] * P + np.arange(P)[None, :]).reshape(-1)
        out = _decode(local, kp[src], vp[src])
        full = np.zeros((w.num_seqs,) + out.shape[1:], np.float32)
        full[mine] = out
        t = torch.from_numpy(full)
        dist.all_reduce(t)  # shards are disjoint: the sum assembles the batch
        tmax = torch.tensor([float(rank + 1)])
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((t.numpy(), float(tmax.item())))
    finally:
        dist.destroy_process_group()


def test_lpt_shards_are_disjoint_complete_and_balanced():
    w = workloads.paged_f16()
    for n in (1, 2, 4, 8):
        shards = shard.lpt_assign(w.seq_lens, n)
        allidx = np.concatenate(shards)
        assert sorted(allidx.tolist()) == list(range(w.num_seqs))
        loads = shard.rank_loads(w.seq_lens, shards)
        assert loads.max() - loads.min() <= int(w.seq_lens.max())
    sub = workloads.subset(w, shard.lpt_assign(w.seq_lens, 4)[1])
    assert sub.block_table.max() == sub.num_pages - 1
    assert (np.unique(sub.block_table[sub.block_table >= 0]) == np.arange(sub.num_pages)).all()


def test_two_gloo_ranks_reassemble_the_unsharded_decode():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got, tmax = q.get(timeout=10)
    w = _global_batch()
    kp, vp = _pools(w, 5)
    assert np.array_equal(got, _decode(w, kp, vp))
    assert tmax == 2.0
