"""The benchmark's synthetic workloads reproduce the sizes the baseline
configurations state (seeded draws; no GPU).

Config 1: decode_f32, 2,101,248 bytes and 1,048,576 flops per step.
Config 2: causal prefill S 2048, 32 heads, D 128: 34,376,515,584 flops
(causal-exact, 4 H D S (S+1) / 2).
Config 3: 64 sequences, ctx U[1024, 8192] seed 2: 309,371 cached tokens
(min 1309, max 8141), 19,369 pages for ctx + 1, KV read (309,371 + 64) x 2 x
8 x 128 x 2 = 1,267,445,760 bytes, 5,069,783,040 flops.
Config 4: 32 sequences, ctx U[8192, 32768] seed 3: 623,873 cached tokens
(min 8995, max 31694), 2080 bytes of int8 K/V + f16 scales per token.
"""
from __future__ import annotations

import numpy as np

from doe_b200 import workloads


def test_config1_decode_f32_sizes():
    d = workloads.decode_f32()
    assert d.q.shape == (8, 64) and d.k.shape == (8, 512, 64) and d.v.shape == (8, 512, 64)
    assert d.bytes_per_step == 2_101_248
    assert d.flops_per_step == 1_048_576
    assert d.scale == 0.125


def test_config2_prefill_flops():
    w = workloads.prefill_f16()
    assert w.q.shape == (2048, 32, 128) and w.k.shape == (2048, 32, 128)
    assert w.q.dtype == np.float16
    assert w.flops == 34_376_515_584


def test_config3_paged_f16_draws():
    w = workloads.paged_f16()
    assert w.num_seqs == 64 and (w.num_heads, w.num_kv_heads, w.head_dim, w.page_size) == (32, 8, 128, 16)
    assert int(w.ctx.sum()) == 309_371 and int(w.ctx.min()) == 1309 and int(w.ctx.max()) == 8141
    assert w.num_pages == 19_369
    b = w.step_bytes()
    assert b["kv_read"] == 1_267_445_760
    assert w.step_flops() == 5_069_783_040
    # the block table is a permutation of the pool: every page used once
    used = w.block_table[w.block_table >= 0]
    assert np.array_equal(np.sort(used), np.arange(w.num_pages))


def test_config4_paged_int8_draws():
    w = workloads.paged_int8()
    assert w.num_seqs == 32 and w.kv_dtype == "int8"
    assert int(w.ctx.sum()) == 623_873 and int(w.ctx.min()) == 8995 and int(w.ctx.max()) == 31694
    assert w.kv_bytes_per_token() == 2080
    used = w.block_table[w.block_table >= 0]
    assert np.array_equal(np.sort(used), np.arange(w.num_pages))


def test_config5_decoder_bytes():
    """Config 5: bf16 linear weights 1,744,830,464 B and f16 KV 2,147,483,648 B
    at ctx 4096 (4 layers, batch 32); the bench's count adds the RMSNorm
    weights (2 x 4096 bf16 per layer) and the appended token (ctx + 1)."""
    from doe_b200.decoder import DecoderConfig

    cfg = DecoderConfig()
    assert (cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.layers, cfg.batch, cfg.ctx) == \
        (4096, 32, 8, 128, 14336, 4, 32, 4096)
    norms = 2 * 2 * cfg.hidden * cfg.layers
    assert cfg.weight_bytes() - norms == 1_744_830_464
    per_token = cfg.batch * cfg.kv_heads * cfg.head_dim * 2 * 2 * cfg.layers
    assert cfg.kv_read_bytes() - per_token == 2_147_483_648
    assert cfg.weight_bytes() + cfg.kv_read_bytes() == 3_892_903_936


def test_config4_strong_split_covers_every_sequence_once():
    """bench.py's config-4 split at N = 2, 4, 8: every one of the 32 sequences
    on exactly one rank, each shard's pages renumbered densely, token loads
    within one sequence of each other (LPT)."""
    import bench

    w = workloads.paged_int8()
    for world in (2, 4, 8):
        shards = [bench.strong_split(w, world, r)[0] for r in range(world)]
        idx = np.concatenate([s.meta["global_index"] for s in shards])
        assert sorted(idx.tolist()) == list(range(w.num_seqs))
        for s in shards:
            used = s.block_table[s.block_table >= 0]
            assert np.array_equal(np.sort(used), np.arange(s.num_pages))
            assert np.array_equal(s.ctx, w.ctx[s.meta["global_index"]])
        loads = [int(s.seq_lens.sum()) for s in shards]
        assert max(loads) - min(loads) <= int(w.seq_lens.max())
