"""Seeded synthetic workloads for the benchmark configurations.

No public dataset is involved: every input is drawn from
`np.random.default_rng(seed)` in the order lengths -> block-table permutation
-> Q -> new K/V (float32 normal draws, cast afterwards).  KV pools of the
decode configs are large (1.2-1.3 GB), so their contents are drawn on the
device with a seeded torch generator.  Algorithmic byte / flop counts per
step (the roofline numerators) are computed here from the drawn lengths.

  decode_f32   config 1: 8 heads, D 64, 512 cached tokens, f32, seed 0
  prefill_f16  config 2: causal, S 2048, 32 heads, D 128, f16 x 0.5, seed 1
  paged_f16    config 3: 64 seqs, 32/8 heads, D 128, page 16, ctx U[1024, 8192], seed 2
  paged_int8   config 4: 32 seqs, 32/8 heads, D 128, page 16, ctx U[8192, 32768], seed 3
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class DecodeF32:
    q: np.ndarray
    k: np.ndarray
    v: np.ndarray
    scale: float
    bytes_per_step: int
    flops_per_step: int


def decode_f32(seed: int = 0, heads: int = 8, head_dim: int = 64, kv_len: int = 512) -> DecodeF32:
    g = np.random.default_rng(seed)
    q = g.standard_normal((heads, head_dim), dtype=np.float32)
    k = g.standard_normal((heads, kv_len, head_dim), dtype=np.float32)
    v = g.standard_normal((heads, kv_len, head_dim), dtype=np.float32)
    nbytes = (2 * heads * kv_len * head_dim + 2 * heads * head_dim) * 4
    flops = 4 * heads * kv_len * head_dim
    return DecodeF32(q, k, v, 1.0 / np.sqrt(head_dim), nbytes, flops)


@dataclass
class PrefillF16:
    q: np.ndarray  # [S, H, D] f16
    k: np.ndarray  # [S, Hkv, D] f16
    v: np.ndarray
    scale: float
    flops: int     # causal-exact: 4 * H * D * S (S + 1) / 2
    io_bytes: int  # q, k, v read + f32 out + the K/V cache write


def prefill_f16(seed: int = 1, seq_len: int = 2048, heads: int = 32, kv_heads: int = 32,
                head_dim: int = 128) -> PrefillF16:
    """Config 2: causal prefill, Q/K/V ~ N(0,1) * 0.5 cast to f16, [B=1, S, H, D]."""
    g = np.random.default_rng(seed)
    q = (g.standard_normal((seq_len, heads, head_dim), dtype=np.float32) * np.float32(0.5)).astype(np.float16)
    k = (g.standard_normal((seq_len, kv_heads, head_dim), dtype=np.float32) * np.float32(0.5)).astype(np.float16)
    v = (g.standard_normal((seq_len, kv_heads, head_dim), dtype=np.float32) * np.float32(0.5)).astype(np.float16)
    flops = 4 * heads * head_dim * seq_len * (seq_len + 1) // 2
    io = (q.nbytes + k.nbytes + v.nbytes) + seq_len * heads * head_dim * 4 + k.nbytes + v.nbytes
    return PrefillF16(q, k, v, 1.0 / float(np.sqrt(head_dim)), flops, io)


@dataclass
class PagedWorkload:
    """A batched decode step over a paged cache (configs 3 and 4)."""

    name: str
    seed: int
    num_seqs: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    page_size: int
    ctx: np.ndarray            # cached tokens before this step's append
    block_table: np.ndarray    # [B, max_pages] int32, -1 unmapped
    num_pages: int
    q: np.ndarray              # [B, H, D] f16
    new_k: np.ndarray          # [B, Hkv, D] f16
    new_v: np.ndarray
    kv_dtype: str
    scale: float
    extra_tokens: int = 0      # room reserved past ctx + 1 (chunk append)
    meta: dict = field(default_factory=dict)

    @property
    def seq_lens(self) -> np.ndarray:
        """Tokens attended by the decode step (context + the appended token)."""
        return (self.ctx + 1).astype(np.int32)

    def kv_bytes_per_token(self) -> int:
        if self.kv_dtype == "f16":
            return 2 * self.num_kv_heads * self.head_dim * 2
        return 2 * self.num_kv_heads * (self.head_dim + 2)  # int8 + f16 scale, K and V

    def step_bytes(self) -> dict:
        """Algorithmic HBM bytes of one fused append + decode step."""
        B, H, Hkv, D = self.num_seqs, self.num_heads, self.num_kv_heads, self.head_dim
        toks = int(self.seq_lens.sum())
        kv = toks * self.kv_bytes_per_token()
        q = B * H * D * 2
        out = B * H * D * 4
        pages = int(sum(-(-int(n) // self.page_size) for n in self.seq_lens))
        table = pages * 4 + B * 4
        new_in = 2 * B * Hkv * D * 2
        new_out = B * self.kv_bytes_per_token()
        total = kv + q + out + table + new_in + new_out
        return {"kv_read": kv, "q": q, "out": out, "table_and_lens": table,
                "new_kv_read": new_in, "append_write": new_out, "total": total}

    def step_flops(self) -> int:
        return 4 * int(self.seq_lens.sum()) * self.num_heads * self.head_dim

    def tokens_per_step(self) -> int:
        return self.num_seqs


def _paged(name, seed, num_seqs, lo, hi, kv_dtype, extra_tokens=0, num_heads=32, num_kv_heads=8,
           head_dim=128, page_size=16) -> PagedWorkload:
    g = np.random.default_rng(seed)
    ctx = g.integers(lo, hi + 1, num_seqs).astype(np.int64)
    need = [-(-(int(c) + 1 + extra_tokens) // page_size) for c in ctx]
    num_pages = int(sum(need))
    perm = g.permutation(num_pages).astype(np.int32)
    max_pages = max(need)
    table = np.full((num_seqs, max_pages), -1, np.int32)
    o = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[o:o + n]
        o += n
    q = g.standard_normal((num_seqs, num_heads, head_dim), dtype=np.float32).astype(np.float16)
    nk = g.standard_normal((num_seqs, num_kv_heads, head_dim), dtype=np.float32).astype(np.float16)
    nv = g.standard_normal((num_seqs, num_kv_heads, head_dim), dtype=np.float32).astype(np.float16)
    return PagedWorkload(name, seed, num_seqs, num_heads, num_kv_heads, head_dim, page_size, ctx,
                         table, num_pages, q, nk, nv, kv_dtype, 1.0 / float(np.sqrt(head_dim)),
                         extra_tokens)


def paged_f16(seed: int = 2, num_seqs: int = 64) -> PagedWorkload:
    """Config 3: 64 sequences, ctx U[1024, 8192], page 16, f16 pools."""
    return _paged("paged_gqa_decode_f16", seed, num_seqs, 1024, 8192, "f16")


def paged_int8(seed: int = 3, num_seqs: int = 32, chunk: int = 512) -> PagedWorkload:
    """Config 4: 32 sequences, ctx U[8192, 32768], int8 pools; room for a 512-token chunk."""
    return _paged("paged_gqa_decode_int8", seed, num_seqs, 8192, 32768, "int8", extra_tokens=chunk)


def concat(parts: list[PagedWorkload], name: str | None = None) -> PagedWorkload:
    """One batch holding every sequence of `parts`, pages renumbered disjointly."""
    base = parts[0]
    tables, off = [], 0
    width = max(p.block_table.shape[1] for p in parts)
    for p in parts:
        t = np.full((p.num_seqs, width), -1, np.int32)
        live = p.block_table >= 0
        t[:, :p.block_table.shape[1]][live] = p.block_table[live] + off
        tables.append(t)
        off += p.num_pages
    return PagedWorkload(name or base.name, base.seed, sum(p.num_seqs for p in parts), base.num_heads,
                         base.num_kv_heads, base.head_dim, base.page_size,
                         np.concatenate([p.ctx for p in parts]), np.concatenate(tables), off,
                         np.concatenate([p.q for p in parts]), np.concatenate([p.new_k for p in parts]),
                         np.concatenate([p.new_v for p in parts]), base.kv_dtype, base.scale,
                         base.extra_tokens)


def subset(w: PagedWorkload, idx) -> PagedWorkload:
    """The sequences `idx` of `w` with their pages renumbered 0..n-1 (one GPU's shard)."""
    idx = np.asarray(idx, dtype=np.int64)
    rows = w.block_table[idx]
    used = np.unique(rows[rows >= 0])
    remap = np.full(w.num_pages, -1, np.int32)
    remap[used] = np.arange(len(used), dtype=np.int32)
    table = np.where(rows >= 0, remap[np.maximum(rows, 0)], -1).astype(np.int32)
    return PagedWorkload(w.name, w.seed, len(idx), w.num_heads, w.num_kv_heads, w.head_dim,
                         w.page_size, w.ctx[idx].copy(), table, int(len(used)), w.q[idx].copy(),
                         w.new_k[idx].copy(), w.new_v[idx].copy(), w.kv_dtype, w.scale,
                         w.extra_tokens, {"global_index": idx})


def small_paged(seed: int, lens, num_heads=32, num_kv_heads=8, head_dim=128, page_size=16,
                kv_dtype="f16", extra_tokens=0, spare_pages=0) -> PagedWorkload:
    """A small paged workload with explicit context lengths (tests)."""
    g = np.random.default_rng(seed)
    ctx = np.asarray(lens, np.int64)
    B = len(ctx)
    need = [-(-(int(c) + 1 + extra_tokens) // page_size) for c in ctx]
    num_pages = int(sum(need)) + spare_pages
    perm = g.permutation(num_pages).astype(np.int32)
    max_pages = max(need) + 1
    table = np.full((B, max_pages), -1, np.int32)
    o = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[o:o + n]
        o += n
    q = g.standard_normal((B, num_heads, head_dim), dtype=np.float32).astype(np.float16)
    nk = g.standard_normal((B, num_kv_heads, head_dim), dtype=np.float32).astype(np.float16)
    nv = g.standard_normal((B, num_kv_heads, head_dim), dtype=np.float32).astype(np.float16)
    return PagedWorkload("small", seed, B, num_heads, num_kv_heads, head_dim, page_size, ctx, table,
                         num_pages, q, nk, nv, kv_dtype, 1.0 / float(np.sqrt(head_dim)), extra_tokens)


def fill_pools(cache, seed: int, std: float = 1.0, chunk_rows: int = 1 << 18) -> None:
    """Fill a PagedKVCache's pools with seeded N(0, std) values on its device.

    f16 pools hold the values; int8 pools hold their quantisation under the
    int8 KV definition (scale = f16(absmax / 127) per token and kv head,
    q = clamp(rint(x / scale), -127, 127)), computed with IEEE division and
    round-half-even on the device."""
    import torch

    gen = torch.Generator(device=cache.k_pool.device)
    gen.manual_seed(seed)
    rows = cache.k_pool.shape[0]
    Hkv, D, P = cache.num_kv_heads, cache.head_dim, cache.page_size
    for pool, scale in ((cache.k_pool, cache.k_scale), (cache.v_pool, cache.v_scale)):
        for r0 in range(0, rows, chunk_rows):
            r1 = min(rows, r0 + chunk_rows)
            x = torch.randn((r1 - r0, Hkv, D), generator=gen, device=pool.device,
                            dtype=torch.float32)
            if std != 1.0:
                x = x * std
            x = x.to(torch.float16)
            if cache.kv_dtype == "f16":
                pool[r0:r1] = x
                continue
            xf = x.float()
            s = (xf.abs().amax(dim=-1) / 127.0).to(torch.float16)
            sf = s.float()
            qv = torch.where(sf[..., None] > 0, torch.round(xf / sf[..., None].clamp_min(1e-30)),
                             torch.zeros_like(xf)).clamp_(-127, 127)
            pool[r0:r1] = qv.to(torch.int8)
            # scales are page-blocked: [num_pages, Hkv, page_size]
            rows_idx = torch.arange(r0, r1, device=pool.device)
            scale[rows_idx // P, :, rows_idx % P] = s
