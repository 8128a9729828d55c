"""numpy restatement of one rank's Llama-style decoder step.

TEST INFRASTRUCTURE ONLY: the parity checker for doe_b200.decoder, imported by
tests/ alone.

Parity unpinned: the reference has no decoder-block kernels and no vectors for
them (its ORT EP runs f32 basic ops only,
runtime/bridge/onnxruntime-ep/src/doe_ort_ep.cc:2062-2341).  This follows the
ONNX operators such a graph is made of -- SimplifiedLayerNormalization
(f32 stash), MatMul, RotaryEmbedding, GroupQueryAttention, Sigmoid, Mul, Add
-- with the attention step through the pinned paged-decode restatement
(oracle.paged_append / oracle.paged_decode over the paged cache, RoPE by
oracle.rope = rope.wgsl), and it rounds where the kernels store: bf16 after
each RMSNorm, SwiGLU and attention, f16 for q / k / v, f32 for the residual
stream.  Products are taken in float64 and rounded to f32.  The split form of
an RMSNorm (one process: the norm's scale applied to the product's rows
instead of before the bf16 rounding) is normed_matmul(..., split=True).

The weights arrive in the shard layout of doe_b200.decoder.shard_layer
(q|k|v rows stacked; gate|up in 128-row blocks of 64 gate then 64 up rows),
unpacked here by that documented layout.
"""
from __future__ import annotations

import numpy as np

from . import paged_append, paged_decode, rope

F32 = np.float32


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round f32 values to the nearest bf16 (ties to even), returned as f32."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(F32)


def rmsnorm(x: np.ndarray, gamma: np.ndarray, eps: float) -> np.ndarray:
    """SimplifiedLayerNormalization: x / sqrt(mean(x^2) + eps) * gamma, rounded to bf16."""
    x = x.astype(F32)
    ms = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    inv = (1.0 / np.sqrt(ms + eps)).astype(F32)
    return bf16_round(x * inv * gamma.astype(F32))


def rms_scale(x: np.ndarray, eps: float) -> np.ndarray:
    """The RMSNorm's per-row scale 1 / sqrt(mean(x^2) + eps) as f32, [rows, 1]."""
    ms = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    return (1.0 / np.sqrt(ms + eps)).astype(F32)


def norm_numerator(x: np.ndarray, gamma: np.ndarray) -> np.ndarray:
    """The split RMSNorm's product input bf16(x * gamma); the product's rows are
    then scaled by rms_scale(x) (doe_linear_bf16_norm)."""
    return bf16_round(x.astype(F32) * gamma.astype(F32))


def normed_matmul(x: np.ndarray, gamma: np.ndarray, w: np.ndarray, eps: float, split: bool) -> np.ndarray:
    """RMSNorm then MatMul: bf16(rmsnorm(x) * gamma) @ w^T, or in the split form
    rms_scale(x) * (bf16(x * gamma) @ w^T), rounded to f32."""
    if not split:
        return matmul(rmsnorm(x, gamma, eps), w)
    p = norm_numerator(x, gamma).astype(np.float64) @ w.astype(np.float64).T
    return (p.astype(F32) * rms_scale(x, eps)).astype(F32)


def matmul(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """x [B, K] @ w[N, K]^T in float64, rounded to f32."""
    return (x.astype(np.float64) @ w.astype(np.float64).T).astype(F32)


def unpack_gate_up(wgu: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    blocks = wgu.reshape(-1, 128, wgu.shape[1])
    return blocks[:, :64].reshape(-1, wgu.shape[1]), blocks[:, 64:].reshape(-1, wgu.shape[1])


def layer_partials(x, L: dict, cache: dict, *, qh: int, kvh: int, head_dim: int, eps: float, scale: float,
                   freq_cis, seq_lens, add_residual: bool, all_reduce=lambda t: t,
                   split_first: bool = False, split_second: bool = False):
    """One rank's decoder layer.  x [B, E] f32 (replicated); L holds the rank's
    bf16-valued f32 arrays wqkv, wo, wgu, wd, g1, g2; cache holds the rank's
    pools (f16 bits) and block table, updated in place by the append.
    `all_reduce` sums a [B, E] f32 array over ranks (identity for one rank).
    split_first / split_second take the layer's first / second RMSNorm in the
    split form (normed_matmul).  Returns the next residual stream."""
    B, D = x.shape[0], head_dim
    qkv = normed_matmul(x, L["g1"], L["wqkv"], eps, split_first)
    q = qkv[:, :qh * D].reshape(B, qh, D).astype(np.float16)
    k = qkv[:, qh * D:(qh + kvh) * D].reshape(B, kvh, D).astype(np.float16)
    v = qkv[:, (qh + kvh) * D:].reshape(B, kvh, D).astype(np.float16)
    pos = seq_lens.astype(np.int64) - 1
    rq = np.stack([rope(q[b][None].astype(F32), freq_cis, position_offset=int(pos[b]))[0] for b in range(B)])
    rk = np.stack([rope(k[b][None].astype(F32), freq_cis, position_offset=int(pos[b]))[0] for b in range(B)])
    rq, rk = rq.astype(np.float16), rk.astype(np.float16)
    paged_append(rk[:, None].view(np.uint16), v[:, None].view(np.uint16), cache["k"], cache["v"],
                 cache["table"], pos.astype(np.int32), page_size=cache["page_size"])
    attn = paged_decode(rq.view(np.uint16), cache["k"], cache["v"], cache["table"], seq_lens, scale,
                        page_size=cache["page_size"])
    attn = bf16_round(attn.reshape(B, qh * D).astype(F32))
    h = matmul(attn, L["wo"])
    if add_residual:
        h = (h + x).astype(F32)
    h = all_reduce(h)
    wg, wu = unpack_gate_up(L["wgu"])
    g, u = normed_matmul(h, L["g2"], wg, eps, split_second), normed_matmul(h, L["g2"], wu, eps, split_second)
    act = bf16_round((g / (F32(1.0) + np.exp(-g)) * u).astype(F32))
    y = matmul(act, L["wd"])
    if add_residual:
        y = (y + h).astype(F32)
    return all_reduce(y)
