"""Llama-style decoder block for batched decode, tensor
parallel by KV head, on the library's own kernels.

This is the host side an ONNX Runtime EP would run for a bf16 decoder graph:
each graph node maps to one C-ABI call (include/doe_cuda.h, "Decoder-block
operators") and the tensor-parallel AllReduce to NCCL:

    SimplifiedLayerNormalization       doe_rmsnorm_bf16 (f32 residual in, bf16 out)
    MatMul q|k|v (fused, Split)         doe_linear_bf16, 3 f16 segments
    RotaryEmbedding + GroupQueryAttention over the paged cache
                                        doe_paged_decode_ex (RoPE of q and the new
                                        K row, fused append, bf16 output)
    MatMul o_proj + Add residual        doe_linear_bf16, f32 out (+ residual on rank 0)
    AllReduce + SimplifiedLayerNorm     world > 1: doe_tp_reduce_rmsnorm (the partial products
                                        summed over peer buffers inside the norm); or NCCL
                                        (torch.distributed) + doe_rmsnorm_bf16
    MatMul gate|up + Sigmoid/Mul        doe_linear_bf16, SwiGLU epilogue
    MatMul down_proj + Add residual     doe_linear_bf16, f32 out (+ residual on rank 0)
    AllReduce (+ next layer's norm)     as after o_proj

Precision: weights and GEMM inputs bf16 with f32 accumulation; the residual
stream f32; q/k/v and the KV cache f16 (every bf16-derived value is exact or
better in f16 at these magnitudes); attention in f32.

Tensor parallelism (Megatron-style, by KV head): rank r of N holds query heads
[r H/N, (r+1) H/N), KV heads [r Hkv/N, ...), the matching o_proj columns, FFN
features [r F/N, ...) of gate/up and the matching down_proj columns.  The
partial o_proj and down_proj products are summed by an all-reduce; rank 0 adds
the residual before it, so the sum is the residual stream.  Weights are
stored as [out_features, in_features] (nn.Linear; an ONNX MatMul initializer
is transposed once at load).  gate|up is packed in 128-row blocks of 64 gate
rows then the 64 matching up rows, the layout the SwiGLU epilogue reads.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .kv import PagedKVCache


@dataclass(frozen=True)
class DecoderConfig:
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    layers: int = 4
    eps: float = 1e-5
    rope_theta: float = 500000.0
    batch: int = 32
    ctx: int = 4096          # cached tokens per sequence before the step
    page_size: int = 16
    weight_std: float = 0.02

    def check(self, world: int) -> None:
        if self.heads * self.head_dim != self.hidden:
            raise ValueError("hidden must equal heads * head_dim")
        if self.head_dim != 128:
            raise ValueError("the paged decode kernel is built for head_dim 128")
        if self.kv_heads % world or self.heads % world:
            raise ValueError(f"{world} ranks do not divide {self.kv_heads} KV heads")
        if (self.ffn // world) % 64 or self.ffn % world:
            raise ValueError("ffn / world must be a multiple of 64")
        if self.hidden % 128:
            raise ValueError("hidden must be a multiple of 128")
        if self.batch > 32:
            raise ValueError("batch <= 32")

    def weight_bytes(self) -> int:
        """bf16 weight bytes of all layers (whole model, all ranks)."""
        D, H, Hkv, E, F = self.head_dim, self.heads, self.kv_heads, self.hidden, self.ffn
        per = (H * D + 2 * Hkv * D) * E + E * H * D + 3 * F * E
        return 2 * (per + 2 * E) * self.layers

    def kv_read_bytes(self) -> int:
        """f16 K and V bytes one step reads (ctx + 1 tokens per sequence, all layers)."""
        return self.batch * (self.ctx + 1) * self.kv_heads * self.head_dim * 2 * 2 * self.layers


def rope_table(positions: int, head_dim: int, theta: float) -> np.ndarray:
    """[positions, D/2, {cos, sin}] f32 with angle pos * theta^(-2i/D) (rope.wgsl's table)."""
    inv = theta ** (-np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    ang = np.arange(positions, dtype=np.float64)[:, None] * inv[None, :]
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def init_layer(cfg: DecoderConfig, seed: int, layer: int, device) -> dict:
    """Full (unsharded) bf16 weights of one layer, N(0, weight_std), seeded on the device."""
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000 + layer)
    D, H, Hkv, E, F = cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.hidden, cfg.ffn

    def w(*shape):
        return (torch.randn(shape, generator=g, device=device) * cfg.weight_std).to(torch.bfloat16)

    return {"wq": w(H * D, E), "wk": w(Hkv * D, E), "wv": w(Hkv * D, E), "wo": w(E, H * D),
            "wg": w(F, E), "wu": w(F, E), "wd": w(E, F),
            "g1": (1.0 + torch.randn(E, generator=g, device=device) * cfg.weight_std).to(torch.bfloat16),
            "g2": (1.0 + torch.randn(E, generator=g, device=device) * cfg.weight_std).to(torch.bfloat16)}


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[F, E] gate and up -> [2F, E] in 128-row blocks of 64 gate rows, 64 up rows."""
    F, E = gate.shape
    return torch.cat([gate.reshape(F // 64, 64, E), up.reshape(F // 64, 64, E)], dim=1).reshape(2 * F, E)


def shard_layer(full: dict, cfg: DecoderConfig, rank: int, world: int) -> dict:
    """Rank `rank`'s slice of a layer for KV-head tensor parallelism over `world` ranks."""
    D = cfg.head_dim
    qh, kvh, f = cfg.heads // world, cfg.kv_heads // world, cfg.ffn // world
    q0, k0, f0 = rank * qh * D, rank * kvh * D, rank * f
    wqkv = torch.cat([full["wq"][q0:q0 + qh * D], full["wk"][k0:k0 + kvh * D], full["wv"][k0:k0 + kvh * D]])
    return {"wqkv": wqkv.contiguous(),
            "wo": full["wo"][:, q0:q0 + qh * D].contiguous(),
            "wgu": pack_gate_up(full["wg"][f0:f0 + f], full["wu"][f0:f0 + f]).contiguous(),
            "wd": full["wd"][:, f0:f0 + f].contiguous(),
            "g1": full["g1"].contiguous(), "g2": full["g2"].contiguous()}


def block_table(cfg: DecoderConfig, seed: int) -> np.ndarray:
    """[batch, pages per sequence] int32: a random permutation of the pool (room for ctx + 1 tokens)."""
    pps = (cfg.ctx + 1 + cfg.page_size - 1) // cfg.page_size
    perm = np.random.default_rng(seed).permutation(cfg.batch * pps).astype(np.int32)
    return perm.reshape(cfg.batch, pps)


class Decoder:
    """One rank's share of the decoder: sharded weights, paged KV caches, buffers.

    step(x) runs all layers for one decode token per sequence on the current
    stream: x [batch, hidden] f32 (the residual stream) is updated in place.
    capture() records the step in a CUDA graph; replay() reruns it."""

    def __init__(self, cfg: DecoderConfig, *, seed: int = 4, rank: int = 0, world: int = 1, group=None,
                 device=None, layers: list[dict] | None = None, caches: list[PagedKVCache] | None = None,
                 reduce: str = "fused", split_norm: bool | None = None):
        """reduce (world > 1): "fused" sums the partial products over peer
        buffers inside the following RMSNorm (doe_tp_reduce_rmsnorm); "nccl"
        all-reduces them with NCCL and normalises separately.
        split_norm (world 1 only; the default there): every RMSNorm after the
        first is split over the products around it (doe_linear_bf16_norm):
        o_proj / down_proj also write bf16(h * gamma) and per-32-column sums
        of squares of h, and the next product scales its rows by
        1 / sqrt(mean(h^2) + eps), so the step has no RMSNorm launch but the
        first."""
        cfg.check(world)
        if reduce not in ("fused", "nccl"):
            raise ValueError("reduce must be 'fused' or 'nccl'")
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        if split_norm is None:
            split_norm = world == 1
        if split_norm and world != 1:
            raise ValueError("split_norm needs world 1: the norm follows the tensor-parallel reduction")
        self.split_norm = split_norm
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        B, D = cfg.batch, cfg.head_dim
        self.qh, self.kvh, self.f = cfg.heads // world, cfg.kv_heads // world, cfg.ffn // world
        if layers is None:
            layers = []
            for l in range(cfg.layers):
                full = init_layer(cfg, seed, l, dev)
                layers.append(shard_layer(full, cfg, rank, world))
                del full
        self.layers = layers
        table = block_table(cfg, seed)
        if caches is None:
            from .workloads import fill_pools
            caches = []
            for l in range(cfg.layers):
                c = PagedKVCache(num_pages=int(table.size), page_size=cfg.page_size, num_kv_heads=self.kvh,
                                 head_dim=D, block_table=table, device=dev)
                fill_pools(c, seed * 1000 + 100 * l + rank)
                caches.append(c)
        self.caches = caches
        self.freq_cis = torch.from_numpy(rope_table(cfg.ctx + 1, D, cfg.rope_theta)).to(dev)
        self.seq_lens = torch.full((B,), cfg.ctx + 1, dtype=torch.int32, device=dev)
        self.scale = 1.0 / float(np.sqrt(D))
        self.status = ops.status_word(dev)
        # activations
        self.xn = torch.empty((B, cfg.hidden), dtype=torch.bfloat16, device=dev)
        self.q = torch.empty((B, self.qh * D), dtype=torch.float16, device=dev)
        self.k = torch.empty((B, self.kvh * D), dtype=torch.float16, device=dev)
        self.v = torch.empty((B, self.kvh * D), dtype=torch.float16, device=dev)
        self.attn = torch.empty((B, self.qh * D), dtype=torch.bfloat16, device=dev)
        self.h = torch.empty((B, cfg.hidden), dtype=torch.float32, device=dev)
        self.act = torch.empty((B, self.f), dtype=torch.bfloat16, device=dev)
        self.ssq = ops.ssq_buffer(cfg.hidden, dev)  # split_norm: the sums of squares of x or h
        n_max = max(cfg.hidden, (self.qh + 2 * self.kvh) * D, 2 * self.f)
        self.lin_ws = torch.zeros(int(ops.abi.lib().doe_linear_workspace_bytes(n_max, 64)), dtype=torch.uint8,
                                  device=dev)
        # the decode's own workspace: its split counters stay zero between calls
        self.dec_ws = ops.decode_workspace(self.caches[0], B, self.qh)
        self.peers = None
        if world > 1 and reduce == "fused":
            from .tp import TpPeers
            self.peers = TpPeers(B, cfg.hidden, group=group, device=dev)
        self.graph = None

    def _all_reduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            torch.distributed.all_reduce(t, group=self.group)

    def step(self, x: torch.Tensor, trace=None) -> torch.Tensor:
        """One decode token per sequence through every layer; x updated in place.

        trace(layer, name, tensor), when given, sees each intermediate right
        after the op that writes it (for stage-by-stage checks; not in graphs)."""
        cfg, B, D = self.cfg, self.cfg.batch, self.cfg.head_dim
        first = self.rank == 0
        fused = self.peers is not None
        split = self.split_norm
        t = trace if trace is not None else (lambda *_: None)
        for li, (L, cache) in enumerate(zip(self.layers, self.caches)):
            t(li, "x", x)
            if li == 0 or not (fused or split):
                ops.rmsnorm(x, L["g1"], cfg.eps, out=self.xn, status=self.status)
            # (fused: the previous layer's reduction already wrote x and its norm;
            # split: the previous down_proj wrote bf16(x * g1) and x's sums of squares)
            t(li, "xn", self.xn)
            ops.linear(self.xn, L["wqkv"], [self.q, self.k, self.v], status=self.status, ws=self.lin_ws,
                       norm_in=(self.ssq, cfg.eps) if split and li > 0 else None)
            t(li, "q", self.q), t(li, "k", self.k), t(li, "v", self.v)
            # seq_lens, the table and this layer's pool rows are written by no
            # kernel of the step but this call's own append (inputs_stable)
            ops.paged_decode(cache, self.q.view(B, self.qh, D), self.seq_lens, self.scale,
                             new_k=self.k.view(B, self.kvh, D), new_v=self.v.view(B, self.kvh, D),
                             out=self.attn.view(B, self.qh, D), status=self.status, freq_cis=self.freq_cis,
                             out_dtype=torch.bfloat16, ws=self.dec_ws, inputs_stable=True)
            t(li, "attn", self.attn)
            if fused:
                # partial o_proj into slot 0 of this rank's peer buffer, then the
                # sum over ranks and the second norm in one launch
                ops.linear(self.attn, L["wo"], [self.peers.slots[0]], residual=x if first else None,
                           status=self.status, ws=self.lin_ws)
                self.peers.reduce_rmsnorm(0, self.h, L["g2"], cfg.eps, self.xn, status=self.status)
            else:
                ops.linear(self.attn, L["wo"], [self.h], residual=x if first else None, status=self.status,
                           ws=self.lin_ws, norm_out=(L["g2"], self.xn, self.ssq) if split else None)
                self._all_reduce(self.h)
                if not split:
                    ops.rmsnorm(self.h, L["g2"], cfg.eps, out=self.xn, status=self.status)
            t(li, "h", self.h)
            t(li, "hn", self.xn)
            ops.linear(self.xn, L["wgu"], [self.act], swiglu=True, status=self.status, ws=self.lin_ws,
                       norm_in=(self.ssq, cfg.eps) if split else None)
            t(li, "act", self.act)
            if fused:
                nxt = self.layers[li + 1] if li + 1 < len(self.layers) else None
                ops.linear(self.act, L["wd"], [self.peers.slots[1]], residual=self.h if first else None,
                           status=self.status, ws=self.lin_ws)
                self.peers.reduce_rmsnorm(1, x, nxt["g1"] if nxt else None, cfg.eps,
                                          self.xn if nxt else None, status=self.status)
            else:
                nxt = self.layers[li + 1] if li + 1 < len(self.layers) else None
                ops.linear(self.act, L["wd"], [x], residual=self.h if first else None, status=self.status,
                           ws=self.lin_ws, norm_out=(nxt["g1"], self.xn, self.ssq) if split and nxt else None)
                self._all_reduce(x)
            t(li, "out", x)
        return x

    def check(self) -> None:
        """Raise on device-side errors of the steps run so far: a tensor-parallel
        reduction timeout (TpTimeoutError, the peers then unusable) or any
        other DOE_DEVICE_ERR_* bit.  Reads the status word: not inside a capture."""
        if self.peers is not None:
            self.peers.check_status(self.status)
        value = int(self.status.item())
        if value:
            raise RuntimeError(f"decoder step: device status {value:#x}")

    def launches_per_step(self) -> int:
        """Kernels of this library per step."""
        if self.split_norm:
            return 5 * self.cfg.layers + 1
        return 7 * self.cfg.layers + (1 if self.peers is not None else 0)

    def capture(self, x: torch.Tensor) -> None:
        """Record step(x) (x's storage fixed) in a CUDA graph; call after an eager warm-up step."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.step(x)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()

    def release(self) -> None:
        """Drop the CUDA graph (before the process group is destroyed when it
        holds NCCL calls) and, after every rank is idle, the peer buffers."""
        self.graph = None
        if self.peers is not None:
            torch.cuda.synchronize(self.device)
            torch.distributed.barrier(group=self.group)
            self.peers.close()
            self.peers = None
