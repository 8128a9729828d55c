"""CPU restatement of the non-attention kernels of Doe's Gemma inference
command streams (bench/inference-pipeline/kernels/*.wgsl), in float32 with
each kernel's own summation order, and a whole-stream replay on top of it.

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path that
doe_cuda_dispatch runs for these kernel names.  Products and sums are
separate float32 operations (numpy never fuses them); WGSL leaves `dot`'s
order and fusing to the implementation, which is why GPU results are held
to 1e-5 * max(|ref|, 1) rather than bit equality.
"""
from __future__ import annotations

import numpy as np

from . import attention_decode_wgsl, attention_prefill_wgsl, rope

F32 = np.float32


def rmsnorm(x: np.ndarray, weight: np.ndarray, size: int, eps: float, rows: int,
            weight_offset: bool = False) -> np.ndarray:
    """rmsnorm.wgsl:14-52 (main) and :54-90 (main_weight_offset): 256 lanes
    each sum v*v over elements lane, lane + 256, ...; a halving tree over the
    lanes; rms = 1 / sqrt(sum / size + eps); out = x * rms * w."""
    x = np.asarray(x, F32).reshape(-1)[:rows * size].reshape(rows, size)
    w = np.asarray(weight, F32).reshape(-1)[:size]
    partial = np.zeros((rows, 256), F32)
    for c in range(0, size, 256):
        blk = x[:, c:c + 256]
        partial[:, :blk.shape[1]] = partial[:, :blk.shape[1]] + blk * blk
    stride = 128
    while stride:
        partial[:, :stride] = partial[:, :stride] + partial[:, stride:2 * stride]
        stride //= 2
    rms = F32(1.0) / np.sqrt(partial[:, 0] / F32(size) + F32(eps))
    g = (F32(1.0) + w) if weight_offset else w
    return (x * rms[:, None]) * g[None, :]


def gemv(matrix: np.ndarray, vector: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """matmul-gemv.wgsl:16-74: 64 lanes per row; lane l accumulates
    dot(vec4 at l*4 + k*256) over k, then the scalar tail, then a halving tree."""
    m = np.asarray(matrix, F32).reshape(-1)[:rows * cols].reshape(rows, cols)
    v = np.asarray(vector, F32).reshape(-1)[:cols]
    vec_cols = cols & ~3
    acc = np.zeros((rows, 64), F32)
    for c in range(0, vec_cols, 256):
        n = min(256, vec_cols - c)
        lanes = n // 4
        mb = m[:, c:c + n].reshape(rows, lanes, 4)
        vb = v[c:c + n].reshape(lanes, 4)
        d = ((mb[:, :, 0] * vb[:, 0] + mb[:, :, 1] * vb[:, 1]) + mb[:, :, 2] * vb[:, 2]) + mb[:, :, 3] * vb[:, 3]
        acc[:, :lanes] = acc[:, :lanes] + d
    for c in range(vec_cols, cols, 64):
        n = min(64, cols - c)
        acc[:, :n] = acc[:, :n] + m[:, c:c + n] * v[c:c + n]
    stride = 32
    while stride:
        acc[:, :stride] = acc[:, :stride] + acc[:, stride:2 * stride]
        stride //= 2
    return acc[:, 0].copy()


def matmul_tiled(a: np.ndarray, b: np.ndarray, M: int, K: int, N: int) -> np.ndarray:
    """matmul-tiled.wgsl: C[m, n] = sum over k4 of dot(A[m, k4:k4+4], B[k4:k4+4, n]),
    accumulated in k order (zero padding past K)."""
    A = np.zeros((M, (K + 3) // 4 * 4), F32)
    A[:, :K] = np.asarray(a, F32).reshape(-1)[:M * K].reshape(M, K)
    B = np.zeros(((K + 3) // 4 * 4, N), F32)
    B[:K] = np.asarray(b, F32).reshape(-1)[:K * N].reshape(K, N)
    acc = np.zeros((M, N), F32)
    for k in range(0, A.shape[1], 4):
        d = ((A[:, k, None] * B[k] + A[:, k + 1, None] * B[k + 1]) + A[:, k + 2, None] * B[k + 2]) + \
            A[:, k + 3, None] * B[k + 3]
        acc = acc + d
    return acc


def gelu(x: np.ndarray) -> np.ndarray:
    """gelu.wgsl:4-7: 0.5 x (1 + tanh(clamp(0.7978845608 (x + 0.044715 x^3), -15, 15)))."""
    x = np.asarray(x, F32)
    inner = F32(0.7978845608) * (x + ((F32(0.044715) * x) * x) * x)
    t = np.tanh(np.clip(inner, F32(-15.0), F32(15.0)).astype(np.float64)).astype(F32)
    return (F32(0.5) * x) * (F32(1.0) + t)


def residual(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """residual.wgsl:5-8."""
    return np.asarray(a, F32) + np.asarray(b, F32)


def sample(logits: np.ndarray, vocab: int) -> int:
    """sample.wgsl:16-52: 256 lanes scan lane, lane + 256, ... keeping the
    first strictly greater value (start -1e30, index 0); a halving tree that
    takes the right value only when strictly greater."""
    lg = np.asarray(logits, F32).reshape(-1)[:vocab]
    best_v = np.full(256, F32(-1e30), F32)
    best_i = np.zeros(256, np.int64)
    for c in range(0, vocab, 256):
        blk = lg[c:c + 256]
        n = blk.shape[0]
        take = blk > best_v[:n]
        best_v[:n] = np.where(take, blk, best_v[:n])
        best_i[:n] = np.where(take, np.arange(c, c + n), best_i[:n])
    stride = 128
    while stride:
        right_v, right_i = best_v[stride:2 * stride].copy(), best_i[stride:2 * stride].copy()
        take = right_v > best_v[:stride]
        best_v[:stride] = np.where(take, right_v, best_v[:stride])
        best_i[:stride] = np.where(take, right_i, best_i[:stride])
        stride //= 2
    return int(best_i[0])


def gather(ids: np.ndarray, table: np.ndarray, seq_len: int, dim: int) -> np.ndarray:
    """gather.wgsl:14-24."""
    t = np.asarray(table, F32).reshape(-1)
    ids = np.asarray(ids, np.uint32).reshape(-1)[:seq_len]
    return np.stack([t[int(i) * dim:(int(i) + 1) * dim] for i in ids]).reshape(-1)


def _u32(data: bytes, n: int) -> list[int]:
    return [int(w) for w in np.frombuffer(data[:4 * n].ljust(4 * n, b"\0"), np.uint32)]


def _f32_word(word: int) -> float:
    return float(np.uint32(word).view(F32))


def run_dispatch(kernel: str, entry_point: str | None, x: int, bufs: dict, binds: dict) -> tuple[int, np.ndarray]:
    """One kernel_dispatch on the CPU.  `bufs` maps handles to bytes (f32 /
    u32 little-endian); `binds` maps binding index -> (handle, size).
    Returns (handle written, its new float32 / uint32 contents)."""
    def arr(b, dtype=F32):
        h, size = binds[b]
        data = bufs.get(h, b"")
        data = data[:size] if size else data
        return np.frombuffer(data.ljust(size or len(data), b"\0"), dtype)

    def uni(b, n=4):
        h, _ = binds[b]
        return _u32(bufs.get(h, b""), n)

    if kernel == "rmsnorm.wgsl":
        size, eps_w = uni(0)[:2]
        out = rmsnorm(arr(1), arr(2), size, _f32_word(eps_w), x, entry_point == "main_weight_offset")
        return binds[3][0], out.reshape(-1)
    if kernel == "matmul-gemv.wgsl":
        rows, cols = uni(0)[:2]
        return binds[3][0], gemv(arr(1), arr(2), min(rows, x), cols)
    if kernel == "matmul-tiled.wgsl":
        M, K, N = uni(3)[:3]
        return binds[2][0], matmul_tiled(arr(0), arr(1), M, K, N).reshape(-1)
    if kernel == "gelu.wgsl":
        a = arr(0)
        n = min(x * 256, a.shape[0], binds[1][1] // 4)
        return binds[1][0], gelu(a[:n])
    if kernel == "residual.wgsl":
        a, b = arr(0), arr(1)
        n = min(x * 256, a.shape[0], b.shape[0], binds[2][1] // 4)
        return binds[2][0], residual(a[:n], b[:n])
    if kernel == "sample.wgsl":
        vocab = uni(0)[0]
        return binds[2][0], np.array([sample(arr(1), vocab)], np.uint32)
    if kernel == "gather.wgsl":
        S, D = uni(0)[:2]
        return binds[3][0], gather(arr(1, np.uint32), arr(2), S, D)
    if kernel == "rope.wgsl":
        S, D, H, off = uni(0)
        qk = arr(1)[:S * H * D].reshape(S, H, D)
        return binds[1][0], rope(qk, arr(2), off).reshape(-1)
    if kernel == "attention-decode.wgsl":
        H, D, L, sc = uni(0)
        q = arr(1)[:H * D].reshape(H, D)
        k = arr(2)[:H * L * D].reshape(H, L, D)
        v = arr(3)[:H * L * D].reshape(H, L, D)
        return binds[4][0], attention_decode_wgsl(q, k, v, _f32_word(sc)).reshape(-1)
    if kernel == "attention-prefill.wgsl":
        S, D, H, sc = uni(0)
        q, k, v = (arr(b)[:H * S * D].reshape(H, S, D) for b in (1, 2, 3))
        return binds[4][0], attention_prefill_wgsl(q, k, v, _f32_word(sc)).reshape(-1)
    raise NotImplementedError(kernel)


def replay(commands, asset_bytes) -> tuple[dict, list]:
    """The whole stream on the CPU: returns the final handle -> bytes map and,
    per kernel_dispatch, (kernel, handle written, its contents).
    asset_bytes(generator, seed, scale, byte_length) supplies buffer_load
    payloads."""
    bufs: dict[int, bytes] = {}
    log = []
    for c in commands:
        kind = c["kind"]
        if kind == "buffer_write":
            data = np.asarray(c["data"], np.uint64).astype(np.uint32).tobytes()
            size = int(c.get("bufferSize", len(data)))
            bufs[int(c["handle"])] = data[:size].ljust(size, b"\0")
        elif kind == "buffer_load":
            bufs[int(c["handle"])] = asset_bytes(c["generator"], int(c["seed"]), float(c["scale"]),
                                                 int(c["byteLength"]))
        elif kind == "kernel_dispatch":
            binds = {int(b["binding"]): (int(b["resource_handle"]), int(b.get("buffer_size", 0)))
                     for b in c["bindings"]}
            h, out = run_dispatch(c["kernel"], c.get("entry_point"), int(c.get("x", 1)), bufs, binds)
            size = next(sz for (hh, sz) in binds.values() if hh == h)
            raw = np.asarray(out).tobytes()
            prev = bufs.get(h, b"\0" * size).ljust(size, b"\0")
            bufs[h] = raw + prev[len(raw):]
            log.append((c["kernel"], h, bufs[h]))
    return bufs, log
