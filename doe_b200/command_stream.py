"""Replays a Doe command stream on the CUDA backend through its C ABI.

Doe's benchmark plans run a model as a flat list of commands
(examples/inference_gemma3_*_commands.json): `buffer_write` (u32 words into
a handle), `buffer_load` (a synthetic weight or cache asset into a handle)
and `kernel_dispatch` (a WGSL kernel name, workgroup counts and handle
bindings).  The Zig runtime feeds each to a backend's execute_command
(runtime/zig/src/backend/backend_iface.zig:15); `replay` does the same
through doe_cuda_dispatch, so every kernel of the stream runs as a CUDA
kernel of libdoe_cuda.so and nothing runs on the host.

`buffer_load` payloads are the reference's deterministic synthetic assets
(bench/lib/synthetic_assets.py:160-222): a splitmix64 sequence from the
command's seed (Steele, Lea and Flood, "Fast splittable pseudorandom number
generators", 2014), each draw's top 53 bits as a uniform in [0, 1) mapped to
[-scale, scale), values below a small magnitude replaced by +-that magnitude,
stored as float32 (or float16).  `synthetic_asset` computes it with numpy,
vectorised over the draws.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from .backend import Bind, CudaBackend

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_MUL0 = np.uint64(0xBF58476D1CE4E5B9)
_MUL1 = np.uint64(0x94D049BB133111EB)


def _splitmix64(seed: int, count: int) -> np.ndarray:
    """The first `count` outputs of splitmix64 seeded with `seed`."""
    with np.errstate(over="ignore"):
        state = np.uint64(seed & (2 ** 64 - 1)) + np.arange(1, count + 1, dtype=np.uint64) * _GAMMA
        z = state
        z = (z ^ (z >> np.uint64(30))) * _MUL0
        z = (z ^ (z >> np.uint64(27))) * _MUL1
        return z ^ (z >> np.uint64(31))


def synthetic_asset(generator: str, seed: int, scale: float, byte_length: int) -> bytes:
    """The payload of a buffer_load command (splitmix64_f32_nonzero_v1 or
    splitmix64_f16_nonzero_v1)."""
    if not scale > 0:
        raise ValueError("synthetic asset scale must be > 0")
    if generator == "splitmix64_f32_nonzero_v1":
        width, min_abs, dtype = 4, max(scale / 1024.0, 2.0 ** -20), np.float32
    elif generator == "splitmix64_f16_nonzero_v1":
        width, min_abs, dtype = 2, max(scale / 256.0, 2.0 ** -12), np.float16
    else:
        raise ValueError(f"unsupported synthetic asset generator {generator!r}")
    if byte_length % width:
        raise ValueError(f"{generator} requires byteLength divisible by {width}")
    z = _splitmix64(int(seed), byte_length // width)
    unit = ((z >> np.uint64(11)) & np.uint64((1 << 53) - 1)).astype(np.float64) * (1.0 / float(1 << 53))
    value = (unit * 2.0 - 1.0) * float(scale)
    small = (value == 0.0) | (np.abs(value) < min_abs)
    value = np.where(small, np.where((z & np.uint64(1)) == 0, min_abs, -min_abs), value)
    return value.astype(dtype).tobytes()


def load_commands(path) -> list[dict]:
    data = json.loads(Path(path).read_text())
    return data["commands"] if isinstance(data, dict) else data


def _binds(cmd: dict) -> list[Bind]:
    out = []
    for b in cmd.get("bindings", []):
        out.append(Bind(int(b["binding"]), int(b["resource_handle"]), offset=int(b.get("offset", 0)),
                        size=int(b.get("buffer_size", 0)), group=int(b.get("group", 0))))
    return out


class Replayer:
    """Executes a stream's commands one at a time on a backend.

    `assets` caches buffer_load payloads across replays, keyed by the
    command's (generator, seed, scale, byteLength)."""

    def __init__(self, backend: CudaBackend | None = None, assets: dict | None = None):
        self.backend = backend if backend is not None else CudaBackend(0)
        self.assets = assets if assets is not None else {}
        self.dispatches: list[dict] = []  # kernel_dispatch commands run so far

    def payload(self, c: dict) -> bytes:
        """The bytes a buffer_write or buffer_load command puts in its handle."""
        if c["kind"] == "buffer_write":
            data = np.asarray(c["data"], dtype=np.uint64).astype(np.uint32).tobytes()
            size = int(c.get("bufferSize", len(data)))
            return data[:size]
        key = (c["generator"], int(c["seed"]), float(c["scale"]), int(c["byteLength"]))
        if key not in self.assets:
            self.assets[key] = synthetic_asset(*key)
        return self.assets[key]

    def execute(self, c: dict) -> None:
        be = self.backend
        kind = str(c.get("kind", "")).lower()
        if kind in ("buffer_write", "buffer_load"):
            data = self.payload(c)
            be.ensure_buffer(int(c["handle"]), max(int(c.get("bufferSize", len(data))), len(data)))
            be.execute_buffer_write_bytes(int(c["handle"]), int(c.get("offset", 0)), np.frombuffer(data, np.uint8))
        elif kind == "kernel_dispatch":
            be.execute_kernel_dispatch(c["kernel"], _binds(c), x=int(c.get("x", 1)), y=int(c.get("y", 1)),
                                       z=int(c.get("z", 1)), entry_point=c.get("entry_point"))
            self.dispatches.append(c)
        else:
            raise ValueError(f"command kind {kind!r} is not part of a replayable stream")

    def capture(self, handle: int, size: int) -> bytes:
        return self.backend.capture_buffer(handle, 0, size)


def replay(commands, backend: CudaBackend | None = None, assets: dict | None = None) -> Replayer:
    """Execute `commands` in order on `backend` (a new one on device 0 when
    None) and wait for the queue; returns the Replayer (its backend holds
    every buffer the stream wrote)."""
    r = Replayer(backend, assets)
    for c in commands:
        r.execute(c)
    r.backend.flush_queue()
    return r
