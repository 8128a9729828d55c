"""Python view of the doe_cuda backend surface (include/doe_cuda.h, backend part).

Method names follow Doe's backend interface
(runtime/zig/src/backend/backend_iface.zig:33-93 BackendIface): buffer writes,
kernel_dispatch commands with handle bindings, flush_queue and
capture_buffer.  Errors raise DoeError carrying the backend's message.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _abi as abi


@dataclass
class Bind:
    """One KernelBinding (runtime/zig/src/model_compute_types.zig:19-35)."""

    binding: int
    handle: int
    offset: int = 0
    size: int = 0  # 0 = the whole buffer from offset
    group: int = 0
    buffer_type: int = 0


class CudaBackend:
    def __init__(self, ordinal: int = 0):
        self._lib = abi.lib()
        h = C.c_void_p()
        rc = self._lib.doe_cuda_open(ordinal, C.byref(h))
        if rc != abi.DOE_OK:
            raise abi.DoeError("doe_cuda_open", rc, abi.op_error())
        self._h = h

    # -- lifecycle -------------------------------------------------------------
    def close(self) -> None:
        if self._h:
            self._lib.doe_cuda_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, fn: str, rc: int) -> None:
        abi.check(fn, rc, self._h)

    @property
    def stream_handle(self) -> int:
        return self._lib.doe_cuda_stream(self._h)

    # -- buffers ---------------------------------------------------------------
    def ensure_buffer(self, handle: int, nbytes: int) -> None:
        self._check("doe_cuda_buffer_ensure", self._lib.doe_cuda_buffer_ensure(self._h, handle, nbytes))

    def execute_buffer_write_bytes(self, handle: int, offset: int, data) -> None:
        buf = np.ascontiguousarray(data)
        self._check("doe_cuda_buffer_write", self._lib.doe_cuda_buffer_write(
            self._h, handle, offset, buf.ctypes.data, buf.nbytes))

    def write_ptr(self, handle: int, offset: int, ptr: int, nbytes: int) -> None:
        """Buffer write from a raw host address (pinned or pageable)."""
        self._check("doe_cuda_buffer_write", self._lib.doe_cuda_buffer_write(
            self._h, handle, offset, ptr, nbytes))

    def write_ptr_async(self, handle: int, offset: int, ptr: int, nbytes: int) -> None:
        """Deferred write from page-locked memory (kept unchanged until flush_queue())."""
        self._check("doe_cuda_buffer_write_async", self._lib.doe_cuda_buffer_write_async(
            self._h, handle, offset, ptr, nbytes))

    def capture_buffer(self, handle: int, offset: int, size: int) -> bytes:
        out = np.empty(size, np.uint8)
        self._check("doe_cuda_buffer_read", self._lib.doe_cuda_buffer_read(
            self._h, handle, offset, out.ctypes.data, size))
        return out.tobytes()

    def read_into(self, handle: int, offset: int, ptr: int, nbytes: int) -> None:
        self._check("doe_cuda_buffer_read", self._lib.doe_cuda_buffer_read(
            self._h, handle, offset, ptr, nbytes))

    def read_into_async(self, handle: int, offset: int, ptr: int, nbytes: int) -> None:
        """Deferred capture into page-locked memory; valid after flush_queue()."""
        self._check("doe_cuda_buffer_read_async", self._lib.doe_cuda_buffer_read_async(
            self._h, handle, offset, ptr, nbytes))

    def release_buffer(self, handle: int) -> None:
        self._check("doe_cuda_buffer_release", self._lib.doe_cuda_buffer_release(self._h, handle))

    def buffer_device_ptr(self, handle: int) -> int:
        p = C.c_void_p()
        self._check("doe_cuda_buffer_device_ptr",
                    self._lib.doe_cuda_buffer_device_ptr(self._h, handle, C.byref(p)))
        return p.value

    # -- commands --------------------------------------------------------------
    def execute_kernel_dispatch(self, kernel: str, bindings: list[Bind], x: int = 1, y: int = 1,
                                z: int = 1, entry_point: str | None = None) -> abi.ExecResult:
        arr = (abi.Binding * max(1, len(bindings)))()
        for i, b in enumerate(bindings):
            arr[i] = abi.Binding(b.binding, b.group, b.handle, b.offset, b.size, b.buffer_type, 0)
        res = abi.ExecResult()
        rc = self._lib.doe_cuda_dispatch(self._h, kernel.encode(),
                                         entry_point.encode() if entry_point else None, x, y, z,
                                         arr, len(bindings), C.byref(res))
        self._check(f"dispatch({kernel})", rc)
        return res

    def kernel_supported(self, kernel: str) -> bool:
        return bool(self._lib.doe_cuda_kernel_supported(kernel.encode()))

    def prewarm_kernel_dispatch(self, kernel: str) -> None:
        self._check("doe_cuda_prewarm_kernel", self._lib.doe_cuda_prewarm_kernel(self._h, kernel.encode()))

    def prewarm_upload_path(self, max_upload_bytes: int) -> None:
        self._check("doe_cuda_prewarm_upload", self._lib.doe_cuda_prewarm_upload(self._h, max_upload_bytes))

    def set_upload_behavior(self, mode: int, submit_every: int) -> None:
        """Flush the queue after every `submit_every` buffer writes (0 counts as
        1; 2**32 - 1 never); `mode` is the upload usage (DOE_UPLOAD_*)."""
        self._check("doe_cuda_set_upload_behavior",
                    self._lib.doe_cuda_set_upload_behavior(self._h, int(mode), int(submit_every)))

    def set_queue_wait_mode(self, mode: int) -> None:
        """QueueWaitMode: 0 process_events, 1 wait_any (flush waits either way)."""
        self._check("doe_cuda_set_queue_wait_mode", self._lib.doe_cuda_set_queue_wait_mode(self._h, int(mode)))

    def set_queue_sync_mode(self, per_command: bool) -> None:
        self._check("doe_cuda_set_queue_sync_mode",
                    self._lib.doe_cuda_set_queue_sync_mode(self._h, int(per_command)))

    def set_gpu_timestamp_mode(self, on: bool) -> None:
        self._check("doe_cuda_set_gpu_timestamp_mode",
                    self._lib.doe_cuda_set_gpu_timestamp_mode(self._h, int(on)))

    def flush_queue(self) -> int:
        ns = C.c_uint64()
        self._check("doe_cuda_flush", self._lib.doe_cuda_flush(self._h, C.byref(ns)))
        return ns.value
