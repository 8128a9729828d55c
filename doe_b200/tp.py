"""Peer buffers for the decoder's tensor-parallel reduction (one process per
GPU of one node).

Each rank allocates one buffer in the library (cudaMalloc + an IPC handle),
the handles are exchanged over the process group, and every rank maps every
peer's buffer.  The library's linear layers write their partial products
into a slot of the rank's own buffer; doe_tp_reduce_rmsnorm sums the slots of
all ranks over NVLink and normalises, in one launch per rank
(include/doe_cuda.h, "Tensor-parallel reduction").
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _abi as abi


class _DevArray:
    """A raw device pointer seen by torch as a tensor (no copy, no ownership)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class TpTimeoutError(RuntimeError):
    """A tensor-parallel reduction gave up waiting for a peer (DOE_DEVICE_ERR_TIMEOUT)."""


class TpPeers:
    """This rank's peer buffer and every other rank's, mapped into this process.

    After a reduction reports DOE_DEVICE_ERR_TIMEOUT, its sums and norms are
    not valid (a late peer's slot was read before it was complete) and the
    ranks' epochs no longer agree: check_status() raises TpTimeoutError and
    marks these peers unusable, so that every later reduce_rmsnorm raises
    until new peer buffers are made on every rank."""

    def __init__(self, rows: int, cols: int, group=None, device=None):
        self.rows, self.cols = rows, cols
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > abi.TP_MAX_RANKS:
            raise ValueError(f"at most {abi.TP_MAX_RANKS} ranks")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = abi.lib()
        nbytes = int(lib.doe_tp_buffer_bytes(rows, cols))
        own = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        abi.check("doe_peer_buffer_create", lib.doe_peer_buffer_create(nbytes, C.byref(own), handle))
        self._own = own.value
        self._opened: list[int] = []
        self.slots = []
        try:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                p = C.c_void_p()
                abi.check("doe_peer_buffer_open",
                          lib.doe_peer_buffer_open((C.c_ubyte * 64).from_buffer_copy(h), C.byref(p)))
                self._opened.append(p.value)
                ptrs.append(p.value)
        except BaseException:
            self.close()
            raise
        self.struct = abi.TpPeers(self.rank, self.world,
                                  (C.c_void_p * abi.TP_MAX_RANKS)(*ptrs, *([None] * (abi.TP_MAX_RANKS - self.world))))
        # this rank's two partial slots as torch tensors (outputs of the linear layers)
        self.slots = []
        for s in range(2):
            ptr = lib.doe_tp_slot_ptr(self._own, s, rows, cols)
            self.slots.append(torch.as_tensor(_DevArray(ptr, (rows, cols), "<f4"), device=self.device))

    failed = False

    def check_status(self, status) -> None:
        """Raise TpTimeoutError if the launch status word (a device int32 tensor
        or its value) holds DOE_DEVICE_ERR_TIMEOUT; the peers are then unusable.
        Reads the device word, so call it after the step, outside graph capture."""
        value = int(status.item()) if hasattr(status, "item") else int(status)
        if value & abi.DOE_DEVICE_ERR_TIMEOUT:
            self.failed = True
            raise TpTimeoutError(
                f"rank {self.rank}: a tensor-parallel reduction timed out waiting for a peer "
                f"(status {value:#x}); its outputs are invalid and the peer buffers must be "
                "recreated on every rank")

    def reduce_rmsnorm(self, slot: int, h_out: torch.Tensor, gamma=None, eps: float = 0.0, xn_out=None,
                       status=None, stream=None) -> None:
        """h_out = sum over ranks of slot `slot`; with gamma also xn_out = RMSNorm(h_out) in bf16."""
        if self.failed:
            raise TpTimeoutError(f"rank {self.rank}: peer buffers unusable after a reduction timeout")
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        l = abi.Launch(s.cuda_stream, None, 0, status.data_ptr() if status is not None else None)
        abi.check("doe_tp_reduce_rmsnorm", abi.lib().doe_tp_reduce_rmsnorm(
            C.byref(self.struct), slot, gamma.data_ptr() if gamma is not None else None, float(eps),
            h_out.data_ptr(), xn_out.data_ptr() if xn_out is not None else None, self.rows, self.cols,
            C.byref(l)))

    def close(self) -> None:
        """Unmap the peers and free this rank's buffer.  Every rank must have
        finished its kernels first: call after a device sync and a barrier."""
        if self._own is None:
            return
        lib = abi.lib()
        self.slots = []
        for p in self._opened:
            lib.doe_peer_buffer_close(p)
        self._opened = []
        lib.doe_peer_buffer_free(self._own)
        self._own = None
