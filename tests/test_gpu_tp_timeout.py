"""A tensor-parallel reduction whose peer never arrives ends with an error
status, not a hang (one GPU).

Two peer buffers in one process stand for ranks 0 and 1 of a world of 2; only
rank 0's reduction runs.  It raises rank 1's flag in the second buffer, then
waits for its own flag from rank 1, which nothing sets.  The wait is bounded
(~2 s of SM clock cycles): the kernel reports DOE_DEVICE_ERR_TIMEOUT in the
status word and returns, and the context stays usable.
"""
from __future__ import annotations

import ctypes as C
import time

import pytest

from doe_b200 import _abi as abi
from doe_b200 import ops

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_reduce_reports_timeout_when_a_peer_never_arrives():
    lib = abi.lib()
    rows, cols = 4, 256
    nbytes = int(lib.doe_tp_buffer_bytes(rows, cols))
    bufs = []
    try:
        for _ in range(2):
            p, h = C.c_void_p(), (C.c_ubyte * 64)()
            abi.check("doe_peer_buffer_create", lib.doe_peer_buffer_create(nbytes, C.byref(p), h))
            bufs.append(p.value)
        peers = abi.TpPeers(0, 2, (C.c_void_p * abi.TP_MAX_RANKS)(*bufs, *([None] * (abi.TP_MAX_RANKS - 2))))
        h_out = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
        status = ops.status_word()
        launch = abi.Launch(torch.cuda.current_stream().cuda_stream, None, 0, status.data_ptr())
        t0 = time.perf_counter()
        abi.check("doe_tp_reduce_rmsnorm", lib.doe_tp_reduce_rmsnorm(
            C.byref(peers), 0, None, 0.0, h_out.data_ptr(), None, rows, cols, C.byref(launch)))
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert int(status.item()) & abi.DOE_DEVICE_ERR_TIMEOUT
        assert 0.5 < waited < 60.0
        # the context still works
        z = torch.full((1024,), 2.0, device="cuda")
        assert float(z.sum().item()) == 2048.0
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.doe_peer_buffer_free(p)
