"""GPU: doe_attention_decode_f32_noalloc, the allocation-free decode entry point.

Some callers of this library cannot give it scratch memory and must not have
it allocate any (a plugin callback with no allocator for temporaries, a
serving loop whose device memory is fixed up front).  This entry point keeps
its split partials in a fixed array inside the library.  The test calls it
through the C ABI twice in a row and compares each result with the regular
entry point (caller-provided workspace) at the f32 tolerance, 1e-5 relative.
It lives in its own file so that it runs after every other test, and it sets
up all it needs itself, so it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from doe_b200 import _abi as abi
from doe_b200 import workloads

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-5


def _regular(q, k, v, scale):
    H, D = q.shape
    L = k.shape[1]
    lib = abi.lib()
    ws_bytes = lib.doe_attention_decode_f32_workspace_bytes(H, D, L)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    out = torch.empty_like(q)
    launch = abi.Launch(torch.cuda.current_stream().cuda_stream, ws.data_ptr(), ws.numel(), None)
    abi.check("doe_attention_decode_f32", lib.doe_attention_decode_f32(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), H, D, L, float(scale), C.byref(launch)))
    return out


def _noalloc(q, k, v, scale, out=None):
    H, D = q.shape
    L = k.shape[1]
    out = torch.empty_like(q) if out is None else out
    rc = abi.lib().doe_attention_decode_f32_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), H, D, L, float(scale),
        torch.cuda.current_stream().cuda_stream)
    abi.check("doe_attention_decode_f32_noalloc", rc)
    return out


def _close(a, b):
    a = a.cpu().numpy().astype(np.float64)
    b = b.cpu().numpy().astype(np.float64)
    assert np.isfinite(a).all()
    assert np.all(np.abs(a - b) <= TOL * np.maximum(np.abs(b), 1.0))


@pytest.mark.parametrize("H,D,L", [(8, 64, 512), (32, 128, 4096), (2, 256, 3000), (4, 64, 7)])
def test_noalloc_matches_regular_entry_point_twice(H, D, L):
    torch.cuda.set_device(0)
    if (H, D, L) == (8, 64, 512):
        w = workloads.decode_f32()
        q, k, v, scale = w.q, w.k, w.v, w.scale
    else:
        g = np.random.default_rng(H + D + L)
        q = g.standard_normal((H, D), dtype=np.float32)
        k = g.standard_normal((H, L, D), dtype=np.float32)
        v = g.standard_normal((H, L, D), dtype=np.float32)
        scale = 1.0 / np.sqrt(D)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    q, k, v = t(q), t(k), t(v)
    ref = _regular(q, k, v, scale)
    first = _noalloc(q, k, v, scale)
    # the second call reuses the scratch array still holding the first call's partials
    second = _noalloc(q, k, v, scale)
    torch.cuda.synchronize()
    _close(first, ref)
    _close(second, ref)


def test_noalloc_rejects_problems_beyond_its_scratch():
    torch.cuda.set_device(0)
    H, D, L = 128, 256, 1 << 16  # 128 heads x 3 splits x 258 floats: beyond 256 KiB
    lib = abi.lib()
    need = lib.doe_attention_decode_f32_workspace_bytes(H, D, L)
    assert need > (1 << 18)
    fake = torch.empty(16, dtype=torch.float32, device="cuda")
    rc = lib.doe_attention_decode_f32_noalloc(fake.data_ptr(), fake.data_ptr(), fake.data_ptr(),
                                              fake.data_ptr(), H, D, L, 1.0, None)
    assert rc == abi.DOE_INVALID_ARGUMENT
    assert "scratch" in abi.op_error()
