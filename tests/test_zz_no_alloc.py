"""GPU: doe_attention_decode_f32_noalloc, the allocation-free decode entry point.

Some callers of this library cannot give it scratch memory and must not have
it allocate any (a plugin callback with no allocator for temporaries, a
serving loop whose device memory is fixed up front).  This entry point keeps
its split partials in a fixed array inside the library.  The test calls it
through the C ABI twice in a row and compares each result with the regular
entry point (caller-provided workspace) and, on shapes whose partials go
through the scratch array, with the CPU oracle, at the f32 tolerance, 1e-5
relative.
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


def _inputs(H, D, L, seed):
    g = np.random.default_rng(seed)
    q = g.standard_normal((H, D), dtype=np.float32)
    k = g.standard_normal((H, L, D), dtype=np.float32)
    v = g.standard_normal((H, L, D), dtype=np.float32)
    return q, k, v


@pytest.mark.parametrize("H,D,L", [(8, 64, 512), (32, 128, 4096), (2, 256, 3000), (4, 64, 7)])
def test_noalloc_matches_regular_entry_point_twice(H, D, L):
    torch.cuda.set_device(0)
    if (H, D, L) == (8, 64, 512):
        w = workloads.decode_f32()
        q, k, v, scale = w.q, w.k, w.v, w.scale
    else:
        q, k, v = _inputs(H, D, L, H + D + L)
        scale = 1.0 / np.sqrt(D)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    q, k, v = t(q), t(k), t(v)
    ref = _regular(q, k, v, scale)
    first = _noalloc(q, k, v, scale)
    second = _noalloc(q, k, v, scale)
    torch.cuda.synchronize()
    _close(first, ref)
    _close(second, ref)


def _splits(H, D, L) -> int:
    """Split partials per head the decode plans (0 for a single split)."""
    ws = abi.lib().doe_attention_decode_f32_workspace_bytes(H, D, L)
    return ws // (H * (D + 2) * 4)


@pytest.mark.parametrize("H,D,L", [(4, 128, 8192), (1, 64, 20000), (2, 256, 3000)])
def test_noalloc_split_path_two_calls_against_oracle(H, D, L):
    """Shapes with more than 16 splits per head: the splits cannot form one
    thread-block cluster, so their partials go through the library's scratch
    array.  Two calls in a row on different inputs: the second must not see
    the first call's partials.  Both against the CPU oracle and the regular
    entry point at 1e-5."""
    import oracle

    torch.cuda.set_device(0)
    assert _splits(H, D, L) > 16, "shape does not take the scratch-array split path"
    assert abi.lib().doe_attention_decode_f32_workspace_bytes(H, D, L) <= abi.DOE_NOALLOC_SCRATCH_BYTES
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    scale = 1.0 / np.sqrt(D)
    host = [_inputs(H, D, L, 100 + i) for i in range(2)]
    dev = [tuple(t(a) for a in h) for h in host]
    outs = [_noalloc(*dev[i], scale) for i in range(2)]
    torch.cuda.synchronize()
    for (q, k, v), (dq, dk, dv), out in zip(host, dev, outs):
        ref = oracle.attention_decode_wgsl(q, k, v, scale)
        got = out.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all()
        assert np.all(np.abs(got - ref) <= TOL * np.maximum(np.abs(ref), 1.0))
        _close(out, _regular(dq, dk, dv, scale))
    # the two problems differ, so equal outputs would mean a stale read
    assert not torch.equal(outs[0], outs[1])


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
