"""GPU: the backend surface -- buffers, kernel_dispatch by kernel / op name, flush.

Command shapes follow Doe's command streams (buffer_write + kernel_dispatch
with handle bindings, e.g. examples/inference_gemma3_270m_decode_1tok_commands.json).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from doe_b200 import _abi as abi
from doe_b200 import ops, workloads
from doe_b200.backend import Bind, CudaBackend

from .gpu_util import within

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture()
def be():
    b = CudaBackend(0)
    yield b
    b.close()


def _u32(*vals) -> np.ndarray:
    out = []
    for v in vals:
        out.append(np.float32(v).view(np.uint32) if isinstance(v, float) else np.uint32(v))
    return np.array(out, np.uint32)


def test_buffer_roundtrip_grow_and_errors(be):
    g = np.random.default_rng(0)
    data = g.integers(0, 256, 10_000, dtype=np.uint8)
    be.execute_buffer_write_bytes(7, 0, data)
    assert be.capture_buffer(7, 0, 10_000) == data.tobytes()
    be.execute_buffer_write_bytes(7, 20_000, data[:100])  # grows, keeps contents
    assert be.capture_buffer(7, 0, 10_000) == data.tobytes()
    assert be.capture_buffer(7, 20_000, 100) == data[:100].tobytes()
    assert be.capture_buffer(7, 10_000, 16) == bytes(16)  # the gap is zero-filled
    with pytest.raises(abi.DoeError) as e:
        be.capture_buffer(99, 0, 4)
    assert e.value.rc == abi.DOE_NOT_FOUND
    with pytest.raises(abi.DoeError) as e:
        be.execute_kernel_dispatch("matmul.wgsl", [])
    assert e.value.rc == abi.DOE_UNSUPPORTED
    with pytest.raises(abi.DoeError) as e:
        be.prewarm_kernel_dispatch("gelu")
    assert e.value.rc == abi.DOE_UNSUPPORTED
    be.prewarm_kernel_dispatch("attention-decode.wgsl")
    be.release_buffer(7)
    with pytest.raises(abi.DoeError):
        be.capture_buffer(7, 0, 4)


def test_deferred_capture_lands_at_flush(be):
    g = np.random.default_rng(1)
    data = g.integers(0, 256, 1 << 20, dtype=np.uint8)
    be.execute_buffer_write_bytes(8, 0, data)
    pinned = torch.zeros(1 << 20, dtype=torch.uint8).pin_memory()
    be.read_into_async(8, 0, pinned.data_ptr(), 1 << 20)
    be.flush_queue()
    assert np.array_equal(pinned.numpy(), data)
    # a deferred write from pinned memory lands before the next kernel / capture
    src = torch.from_numpy(data[::-1].copy()).pin_memory()
    be.write_ptr_async(8, 0, src.data_ptr(), 1 << 20)
    be.read_into_async(8, 0, pinned.data_ptr(), 1 << 20)
    be.flush_queue()
    assert np.array_equal(pinned.numpy(), data[::-1])
    # pageable destinations are refused (the copy would outlive the call)
    host = np.zeros(16, np.uint8)
    with pytest.raises(abi.DoeError) as e:
        be.read_into_async(8, 0, host.ctypes.data, 16)
    assert e.value.rc == abi.DOE_INVALID_ARGUMENT


def test_attention_decode_wgsl_dispatch(be):
    w = workloads.decode_f32()
    be.execute_buffer_write_bytes(1, 0, _u32(8, 64, 512, float(np.float32(w.scale))))
    be.execute_buffer_write_bytes(2, 0, w.q)
    be.execute_buffer_write_bytes(3, 0, w.k)
    be.execute_buffer_write_bytes(4, 0, w.v)
    be.set_gpu_timestamp_mode(True)
    be.set_queue_sync_mode(True)
    res = be.execute_kernel_dispatch(
        "attention-decode.wgsl",
        [Bind(0, 1, size=16), Bind(1, 2), Bind(2, 3), Bind(3, 4), Bind(4, 5, size=8 * 64 * 4)], x=8)
    assert res.status == 0 and res.dispatch_count == 1 and res.gpu_timestamp_valid == 1
    out = np.frombuffer(be.capture_buffer(5, 0, 8 * 64 * 4), np.float32).reshape(8, 64)
    within(out, oracle.attention_decode_wgsl(w.q, w.k, w.v, w.scale), 1e-5)


def test_head256_dispatch_paged(be):
    g = np.random.default_rng(4)
    H, Hkv, D, L, page = 4, 1, 256, 70, 16
    rows = 80
    q = g.standard_normal((3, H, D), dtype=np.float32)
    k = g.standard_normal((rows, Hkv, D), dtype=np.float32).astype(np.float16)
    v = g.standard_normal((rows, Hkv, D), dtype=np.float32).astype(np.float16)
    pt = g.permutation(rows // page).astype(np.uint32)
    u = dict(num_heads=H, num_kv_heads=Hkv, head_dim=D, seq_len=L, query_len=3, scale=0.0625,
             is_causal=1, start_pos=67, attn_softcap=30.0, sliding_window=0, kv_len_source=0,
             kv_start=0, page_size=page, kv_layout=2)
    uni = np.array([u[n] if not isinstance(u[n], float) else np.float32(u[n]).view(np.uint32)
                    for n in ("num_heads", "num_kv_heads", "head_dim", "seq_len", "query_len", "scale",
                              "is_causal", "start_pos", "attn_softcap", "sliding_window",
                              "kv_len_source", "kv_start", "page_size", "kv_layout")] + [0], np.uint32)
    for h, arr in ((10, uni), (11, q), (12, k), (13, v), (15, np.array([0], np.uint32)), (16, pt)):
        be.execute_buffer_write_bytes(h, 0, arr)
    be.execute_kernel_dispatch("attention_head256_f16kv.wgsl",
                               [Bind(0, 10, size=64), Bind(1, 11), Bind(2, 12), Bind(3, 13),
                                Bind(4, 14, size=q.nbytes), Bind(5, 15), Bind(6, 16)])
    be.flush_queue()
    out = np.frombuffer(be.capture_buffer(14, 0, q.nbytes), np.float32).reshape(q.shape)
    ref = oracle.attention_online_f16kv(u, q, k.view(np.uint16), v.view(np.uint16), None, pt)
    within(out, ref, 1e-5)
    # the fixed-head-dim kernel name rejects another head_dim explicitly
    uni2 = uni.copy()
    uni2[2] = 128
    be.execute_buffer_write_bytes(10, 0, uni2)
    with pytest.raises(abi.DoeError) as e:
        be.execute_kernel_dispatch("attention_head256_f16kv.wgsl",
                                   [Bind(0, 10, size=64), Bind(1, 11), Bind(2, 12), Bind(3, 13),
                                    Bind(4, 14), Bind(5, 15), Bind(6, 16)])
    assert e.value.rc == abi.DOE_INVALID_ARGUMENT


def test_kv_write_read_dispatch_exact_and_position_error(be):
    g = np.random.default_rng(6)
    heads, max_len, D = 3, 40, 64
    kp = g.standard_normal((heads, D), dtype=np.float32)
    vp = g.standard_normal((heads, D), dtype=np.float32)
    be.execute_buffer_write_bytes(20, 0, _u32(heads, max_len, D, 4))
    be.execute_buffer_write_bytes(21, 0, kp)
    be.execute_buffer_write_bytes(22, 0, vp)
    be.ensure_buffer(23, heads * max_len * D * 4)
    be.ensure_buffer(24, heads * max_len * D * 4)
    be.execute_buffer_write_bytes(25, 0, np.array([17], np.uint32))
    binds = [Bind(0, 20, size=16), Bind(1, 21), Bind(2, 22), Bind(3, 23), Bind(4, 24), Bind(5, 25, size=4)]
    be.execute_kernel_dispatch("kv_write", binds)
    be.flush_queue()
    kc = np.frombuffer(be.capture_buffer(23, 0, heads * max_len * D * 4), np.float32).reshape(heads, max_len, D)
    exp = np.zeros((heads, max_len, D), np.float32)
    for h in range(heads):
        oracle.kv_write_dense(kp[h], vp[h], exp[h], np.zeros_like(exp[h]), 17)
    assert np.array_equal(kc, exp)
    # read back rows [15, 20)
    be.execute_buffer_write_bytes(26, 0, _u32(heads, max_len, D, 4, 15, 5))
    be.execute_kernel_dispatch("kv_read", [Bind(0, 26, size=24), Bind(1, 23), Bind(2, 24),
                                           Bind(3, 27, size=heads * 5 * D * 4),
                                           Bind(4, 28, size=heads * 5 * D * 4)])
    ko = np.frombuffer(be.capture_buffer(27, 0, heads * 5 * D * 4), np.float32).reshape(heads, 5, D)
    assert np.array_equal(ko, exp[:, 15:20])
    # position >= max_seq_len: nothing written, flush reports OUT_OF_RANGE
    be.execute_buffer_write_bytes(25, 0, np.array([max_len], np.uint32))
    be.execute_kernel_dispatch("kv_write", binds)
    with pytest.raises(abi.DoeError) as e:
        be.flush_queue()
    assert e.value.rc == abi.DOE_OUT_OF_RANGE
    kc2 = np.frombuffer(be.capture_buffer(23, 0, heads * max_len * D * 4), np.float32).reshape(heads, max_len, D)
    assert np.array_equal(kc2, exp)
    be.flush_queue()  # the error word was cleared


def test_rope_dispatch(be):
    g = np.random.default_rng(8)
    S, H, D, off = 6, 4, 64, 3
    x = g.standard_normal((S, H, D), dtype=np.float32)
    ang = g.uniform(-3, 3, (S + off, D // 2)).astype(np.float32)
    fc = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32).reshape(-1)
    be.execute_buffer_write_bytes(30, 0, _u32(S, D, H, off))
    be.execute_buffer_write_bytes(31, 0, x)
    be.execute_buffer_write_bytes(32, 0, fc)
    be.execute_kernel_dispatch("rope.wgsl", [Bind(0, 30, size=16), Bind(1, 31), Bind(2, 32)])
    out = np.frombuffer(be.capture_buffer(31, 0, x.nbytes), np.float32).reshape(x.shape)
    assert np.array_equal(out, oracle.rope(x, fc, off))


def test_paged_decode_dispatch_matches_operator(be):
    w = workloads.small_paged(3, [10, 200, 33])
    from doe_b200.kv import PagedKVCache
    c = PagedKVCache(num_pages=w.num_pages, page_size=w.page_size, num_kv_heads=w.num_kv_heads,
                     head_dim=w.head_dim, block_table=w.block_table)
    workloads.fill_pools(c, 5)
    kp = c.k_pool.cpu().numpy()
    vp = c.v_pool.cpu().numpy()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ref = ops.paged_decode(c, t(w.q), t(w.seq_lens), w.scale, new_k=t(w.new_k), new_v=t(w.new_v))
    torch.cuda.synchronize()
    uni = _u32(w.num_seqs, w.num_heads, w.num_kv_heads, w.head_dim, w.page_size, w.num_pages,
               w.block_table.shape[1], 0, float(np.float32(w.scale)), 0)
    for h, arr in ((40, uni), (41, w.q), (42, kp), (43, vp), (44, w.block_table), (45, w.seq_lens),
                   (47, w.new_k), (48, w.new_v)):
        be.execute_buffer_write_bytes(h, 0, arr)
    be.execute_kernel_dispatch("attention_paged_decode",
                               [Bind(0, 40, size=40), Bind(1, 41), Bind(2, 42), Bind(3, 43), Bind(4, 44),
                                Bind(5, 45), Bind(6, 46, size=w.num_seqs * w.num_heads * w.head_dim * 4),
                                Bind(7, 47), Bind(8, 48)])
    out = np.frombuffer(be.capture_buffer(46, 0, w.num_seqs * w.num_heads * w.head_dim * 4), np.float32)
    assert np.array_equal(out.reshape(ref.shape), ref.cpu().numpy())
    assert np.array_equal(np.frombuffer(be.capture_buffer(42, 0, kp.nbytes), np.float16).reshape(kp.shape),
                          c.k_pool.cpu().numpy())


def test_queued_steps_on_alternating_buffers_match_synchronous_steps(be):
    # writes run on the backend's copy stream and kernels on its compute
    # stream, ordered per buffer by events; four decode steps queued back to
    # back (new queries each step, two buffer sets alternating, deferred
    # captures) must give what one synchronous step at a time gives
    w = workloads.small_paged(4, [40, 300, 7, 129])
    g = np.random.default_rng(8)
    qs = [g.standard_normal(w.q.shape, dtype=np.float32).astype(np.float16) for _ in range(4)]
    out_bytes = w.num_seqs * w.num_heads * w.head_dim * 4
    uni = _u32(w.num_seqs, w.num_heads, w.num_kv_heads, w.head_dim, w.page_size, w.num_pages,
               w.block_table.shape[1], 0, float(np.float32(w.scale)), 0)
    from doe_b200.kv import PagedKVCache
    c = PagedKVCache(num_pages=w.num_pages, page_size=w.page_size, num_kv_heads=w.num_kv_heads,
                     head_dim=w.head_dim, block_table=w.block_table)
    workloads.fill_pools(c, 6)
    kp, vp = c.k_pool.cpu().numpy(), c.v_pool.cpu().numpy()

    def setup(b):
        for h, arr in ((60, uni), (62, kp), (63, vp), (64, w.block_table)):
            b.execute_buffer_write_bytes(h, 0, arr)

    def binds(o):
        return [Bind(0, 60, size=40), Bind(1, 70 + o), Bind(2, 62), Bind(3, 63), Bind(4, 64), Bind(5, 71 + o),
                Bind(6, 72 + o, size=out_bytes), Bind(7, 73 + o), Bind(8, 74 + o)]

    def upload(b, i, o):
        for h, arr in ((70 + o, qs[i]), (71 + o, w.seq_lens), (73 + o, w.new_k), (74 + o, w.new_v)):
            b.execute_buffer_write_bytes(h, 0, arr)

    setup(be)
    expected = []
    for i in range(4):  # one step at a time, synchronous captures
        upload(be, i, 0)
        be.execute_kernel_dispatch("attention_paged_decode", binds(0))
        expected.append(np.frombuffer(be.capture_buffer(72, 0, out_bytes), np.float32).copy())
    b2 = CudaBackend(0)
    try:
        setup(b2)
        outs = [torch.zeros(out_bytes, dtype=torch.uint8).pin_memory() for _ in range(4)]
        for i in range(4):  # queued
            o = 10 * (i & 1)
            upload(b2, i, o)
            b2.execute_kernel_dispatch("attention_paged_decode", binds(o))
            b2.read_into_async(72 + o, 0, outs[i].data_ptr(), out_bytes)
        b2.flush_queue()
        for i in range(4):
            assert np.array_equal(outs[i].numpy().view(np.float32), expected[i]), f"step {i}"
    finally:
        b2.close()


def _uniform15(**u) -> np.ndarray:
    names = ("num_heads", "num_kv_heads", "head_dim", "seq_len", "query_len", "scale", "is_causal",
             "start_pos", "attn_softcap", "sliding_window", "kv_len_source", "kv_start", "page_size",
             "kv_layout")
    return np.array([np.float32(u[n]).view(np.uint32) if isinstance(u[n], float) else u[n] for n in names]
                    + [0], np.uint32)


@pytest.fixture(scope="module")
def prefill_config2_case():
    """Config 2 shapes with f32 queries (not f16-representable, so the
    dispatch's f16 rounding of Q is exercised) and the oracle over every row."""
    w = workloads.prefill_f16()
    S, H, D = w.q.shape
    q = np.random.default_rng(12).standard_normal((S, H, D), dtype=np.float32) * np.float32(0.5)
    u = dict(num_heads=H, num_kv_heads=w.k.shape[1], head_dim=D, seq_len=S, query_len=S,
             scale=float(np.float32(w.scale)), is_causal=1, start_pos=0, attn_softcap=0.0,
             sliding_window=0, kv_len_source=0, kv_start=0, page_size=16, kv_layout=0)
    ref = oracle.attention_online_f16kv(u, q, w.k.view(np.uint16), w.v.view(np.uint16))
    return w, q, u, ref


@pytest.mark.parametrize("name", ["attention_prefill", "attention_prefill_kv_axis_sharded"])
def test_exec_v1_prefill_runs_tcgen05_prefill(be, name, prefill_config2_case):
    """The exec-v1 prefill ops (emit_csl_exec_v1.zig:118,125) on config 2's
    shapes take the tensor-core prefill: the launch list holds prefill_kernel,
    and every output row is within 2e-3 of the oracle."""
    w, q, u, ref = prefill_config2_case
    for h, arr in ((80, _uniform15(**u)), (81, q), (82, w.k), (83, w.v)):
        be.execute_buffer_write_bytes(h, 0, arr)
    be.flush_queue()
    binds = [Bind(0, 80, size=64), Bind(1, 81), Bind(2, 82), Bind(3, 83), Bind(4, 84, size=q.nbytes)]
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        be.execute_kernel_dispatch(name, binds)
        be.flush_queue()
    kernels = [e.key for e in prof.key_averages()]
    assert any("prefill_kernel" in k for k in kernels), kernels
    assert not any("attn_online_generic" in k for k in kernels), kernels
    out = np.frombuffer(be.capture_buffer(84, 0, q.nbytes), np.float32).reshape(q.shape)
    within(out, ref, 2e-3)


def test_exec_v1_prefill_other_uniforms_run_head256_kernel(be):
    """attention_prefill with a softcap, a query chunk after earlier keys and
    GQA is not a whole-prompt prefill: it runs the head256 kernel and matches
    the oracle at the f32 bound."""
    g = np.random.default_rng(14)
    S, Q0, H, Hkv, D = 96, 64, 4, 2, 128
    q = g.standard_normal((S - Q0, H, D), dtype=np.float32)
    k = g.standard_normal((S, Hkv, D), dtype=np.float32).astype(np.float16)
    v = g.standard_normal((S, Hkv, D), dtype=np.float32).astype(np.float16)
    u = dict(num_heads=H, num_kv_heads=Hkv, head_dim=D, seq_len=S, query_len=S - Q0, scale=0.088,
             is_causal=1, start_pos=Q0, attn_softcap=20.0, sliding_window=0, kv_len_source=0,
             kv_start=0, page_size=16, kv_layout=0)
    for h, arr in ((90, _uniform15(**u)), (91, q), (92, k), (93, v)):
        be.execute_buffer_write_bytes(h, 0, arr)
    binds = [Bind(0, 90, size=64), Bind(1, 91), Bind(2, 92), Bind(3, 93), Bind(4, 94, size=q.nbytes)]
    be.execute_kernel_dispatch("attention_prefill", binds)
    out = np.frombuffer(be.capture_buffer(94, 0, q.nbytes), np.float32).reshape(q.shape)
    within(out, oracle.attention_online_f16kv(u, q, k.view(np.uint16), v.view(np.uint16)), 1e-5)


def test_upload_behavior_flushes_every_n_writes(be):
    """set_upload_behavior (backend_iface.zig:17): writes still land in order
    with a flush every 2 writes; unknown usage modes are refused."""
    g = np.random.default_rng(15)
    be.set_upload_behavior(abi.DOE_UPLOAD_COPY_DST, 2)
    chunks = [g.integers(0, 256, 4096, dtype=np.uint8) for _ in range(5)]
    for i, c in enumerate(chunks):
        be.execute_buffer_write_bytes(95, i * 4096, c)
    assert be.capture_buffer(95, 0, 5 * 4096) == np.concatenate(chunks).tobytes()
    be.set_upload_behavior(abi.DOE_UPLOAD_COPY_DST_COPY_SRC, 0xFFFFFFFF)
    with pytest.raises(abi.DoeError) as e:
        be.set_upload_behavior(7, 1)
    assert e.value.rc == abi.DOE_INVALID_ARGUMENT
