"""GPU parity: f32 decode (config 1), the generic head256 kernel, prefill.wgsl, stitch.

Every comparison is against the CPU oracle (oracle/), itself pinned to the
reference's golden vectors in test_oracle_golden.py.  Tolerances: f32 paths
1e-5 relative (|o - ref| <= 1e-5 * max(|ref|, 1)).
"""
from __future__ import annotations

import hashlib
import json
import zlib

import numpy as np
import pytest

import oracle
from doe_b200 import ops, workloads

from .gpu_util import within

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

F32_TOL = 1e-5


def _t(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)  # same bits; torch's uint32 support is partial
    return torch.from_numpy(a).cuda()


def test_config1_decode_f32_matches_oracle():
    w = workloads.decode_f32()
    out = ops.attention_decode_f32(_t(w.q), _t(w.k), _t(w.v), w.scale).cpu().numpy()
    ref = oracle.attention_decode_wgsl(w.q, w.k, w.v, w.scale)
    within(out, ref, F32_TOL)


@pytest.mark.parametrize("H,D,L", [(1, 64, 1), (3, 64, 2), (8, 64, 63), (8, 64, 65), (2, 32, 700),
                                   (4, 100, 129), (2, 128, 2048), (2, 128, 2049), (1, 256, 5000),
                                   (16, 8, 3)])
def test_decode_f32_shapes(H, D, L):
    g = np.random.default_rng(H * 1000 + D + L)
    q = g.standard_normal((H, D), dtype=np.float32)
    k = g.standard_normal((H, L, D), dtype=np.float32)
    v = g.standard_normal((H, L, D), dtype=np.float32)
    scale = 1.0 / np.sqrt(D)
    out = ops.attention_decode_f32(_t(q), _t(k), _t(v), scale).cpu().numpy()
    within(out, oracle.attention_decode_wgsl(q, k, v, scale), F32_TOL)


def test_decode_sim_seed11_golden(golden_dir):
    z = np.load(golden_dir / "decode_sim_seed11.npz")
    out = ops.attention_decode_f32(_t(z["q"][:, 0]), _t(z["k"]), _t(z["v"]), float(z["scale"][0]))
    atol, rtol = z["tol"]
    np.testing.assert_allclose(out.cpu().numpy(), z["expected"], atol=atol, rtol=rtol)
    within(out.cpu().numpy(), z["expected"], F32_TOL)


def test_attention_slice_kat(golden_dir):
    kat = json.loads((golden_dir / "attention_slice_kat.json").read_text())
    q = np.array(kat["q_u32"], np.uint32).view(np.float32)[None]
    k = np.array(kat["k_u32"], np.uint32).view(np.float32).reshape(1, 8, 8)
    v = np.zeros((1, 8, 8), np.float32)
    v[0, :, :2] = np.array(kat["v_u32"], np.uint32).view(np.float32).reshape(8, 2)
    scale = float(np.array(kat["uniform_u32"][2], np.uint32).view(np.float32))
    out = ops.attention_decode_f32(_t(q), _t(k), _t(v), scale).cpu().numpy()[0, :2]
    for meta in kat["exact"].values():
        within(out, np.array(meta["exactReferenceLogits"]), F32_TOL)


def test_zero_input_canary(golden_dir):
    shas = json.loads((golden_dir / "canary.json").read_text())["canary_output_sha256"]
    for D, L in ((256, 15), (256, 1)):
        z = torch.zeros((1, L, D), dtype=torch.float32, device="cuda")
        out = ops.attention_decode_f32(torch.zeros((1, D), device="cuda"), z, z, 1.0)
        assert hashlib.sha256(out.cpu().numpy()[0].tobytes()).hexdigest() == shas[str(D)]
    for D, L in ((256, 15), (512, 7)):
        u = dict(num_heads=1, num_kv_heads=1, head_dim=D, seq_len=L, query_len=1, scale=1.0,
                 is_causal=0, start_pos=0, attn_softcap=0.0, sliding_window=0, kv_len_source=0,
                 kv_start=0, page_size=16, kv_layout=0)
        zk = torch.zeros((L, 1, D), dtype=torch.float16, device="cuda")
        out = ops.attention_online(u, torch.zeros((1, 1, D), device="cuda"), zk, zk)
        assert hashlib.sha256(out.cpu().numpy()[0, 0].tobytes()).hexdigest() == shas[str(D)]


def _online_case(seed, *, H, Hkv, D, qlen, kvlen, causal=0, start_pos=0, softcap=0.0, window=0,
                 layout=0, page=16, kv_start=0, len_source=0, kv_rows=None):
    g = np.random.default_rng(seed)
    rows = kv_rows if kv_rows is not None else (kv_start + kvlen)
    q = g.standard_normal((qlen, H, D), dtype=np.float32)
    kf = g.standard_normal((rows, Hkv, D), dtype=np.float32).astype(np.float16)
    vf = g.standard_normal((rows, Hkv, D), dtype=np.float32).astype(np.float16)
    u = dict(num_heads=H, num_kv_heads=Hkv, head_dim=D, seq_len=kvlen, query_len=qlen,
             scale=1.0 / np.sqrt(D), is_causal=causal, start_pos=start_pos, attn_softcap=softcap,
             sliding_window=window, kv_len_source=len_source, kv_start=kv_start, page_size=page,
             kv_layout=layout)
    pt = None
    if layout == 2:
        npages = -(-rows // page)
        pt = g.permutation(npages).astype(np.uint32)
    klb = np.array([kvlen], np.uint32)
    if len_source:
        u["seq_len"] = 0  # the buffer wins
    return u, q, kf, vf, klb, pt


@pytest.mark.parametrize("case", [
    dict(H=4, Hkv=4, D=64, qlen=1, kvlen=300),
    dict(H=8, Hkv=2, D=128, qlen=40, kvlen=40, causal=1),
    dict(H=8, Hkv=2, D=128, qlen=33, kvlen=100, causal=1, start_pos=67),
    dict(H=4, Hkv=1, D=256, qlen=5, kvlen=70, causal=1, start_pos=65, window=20),
    dict(H=2, Hkv=2, D=64, qlen=3, kvlen=50, softcap=5.0),
    dict(H=2, Hkv=1, D=64, qlen=2, kvlen=40, layout=1, window=16, kv_rows=16),
    dict(H=4, Hkv=2, D=128, qlen=2, kvlen=90, layout=2, page=16, kv_rows=96),
    dict(H=4, Hkv=2, D=128, qlen=1, kvlen=77, len_source=1),
    dict(H=2, Hkv=2, D=512, qlen=2, kvlen=45, causal=1, start_pos=43),
    dict(H=2, Hkv=2, D=96, qlen=1, kvlen=33, kv_start=10, causal=1, start_pos=42),
])
def test_online_generic_matches_oracle(case):
    u, q, kf, vf, klb, pt = _online_case(zlib.crc32(json.dumps(case, sort_keys=True).encode()), **case)
    kb, vb = kf.view(np.uint16), vf.view(np.uint16)
    ref = oracle.attention_online_f16kv(u, q, kb, vb, klb, pt)
    out = ops.attention_online(u, _t(q), _t(kf), _t(vf), _t(klb), None if pt is None else _t(pt))
    within(out.cpu().numpy(), ref, F32_TOL)


def test_prefill_wgsl_matches_oracle():
    g = np.random.default_rng(77)
    H, S, D = 2, 100, 64
    q, k, v = (g.standard_normal((H, S, D), dtype=np.float32) for _ in range(3))
    out = ops.attention_prefill_wgsl(_t(q), _t(k), _t(v), 0.125).cpu().numpy()
    within(out, oracle.attention_prefill_wgsl(q, k, v, 0.125), F32_TOL)


def test_stitch_matches_reference_golden(golden_dir):
    z = np.load(golden_dir / "stitch_reference.npz")
    for i in range(int(z["count"][0])):
        parts = z[f"c{i}_partials"]
        out = ops.stitch(_t(parts[None])).cpu().numpy()[0]
        np.testing.assert_allclose(out, z[f"c{i}_out"], rtol=2e-6, atol=1e-7)
