"""Command-stream replay, host side (no GPU).

- The buffer_load asset generator (doe_b200/command_stream.py, the
  reference's splitmix64 nonzero generators, bench/lib/synthetic_assets.py:
  160-222) reproduces the sha256 of payloads the reference's own generator
  made (tests/golden/synthetic_assets.json, written by make_golden.py): five
  small cases and every buffer_load of the Gemma 3 270M decode stream.
- The CPU restatements of the stream's kernels (oracle/pipeline.py) against
  plain float64 numpy of the same formulas, and sample.wgsl's tie order.
- The whole 270M decode stream replays on the CPU oracle to one token.
"""
from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from doe_b200 import command_stream as cs
from oracle import pipeline as opl


@pytest.fixture(scope="module")
def streams(golden_dir):
    return json.loads((golden_dir / "gemma_command_streams.json").read_text())["streams"]


def test_generator_matches_reference_hashes(golden_dir, streams):
    d = json.loads((golden_dir / "synthetic_assets.json").read_text())
    for c in d["cases"]:
        data = cs.synthetic_asset(c["generator"], c["seed"], c["scale"], c["byteLength"])
        assert data[:32].hex() == c["head_hex"], c
        assert hashlib.sha256(data).hexdigest() == c["sha256"], c
    loads = {c["handle"]: c for c in streams["inference_gemma3_270m_decode_1tok_commands"]
             if c["kind"] == "buffer_load"}
    assert len(d["inference_gemma3_270m_decode_1tok"]) == len(loads) > 0
    for a in d["inference_gemma3_270m_decode_1tok"]:
        c = loads[a["handle"]]
        data = cs.synthetic_asset(c["generator"], c["seed"], c["scale"], c["byteLength"])
        assert hashlib.sha256(data).hexdigest() == a["sha256"], a["handle"]


def test_generator_rejects_bad_arguments():
    with pytest.raises(ValueError):
        cs.synthetic_asset("splitmix64_f32_nonzero_v1", 1, 0.0, 16)
    with pytest.raises(ValueError):
        cs.synthetic_asset("splitmix64_f32_nonzero_v1", 1, 1.0, 10)
    with pytest.raises(ValueError):
        cs.synthetic_asset("uniform", 1, 1.0, 16)


def test_kernel_restatements_against_float64():
    g = np.random.default_rng(1)
    x = g.standard_normal((3, 1000), dtype=np.float32)
    w = g.standard_normal(1000, dtype=np.float32)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * w
    assert np.allclose(opl.rmsnorm(x, w, 1000, 1e-6, 3), ref, rtol=1e-5, atol=1e-6)
    ref1 = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * (1 + w)
    assert np.allclose(opl.rmsnorm(x, w, 1000, 1e-6, 3, weight_offset=True), ref1, rtol=1e-5, atol=1e-6)
    m = g.standard_normal((70, 1030), dtype=np.float32)
    v = g.standard_normal(1030, dtype=np.float32)
    assert np.allclose(opl.gemv(m, v, 70, 1030), m.astype(np.float64) @ v, rtol=1e-5, atol=1e-4)
    a = g.standard_normal((5, 37), dtype=np.float32)
    b = g.standard_normal((37, 11), dtype=np.float32)
    assert np.allclose(opl.matmul_tiled(a, b, 5, 37, 11), a.astype(np.float64) @ b, rtol=1e-5, atol=1e-5)
    z = np.linspace(-30, 30, 1001, dtype=np.float32)
    inner = np.clip(0.7978845608 * (z + 0.044715 * z.astype(np.float64) ** 3), -15, 15)
    assert np.allclose(opl.gelu(z), 0.5 * z * (1 + np.tanh(inner)), rtol=1e-6, atol=1e-6)


def test_sample_tie_order_and_floor():
    lg = np.full(1000, -5.0, np.float32)
    lg[700] = lg[300] = lg[44] = 2.0    # 700 % 256 = 188, 300 % 256 = 44, 44 % 256 = 44
    assert opl.sample(lg, 1000) == 44   # smallest index mod 256, then smallest index
    lg[44] = 1.0
    assert opl.sample(lg, 1000) == 300
    lg[:] = -1e30                       # nothing above -1e30: token 0
    assert opl.sample(lg, 1000) == 0
    lg[999] = np.nan
    lg[5] = -1e29
    assert opl.sample(lg, 1000) == 5


def test_270m_decode_stream_replays_on_the_oracle(streams):
    cmds = streams["inference_gemma3_270m_decode_1tok_commands"]
    bufs, log = opl.replay(cmds, cs.synthetic_asset)
    kernels = [k for k, _, _ in log]
    assert kernels.count("matmul-gemv.wgsl") == 8 and kernels[-1] == "sample.wgsl"
    token = int(np.frombuffer(log[-1][2], np.uint32)[0])
    assert 0 <= token < 4096
    for _, _, data in log:
        assert np.isfinite(np.frombuffer(data, np.float32)).all()
