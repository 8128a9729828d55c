"""The ORT plugin EP's basic operators, host side (no GPU).

- The numpy restatement (oracle/ort_ep.py) reproduces every case of the
  reference EP's session smoke test within its absolute tolerance 1e-5
  (runtime/bridge/onnxruntime-ep/src/doe_ort_ep_session_smoke.cc:578-584,
  808-950; fixture tests/golden/ort_ep_smoke_cases.json).
- doe_b200.ort_ep.validate applies the EP's runtime shape rules with its
  messages before any device call.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from doe_b200 import ort_ep
from oracle import ort_ep as oep


def _cases(golden_dir):
    return json.loads((golden_dir / "ort_ep_smoke_cases.json").read_text())


def test_fixture_covers_every_smoke_case(golden_dir):
    d = _cases(golden_dir)
    names = {c["name"] for c in d["cases"]}
    assert names == set(oep.KINDS), names ^ set(oep.KINDS)
    assert d["tolerance_abs"] == 1e-5
    assert names <= set(ort_ep.KINDS)


def test_oracle_matches_reference_smoke_cases(golden_dir):
    d = _cases(golden_dir)
    for c in d["cases"]:
        ins = [np.asarray(v, np.float32).reshape(dims) for v, dims in zip(c["inputs"], c["input_dims"])]
        got = oep.KINDS[c["name"]](ins)
        assert list(got.shape) == c["output_dims"], c["name"]
        exp = np.asarray(c["expected"], np.float32).reshape(c["output_dims"])
        assert np.abs(got - exp).max() <= d["tolerance_abs"], (c["name"], got, exp)


def test_oracle_matmul_folds_in_order():
    # 2^24 + 1 - 1: left to right in f32 the +1 is lost; a float64 product would keep it
    a = np.array([[1.0, 1.0, -1.0]], np.float32)
    b = np.array([[2.0 ** 24], [1.0], [2.0 ** 24]], np.float32)
    assert oep.matmul(a, b)[0, 0] == 0.0


def test_oracle_softmax_and_layernorm_edges():
    assert oep.softmax(np.zeros((3, 0), np.float32)).shape == (3, 0)
    s = oep.softmax(np.array([[-np.inf, 0.0]], np.float32))
    assert s.tolist() == [[0.0, 1.0]]
    y = oep.layernorm(np.full((2, 4), 3.0, np.float32), np.ones(4, np.float32))
    assert np.all(y == 0.0)


def _meta(*shape):
    return torch.empty(shape, device="meta")


def test_validate_shapes_and_messages():
    assert ort_ep.validate("add", _meta(2, 3), _meta(2, 3)) == (2, 3)
    with pytest.raises(ort_ep.InvalidGraph, match=r"Add slice requires exact-shape float32 tensors; input0 has "
                                                  r"shape \[2, 3\] while input1 has shape \[3, 2\]"):
        ort_ep.validate("add", _meta(2, 3), _meta(3, 2))
    assert ort_ep.validate("matmul", _meta(4, 5), _meta(5, 6)) == (4, 6)
    with pytest.raises(ort_ep.InvalidGraph, match="requires rank-2 float32 inputs"):
        ort_ep.validate("matmul", _meta(2, 3, 4), _meta(4, 5))
    with pytest.raises(ort_ep.InvalidGraph, match="exact matrix inner dimensions"):
        ort_ep.validate("matmul", _meta(2, 3), _meta(4, 5))
    with pytest.raises(ort_ep.InvalidGraph, match=r"Gemm slice .* gemm_bias has shape \[2\]"):
        ort_ep.validate("gemm", _meta(2, 3), _meta(3, 2), _meta(2))
    with pytest.raises(ort_ep.InvalidGraph, match=r"MatMul->Add->Relu slice .* add_input"):
        ort_ep.validate("matmul_add_relu", _meta(2, 3), _meta(3, 2), _meta(1, 2))
    assert ort_ep.validate("gemm_relu_gemm", _meta(1, 2), _meta(2, 3), _meta(1, 3), _meta(3, 2),
                           _meta(1, 2)) == (1, 2)
    with pytest.raises(ort_ep.InvalidGraph, match="hidden_bias"):
        ort_ep.validate("gemm_relu_gemm", _meta(1, 2), _meta(2, 3), _meta(1, 4), _meta(3, 2), _meta(1, 2))
    with pytest.raises(ort_ep.InvalidGraph, match="rank >= 1"):
        ort_ep.validate("softmax", _meta())
    with pytest.raises(ort_ep.InvalidGraph, match="scale length must match"):
        ort_ep.validate("layernorm", _meta(2, 4), _meta(3))
    assert ort_ep.validate("concat", _meta(2, 3, 4), _meta(2, 5, 4), axis=1) == (2, 8, 4)
    assert ort_ep.validate("concat", _meta(2, 3), _meta(2, 3), axis=-1) == (2, 6)
    with pytest.raises(ort_ep.InvalidGraph, match="non-axis"):
        ort_ep.validate("concat", _meta(2, 3), _meta(3, 3), axis=1)
    with pytest.raises(ort_ep.InvalidGraph, match="out of range"):
        ort_ep.validate("concat", _meta(2, 3), _meta(2, 3), axis=2)
    with pytest.raises(ValueError, match="unknown op kind"):
        ort_ep.validate("conv", _meta(1))
    with pytest.raises(ort_ep.InvalidGraph, match="takes 2 inputs"):
        ort_ep.validate("add", _meta(1))


def test_execute_needs_cuda_tensors():
    with pytest.raises(ValueError, match="CUDA float32"):
        ort_ep.execute("relu", torch.zeros(4))
