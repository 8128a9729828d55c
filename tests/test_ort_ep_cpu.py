"""The ORT plugin EP's basic operators, host side (no GPU).

- The numpy restatement (oracle/ort_ep.py) reproduces every case of the
  reference EP's session smoke test within its absolute tolerance 1e-5
  (runtime/bridge/onnxruntime-ep/src/doe_ort_ep_session_smoke.cc:578-584,
  808-950; fixture tests/golden/ort_ep_smoke_cases.json).
- doe_b200.ort_ep.validate applies the EP's runtime shape rules with its
  messages before any device call, and the C ABI's doe_ep_* entry points
  reject bad arguments before any launch.
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


def test_c_abi_validation_precedes_any_launch():
    """The doe_ep_* entry points reject bad calls on the host: nothing below
    reaches a kernel (the fake pointers are never dereferenced)."""
    import ctypes as C

    from doe_b200 import _abi as abi

    lib = abi.lib()
    x, y = 0x10000, 0x20000  # 16-byte aligned, disjoint for n <= 4096
    inval = abi.DOE_INVALID_ARGUMENT
    assert lib.doe_ep_unary_f32(9, x, y, 4, None) == inval
    assert "unknown op" in abi.op_error()
    assert lib.doe_ep_unary_f32(abi.EP_RELU, None, y, 4, None) == inval
    assert lib.doe_ep_unary_f32(abi.EP_RELU, x, x + 4, 100, None) == inval
    assert "overlap" in abi.op_error()
    assert lib.doe_ep_unary_f32(abi.EP_RELU, None, None, 0, None) == abi.DOE_OK  # empty: nothing to do
    assert lib.doe_ep_binary_f32(5, x, x, y, 4, None) == inval
    assert lib.doe_ep_binary_f32(abi.EP_ADD, x, y + 8, y, 16, None) == inval  # b partly overlaps y
    assert lib.doe_ep_softmax_f32(x, y, 1 << 40, 4096, None) == inval
    assert lib.doe_ep_softmax_f32(None, None, 0, 5, None) == abi.DOE_OK
    assert lib.doe_ep_softmax_f32(None, None, 5, 0, None) == abi.DOE_OK  # empty axis (ExecuteSoftmax)
    assert lib.doe_ep_layernorm_f32(x, x + 64, -1.0, y, 1, 4, None) == inval
    assert "epsilon" in abi.op_error()
    assert lib.doe_ep_layernorm_f32(x, y + 16, 1e-5, y, 2, 16, None) == inval  # scale inside y
    assert lib.doe_ep_concat_f32(x, x + 4096, x + 32, 1, 4, 4, 4, None) == inval  # y over a
    assert lib.doe_ep_matmul_f32(x, x, None, y, 4, 4, 4, 2, None) == inval
    assert "flags" in abi.op_error()
    assert lib.doe_ep_matmul_f32(x, x, None, y, 1 << 31, 4, 4, 0, None) == inval
    assert lib.doe_ep_matmul_f32(x, x, None, y, 65535 * 128 + 1, 1, 1, 0, None) == inval
    assert lib.doe_ep_matmul_f32(x, x + 0x1000, None, x + 8, 4, 4, 4, 0, None) == inval  # y over a
    assert lib.doe_ep_matmul_f32(None, None, None, None, 0, 4, 4, 0, None) == abi.DOE_OK
    rc = lib.doe_ep_gemm_relu_gemm_f32(x, x, x, x, x, y, 2, 2, 2, 2, None)
    assert rc == inval and "workspace" in abi.op_error()
    assert lib.doe_ep_gemm_relu_gemm_workspace_bytes(32, 1000) == 128000
    l = abi.Launch(None, None, 0, None)
    assert lib.doe_ep_gemm_relu_gemm_f32(x, x, x, x, x, y, 0, 2, 2, 2, C.byref(l)) == abi.DOE_OK
