"""The ORT plugin EP's basic f32 operators on device tensors.

The reference EP claims ONNX nodes of these kinds and runs each on the host
(runtime/bridge/onnxruntime-ep/src/doe_ort_ep.cc:1899-2401).  `execute(kind,
*inputs)` is the GPU form of its Compute dispatch: the same op kinds (the
names its session smoke test uses), the same shape checks and messages
(ValidateSameRuntimeShape, ValidateRuntimeMatMulShape, :1864-1897; the
Softmax / LayerNorm rank and scale checks, :2031, :2079-2084), and one
libdoe_cuda kernel per node.  Inputs are CUDA float32 tensors; the result is
a new CUDA float32 tensor.  There is no host fallback.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _abi as abi
from .ops import _launch

KINDS = ("identity", "add", "relu", "sigmoid", "tanh", "gelu", "matmul", "gemm", "gemm_relu_gemm", "matmul_add",
         "matmul_add_relu", "add_relu", "softmax", "layernorm", "concat")

_UNARY = {"identity": abi.EP_IDENTITY, "relu": abi.EP_RELU, "sigmoid": abi.EP_SIGMOID, "tanh": abi.EP_TANH,
          "gelu": abi.EP_GELU}
_BINARY = {"add": abi.EP_ADD, "add_relu": abi.EP_ADD_RELU}
_INPUTS = {**{k: 1 for k in _UNARY}, **{k: 2 for k in _BINARY}, "matmul": 2, "gemm": 3, "matmul_add": 3,
           "matmul_add_relu": 3, "gemm_relu_gemm": 5, "softmax": 1, "layernorm": 2, "concat": 2}
LAYERNORM_EPSILON = 1e-5  # kDefaultLayerNormEpsilon (doe_ort_ep.cc:52)


class InvalidGraph(ValueError):
    """A node whose runtime shapes the EP rejects (ORT_INVALID_GRAPH)."""


# CompiledOpKindName (doe_ort_ep.cc:183-217): the name a kind's messages use
OP_NAMES = {"identity": "Identity", "add": "Add", "relu": "Relu", "sigmoid": "Sigmoid", "tanh": "Tanh",
            "gelu": "Gelu", "matmul": "MatMul", "gemm": "Gemm", "gemm_relu_gemm": "Gemm->Relu->Gemm",
            "matmul_add": "MatMul->Add", "matmul_add_relu": "MatMul->Add->Relu", "add_relu": "Add->Relu",
            "softmax": "Softmax", "layernorm": "LayerNormalization", "concat": "Concat"}


def _shape(t) -> str:
    """ShapeString (doe_ort_ep.cc:433): [d0, d1, ...]."""
    return "[" + ", ".join(str(d) for d in t.shape) + "]"


def _same_shape(kind, lhs_name, lhs, rhs_name, rhs) -> None:
    """ValidateSameRuntimeShape (doe_ort_ep.cc:1847-1862)."""
    if tuple(lhs.shape) != tuple(rhs.shape):
        raise InvalidGraph(f"Doe ORT plugin EP {OP_NAMES[kind]} slice requires exact-shape float32 tensors; "
                           f"{lhs_name} has shape {_shape(lhs)} while {rhs_name} has shape {_shape(rhs)}.")


def _matmul_shape(lhs, rhs) -> tuple[int, int, int]:
    if lhs.dim() != 2 or rhs.dim() != 2:
        raise InvalidGraph(f"Doe ORT plugin EP MatMul slice requires rank-2 float32 inputs; input0 has shape "
                           f"{_shape(lhs)} and input1 has shape {_shape(rhs)}.")
    if lhs.shape[1] != rhs.shape[0]:
        raise InvalidGraph(f"Doe ORT plugin EP MatMul slice requires exact matrix inner dimensions; input0 has "
                           f"shape {_shape(lhs)} and input1 has shape {_shape(rhs)}.")
    return lhs.shape[0], lhs.shape[1], rhs.shape[1]


def validate(kind: str, *inputs, axis: int | None = None) -> tuple:
    """The EP's runtime checks for one node; returns the output shape."""
    if kind not in _INPUTS:
        raise ValueError(f"unknown op kind {kind!r}; expected one of {', '.join(KINDS)}")
    if len(inputs) != _INPUTS[kind]:
        raise InvalidGraph(f"Doe ORT plugin EP {kind} takes {_INPUTS[kind]} inputs, got {len(inputs)}.")
    if kind in _UNARY:
        return tuple(inputs[0].shape)
    if kind in _BINARY:
        _same_shape(kind, "input0", inputs[0], "input1", inputs[1])
        return tuple(inputs[0].shape)
    if kind in ("matmul", "gemm", "matmul_add", "matmul_add_relu"):
        m, _, n = _matmul_shape(inputs[0], inputs[1])
        if kind != "matmul":
            out = torch.empty((m, n), device="meta")
            _same_shape(kind, "matmul_output", out, "gemm_bias" if kind == "gemm" else "add_input", inputs[2])
        return (m, n)
    if kind == "gemm_relu_gemm":
        x, w1, b1, w2, b2 = inputs
        b, _, hdim = _matmul_shape(x, w1)
        _same_shape(kind, "hidden_gemm_output", torch.empty((b, hdim), device="meta"), "hidden_bias", b1)
        _, _, odim = _matmul_shape(torch.empty((b, hdim), device="meta"), w2)
        _same_shape(kind, "output_gemm_output", torch.empty((b, odim), device="meta"), "output_bias", b2)
        return (b, odim)
    if kind == "softmax":
        if inputs[0].dim() == 0:
            raise InvalidGraph("Doe ORT plugin EP Softmax requires a tensor with rank >= 1.")
        return tuple(inputs[0].shape)
    if kind == "layernorm":
        x, scale = inputs
        if x.dim() == 0:
            raise InvalidGraph("Doe ORT plugin EP LayerNormalization requires a tensor with rank >= 1.")
        if scale.numel() != x.shape[-1]:
            raise InvalidGraph("Doe ORT plugin EP LayerNormalization scale length must match the last input "
                               "dimension.")
        return tuple(x.shape)
    # concat
    a, b = inputs
    if a.dim() != b.dim() or a.dim() == 0:
        raise InvalidGraph("Doe ORT plugin EP Concat requires two inputs of the same rank >= 1.")
    ax = 0 if axis is None else axis
    ax = ax + a.dim() if ax < 0 else ax
    if not 0 <= ax < a.dim():
        raise InvalidGraph(f"Doe ORT plugin EP Concat axis {axis} is out of range for rank {a.dim()}.")
    for i in range(a.dim()):
        if i != ax and a.shape[i] != b.shape[i]:
            raise InvalidGraph("Doe ORT plugin EP Concat inputs must match in every non-axis dimension.")
    out = list(a.shape)
    out[ax] = a.shape[ax] + b.shape[ax]
    return tuple(out)


def _dev(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda or t.dtype != torch.float32:
        raise ValueError(f"{name} must be a CUDA float32 tensor")
    return t.contiguous()


def execute(kind: str, *inputs, axis: int | None = None, epsilon: float = LAYERNORM_EPSILON, status=None,
            stream=None) -> torch.Tensor:
    """Run one EP node kind on device tensors and return its output."""
    out_shape = validate(kind, *inputs, axis=axis)
    xs = [_dev(t, f"input{i}") for i, t in enumerate(inputs)]
    dev = xs[0].device
    y = torch.empty(out_shape, dtype=torch.float32, device=dev)
    lib = abi.lib()
    if kind == "gemm_relu_gemm":
        b, hdim = xs[0].shape[0], xs[1].shape[1]
        ws = int(lib.doe_ep_gemm_relu_gemm_workspace_bytes(b, hdim))
        l = _launch(ws, status, stream, dev)
    else:
        l = _launch(0, status, stream, dev)
    p = [t.data_ptr() for t in xs]
    if kind in _UNARY:
        rc = lib.doe_ep_unary_f32(_UNARY[kind], p[0], y.data_ptr(), y.numel(), C.byref(l))
    elif kind in _BINARY:
        rc = lib.doe_ep_binary_f32(_BINARY[kind], p[0], p[1], y.data_ptr(), y.numel(), C.byref(l))
    elif kind in ("matmul", "gemm", "matmul_add", "matmul_add_relu"):
        m, k, n = xs[0].shape[0], xs[0].shape[1], xs[1].shape[1]
        flags = abi.EP_MATMUL_RELU if kind == "matmul_add_relu" else 0
        rc = lib.doe_ep_matmul_f32(p[0], p[1], p[2] if len(p) > 2 else None, y.data_ptr(), m, k, n, flags,
                                   C.byref(l))
    elif kind == "gemm_relu_gemm":
        b, i, hdim, o = xs[0].shape[0], xs[0].shape[1], xs[1].shape[1], xs[3].shape[1]
        rc = lib.doe_ep_gemm_relu_gemm_f32(*p, y.data_ptr(), b, i, hdim, o, C.byref(l))
    elif kind == "softmax":
        cols = xs[0].shape[-1]
        rc = lib.doe_ep_softmax_f32(p[0], y.data_ptr(), xs[0].numel() // cols if cols else 0, cols, C.byref(l))
    elif kind == "layernorm":
        cols = xs[0].shape[-1]
        rc = lib.doe_ep_layernorm_f32(p[0], p[1], float(epsilon), y.data_ptr(),
                                      xs[0].numel() // cols if cols else 0, cols, C.byref(l))
    else:  # concat
        a, b = xs
        ax = 0 if axis is None else (axis + a.dim() if axis < 0 else axis)
        outer = 1
        for d in a.shape[:ax]:
            outer *= d
        inner = 1
        for d in a.shape[ax + 1:]:
            inner *= d
        rc = lib.doe_ep_concat_f32(p[0], p[1], y.data_ptr(), outer, a.shape[ax], b.shape[ax], inner, C.byref(l))
    abi.check(f"doe_ep {kind}", rc)
    return y


__all__ = ["KINDS", "LAYERNORM_EPSILON", "OP_NAMES", "InvalidGraph", "execute", "validate"]
