"""numpy restatement of the ORT plugin EP's basic f32 operators.

TEST INFRASTRUCTURE ONLY: the parity checker for doe_b200.ort_ep, imported by
tests/ alone.

Each function follows one host compute kernel of the reference EP
(runtime/bridge/onnxruntime-ep/src/doe_ort_ep.cc) loop for loop, in f32 with
the same operation order: products rounded to f32 and added left to right
over k, row sums folded left to right, Softmax multiplying by 1 / sum.
Parity is pinned by the EP's own session smoke cases
(runtime/bridge/onnxruntime-ep/src/doe_ort_ep_session_smoke.cc:808-950,
checked there with an absolute tolerance of 1e-5, :578-584), copied into
tests/golden/ort_ep_smoke_cases.json by tests/golden/make_golden.py.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=F32)


def identity(x):
    """ExecuteIdentity (:1919): a copy."""
    return _f32(x).copy()


def add(a, b):
    """ExecuteAdd (:1933)."""
    return _f32(a) + _f32(b)


def relu(x):
    """ReluValue (:1899): value < 0 ? 0 : value (NaN passes through)."""
    x = _f32(x)
    return np.where(x < 0, F32(0), x).astype(F32)


def sigmoid(x):
    """SigmoidValue (:1903): 1 / (1 + exp(-x)) in f32."""
    x = _f32(x)
    with np.errstate(over="ignore"):
        return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)


def tanh(x):
    """TanhValue (:1907)."""
    return np.tanh(_f32(x)).astype(F32)


def gelu(x):
    """GeluValue (:1914): 0.5 * x * (1 + erf(x / sqrt(2))), f32 steps, erf of the f32 argument."""
    x = _f32(x)
    arg = (x * F32(0.70710678118654752440)).astype(F32)
    erf = np.vectorize(math.erf, otypes=[np.float64])(arg.astype(np.float64)).astype(F32)
    return (F32(0.5) * x * (F32(1) + erf)).astype(F32)


def add_relu(a, b):
    """ExecuteAddRelu (:2380)."""
    return relu(add(a, b))


def softmax(x):
    """ExecuteSoftmax (:2021): per last-axis row, exp(x - max) folded left to right,
    then multiplied by 1 / sum (0 when the sum is 0)."""
    x = _f32(x)
    if x.ndim == 0:
        raise ValueError("Softmax requires a tensor with rank >= 1")
    cols = x.shape[-1]
    if cols == 0:
        return x.copy()
    r = x.reshape(-1, cols)
    m = r.max(axis=1)
    e = np.exp((r - m[:, None]).astype(F32)).astype(F32)
    s = np.zeros(r.shape[0], F32)
    for i in range(cols):
        s = (s + e[:, i]).astype(F32)
    inv = np.where(s != 0, F32(1) / np.where(s != 0, s, F32(1)), F32(0)).astype(F32)
    return (e * inv[:, None]).astype(F32).reshape(x.shape)


def layernorm(x, scale, epsilon: float = 1e-5):
    """ExecuteLayerNorm (:2062): scale only; mean and variance folded left to
    right and multiplied by 1 / cols; y = (x - mean) * (1 / sqrt(var + eps)) * scale."""
    x = _f32(x)
    cols = x.shape[-1]
    scale = _f32(scale)
    if scale.size != cols:
        raise ValueError("LayerNormalization scale length must match the last input dimension")
    if cols == 0:
        return x.copy()
    r = x.reshape(-1, cols)
    inv_last = F32(1) / F32(cols)
    mean = np.zeros(r.shape[0], F32)
    for i in range(cols):
        mean = (mean + r[:, i]).astype(F32)
    mean = (mean * inv_last).astype(F32)
    var = np.zeros(r.shape[0], F32)
    for i in range(cols):
        d = (r[:, i] - mean).astype(F32)
        var = (var + (d * d).astype(F32)).astype(F32)
    var = (var * inv_last).astype(F32)
    inv_std = (F32(1) / np.sqrt((var + F32(epsilon)).astype(F32))).astype(F32)
    y = (((r - mean[:, None]).astype(F32) * inv_std[:, None]).astype(F32) * scale[None, :]).astype(F32)
    return y.reshape(x.shape)


def concat(a, b, axis: int):
    """ExecuteConcat (:2110): input0 then input1 along `axis`."""
    return np.concatenate([_f32(a), _f32(b)], axis=axis)


def matmul(a, b, addend=None, relu_out: bool = False):
    """ExecuteMatMul / ExecuteGemm / ExecuteMatMulAdd / ExecuteMatMulAddRelu
    (:2165-2378): rank-2 [m, k] x [k, n], sum += a[m, k] * b[k, n] over k in
    order (each product rounded to f32), then + addend, then relu."""
    a, b = _f32(a), _f32(b)
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"MatMul requires rank-2 inputs with matching inner dims; got {a.shape} and {b.shape}")
    acc = np.zeros((a.shape[0], b.shape[1]), F32)
    for k in range(a.shape[1]):
        acc = (acc + (a[:, k, None] * b[None, k, :]).astype(F32)).astype(F32)
    if addend is not None:
        acc = (acc + _f32(addend)).astype(F32)
    return relu(acc) if relu_out else acc


def gemm_relu_gemm(x, w1, b1, w2, b2):
    """ExecuteGemmReluGemm (:2236): relu(x w1 + b1) w2 + b2."""
    return matmul(matmul(x, w1, b1, relu_out=True), w2, b2)


# op kind (the smoke cases' names) -> function of the case's inputs
KINDS = {
    "identity": lambda i: identity(*i),
    "add": lambda i: add(*i),
    "relu": lambda i: relu(*i),
    "sigmoid": lambda i: sigmoid(*i),
    "tanh": lambda i: tanh(*i),
    "gelu": lambda i: gelu(*i),
    "matmul": lambda i: matmul(*i),
    "gemm": lambda i: matmul(i[0], i[1], i[2]),
    "gemm_relu_gemm": lambda i: gemm_relu_gemm(*i),
    "matmul_add": lambda i: matmul(i[0], i[1], i[2]),
    "matmul_add_relu": lambda i: matmul(i[0], i[1], i[2], relu_out=True),
    "add_relu": lambda i: add_relu(*i),
    "softmax": lambda i: softmax(*i),
    "layernorm": lambda i: layernorm(*i),
}
