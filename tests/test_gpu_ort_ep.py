"""GPU parity of the ORT plugin EP's basic operators (doe_ep_*_f32).

- Every case of the reference EP's session smoke test, through the GPU,
  within its absolute tolerance 1e-5 (tests/golden/ort_ep_smoke_cases.json).
- Seeded random shapes against the numpy restatement (oracle/ort_ep.py):
  |y - ref| <= 1e-5 * max(|ref|, 1), the f32 bar.  Relu, Identity, Add,
  AddRelu and Concat are exact.
- Edge cases: empty tensors, lengths that are not a multiple of 4 and
  misaligned views, rows longer than the shared-memory cache, in-place
  element-wise and row ops, rows of -inf, matmul sizes off the 128 tile.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from doe_b200 import _abi as abi
from doe_b200 import ort_ep
from oracle import ort_ep as oep
from tests.gpu_util import within

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-5


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def _n(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_reference_smoke_cases(golden_dir):
    d = json.loads((golden_dir / "ort_ep_smoke_cases.json").read_text())
    for c in d["cases"]:
        ins = [_t(np.asarray(v, np.float32).reshape(dims)) for v, dims in zip(c["inputs"], c["input_dims"])]
        got = _n(ort_ep.execute(c["name"], *ins))
        exp = np.asarray(c["expected"], np.float32).reshape(c["output_dims"])
        assert np.abs(got - exp).max() <= d["tolerance_abs"], (c["name"], got, exp)


@pytest.mark.parametrize("kind", ["identity", "relu", "sigmoid", "tanh", "gelu"])
@pytest.mark.parametrize("n", [1, 7, 4096, 1000003])
def test_unary_matches_oracle(kind, n):
    g = np.random.default_rng(n)
    x = (g.standard_normal(n, dtype=np.float32) * 4).astype(np.float32)
    x[:: 97] = 0.0
    got = _n(ort_ep.execute(kind, _t(x)))
    ref = oep.KINDS[kind]([x])
    if kind in ("identity", "relu"):
        assert np.array_equal(got, ref)
    else:
        within(got, ref, TOL)


@pytest.mark.parametrize("kind", ["add", "add_relu"])
@pytest.mark.parametrize("shape", [(3, 5), (1024, 1027), (2, 3, 4)])
def test_binary_exact(kind, shape):
    g = np.random.default_rng(sum(shape))
    a, b = g.standard_normal(shape, dtype=np.float32), g.standard_normal(shape, dtype=np.float32)
    got = _n(ort_ep.execute(kind, _t(a), _t(b)))
    assert np.array_equal(got, oep.KINDS[kind]([a, b]))


def test_unaligned_views_and_in_place():
    lib = abi.lib()
    g = np.random.default_rng(5)
    x = _t(g.standard_normal(1001, dtype=np.float32))
    ref = oep.gelu(_n(x)[1:])
    y = torch.empty(1001, device="cuda")
    l = abi.Launch(torch.cuda.current_stream().cuda_stream, None, 0, None)
    import ctypes as C
    # x + 1 element: 4-byte aligned only, so the scalar path runs
    abi.check("unary", lib.doe_ep_unary_f32(abi.EP_GELU, x.data_ptr() + 4, y.data_ptr() + 4, 1000, C.byref(l)))
    within(_n(y)[1:], ref, TOL)
    # in place
    z = x.clone()
    abi.check("unary", lib.doe_ep_unary_f32(abi.EP_TANH, z.data_ptr(), z.data_ptr(), 1001, C.byref(l)))
    within(_n(z), oep.tanh(_n(x)), TOL)
    # a partial overlap is refused
    rc = lib.doe_ep_unary_f32(abi.EP_RELU, x.data_ptr(), x.data_ptr() + 4, 1000, C.byref(l))
    assert rc == 3 and b"overlap" in lib.doe_cuda_op_last_error()


@pytest.mark.parametrize("shape", [(1, 4), (7, 33), (256, 4096), (3, 20000), (5, 1)])
def test_softmax_matches_oracle(shape):
    g = np.random.default_rng(shape[1])
    x = (g.standard_normal(shape, dtype=np.float32) * 3).astype(np.float32)
    got = _n(ort_ep.execute("softmax", _t(x)))
    within(got, oep.softmax(x), TOL)
    assert np.allclose(got.sum(axis=-1), 1.0, atol=1e-5)


def test_softmax_edges_and_in_place():
    x = np.array([[-np.inf, 0.0, -np.inf], [1.0, 1.0, 1.0]], np.float32)
    got = _n(ort_ep.execute("softmax", _t(x)))
    assert got.tolist() == oep.softmax(x).tolist()
    assert ort_ep.execute("softmax", _t(np.zeros((3, 0), np.float32))).shape == (3, 0)
    import ctypes as C
    g = np.random.default_rng(9)
    xs = g.standard_normal((64, 300), dtype=np.float32)
    t = _t(xs)
    l = abi.Launch(torch.cuda.current_stream().cuda_stream, None, 0, None)
    abi.check("softmax", abi.lib().doe_ep_softmax_f32(t.data_ptr(), t.data_ptr(), 64, 300, C.byref(l)))
    within(_n(t), oep.softmax(xs), TOL)


@pytest.mark.parametrize("shape", [(1, 4), (9, 100), (128, 4096), (2, 17000)])
def test_layernorm_matches_oracle(shape):
    g = np.random.default_rng(shape[0] + shape[1])
    x = (g.standard_normal(shape, dtype=np.float32) * 2 + 0.5).astype(np.float32)
    scale = g.standard_normal(shape[1], dtype=np.float32)
    got = _n(ort_ep.execute("layernorm", _t(x), _t(scale)))
    within(got, oep.layernorm(x, scale), TOL)


def test_layernorm_constant_rows_and_epsilon():
    x = np.full((3, 8), 2.5, np.float32)
    got = _n(ort_ep.execute("layernorm", _t(x), _t(np.ones(8, np.float32))))
    assert np.all(got == 0.0)
    g = np.random.default_rng(3)
    x = g.standard_normal((4, 64), dtype=np.float32) * 1e-3
    s = np.ones(64, np.float32)
    within(_n(ort_ep.execute("layernorm", _t(x), _t(s), epsilon=1e-2)), oep.layernorm(x, s, 1e-2), TOL)


@pytest.mark.parametrize("shapes,axis", [(((2, 3), (2, 5)), 1), (((4, 3, 2), (1, 3, 2)), 0),
                                         (((2, 3, 7), (2, 3, 1)), -1), (((5,), (0,)), 0)])
def test_concat_exact(shapes, axis):
    g = np.random.default_rng(len(shapes[0]))
    a = g.standard_normal(shapes[0], dtype=np.float32)
    b = g.standard_normal(shapes[1], dtype=np.float32)
    got = _n(ort_ep.execute("concat", _t(a), _t(b), axis=axis))
    assert np.array_equal(got, oep.concat(a, b, axis))


@pytest.mark.parametrize("m,k,n", [(2, 3, 2), (1, 1, 1), (129, 65, 131), (256, 512, 384), (7, 1000, 3),
                                   (130, 68, 260), (1, 4, 4)])
def test_matmul_family_matches_oracle(m, k, n):
    g = np.random.default_rng(m * 7 + k * 3 + n)
    a = g.standard_normal((m, k), dtype=np.float32)
    b = (g.standard_normal((k, n), dtype=np.float32) / np.sqrt(k)).astype(np.float32)
    c = g.standard_normal((m, n), dtype=np.float32)
    within(_n(ort_ep.execute("matmul", _t(a), _t(b))), oep.matmul(a, b), TOL)
    within(_n(ort_ep.execute("gemm", _t(a), _t(b), _t(c))), oep.matmul(a, b, c), TOL)
    within(_n(ort_ep.execute("matmul_add", _t(a), _t(b), _t(c))), oep.matmul(a, b, c), TOL)
    within(_n(ort_ep.execute("matmul_add_relu", _t(a), _t(b), _t(c))), oep.matmul(a, b, c, relu_out=True), TOL)


def test_matmul_empty_inner_dimension_gives_addend():
    c = np.arange(6, dtype=np.float32).reshape(2, 3) - 2
    got = _n(ort_ep.execute("matmul_add_relu", _t(np.zeros((2, 0))), _t(np.zeros((0, 3))), _t(c)))
    assert np.array_equal(got, np.maximum(c, 0))


@pytest.mark.parametrize("b,i,h,o", [(1, 2, 3, 2), (33, 100, 257, 10), (32, 64, 256, 16)])
def test_gemm_relu_gemm_matches_oracle(b, i, h, o):
    g = np.random.default_rng(b + i + h + o)
    x = g.standard_normal((b, i), dtype=np.float32)
    w1 = (g.standard_normal((i, h), dtype=np.float32) / np.sqrt(i)).astype(np.float32)
    b1 = g.standard_normal((b, h), dtype=np.float32) * 0.1
    w2 = (g.standard_normal((h, o), dtype=np.float32) / np.sqrt(h)).astype(np.float32)
    b2 = g.standard_normal((b, o), dtype=np.float32) * 0.1
    got = _n(ort_ep.execute("gemm_relu_gemm", *map(_t, (x, w1, b1, w2, b2))))
    within(got, oep.gemm_relu_gemm(x, w1, b1, w2, b2), TOL)


def test_gemm_relu_gemm_needs_workspace():
    import ctypes as C
    lib = abi.lib()
    z = torch.zeros((4, 4), device="cuda")
    l = abi.Launch(torch.cuda.current_stream().cuda_stream, None, 0, None)
    rc = lib.doe_ep_gemm_relu_gemm_f32(*(z.data_ptr(),) * 6, 2, 2, 2, 2, C.byref(l))
    assert rc == 3 and b"workspace" in lib.doe_cuda_op_last_error()
    assert lib.doe_ep_gemm_relu_gemm_workspace_bytes(3, 5) == 256
