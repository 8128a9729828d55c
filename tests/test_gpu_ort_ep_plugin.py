"""GPU: the compiled ORT plugin EP (doe_b200/libdoe_ort_ep.so) end to end
through its C ABI, driven by the fake ONNX Runtime host: GetCapability on an
ONNX graph, Compile of the claimed group, Compute with device tensors on a
CUDA stream.

- Every case of the reference EP's session smoke test
  (runtime/bridge/onnxruntime-ep/src/doe_ort_ep_session_smoke.cc:808-950, in
  tests/golden/ort_ep_smoke_cases.json), each as the ONNX node or fused chain
  the reference claims, within the smoke test's absolute 1e-5.
- Seeded shapes against the numpy restatement (oracle/ort_ep.py) at
  1e-5 * max(|ref|, 1), the f32 bar, with fused MatMul->Add->Relu and
  Gemm->Relu->Gemm groups.
- The decoder-block nodes: SimplifiedLayerNormalization (f32 X, bf16 scale)
  within one bf16 ulp of the oracle's RMSNorm, and a bf16 MatMul by a
  constant weight within 2^-7 of the float64 product of the same values.
- The factory's device allocator, data transfer and sync stream: a round
  trip host -> device -> device -> host returns the same bytes.
- Runtime shape errors come back as ORT_INVALID_GRAPH with the reference's
  message, and the EP's debug counters count each Compute.
"""
from __future__ import annotations

import ctypes as C
import json

import numpy as np
import pytest

from doe_b200 import build as dbuild
from oracle import decoder as odec
from oracle import ort_ep as oep
from tests.gpu_util import within
from tests.ort_host import BFLOAT16, FLOAT, GRAPH_INPUT, GRAPH_OUTPUT, INITIALIZER, EpError, FakeOrt

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

EP = dbuild.EP_LIB
TOL = 1e-5
ORT_INVALID_GRAPH = 10


@pytest.fixture(scope="module")
def ort():
    assert EP.exists(), "libdoe_ort_ep.so is not built"
    h = FakeOrt(EP)
    yield h
    h.close()


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()


# One ONNX graph per reference kind: (nodes, input names, output name).  Each
# node: (name, op, inputs, outputs, attrs).
def _graph(ort, kind, in_shapes, out_shape):
    g = ort.graph()
    names = [f"in{i}" for i in range(len(in_shapes))]
    for n, s in zip(names, in_shapes):
        g.value(n, FLOAT, list(s), GRAPH_INPUT)
    mm = [in_shapes[0][0], in_shapes[1][-1]] if len(in_shapes) > 1 and len(in_shapes[0]) == 2 else None
    single = {"identity": "Identity", "relu": "Relu", "sigmoid": "Sigmoid", "tanh": "Tanh", "gelu": "Gelu",
              "softmax": "Softmax", "add": "Add", "matmul": "MatMul", "gemm": "Gemm",
              "layernorm": "LayerNormalization"}
    if kind in single:
        g.value("y", FLOAT, list(out_shape), GRAPH_OUTPUT)
        g.node(kind, single[kind], names, ["y"])
    elif kind == "concat":
        g.value("y", FLOAT, list(out_shape), GRAPH_OUTPUT)
        axis = next(i for i in range(len(in_shapes[0])) if in_shapes[0][i] != in_shapes[1][i]) \
            if in_shapes[0] != in_shapes[1] else 0
        g.node(kind, "Concat", names, ["y"], axis=axis)
    elif kind == "add_relu":
        g.value("s", FLOAT, list(out_shape)), g.value("y", FLOAT, list(out_shape), GRAPH_OUTPUT)
        g.node("add", "Add", names, ["s"]), g.node("relu", "Relu", ["s"], ["y"])
    elif kind in ("matmul_add", "matmul_add_relu"):
        g.value("p", FLOAT, mm)
        last = "y" if kind == "matmul_add" else "s"
        g.value(last, FLOAT, mm, GRAPH_OUTPUT if kind == "matmul_add" else 0)
        g.node("mm", "MatMul", names[:2], ["p"])
        g.node("add", "Add", ["p", names[2]], [last])
        if kind == "matmul_add_relu":
            g.value("y", FLOAT, mm, GRAPH_OUTPUT)
            g.node("relu", "Relu", ["s"], ["y"])
    elif kind == "gemm_relu_gemm":
        hid = [in_shapes[0][0], in_shapes[1][1]]
        g.value("h", FLOAT, hid), g.value("hr", FLOAT, hid), g.value("y", FLOAT, list(out_shape), GRAPH_OUTPUT)
        g.node("g1", "Gemm", names[:3], ["h"]), g.node("r", "Relu", ["h"], ["hr"])
        g.node("g2", "Gemm", ["hr", names[3], names[4]], ["y"])
    else:
        raise ValueError(kind)
    return g


def _run(ort, kind, ins, out_shape, stream=None):
    g = _graph(ort, kind, [x.shape for x in ins], out_shape)
    groups = ort.capability(g)
    assert len(groups) == 1, (kind, groups)
    ci = ort.compile(g, 0, f"doe_{kind}")
    out = torch.full(tuple(out_shape), float("nan"), device="cuda")
    dims = ort.compute(ci, [_t(x) for x in ins], out, stream=stream)
    torch.cuda.synchronize()
    assert dims == tuple(out_shape)
    return out.cpu().numpy()


def test_reference_smoke_cases(ort, golden_dir):
    d = json.loads((golden_dir / "ort_ep_smoke_cases.json").read_text())
    for c in d["cases"]:
        ins = [np.asarray(v, np.float32).reshape(dims) for v, dims in zip(c["inputs"], c["input_dims"])]
        got = _run(ort, c["name"], ins, c["output_dims"])
        exp = np.asarray(c["expected"], np.float32).reshape(c["output_dims"])
        assert np.abs(got - exp).max() <= d["tolerance_abs"], (c["name"], got, exp)


@pytest.mark.parametrize("kind", ["identity", "relu", "sigmoid", "tanh", "gelu", "softmax"])
def test_unary_and_softmax_against_oracle(ort, kind):
    x = (np.random.default_rng(3).standard_normal((257, 1000), dtype=np.float32) * 3).astype(np.float32)
    got = _run(ort, kind, [x], x.shape)
    within(got, oep.KINDS[kind]([x]), TOL)


def test_fused_groups_against_oracle(ort):
    g = np.random.default_rng(4)
    a = g.standard_normal((130, 300), dtype=np.float32)
    b = g.standard_normal((300, 190), dtype=np.float32) / np.float32(np.sqrt(300))
    c = g.standard_normal((130, 190), dtype=np.float32)
    within(_run(ort, "matmul_add_relu", [a, b, c], (130, 190)), oep.matmul(a, b, c, relu_out=True), TOL)
    within(_run(ort, "matmul_add", [a, b, c], (130, 190)), oep.matmul(a, b, c), TOL)
    w1 = g.standard_normal((300, 64), dtype=np.float32) / np.float32(np.sqrt(300))
    b1 = g.standard_normal((130, 64), dtype=np.float32)
    w2 = g.standard_normal((64, 33), dtype=np.float32) / np.float32(8)
    b2 = g.standard_normal((130, 33), dtype=np.float32)
    within(_run(ort, "gemm_relu_gemm", [a, w1, b1, w2, b2], (130, 33)), oep.gemm_relu_gemm(a, w1, b1, w2, b2), TOL)
    x, s = g.standard_normal((64, 4096), dtype=np.float32), g.standard_normal(4096, dtype=np.float32)
    within(_run(ort, "layernorm", [x, s], x.shape), oep.layernorm(x, s), TOL)
    p, q = g.standard_normal((4, 3, 8), dtype=np.float32), g.standard_normal((4, 5, 8), dtype=np.float32)
    assert np.array_equal(_run(ort, "concat", [p, q], (4, 8, 8)), oep.concat(p, q, 1))


def test_compute_on_a_given_stream(ort):
    x = np.random.default_rng(5).standard_normal((1024, 1024), dtype=np.float32)
    s = torch.cuda.Stream()
    got = _run(ort, "gelu", [x], x.shape, stream=s)
    within(got, oep.gelu(x), TOL)


def test_runtime_shape_error_is_invalid_graph(ort):
    g = _graph(ort, "add", [(2, 3), (2, 3)], (2, 3))
    ort.capability(g)
    ci = ort.compile(g, 0)
    out = torch.empty((2, 3), device="cuda")
    with pytest.raises(EpError) as e:
        ort.compute(ci, [_t(np.zeros((2, 3), np.float32)), _t(np.zeros((3, 2), np.float32))], out)
    assert e.value.code == ORT_INVALID_GRAPH
    assert "requires exact-shape float32 tensors; input0 has shape [2, 3] while input1 has shape [3, 2]" in e.value.msg


def test_decoder_rmsnorm_and_bf16_linear(ort):
    g_ = np.random.default_rng(6)
    rows, hid, n = 32, 4096, 1024
    h = g_.standard_normal((rows, hid), dtype=np.float32)
    gamma = torch.from_numpy(g_.standard_normal(hid, dtype=np.float32) * 0.02 + 1).to(torch.bfloat16)
    w = (torch.from_numpy(g_.standard_normal((hid, n), dtype=np.float32)) * 0.02).to(torch.bfloat16)
    g = ort.graph()
    g.value("h", FLOAT, [rows, hid], GRAPH_INPUT)
    g.value("gamma", BFLOAT16, [hid], GRAPH_INPUT)
    g.value("xn", BFLOAT16, [rows, hid])
    g.node("norm", "SimplifiedLayerNormalization", ["h", "gamma"], ["xn"], axis=-1, epsilon=1e-5)
    g.value("w", BFLOAT16, [hid, n], INITIALIZER, w.view(torch.int16).numpy())
    g.value("y", BFLOAT16, [rows, n], GRAPH_OUTPUT)
    g.node("proj", "MatMul", ["xn", "w"], ["y"])
    assert ort.capability(g) == [["norm"], ["proj"]]
    c_norm, c_proj = ort.compile(g, 0, "norm"), ort.compile(g, 1, "proj")
    xn = torch.empty((rows, hid), dtype=torch.bfloat16, device="cuda")
    assert ort.compute(c_norm, [_t(h), gamma.cuda()], xn) == (rows, hid)
    y = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    assert ort.compute(c_proj, [xn], y) == (rows, n)
    torch.cuda.synchronize()
    xn_ref = odec.rmsnorm(h, gamma.float().numpy(), 1e-5)
    assert np.allclose(xn.float().cpu().numpy(), xn_ref, rtol=2.0 ** -7, atol=1e-6)
    ref = odec.matmul(xn.float().cpu().numpy(), w.float().numpy().T)
    err = np.abs(y.float().cpu().numpy() - ref) / np.maximum(np.abs(ref), 1.0)
    assert err.max() <= 2.0 ** -7
    claimed, computed = C.c_uint64(), C.c_uint64()
    C.CDLL(str(EP)).DoeOrtEpGetDecoderCounters(C.byref(claimed), C.byref(computed))
    assert computed.value >= 2


def test_allocator_data_transfer_and_stream_round_trip(ort):
    src = np.random.default_rng(7).integers(0, 256, 3 << 20, dtype=np.uint8)
    dst = np.zeros_like(src)
    rc = ort.lib.fh_device_roundtrip(ort.h, src.ctypes.data, dst.ctypes.data, src.nbytes)
    assert rc == 0, ort.error()
    assert np.array_equal(src, dst)


def test_supported_devices_register_device_memory(ort):
    n, vendor, dev, mem = C.c_int(), C.c_uint32(), C.c_uint32(), C.c_int()
    assert ort.lib.fh_supported_devices(ort.h, C.byref(n), C.byref(vendor), C.byref(dev), C.byref(mem)) == 0
    assert n.value == min(2, torch.cuda.device_count())  # the CPU device is not taken
    assert (vendor.value, dev.value, mem.value) == (0x10DE, 0, 1)  # NVIDIA, ordinal 0, GPU memory
