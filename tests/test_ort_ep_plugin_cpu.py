"""The compiled ORT plugin EP (doe_b200/libdoe_ort_ep.so) on the CPU: its
exports, factory and EP names, the nodes GetCapability claims and the groups
it fuses, the debug counters, and Compile -- all host logic, driven through
the EP's C ABI by the fake ONNX Runtime host (tests/ort_host).

The claim rules follow the reference EP (runtime/bridge/onnxruntime-ep/src/
doe_ort_ep.cc:762-1002 GetSupportedNodeSpec, :1004-1395 the fusions,
:2615-2717 GetCapability): float32 tensors with static shapes; MatMul -> Add
(-> Relu), Add -> Relu and Gemm -> Relu -> Gemm fused when each link's output
has exactly one consumer and is not a graph output; Gemm only with alpha =
beta = 1 and no transposes.  Added here: SimplifiedLayerNormalization (f32 X,
bf16 scale / Y) and a bf16 MatMul by a constant initializer.
"""
from __future__ import annotations

import ctypes as C
import subprocess

import numpy as np
import pytest

from doe_b200 import build as dbuild

ort_host = pytest.importorskip("tests.ort_host")
from tests.ort_host import BFLOAT16, FLOAT, FLOAT16, GRAPH_INPUT, GRAPH_OUTPUT, INITIALIZER  # noqa: E402

EP = dbuild.EP_LIB
COUNTER_FIELDS = (
    "get_capability_calls claimed_nodes claimed_identity_nodes claimed_add_nodes claimed_relu_nodes "
    "claimed_sigmoid_nodes claimed_tanh_nodes claimed_gelu_nodes claimed_matmul_nodes claimed_gemm_nodes "
    "claimed_softmax_nodes claimed_layernorm_nodes claimed_concat_nodes compile_calls compiled_identity_groups "
    "compiled_add_groups compiled_relu_groups compiled_sigmoid_groups compiled_tanh_groups compiled_gelu_groups "
    "compiled_matmul_groups compiled_gemm_groups compiled_gemm_relu_gemm_groups compiled_matmul_add_groups "
    "compiled_matmul_add_relu_groups compiled_add_relu_groups compiled_softmax_groups compiled_layernorm_groups "
    "compiled_concat_groups create_state_calls compute_calls compute_identity_calls compute_add_calls "
    "compute_relu_calls compute_sigmoid_calls compute_tanh_calls compute_gelu_calls compute_matmul_calls "
    "compute_gemm_calls compute_gemm_relu_gemm_calls compute_matmul_add_calls compute_matmul_add_relu_calls "
    "compute_add_relu_calls compute_softmax_calls compute_layernorm_calls compute_concat_calls "
    "release_state_calls").split()


class Counters(C.Structure):
    """DoeOrtEpDebugCounters (runtime/bridge/onnxruntime-ep/src/doe_ort_ep.h:10-59)."""

    _fields_ = [(f, C.c_uint64) for f in COUNTER_FIELDS]


def counters() -> dict:
    lib = C.CDLL(str(EP))
    c = Counters()
    lib.DoeOrtEpGetDebugCounters(C.byref(c))
    return {f: getattr(c, f) for f in COUNTER_FIELDS}


@pytest.fixture()
def ort():
    if not EP.exists():
        dbuild.build()
        if dbuild.build_ort_ep() is None:
            pytest.skip("ONNX Runtime headers unavailable: libdoe_ort_ep.so not built")
    C.CDLL(str(EP)).DoeOrtEpResetDebugCounters()
    h = ort_host.FakeOrt(EP)
    yield h
    h.close()


def test_exports():
    out = subprocess.run(["nm", "-D", "--defined-only", str(EP)], capture_output=True, text=True,
                         check=True).stdout
    for sym in ("CreateEpFactories", "ReleaseEpFactory", "DoeOrtEpResetDebugCounters", "DoeOrtEpGetDebugCounters"):
        assert f" T {sym}" in out, sym


def test_names(ort):
    assert ort.lib.fh_ep_name(ort.h) == b"DoeExecutionProvider"
    assert ort.lib.fh_factory_name(ort.h) == b"DoeExecutionProvider"


def f32(g, name, shape, kind=0):
    return g.value(name, FLOAT, shape, kind)


def test_single_ops_claimed(ort):
    g = ort.graph()
    f32(g, "x", [4, 8], GRAPH_INPUT)
    prev = "x"
    for i, op in enumerate(("Identity", "Relu", "Sigmoid", "Tanh", "Gelu", "Softmax")):
        f32(g, f"y{i}", [4, 8], GRAPH_OUTPUT if i == 5 else 0)
        g.node(op, op, [prev], [f"y{i}"])
        prev = f"y{i}"
    groups = ort.capability(g)
    assert groups == [["Identity"], ["Relu"], ["Sigmoid"], ["Tanh"], ["Gelu"], ["Softmax"]]
    c = counters()
    assert c["get_capability_calls"] == 1 and c["claimed_nodes"] == 6
    assert c["claimed_relu_nodes"] == 1 and c["claimed_softmax_nodes"] == 1


def test_matmul_add_relu_fused_and_compiled(ort):
    g = ort.graph()
    f32(g, "a", [3, 5], GRAPH_INPUT), f32(g, "b", [5, 7], GRAPH_INPUT), f32(g, "c", [3, 7], GRAPH_INPUT)
    f32(g, "mm", [3, 7]), f32(g, "sum", [3, 7]), f32(g, "y", [3, 7], GRAPH_OUTPUT)
    g.node("mm", "MatMul", ["a", "b"], ["mm"])
    g.node("add", "Add", ["c", "mm"], ["sum"])  # the product as Add's second input
    g.node("relu", "Relu", ["sum"], ["y"])
    assert ort.capability(g) == [["mm", "add", "relu"]]
    ort.compile(g, 0, "fused_mm")
    c = counters()
    assert (c["claimed_matmul_nodes"], c["claimed_add_nodes"], c["claimed_relu_nodes"]) == (1, 1, 1)
    assert c["compiled_matmul_add_relu_groups"] == 1 and c["compile_calls"] == 1 and c["create_state_calls"] == 1


def test_gemm_relu_gemm_and_add_relu(ort):
    g = ort.graph()
    f32(g, "x", [2, 4], GRAPH_INPUT), f32(g, "w1", [4, 6], GRAPH_INPUT), f32(g, "b1", [2, 6], GRAPH_INPUT)
    f32(g, "w2", [6, 3], GRAPH_INPUT), f32(g, "b2", [2, 3], GRAPH_INPUT)
    f32(g, "h", [2, 6]), f32(g, "hr", [2, 6]), f32(g, "o", [2, 3])
    f32(g, "p", [2, 3], GRAPH_INPUT), f32(g, "s", [2, 3]), f32(g, "y", [2, 3], GRAPH_OUTPUT)
    g.node("g1", "Gemm", ["x", "w1", "b1"], ["h"])
    g.node("r1", "Relu", ["h"], ["hr"])
    g.node("g2", "Gemm", ["hr", "w2", "b2"], ["o"])
    g.node("add", "Add", ["o", "p"], ["s"])
    g.node("r2", "Relu", ["s"], ["y"])
    assert ort.capability(g) == [["g1", "r1", "g2"], ["add", "r2"]]
    ort.compile(g, 0), ort.compile(g, 1)
    c = counters()
    assert c["claimed_gemm_nodes"] == 2 and c["claimed_relu_nodes"] == 2 and c["claimed_add_nodes"] == 1
    assert c["compiled_gemm_relu_gemm_groups"] == 1 and c["compiled_add_relu_groups"] == 1


def test_no_fusion_across_shared_or_graph_outputs(ort):
    g = ort.graph()
    f32(g, "a", [2, 2], GRAPH_INPUT), f32(g, "b", [2, 2], GRAPH_INPUT)
    f32(g, "mm", [2, 2]), f32(g, "s1", [2, 2], GRAPH_OUTPUT), f32(g, "s2", [2, 2], GRAPH_OUTPUT)
    g.node("mm", "MatMul", ["a", "b"], ["mm"])
    g.node("add1", "Add", ["mm", "a"], ["s1"])
    g.node("add2", "Add", ["mm", "b"], ["s2"])  # two consumers: no MatMul->Add fusion
    assert ort.capability(g) == [["mm"], ["add1"], ["add2"]]
    g2 = ort.graph()
    f32(g2, "x", [2, 2], GRAPH_INPUT), f32(g2, "y", [2, 2], GRAPH_INPUT), f32(g2, "s", [2, 2], GRAPH_OUTPUT)
    f32(g2, "r", [2, 2], GRAPH_OUTPUT)
    g2.node("add", "Add", ["x", "y"], ["s"])
    g2.node("relu", "Relu", ["s"], ["r"])  # s is a graph output: Add and Relu stay apart
    assert ort.capability(g2) == [["add"], ["relu"]]


def test_unsupported_nodes_stay_with_ort(ort):
    g = ort.graph()
    g.value("h", FLOAT16, [4], GRAPH_INPUT), g.value("h2", FLOAT16, [4], GRAPH_OUTPUT)
    g.node("add16", "Add", ["h", "h"], ["h2"])                        # float16
    f32(g, "a", [2, 3], GRAPH_INPUT), f32(g, "b", [2, 3], GRAPH_INPUT), f32(g, "c", [2, 2], GRAPH_INPUT)
    f32(g, "gy", [2, 2], GRAPH_OUTPUT)
    g.node("gemm_t", "Gemm", ["a", "b", "c"], ["gy"], transB=1)       # a transpose
    f32(g, "d", [-1, 3], GRAPH_INPUT), f32(g, "dy", [-1, 3], GRAPH_OUTPUT)
    g.node("relu_dyn", "Relu", ["d"], ["dy"])                          # a dynamic shape
    f32(g, "e", [3], GRAPH_INPUT), f32(g, "ey", [3], GRAPH_OUTPUT)
    g.node("conv", "Conv", ["e"], ["ey"])                              # an op it does not run
    g.node("relu_ms", "Relu", ["e"], ["ey"], domain="com.example")     # another domain
    assert ort.capability(g) == []


def test_matmul_output_shape_inferred_when_untyped(ort):
    g = ort.graph()
    f32(g, "a", [3, 4], GRAPH_INPUT), f32(g, "b", [4, 5], GRAPH_INPUT)
    g.value("y", 0, None, GRAPH_OUTPUT)
    g.node("mm", "MatMul", ["a", "b"], ["y"])
    assert ort.capability(g) == [["mm"]]


def test_concat_axis_and_layernorm_rules(ort):
    g = ort.graph()
    f32(g, "a", [2, 3, 4], GRAPH_INPUT), f32(g, "b", [2, 5, 4], GRAPH_INPUT), f32(g, "y", [2, 8, 4], GRAPH_OUTPUT)
    g.node("cat", "Concat", ["a", "b"], ["y"], axis=-2)
    f32(g, "x", [6, 16], GRAPH_INPUT), f32(g, "s", [16], GRAPH_INPUT), f32(g, "ln", [6, 16], GRAPH_OUTPUT)
    g.node("ln", "LayerNormalization", ["x", "s"], ["ln"])
    f32(g, "s_bad", [8], GRAPH_INPUT), f32(g, "ln2", [6, 16], GRAPH_OUTPUT)
    g.node("ln_bad", "LayerNormalization", ["x", "s_bad"], ["ln2"])  # scale length != last dim
    assert ort.capability(g) == [["cat"], ["ln"]]


def test_decoder_nodes_claimed(ort):
    g = ort.graph()
    f32(g, "h", [32, 4096], GRAPH_INPUT)
    g.value("gamma", BFLOAT16, [4096], INITIALIZER, np.ones(4096, np.uint16))
    g.value("xn", BFLOAT16, [32, 4096])
    g.node("norm", "SimplifiedLayerNormalization", ["h", "gamma"], ["xn"], axis=-1, epsilon=1e-5)
    g.value("w", BFLOAT16, [4096, 256], INITIALIZER, np.zeros((4096, 256), np.uint16))
    g.value("y", BFLOAT16, [32, 256], GRAPH_OUTPUT)
    g.node("proj", "MatMul", ["xn", "w"], ["y"])
    g.value("w_in", BFLOAT16, [4096, 256], GRAPH_INPUT)  # not a constant: left to ORT
    g.value("y2", BFLOAT16, [32, 256], GRAPH_OUTPUT)
    g.node("proj_dyn", "MatMul", ["xn", "w_in"], ["y2"])
    assert ort.capability(g) == [["norm"], ["proj"]]
    claimed, computed = C.c_uint64(), C.c_uint64()
    C.CDLL(str(EP)).DoeOrtEpGetDecoderCounters(C.byref(claimed), C.byref(computed))
    assert claimed.value == 2 and computed.value == 0


def test_claims_follow_graph_order(ort):
    # nodes are visited in graph order: an Add listed before the MatMul that
    # feeds it is claimed on its own, and the MatMul's one consumer is then
    # taken, so the two are not fused (doe_ort_ep.cc:2636-2713)
    g = ort.graph()
    f32(g, "c", [3, 7], GRAPH_INPUT), f32(g, "a", [3, 5], GRAPH_INPUT), f32(g, "b", [5, 7], GRAPH_INPUT)
    f32(g, "mm", [3, 7]), f32(g, "y", [3, 7], GRAPH_OUTPUT)
    g.node("add", "Add", ["c", "mm"], ["y"])
    g.node("mm", "MatMul", ["a", "b"], ["mm"])
    assert ort.capability(g) == [["add"], ["mm"]]
