"""TEST INFRASTRUCTURE: ctypes front end of the fake ONNX Runtime host
(fake_ort_host.cpp), which drives libdoe_ort_ep.so through its C ABI the way
ORT's session would: GetSupportedDevices, GetCapability on a graph, Compile
of each claimed group, CreateState and Compute with a kernel context.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libfake_ort_host.so"
SRC = HERE / "fake_ort_host.cpp"

# ONNXTensorElementDataType values (onnxruntime_c_api.h)
FLOAT, UINT8, INT8, INT32, INT64, FLOAT16, BFLOAT16 = 1, 2, 3, 6, 7, 10, 16
# value kinds of fh_value
INTERMEDIATE, GRAPH_INPUT, GRAPH_OUTPUT, INITIALIZER = 0, 1, 2, 3


def build(force: bool = False) -> Path | None:
    """Compile libfake_ort_host.so against ONNX Runtime's C API headers (the
    same directory the EP is built with); None when the headers are absent."""
    import sys

    sys.path.insert(0, str(HERE.parents[1]))
    from doe_b200.build import host_cxx, ort_include_dir

    inc = ort_include_dir()
    if inc is None:
        return LIB if LIB.exists() else None
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    subprocess.run([host_cxx(), "-std=c++17", "-O1", "-fPIC", "-shared", "-Wall", "-I", str(inc),
                    str(SRC), "-o", str(LIB), "-ldl"], check=True)
    return LIB


class EpError(RuntimeError):
    def __init__(self, what: str, code: int, msg: str):
        super().__init__(f"{what}: ORT error {code}: {msg}")
        self.code = code
        self.msg = msg


class Graph:
    """An ONNX graph built value by value and node by node."""

    def __init__(self, host: "FakeOrt"):
        self.h = host
        self.g = host.lib.fh_graph_new()
        self.values: dict[str, int] = {}
        self.nodes: dict[str, int] = {}

    def value(self, name: str, elem: int, shape, kind: int = INTERMEDIATE, data: np.ndarray | None = None):
        dims = (C.c_int64 * max(1, len(shape or ())))(*(shape or ()))
        rank = -1 if shape is None else len(shape)
        idx = self.h.lib.fh_value(self.g, name.encode(), elem, rank, dims, kind)
        if data is not None:
            buf = np.ascontiguousarray(data)
            self.h.lib.fh_set_initializer(self.g, idx, buf.ctypes.data, buf.nbytes)
        self.values[name] = idx
        return idx

    def node(self, name: str, op: str, ins, outs, domain: str = "", **attrs):
        a = (C.c_int * max(1, len(ins)))(*[self.values[i] for i in ins])
        b = (C.c_int * max(1, len(outs)))(*[self.values[o] for o in outs])
        idx = self.h.lib.fh_node(self.g, name.encode(), op.encode(), domain.encode(), len(ins), a, len(outs), b)
        for k, v in attrs.items():
            if isinstance(v, float):
                self.h.lib.fh_attr_float(self.g, idx, k.encode(), v)
            else:
                self.h.lib.fh_attr_int(self.g, idx, k.encode(), int(v))
        self.nodes[name] = idx
        return idx

    def __del__(self):
        try:
            self.h.lib.fh_graph_free(self.g)
        except Exception:
            pass


class FakeOrt:
    """One EP (CUDA ordinal 0) of libdoe_ort_ep.so inside the fake host."""

    def __init__(self, ep_path: Path, name: str = "DoeExecutionProvider"):
        lib_path = build()
        if lib_path is None:
            raise RuntimeError("libfake_ort_host.so is missing and ONNX Runtime headers are unavailable")
        self.lib = C.CDLL(str(lib_path))
        L = self.lib
        P, I, I64, U32, SZ = C.c_void_p, C.c_int, C.c_int64, C.c_uint32, C.c_size_t
        for fn, res, args in (
                ("fh_last_error", C.c_char_p, []), ("fh_graph_new", P, []), ("fh_graph_free", None, [P]),
                ("fh_value", I, [P, C.c_char_p, I, I, C.POINTER(I64), I]),
                ("fh_set_initializer", I, [P, I, P, SZ]),
                ("fh_node", I, [P, C.c_char_p, C.c_char_p, C.c_char_p, I, C.POINTER(I), I, C.POINTER(I)]),
                ("fh_attr_int", I, [P, I, C.c_char_p, I64]), ("fh_attr_float", I, [P, I, C.c_char_p, C.c_float]),
                ("fh_load", P, [C.c_char_p, C.c_char_p]), ("fh_unload", None, [P]),
                ("fh_ep_name", C.c_char_p, [P]), ("fh_factory_name", C.c_char_p, [P]),
                ("fh_supported_devices", I, [P, C.POINTER(I), C.POINTER(U32), C.POINTER(U32), C.POINTER(I)]),
                ("fh_get_capability", I, [P, P]), ("fh_group", I, [P, P, I, C.POINTER(I), I]),
                ("fh_compile", I, [P, P, I, C.c_char_p]),
                ("fh_compute", I, [P, I, I, C.POINTER(P), C.POINTER(I), C.POINTER(I), C.POINTER(I64), P, I, SZ,
                                   C.POINTER(I), C.POINTER(I64), P]),
                ("fh_device_roundtrip", I, [P, P, P, SZ]), ("fh_install_crash_handler", None, [])):
            f = getattr(L, fn)
            f.restype = res
            f.argtypes = args
        if os.environ.get("DOE_FAKE_ORT_BACKTRACE"):
            L.fh_install_crash_handler()  # native frames of a crash on stderr
        self.h = L.fh_load(str(ep_path).encode(), name.encode())
        if not self.h:
            raise RuntimeError(f"loading the EP failed: {self.error()}")

    def error(self) -> str:
        return (self.lib.fh_last_error() or b"").decode()

    def close(self):
        if self.h:
            self.lib.fh_unload(self.h)
            self.h = None

    def graph(self) -> Graph:
        return Graph(self)

    def capability(self, g: Graph) -> list[list[str]]:
        """Groups claimed by GetCapability, as lists of node names."""
        n = self.lib.fh_get_capability(self.h, g.g)
        if n < 0:
            raise EpError("GetCapability", -1, self.error())
        names = {v: k for k, v in g.nodes.items()}
        out = []
        for i in range(n):
            buf = (C.c_int * 8)()
            k = self.lib.fh_group(self.h, g.g, i, buf, 8)
            out.append([names[buf[j]] for j in range(k)])
        return out

    def compile(self, g: Graph, group: int, name: str = "fused") -> int:
        ci = self.lib.fh_compile(self.h, g.g, group, name.encode())
        if ci < 0:
            raise EpError("Compile", -1, self.error())
        return ci

    def compute(self, ci: int, inputs, out, stream=None) -> tuple:
        """Compute with torch CUDA inputs into the torch CUDA tensor `out`
        (its numel is the capacity); returns the output dims the EP set."""
        import torch

        types = {torch.float32: FLOAT, torch.bfloat16: BFLOAT16, torch.float16: FLOAT16, torch.int32: INT32}
        n = len(inputs)
        data = (C.c_void_p * max(1, n))(*[t.data_ptr() for t in inputs])
        tys = (C.c_int * max(1, n))(*[types[t.dtype] for t in inputs])
        ranks = (C.c_int * max(1, n))(*[t.dim() for t in inputs])
        flat = [d for t in inputs for d in t.shape]
        dims = (C.c_int64 * max(1, len(flat)))(*flat)
        orank = C.c_int()
        odims = (C.c_int64 * 8)()
        s = None if stream is None else stream.cuda_stream
        rc = self.lib.fh_compute(self.h, ci, n, data, tys, ranks, dims, out.data_ptr(), types[out.dtype],
                                 out.numel() * out.element_size(), C.byref(orank), odims, s)
        if rc != 0:
            raise EpError("Compute", rc, self.error())
        return tuple(odims[i] for i in range(orank.value))
