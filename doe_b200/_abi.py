"""ctypes bindings of libdoe_cuda.so (include/doe_cuda.h).

The library is loaded from this package directory; a missing or unloadable
library raises immediately -- there is no host fallback for any op.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libdoe_cuda.so"

DOE_OK = 0
DOE_UNSUPPORTED = 1
DOE_ERROR = 2
DOE_INVALID_ARGUMENT = 3
DOE_OUT_OF_RANGE = 4
DOE_NOT_FOUND = 5
DOE_CUDA_ERROR = 6
DOE_NO_DEVICE = 7

STATUS_NAMES = {
    DOE_OK: "DOE_OK", DOE_UNSUPPORTED: "DOE_UNSUPPORTED", DOE_ERROR: "DOE_ERROR",
    DOE_INVALID_ARGUMENT: "DOE_INVALID_ARGUMENT", DOE_OUT_OF_RANGE: "DOE_OUT_OF_RANGE",
    DOE_NOT_FOUND: "DOE_NOT_FOUND", DOE_CUDA_ERROR: "DOE_CUDA_ERROR", DOE_NO_DEVICE: "DOE_NO_DEVICE",
}

DOE_DEVICE_ERR_PAGE = 0x1
DOE_DEVICE_ERR_POSITION = 0x2
DOE_DEVICE_ERR_LENGTH = 0x4
DOE_DEVICE_ERR_TIMEOUT = 0x8

DOE_KV_F16 = 0
DOE_KV_INT8 = 1

# set_upload_behavior usage modes
DOE_UPLOAD_COPY_DST_COPY_SRC = 0
DOE_UPLOAD_COPY_DST = 1

# bytes of the scratch array behind doe_attention_decode_f32_noalloc
DOE_NOALLOC_SCRATCH_BYTES = 1 << 18


class DoeError(RuntimeError):
    def __init__(self, fn: str, rc: int, msg: str = ""):
        super().__init__(f"{fn} -> {STATUS_NAMES.get(rc, rc)}: {msg}")
        self.rc = rc


class Launch(C.Structure):
    _fields_ = [("stream", C.c_void_p), ("workspace", C.c_void_p),
                ("workspace_bytes", C.c_uint64), ("status", C.c_void_p)]


class Binding(C.Structure):
    _fields_ = [("binding", C.c_uint32), ("group", C.c_uint32), ("handle", C.c_uint64),
                ("offset", C.c_uint64), ("size", C.c_uint64), ("buffer_type", C.c_uint32),
                ("reserved", C.c_uint32)]


class ExecResult(C.Structure):
    _fields_ = [("status", C.c_int32), ("dispatch_count", C.c_uint32), ("setup_ns", C.c_uint64),
                ("encode_ns", C.c_uint64), ("submit_wait_ns", C.c_uint64),
                ("gpu_timestamp_ns", C.c_uint64), ("gpu_timestamp_attempted", C.c_uint32),
                ("gpu_timestamp_valid", C.c_uint32)]


class AttnUniforms(C.Structure):
    _fields_ = [(n, C.c_float if n in ("scale", "attn_softcap") else C.c_uint32) for n in (
        "num_heads", "num_kv_heads", "head_dim", "seq_len", "query_len", "scale", "is_causal",
        "start_pos", "attn_softcap", "sliding_window", "kv_len_source", "kv_start", "page_size",
        "kv_layout", "pad")]


class PagedKV(C.Structure):
    _fields_ = [("k_pool", C.c_void_p), ("v_pool", C.c_void_p), ("k_scale", C.c_void_p),
                ("v_scale", C.c_void_p), ("kv_dtype", C.c_uint32), ("num_pages", C.c_uint32),
                ("page_size", C.c_uint32), ("num_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("max_pages_per_seq", C.c_uint32), ("block_table", C.c_void_p)]


class DecodeOptions(C.Structure):
    """doe_decode_options: RoPE table, sliding window, softcap of the paged decode."""

    _fields_ = [("freq_cis", C.c_void_p), ("rope_positions", C.c_uint32), ("sliding_window", C.c_uint32),
                ("attn_softcap", C.c_float), ("flags", C.c_uint32)]


DECODE_OUT_BF16 = 0x1
DECODE_COUNTERS_ZEROED = 0x2
DECODE_INPUTS_STABLE = 0x4
LINEAR_STORE, LINEAR_SWIGLU = 0, 1
DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2
EP_IDENTITY, EP_RELU, EP_SIGMOID, EP_TANH, EP_GELU = 0, 1, 2, 3, 4
EP_ADD, EP_ADD_RELU = 0, 1
EP_MATMUL_RELU = 0x1


TP_MAX_RANKS = 8


class TpPeers(C.Structure):
    """doe_tp_peers: this rank, the world size and every rank's peer buffer mapped here."""

    _fields_ = [("rank", C.c_uint32), ("world", C.c_uint32), ("buffers", C.c_void_p * TP_MAX_RANKS)]


class LinearOut(C.Structure):
    """doe_linear_out: output segments, dtype and epilogue of doe_linear_bf16."""

    _fields_ = [("out", C.c_void_p * 3), ("width", C.c_uint32 * 3), ("dtype", C.c_uint32),
                ("epilogue", C.c_uint32), ("residual", C.c_void_p)]


class LinearNorm(C.Structure):
    """doe_linear_norm: the RMSNorm split over two doe_linear_bf16_norm products."""

    _fields_ = [("gamma", C.c_void_p), ("normed_out", C.c_void_p), ("ssq_out", C.c_void_p),
                ("ssq_in", C.c_void_p), ("eps", C.c_float)]


_P = C.c_void_p
_U32 = C.c_uint32
_U64 = C.c_uint64
_I = C.c_int
_F = C.c_float
_LP = C.POINTER(Launch)

# name -> (restype, argtypes); every function declared in include/doe_cuda.h
SIGNATURES = {
    "doe_cuda_abi_version": (_I, []),
    "doe_cuda_device_count": (_I, [C.POINTER(_I)]),
    "doe_cuda_op_last_error": (C.c_char_p, []),
    "doe_cuda_open": (_I, [_I, C.POINTER(_P)]),
    "doe_cuda_close": (_I, [_P]),
    "doe_cuda_last_error": (C.c_char_p, [_P]),
    "doe_cuda_stream": (_P, [_P]),
    "doe_cuda_buffer_ensure": (_I, [_P, _U64, _U64]),
    "doe_cuda_buffer_write": (_I, [_P, _U64, _U64, _P, _U64]),
    "doe_cuda_buffer_write_async": (_I, [_P, _U64, _U64, _P, _U64]),
    "doe_cuda_buffer_read": (_I, [_P, _U64, _U64, _P, _U64]),
    "doe_cuda_buffer_read_async": (_I, [_P, _U64, _U64, _P, _U64]),
    "doe_cuda_buffer_release": (_I, [_P, _U64]),
    "doe_cuda_buffer_size": (_I, [_P, _U64, C.POINTER(_U64)]),
    "doe_cuda_buffer_device_ptr": (_I, [_P, _U64, C.POINTER(_P)]),
    "doe_cuda_dispatch": (_I, [_P, C.c_char_p, C.c_char_p, _U32, _U32, _U32, C.POINTER(Binding),
                               _U32, C.POINTER(ExecResult)]),
    "doe_cuda_kernel_supported": (_I, [C.c_char_p]),
    "doe_cuda_prewarm_kernel": (_I, [_P, C.c_char_p]),
    "doe_cuda_prewarm_upload": (_I, [_P, _U64]),
    "doe_cuda_set_queue_sync_mode": (_I, [_P, _I]),
    "doe_cuda_set_upload_behavior": (_I, [_P, _I, C.c_uint32]),
    "doe_cuda_set_queue_wait_mode": (_I, [_P, _I]),
    "doe_cuda_set_gpu_timestamp_mode": (_I, [_P, _I]),
    "doe_cuda_flush": (_I, [_P, C.POINTER(_U64)]),
    "doe_attention_decode_f32_workspace_bytes": (_U64, [_U32, _U32, _U32]),
    "doe_attention_decode_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _F, _LP]),
    "doe_attention_online": (_I, [C.POINTER(AttnUniforms), _P, _P, _P, _U32, _P, _P, _P, _LP]),
    "doe_attention_prefill_wgsl_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _F, _LP]),
    "doe_attention_stitch_f32": (_I, [_P, _U32, _U32, _U32, _P, _LP]),
    "doe_attention_prefill_f16": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _F, _U32,
                                       C.POINTER(PagedKV), _U32, _U32, _LP]),
    "doe_paged_decode_workspace_bytes": (_U64, [C.POINTER(PagedKV), _U32, _U32, _U32]),
    "doe_paged_decode": (_I, [C.POINTER(PagedKV), _U32, _U32, _P, _P, _P, _P, _F, _P, _U32, _LP]),
    "doe_paged_append": (_I, [C.POINTER(PagedKV), _U32, _U32, _P, _P, _P, _LP]),
    "doe_paged_append_rope": (_I, [C.POINTER(PagedKV), _U32, _U32, _P, _P, _P, _P, _U32, _LP]),
    "doe_paged_decode_rope": (_I, [C.POINTER(PagedKV), _U32, _U32, _P, _P, _P, _P, _F, _P, _U32, _P, _U32,
                                   _LP]),
    "doe_paged_decode_ex": (_I, [C.POINTER(PagedKV), _U32, _U32, _P, _P, _P, _P, _F, _P, _U32,
                                 C.POINTER(DecodeOptions), _LP]),
    "doe_paged_gather": (_I, [C.POINTER(PagedKV), _U32, _U32, _U32, _P, _P, _P, _P, _LP]),
    "doe_kv_write_dense": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _LP]),
    "doe_kv_read_dense": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _U32, _LP]),
    "doe_rope_f32": (_I, [_P, _P, _U32, _U32, _U32, _U32, _LP]),
    "doe_rmsnorm_bf16": (_I, [_P, _P, _F, _P, _U32, _U32, _LP]),
    "doe_ep_unary_f32": (_I, [_U32, _P, _P, _U64, _LP]),
    "doe_ep_binary_f32": (_I, [_U32, _P, _P, _P, _U64, _LP]),
    "doe_ep_softmax_f32": (_I, [_P, _P, _U64, _U32, _LP]),
    "doe_ep_layernorm_f32": (_I, [_P, _P, _F, _P, _U64, _U32, _LP]),
    "doe_ep_concat_f32": (_I, [_P, _P, _P, _U64, _U64, _U64, _U64, _LP]),
    "doe_ep_matmul_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _LP]),
    "doe_rmsnorm_f32": (_I, [_P, _P, _P, _U32, _U32, C.c_float, _U32, _LP]),
    "doe_gemv_f32": (_I, [_P, _P, _P, _U32, _U32, _LP]),
    "doe_gelu_tanh_f32": (_I, [_P, _P, C.c_uint64, _LP]),
    "doe_argmax_f32": (_I, [_P, _U32, _P, _LP]),
    "doe_gather_rows_f32": (_I, [_P, _P, C.c_uint64, _P, _U32, _U32, _LP]),
    "doe_ep_gemm_relu_gemm_workspace_bytes": (_U64, [_U32, _U32]),
    "doe_ep_gemm_relu_gemm_f32": (_I, [_P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _LP]),
    "doe_linear_workspace_bytes": (_U64, [_U32, _U32]),
    "doe_linear_bf16": (_I, [_P, _P, _U32, _U32, _U32, C.POINTER(LinearOut), _LP]),
    "doe_linear_bf16_norm": (_I, [_P, _P, _U32, _U32, _U32, C.POINTER(LinearOut), C.POINTER(LinearNorm), _LP]),
    "doe_tp_buffer_bytes": (_U64, [_U32, _U32]),
    "doe_tp_slot_ptr": (_P, [_P, _U32, _U32, _U32]),
    "doe_peer_buffer_create": (_I, [_U64, C.POINTER(_P), _P]),
    "doe_peer_buffer_open": (_I, [_P, C.POINTER(_P)]),
    "doe_peer_buffer_close": (_I, [_P]),
    "doe_peer_buffer_free": (_I, [_P]),
    "doe_tp_reduce_rmsnorm": (_I, [C.POINTER(TpPeers), _U32, _P, _F, _P, _P, _U32, _U32, _LP]),
    "doe_attention_decode_f32_noalloc": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _F, _P]),
    "doe_kv_pool_create": (_I, [_U32, _U32, _U32, _U32, C.POINTER(_P)]),
    "doe_kv_pool_destroy": (_I, [_P]),
    "doe_kv_pool_reserve": (_I, [_P, _U32, _U32]),
    "doe_kv_pool_release": (_I, [_P, _U32]),
    "doe_kv_pool_free_pages": (_I, [_P, C.POINTER(_U32)]),
    "doe_kv_pool_seq_pages": (_I, [_P, _U32, C.POINTER(_U32)]),
    "doe_kv_pool_block_table": (_I, [_P, _P, _U64]),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load libdoe_cuda.so (raises if it is missing: build it with doe_b200.build)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing; run `python -m doe_b200.build` first")
        _lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def op_error() -> str:
    msg = lib().doe_cuda_op_last_error()
    return msg.decode() if msg else ""


def check(fn: str, rc: int, ctx=None) -> None:
    if rc != DOE_OK:
        if ctx is not None:
            msg = lib().doe_cuda_last_error(ctx)
            msg = msg.decode() if msg else ""
        else:
            msg = op_error()
        raise DoeError(fn, rc, msg)
