"""numpy front end for the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY.  This package is the parity checker for the
sm_100a kernels and the timed CPU baseline.  It may be imported by tests/,
``__graft_entry__.smoke()`` and bench.py's CPU legs, never by the shipped
package ``doe_b200``.  Each wrapper names the reference source it restates;
the C file carries the file:line citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

OK = 0
EINVAL = -1
ERANGE = -2
EZERO = -3


class OracleError(RuntimeError):
    def __init__(self, fn: str, rc: int):
        super().__init__(f"{fn} rejected its input (rc={rc})")
        self.rc = rc


def build() -> Path:
    """Compile liboracle.so with the Makefile beside this file."""
    env = dict(os.environ)
    env.pop("CC", None)
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True, env=env)
    return _LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(_LIB_PATH))
        _declare(_lib)
    return _lib


_P = C.c_void_p
_U32 = C.c_uint32
_U64 = C.c_uint64
_F = C.c_float
_D = C.c_double
_I = C.c_int


class AttnUniforms(C.Structure):
    """The reference kernel's uniform block (attention_head256_f16kv.wgsl:14-30)."""

    _fields_ = [
        ("num_heads", _U32), ("num_kv_heads", _U32), ("head_dim", _U32),
        ("seq_len", _U32), ("query_len", _U32), ("scale", _F),
        ("is_causal", _U32), ("start_pos", _U32), ("attn_softcap", _F),
        ("sliding_window", _U32), ("kv_len_source", _U32), ("kv_start", _U32),
        ("page_size", _U32), ("kv_layout", _U32),
    ]


def _declare(l: C.CDLL) -> None:
    sig = {
        "doe_oracle_h2f_array": (None, [_P, _P, _U64]),
        "doe_oracle_f2h_array": (None, [_P, _P, _U64]),
        "doe_oracle_attention_decode_wgsl_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _F]),
        "doe_oracle_attention_decode_wgsl_f64": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _D]),
        "doe_oracle_attention_prefill_wgsl_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _F]),
        "doe_oracle_attention_two_pass_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _F, _U32, _U32]),
        "doe_oracle_emit_local_partials_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _F]),
        "doe_oracle_stitch_partials_f32": (_I, [_P, _U32, _U32, _P]),
        "doe_oracle_attention_online_f16kv": (_I, [C.POINTER(AttnUniforms), _P, _P, _P, _P, _P, _P, _I]),
        "doe_oracle_paged_decode": (_I, [_U32, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P,
                                         _U32, _P, _P, _F, _P, _I]),
        "doe_oracle_paged_decode_ex": (_I, [_U32, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P,
                                            _U32, _P, _P, _F, _U32, _F, _P, _I]),
        "doe_oracle_kv_write_dense": (_I, [_P, _P, _P, _P, _U32, _U32, _U32]),
        "doe_oracle_kv_read_dense": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32]),
        "doe_oracle_paged_append": (_I, [_U32, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P,
                                         _P, _P, _U32, _P, _P, _I]),
        "doe_oracle_paged_gather": (_I, [_U32, _U32, _U32, _U32, _P, _U32, _U32, _U32, _P, _P]),
        "doe_oracle_quantize_rows_int8": (None, [_P, _U64, _U32, _P, _P]),
        "doe_oracle_rope_f32": (_I, [_P, _P, _U32, _U32, _U32, _U32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(l, name)
        fn.restype = res
        fn.argtypes = args


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _check(fn: str, rc: int) -> None:
    if rc != OK:
        raise OracleError(fn, rc)


# ---- binary16 -------------------------------------------------------------
def h2f(bits: np.ndarray) -> np.ndarray:
    src = _c(bits, np.uint16)
    out = np.empty(src.shape, np.float32)
    lib().doe_oracle_h2f_array(_ptr(src), _ptr(out), src.size)
    return out


def f2h(x: np.ndarray) -> np.ndarray:
    src = _c(x, np.float32)
    out = np.empty(src.shape, np.uint16)
    lib().doe_oracle_f2h_array(_ptr(src), _ptr(out), src.size)
    return out


# ---- attention-decode.wgsl / attention-prefill.wgsl ------------------------
def attention_decode_wgsl(q, k, v, scale, *, f64: bool = False) -> np.ndarray:
    """q [H,D], k/v [H,L,D] -> out [H,D] (attention-decode.wgsl:46-136)."""
    dt = np.float64 if f64 else np.float32
    q, k, v = _c(q, dt), _c(k, dt), _c(v, dt)
    H, D = q.shape
    L = k.shape[1]
    if k.shape != (H, L, D) or v.shape != (H, L, D):
        raise ValueError("k/v must be [H, L, D] matching q [H, D]")
    out = np.zeros((H, D), dt)
    fn = "doe_oracle_attention_decode_wgsl_" + ("f64" if f64 else "f32")
    _check(fn, getattr(lib(), fn)(_ptr(q), _ptr(k), _ptr(v), _ptr(out), H, D, L, float(scale)))
    return out


def attention_prefill_wgsl(q, k, v, scale) -> np.ndarray:
    """Causal [H,S,D] f32 (attention-prefill.wgsl:19-112)."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    H, S, D = q.shape
    out = np.zeros_like(q)
    _check("prefill_wgsl", lib().doe_oracle_attention_prefill_wgsl_f32(
        _ptr(q), _ptr(k), _ptr(v), _ptr(out), S, D, H, float(scale)))
    return out


def attention_two_pass(q, k, v, scale, causal_mode: int = 0, window: int = 0) -> np.ndarray:
    """Single-Q two-pass f32 (reference_interpreter.zig:1095-1289)."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    D = q.shape[0]
    L = k.shape[0]
    out = np.zeros(D, np.float32)
    _check("two_pass", lib().doe_oracle_attention_two_pass_f32(
        _ptr(q), _ptr(k), _ptr(v), _ptr(out), D, L, float(scale), causal_mode, window))
    return out


def emit_local_partials(q, k_local, v_local, slot_base: int, kv_len: int, scale=1.0) -> np.ndarray:
    q, k, v = _c(q, np.float32), _c(k_local, np.float32), _c(v_local, np.float32)
    D = q.shape[0]
    slots = k.shape[0]
    out = np.zeros(D + 2, np.float32)
    _check("emit_local_partials", lib().doe_oracle_emit_local_partials_f32(
        _ptr(q), _ptr(k), _ptr(v), _ptr(out), D, slots, slot_base, kv_len, float(scale)))
    return out


def stitch(partials) -> np.ndarray:
    """[n, D+2] f32 partials -> [D] (attention_kv_axis_sharded_stitch.py:46-90)."""
    p = _c(partials, np.float32)
    n, w = p.shape
    out = np.zeros(w - 2, np.float32)
    _check("stitch", lib().doe_oracle_stitch_partials_f32(_ptr(p), n, w - 2, _ptr(out)))
    return out


# ---- head256-style online softmax ----------------------------------------
def attention_online_f16kv(u: dict, q, k_bits, v_bits, kv_len_buffer=None,
                           page_table=None, threads: int = 0) -> np.ndarray:
    """Q [query_len,H,D] f32; K/V [pos,Hkv,D] f16 bits (attention_head256_f16kv.wgsl)."""
    uni = AttnUniforms(**u)
    q = _c(q, np.float32)
    k = _c(k_bits, np.uint16)
    v = _c(v_bits, np.uint16)
    out = np.zeros(q.shape, np.float32)
    klb = None if kv_len_buffer is None else _c(kv_len_buffer, np.uint32)
    pt = None if page_table is None else _c(page_table, np.uint32)
    _check("online_f16kv", lib().doe_oracle_attention_online_f16kv(
        C.byref(uni), _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(klb), _ptr(pt), threads))
    return out


def paged_decode(q_bits, k_pool, v_pool, block_table, kv_lens, scale, *, page_size: int,
                 k_scale=None, v_scale=None, threads: int = 0, sliding_window: int = 0,
                 softcap: float = 0.0) -> np.ndarray:
    """Batched paged GQA decode; pools f16 bits (uint16) or int8 + f16 scales.

    sliding_window > 0 keeps the last sliding_window keys; softcap > 0 caps
    each scaled score as tanh(s / softcap) * softcap."""
    q = _c(q_bits, np.uint16)
    B, H, D = q.shape
    int8 = k_pool.dtype == np.int8
    kp = _c(k_pool, np.int8 if int8 else np.uint16)
    vp = _c(v_pool, np.int8 if int8 else np.uint16)
    Hkv = kp.shape[1]
    num_pages = kp.shape[0] // page_size
    bt = _c(block_table, np.int32)
    kl = _c(kv_lens, np.int32)
    ks = None if k_scale is None else _c(k_scale, np.uint16)
    vs = None if v_scale is None else _c(v_scale, np.uint16)
    out = np.zeros((B, H, D), np.float32)
    _check("paged_decode", lib().doe_oracle_paged_decode_ex(
        B, H, Hkv, D, page_size, num_pages, bt.shape[1], _ptr(q), _ptr(kp), _ptr(vp),
        _ptr(ks), _ptr(vs), 1 if int8 else 0, _ptr(bt), _ptr(kl), float(scale), int(sliding_window),
        float(softcap), _ptr(out), threads))
    return out


_FAST_PATH = _HERE / "libcpu_baseline.so"
_fast = None


def cpu_features() -> set[str]:
    """CPU flags of this host (Linux /proc/cpuinfo); empty when unreadable."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("flags"):
                return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def fast_decode_available() -> bool:
    return {"avx2", "f16c"} <= cpu_features()


def _fast_lib() -> C.CDLL:
    global _fast
    if _fast is None:
        if not _FAST_PATH.exists():
            build()
        _fast = C.CDLL(str(_FAST_PATH))
        _fast.doe_cpu_paged_decode.restype = _I
        _fast.doe_cpu_paged_decode.argtypes = [_U32, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P,
                                               _U32, _P, _P, _F, _U32, _F, _P, _I]
    return _fast


def cpu_paged_decode(q_bits, k_pool, v_pool, block_table, kv_lens, scale, *, page_size: int,
                     k_scale=None, v_scale=None, threads: int = 0, sliding_window: int = 0,
                     softcap: float = 0.0) -> np.ndarray:
    """paged_decode's result from the CPU-organised build (cpu_baseline.c):
    the same float order, bit-identical, for timing on the host.  Needs AVX2
    and F16C (fast_decode_available())."""
    if not fast_decode_available():
        raise RuntimeError("cpu_paged_decode needs a CPU with AVX2 and F16C")
    q = _c(q_bits, np.uint16)
    B, H, D = q.shape
    int8 = k_pool.dtype == np.int8
    kp = _c(k_pool, np.int8 if int8 else np.uint16)
    vp = _c(v_pool, np.int8 if int8 else np.uint16)
    Hkv = kp.shape[1]
    bt = _c(block_table, np.int32)
    kl = _c(kv_lens, np.int32)
    ks = None if k_scale is None else _c(k_scale, np.uint16)
    vs = None if v_scale is None else _c(v_scale, np.uint16)
    out = np.zeros((B, H, D), np.float32)
    _check("cpu_paged_decode", _fast_lib().doe_cpu_paged_decode(
        B, H, Hkv, D, page_size, kp.shape[0] // page_size, bt.shape[1], _ptr(q), _ptr(kp), _ptr(vp),
        _ptr(ks), _ptr(vs), 1 if int8 else 0, _ptr(bt), _ptr(kl), float(scale), int(sliding_window),
        float(softcap), _ptr(out), threads))
    return out


def paged_append(new_k_bits, new_v_bits, k_pool, v_pool, block_table, positions, *,
                 page_size: int, k_scale=None, v_scale=None, threads: int = 0) -> None:
    """In-place append of new_k/new_v [B, T, Hkv, D] f16 bits into the pools."""
    nk = _c(new_k_bits, np.uint16)
    nv = _c(new_v_bits, np.uint16)
    B, T, Hkv, D = nk.shape
    int8 = k_pool.dtype == np.int8
    for a in (k_pool, v_pool, k_scale, v_scale):
        if a is not None and not a.flags.c_contiguous:
            raise ValueError("pools must be C-contiguous (written in place)")
    bt = _c(block_table, np.int32)
    pos = _c(positions, np.int32)
    num_pages = k_pool.shape[0] // page_size
    _check("paged_append", lib().doe_oracle_paged_append(
        B, T, Hkv, D, page_size, num_pages, bt.shape[1], _ptr(nk), _ptr(nv), _ptr(k_pool),
        _ptr(v_pool), _ptr(k_scale), _ptr(v_scale), 1 if int8 else 0, _ptr(bt), _ptr(pos), threads))


def paged_gather(pool, block_row, length: int, *, page_size: int) -> np.ndarray:
    pool = np.ascontiguousarray(pool)
    rows, Hkv, D = pool.shape
    row = _c(block_row, np.int32)
    out = np.zeros((length, Hkv, D), pool.dtype)
    _check("paged_gather", lib().doe_oracle_paged_gather(
        Hkv, D, page_size, rows // page_size, _ptr(row), row.shape[0], length,
        pool.dtype.itemsize, _ptr(pool), _ptr(out)))
    return out


def quantize_rows_int8(x_bits) -> tuple[np.ndarray, np.ndarray]:
    """[rows, D] f16 bits -> (int8 [rows, D], f16 scale bits [rows])."""
    x = _c(x_bits, np.uint16)
    D = x.shape[-1]
    rows = x.size // D
    q = np.zeros(x.shape, np.int8)
    s = np.zeros(x.shape[:-1], np.uint16)
    lib().doe_oracle_quantize_rows_int8(_ptr(x), rows, D, _ptr(q), _ptr(s))
    return q, s


def kv_write_dense(k_proj, v_proj, k_cache, v_cache, position: int) -> None:
    max_seq_len, D = k_cache.shape
    kp, vp = _c(k_proj, np.float32), _c(v_proj, np.float32)
    _check("kv_write", lib().doe_oracle_kv_write_dense(
        _ptr(kp), _ptr(vp), _ptr(k_cache), _ptr(v_cache), position, max_seq_len, D))


def kv_read_dense(k_cache, v_cache, read_start: int, read_len: int):
    max_seq_len, D = k_cache.shape
    ko = np.zeros((read_len, D), np.float32)
    vo = np.zeros((read_len, D), np.float32)
    _check("kv_read", lib().doe_oracle_kv_read_dense(
        _ptr(_c(k_cache, np.float32)), _ptr(_c(v_cache, np.float32)), _ptr(ko), _ptr(vo),
        read_start, read_len, max_seq_len, D))
    return ko, vo


def rope(qk, freq_cis, position_offset: int = 0) -> np.ndarray:
    """[S,H,D] f32 rotated in a copy (rope.wgsl:12-35)."""
    x = np.array(qk, dtype=np.float32, order="C", copy=True)
    S, H, D = x.shape
    f = _c(freq_cis, np.float32)
    _check("rope", lib().doe_oracle_rope_f32(_ptr(x), _ptr(f), S, H, D, position_offset))
    return x
