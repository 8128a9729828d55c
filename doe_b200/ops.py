"""torch-facing wrappers of the operator surface (include/doe_cuda.h).

Each wrapper validates shapes / dtypes, passes raw device pointers and the
current torch stream to libdoe_cuda.so, and raises DoeError on a non-OK
status.  Nothing here computes on the host.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _abi as abi
from .kv import PagedKVCache

_WS: dict[int, torch.Tensor] = {}


def workspace(nbytes: int, device=None) -> torch.Tensor:
    """A cached device scratch buffer of at least nbytes (grown on demand)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WS[key] = buf
    return buf


def _launch(ws_bytes: int = 0, status: torch.Tensor | None = None, stream=None, device=None) -> abi.Launch:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    ws = workspace(ws_bytes, device) if ws_bytes else None
    return abi.Launch(s.cuda_stream, ws.data_ptr() if ws is not None else None,
                      ws.numel() if ws is not None else 0,
                      status.data_ptr() if status is not None else None)


def _need(t: torch.Tensor, dtype, name: str) -> None:
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")


def status_word(device=None) -> torch.Tensor:
    """A zeroed device int32 that kernels OR DOE_DEVICE_ERR_* bits into."""
    return torch.zeros(1, dtype=torch.int32, device=device or "cuda")


def attention_decode_f32(q, k_cache, v_cache, scale: float, out=None, status=None, stream=None):
    """attention-decode.wgsl: q [H,D], k/v [H,L,D] f32 -> [H,D]."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, torch.float32, n)
    H, D = q.shape
    L = k_cache.shape[1]
    out = torch.empty_like(q) if out is None else out
    lib = abi.lib()
    ws = lib.doe_attention_decode_f32_workspace_bytes(H, D, L)
    l = _launch(ws, status, stream, q.device)
    abi.check("doe_attention_decode_f32", lib.doe_attention_decode_f32(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), H, D, L, float(scale),
        C.byref(l)))
    return out


def attention_online(u: dict, q, k, v, kv_len_buffer=None, page_table=None, out=None, status=None,
                     stream=None):
    """attention_head256_f16kv.wgsl semantics: q [query_len,H,D] f32, k/v [pos,Hkv,D] f16|f32."""
    _need(q, torch.float32, "q")
    kv_elem = 1 if k.dtype == torch.float32 else 0
    uni = abi.AttnUniforms(**{**u, "pad": 0})
    out = torch.zeros_like(q) if out is None else out
    l = _launch(0, status, stream, q.device)
    abi.check("doe_attention_online", abi.lib().doe_attention_online(
        C.byref(uni), q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_elem, out.data_ptr(),
        kv_len_buffer.data_ptr() if kv_len_buffer is not None else None,
        page_table.data_ptr() if page_table is not None else None, C.byref(l)))
    return out


def attention_prefill_wgsl(q, k, v, scale: float, out=None, status=None, stream=None):
    """attention-prefill.wgsl: causal, [H,S,D] f32."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, torch.float32, n)
    H, S, D = q.shape
    out = torch.empty_like(q) if out is None else out
    l = _launch(0, status, stream, q.device)
    abi.check("doe_attention_prefill_wgsl_f32", abi.lib().doe_attention_prefill_wgsl_f32(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), S, D, H, float(scale), C.byref(l)))
    return out


def stitch(partials, out=None, stream=None):
    """[rows, shards, D+2] f32 partials -> [rows, D]."""
    _need(partials, torch.float32, "partials")
    rows, shards, w = partials.shape
    out = torch.empty((rows, w - 2), dtype=torch.float32, device=partials.device) if out is None else out
    l = _launch(0, None, stream, partials.device)
    abi.check("doe_attention_stitch_f32", abi.lib().doe_attention_stitch_f32(
        partials.data_ptr(), rows, shards, w - 2, out.data_ptr(), C.byref(l)))
    return out


def paged_decode(cache: PagedKVCache, q, seq_lens, scale: float, new_k=None, new_v=None, out=None,
                 split_pages: int = 0, status=None, stream=None, freq_cis=None, sliding_window: int = 0,
                 softcap: float = 0.0, out_dtype=torch.float32, ws=None, inputs_stable: bool = False):
    """Batched GQA decode: q [B,H,D] f16, seq_lens [B] int32 -> out [B,H,D] f32.

    With new_k/new_v ([B,Hkv,D] f16) the new token is first written at
    position seq_lens[b] - 1 (quantised for int8 caches).  With freq_cis
    ([positions, D/2, 2] f32 RoPE table) the query and the new K row are
    rotated at position seq_lens[b] - 1 first (doe_paged_decode_rope).
    sliding_window > 0 keeps the last sliding_window keys and softcap > 0
    caps each scaled score as softcap * tanh(s / softcap) (doe_paged_decode_ex).
    out_dtype torch.bfloat16 writes a bf16 output (DOE_DECODE_OUT_BF16).
    `ws`: a workspace kept for paged decodes alone, zeroed when created
    (decode_workspace); its split counters then need no clearing per call
    (DOE_DECODE_COUNTERS_ZEROED).  inputs_stable: seq_lens, the block table and
    the pool rows (other than the appended ones) are final before the call is
    enqueued, so the first copies may start before the preceding kernel ends
    (DOE_DECODE_INPUTS_STABLE)."""
    _need(q, torch.float16, "q")
    _need(seq_lens, torch.int32, "seq_lens")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be float32 or bfloat16")
    B, H, D = q.shape
    out = torch.empty((B, H, D), dtype=out_dtype, device=q.device) if out is None else out
    _need(out, out_dtype, "out")
    flags = abi.DECODE_OUT_BF16 if out_dtype == torch.bfloat16 else 0
    if ws is not None:
        flags |= abi.DECODE_COUNTERS_ZEROED
    if inputs_stable:
        flags |= abi.DECODE_INPUTS_STABLE
    kv = cache.struct()
    lib = abi.lib()
    need = lib.doe_paged_decode_workspace_bytes(C.byref(kv), B, H, split_pages)
    if ws is None:
        l = _launch(need, status, stream, q.device)
    else:
        if ws.numel() < need:
            raise ValueError(f"decode workspace of {need} bytes needed, {ws.numel()} given")
        s = stream if stream is not None else torch.cuda.current_stream(q.device)
        l = abi.Launch(s.cuda_stream, ws.data_ptr(), ws.numel(), status.data_ptr() if status is not None else None)
    nk = new_k.data_ptr() if new_k is not None else None
    nv = new_v.data_ptr() if new_v is not None else None
    if sliding_window or softcap or flags:
        if freq_cis is not None:
            _need(freq_cis, torch.float32, "freq_cis")
        opts = abi.DecodeOptions(freq_cis.data_ptr() if freq_cis is not None else None,
                                 freq_cis.shape[0] if freq_cis is not None else 0, int(sliding_window),
                                 float(softcap), flags)
        abi.check("doe_paged_decode_ex", lib.doe_paged_decode_ex(
            C.byref(kv), B, H, q.data_ptr(), seq_lens.data_ptr(), nk, nv, float(scale), out.data_ptr(),
            split_pages, C.byref(opts), C.byref(l)))
    elif freq_cis is None:
        abi.check("doe_paged_decode", lib.doe_paged_decode(
            C.byref(kv), B, H, q.data_ptr(), seq_lens.data_ptr(), nk, nv, float(scale), out.data_ptr(),
            split_pages, C.byref(l)))
    else:
        _need(freq_cis, torch.float32, "freq_cis")
        abi.check("doe_paged_decode_rope", lib.doe_paged_decode_rope(
            C.byref(kv), B, H, q.data_ptr(), seq_lens.data_ptr(), nk, nv, float(scale), out.data_ptr(),
            split_pages, freq_cis.data_ptr(), freq_cis.shape[0], C.byref(l)))
    return out


def decode_workspace(cache: PagedKVCache, num_seqs: int, num_heads: int, split_pages: int = 0) -> torch.Tensor:
    """A zeroed workspace for paged decodes alone (pass as paged_decode(ws=...))."""
    kv = cache.struct()
    need = int(abi.lib().doe_paged_decode_workspace_bytes(C.byref(kv), num_seqs, num_heads, split_pages))
    return torch.zeros(max(need, 256), dtype=torch.uint8, device=cache.k_pool.device)


def paged_append(cache: PagedKVCache, new_k, new_v, positions, status=None, stream=None, freq_cis=None):
    """Write new_k/new_v [B,T,Hkv,D] f16 at positions[b] + t (quantising int8 caches).

    With freq_cis ([positions, D/2, 2] f32 RoPE table) each K row is first
    rotated at its position (doe_paged_append_rope)."""
    _need(new_k, torch.float16, "new_k")
    _need(new_v, torch.float16, "new_v")
    _need(positions, torch.int32, "positions")
    B, T = new_k.shape[:2]
    kv = cache.struct()
    l = _launch(0, status, stream, new_k.device)
    if freq_cis is None:
        abi.check("doe_paged_append", abi.lib().doe_paged_append(
            C.byref(kv), B, T, new_k.data_ptr(), new_v.data_ptr(), positions.data_ptr(), C.byref(l)))
    else:
        _need(freq_cis, torch.float32, "freq_cis")
        abi.check("doe_paged_append_rope", abi.lib().doe_paged_append_rope(
            C.byref(kv), B, T, new_k.data_ptr(), new_v.data_ptr(), positions.data_ptr(), freq_cis.data_ptr(),
            freq_cis.shape[0], C.byref(l)))


def paged_gather(cache: PagedKVCache, seq: int, start: int, length: int, status=None, stream=None):
    """kv_read: tokens [start, start+length) of one sequence -> (k, v[, k_scale, v_scale])."""
    shape = (length, cache.num_kv_heads, cache.head_dim)
    k = torch.empty(shape, dtype=cache.k_pool.dtype, device=cache.k_pool.device)
    v = torch.empty_like(k)
    ks = vs = None
    if cache.kv_dtype == "int8":
        ks = torch.empty((length, cache.num_kv_heads), dtype=torch.float16, device=k.device)
        vs = torch.empty_like(ks)
    kv = cache.struct()
    l = _launch(0, status, stream, k.device)
    abi.check("doe_paged_gather", abi.lib().doe_paged_gather(
        C.byref(kv), seq, start, length, k.data_ptr(), v.data_ptr(),
        ks.data_ptr() if ks is not None else None, vs.data_ptr() if vs is not None else None,
        C.byref(l)))
    return (k, v) if ks is None else (k, v, ks, vs)


def kv_write_dense(k_proj, v_proj, k_cache, v_cache, positions, status=None, stream=None):
    """proj [heads, D], caches [heads, max_seq_len, D] (f16|f32), positions u32 [1|heads]."""
    heads, max_len, D = k_cache.shape
    eb = k_cache.element_size()
    l = _launch(0, status, stream, k_cache.device)
    abi.check("doe_kv_write_dense", abi.lib().doe_kv_write_dense(
        k_proj.data_ptr(), v_proj.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        positions.data_ptr(), positions.numel(), heads, max_len, D, eb, C.byref(l)))


def kv_read_dense(k_cache, v_cache, read_start: int, read_len: int, status=None, stream=None):
    heads, max_len, D = k_cache.shape
    ko = torch.empty((heads, read_len, D), dtype=k_cache.dtype, device=k_cache.device)
    vo = torch.empty_like(ko)
    l = _launch(0, status, stream, k_cache.device)
    abi.check("doe_kv_read_dense", abi.lib().doe_kv_read_dense(
        k_cache.data_ptr(), v_cache.data_ptr(), ko.data_ptr(), vo.data_ptr(), heads, read_start,
        read_len, max_len, D, k_cache.element_size(), C.byref(l)))
    return ko, vo


def rope(qk, freq_cis, position_offset: int = 0, stream=None):
    """rope.wgsl in place on qk [S,H,D] f32."""
    _need(qk, torch.float32, "qk")
    S, H, D = qk.shape
    l = _launch(0, None, stream, qk.device)
    abi.check("doe_rope_f32", abi.lib().doe_rope_f32(
        qk.data_ptr(), freq_cis.data_ptr(), S, H, D, position_offset, C.byref(l)))
    return qk


def attention_prefill_f16(q, k, v, scale: float, causal: bool = True, cache: PagedKVCache | None = None,
                          cache_seq: int = 0, cache_start: int = 0, out=None, status=None, stream=None):
    """tcgen05 prefill: q [S,H,128], k/v [S,Hkv,128] f16 -> out [S,H,128] f32.

    With `cache`, the prompt's K/V rows are also written into the paged cache."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, torch.float16, n)
    S, H, D = q.shape
    Hkv = k.shape[1]
    out = torch.empty((S, H, D), dtype=torch.float32, device=q.device) if out is None else out
    kv = cache.struct() if cache is not None else None
    l = _launch(0, status, stream, q.device)
    abi.check("doe_attention_prefill_f16", abi.lib().doe_attention_prefill_f16(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), S, H, Hkv, D, float(scale),
        1 if causal else 0, C.byref(kv) if kv is not None else None, cache_seq, cache_start,
        C.byref(l)))
    return out


_LINEAR_WS: dict[int, torch.Tensor] = {}


def linear_workspace(n_out: int, k: int, device=None) -> torch.Tensor:
    """The zero-initialised workspace doe_linear_bf16 keeps its tile counters in.

    Separate from `workspace()`: its counters must be zero before a call, and
    every call that completes without a timeout leaves them zero again."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    need = int(abi.lib().doe_linear_workspace_bytes(n_out, k))
    buf = _LINEAR_WS.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.zeros(need, dtype=torch.uint8, device=dev)
        _LINEAR_WS[key] = buf
    return buf


_DTYPES = {torch.bfloat16: abi.DTYPE_BF16, torch.float16: abi.DTYPE_F16, torch.float32: abi.DTYPE_F32}


def rmsnorm(x, gamma, eps: float, out=None, status=None, stream=None):
    """x [rows, cols] f32, gamma [cols] bf16 -> bf16 x / sqrt(mean(x^2) + eps) * gamma."""
    _need(x, torch.float32, "x")
    _need(gamma, torch.bfloat16, "gamma")
    rows, cols = x.shape
    out = torch.empty((rows, cols), dtype=torch.bfloat16, device=x.device) if out is None else out
    _need(out, torch.bfloat16, "out")
    l = _launch(0, status, stream, x.device)
    abi.check("doe_rmsnorm_bf16", abi.lib().doe_rmsnorm_bf16(
        x.data_ptr(), gamma.data_ptr(), float(eps), out.data_ptr(), rows, cols, C.byref(l)))
    return out


def ssq_buffer(cols: int, device=None) -> torch.Tensor:
    """The [cols / 32, 32] f32 sums of squares a norm-producing linear writes."""
    return torch.zeros((cols // 32, 32), dtype=torch.float32, device=device)


def linear(x, w, outs, *, swiglu: bool = False, residual=None, status=None, stream=None, ws=None,
           norm_out=None, norm_in=None):
    """doe_linear_bf16: x [batch, k] bf16 times w [n_out, k] bf16 transposed.

    `outs` is a list of 1-3 contiguous tensors of one dtype (bf16, f16 or f32),
    each [batch, width]; with swiglu=True a single [batch, n_out/2] output of
    silu(gate) * up (w packed in 128-row blocks: 64 gate rows, 64 up rows).
    `residual` ([batch, n_out] f32, f32 output) is added to the product.

    The RMSNorm between two products (doe_linear_bf16_norm): norm_out =
    (gamma [n_out] bf16, normed [batch, n_out] bf16, ssq (ssq_buffer(n_out)))
    makes this product (f32, one segment) also write bf16(y * gamma) and its
    per-32-column sums of squares; norm_in = (ssq, eps), with x such a normed
    output, scales each row of this product by 1 / sqrt(mean(h^2) + eps)."""
    _need(x, torch.bfloat16, "x")
    _need(w, torch.bfloat16, "w")
    batch, k = x.shape
    n_out = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"w is {tuple(w.shape)}, x is {tuple(x.shape)}")
    if not 1 <= len(outs) <= 3:
        raise ValueError("1 to 3 output segments")
    dt = outs[0].dtype
    lo = abi.LinearOut()
    for i, o in enumerate(outs):
        _need(o, dt, f"outs[{i}]")
        lo.out[i] = o.data_ptr()
        lo.width[i] = o.shape[-1] if not swiglu else 0
    lo.dtype = _DTYPES[dt]
    lo.epilogue = abi.LINEAR_SWIGLU if swiglu else abi.LINEAR_STORE
    if residual is not None:
        _need(residual, torch.float32, "residual")
        lo.residual = residual.data_ptr()
    ws = linear_workspace(n_out, k, x.device) if ws is None else ws
    s = stream if stream is not None else torch.cuda.current_stream(x.device)
    l = abi.Launch(s.cuda_stream, ws.data_ptr(), ws.numel(), status.data_ptr() if status is not None else None)
    if norm_out is None and norm_in is None:
        abi.check("doe_linear_bf16", abi.lib().doe_linear_bf16(
            x.data_ptr(), w.data_ptr(), batch, n_out, k, C.byref(lo), C.byref(l)))
        return outs
    ln = abi.LinearNorm()
    if norm_out is not None:
        gamma, normed, ssq = norm_out
        _need(gamma, torch.bfloat16, "norm_out gamma")
        _need(normed, torch.bfloat16, "norm_out normed")
        _need(ssq, torch.float32, "norm_out ssq")
        if gamma.numel() != n_out or normed.shape != (batch, n_out) or ssq.numel() != n_out:
            raise ValueError("norm_out: gamma [n_out], normed [batch, n_out], ssq [n_out / 32, 32]")
        ln.gamma, ln.normed_out, ln.ssq_out = gamma.data_ptr(), normed.data_ptr(), ssq.data_ptr()
    if norm_in is not None:
        ssq, eps = norm_in
        _need(ssq, torch.float32, "norm_in ssq")
        if ssq.numel() != k:
            raise ValueError("norm_in: ssq [k / 32, 32]")
        ln.ssq_in, ln.eps = ssq.data_ptr(), float(eps)
    abi.check("doe_linear_bf16_norm", abi.lib().doe_linear_bf16_norm(
        x.data_ptr(), w.data_ptr(), batch, n_out, k, C.byref(lo), C.byref(ln), C.byref(l)))
    return outs
