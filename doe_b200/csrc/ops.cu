// ops.cu -- the operator surface of include/doe_cuda.h: argument checks and
// launches on caller-owned device memory.  No entry point runs work on the
// host; an unsupported shape returns DOE_UNSUPPORTED with a message.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace doe {

static thread_local char g_op_error[512] = "";

void set_op_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_op_error, sizeof(g_op_error), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t err, const char* where) {
  if (err == cudaSuccess) return DOE_OK;
  set_op_error("%s: %s (%s)", where, cudaGetErrorName(err), cudaGetErrorString(err));
  if (err == cudaErrorNoDevice || err == cudaErrorInvalidDevice) return DOE_NO_DEVICE;
  return DOE_CUDA_ERROR;
}

}  // namespace doe

using namespace doe;

namespace {

const doe_launch kDefaultLaunch = {nullptr, nullptr, 0, nullptr};

const doe_launch* launch_or_default(const doe_launch* l) { return l ? l : &kDefaultLaunch; }

int invalid(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_op_error("%s", buf);
  return DOE_INVALID_ARGUMENT;
}

int check_paged_kv(const doe_paged_kv* kv, const char* fn) {
  if (!kv) return invalid("%s: kv is null", fn);
  if (!kv->k_pool || !kv->v_pool || !kv->block_table)
    return invalid("%s: k_pool, v_pool and block_table are required", fn);
  if (kv->kv_dtype > DOE_KV_INT8) return invalid("%s: unknown kv_dtype %u", fn, kv->kv_dtype);
  if (kv->kv_dtype == DOE_KV_INT8 && (!kv->k_scale || !kv->v_scale))
    return invalid("%s: int8 pools need k_scale and v_scale", fn);
  if (kv->page_size == 0 || kv->page_size % 16 != 0)
    return invalid("%s: page_size must be a positive multiple of 16 (got %u)", fn, kv->page_size);
  if (kv->num_kv_heads == 0 || kv->head_dim == 0 || kv->num_pages == 0)
    return invalid("%s: num_kv_heads, head_dim and num_pages must be positive", fn);
  if (kv->max_pages_per_seq == 0) return invalid("%s: max_pages_per_seq must be positive", fn);
  return DOE_OK;
}

}  // namespace

extern "C" {

int doe_cuda_abi_version(void) { return DOE_CUDA_ABI_VERSION; }

int doe_cuda_device_count(int* count) {
  if (!count) return DOE_INVALID_ARGUMENT;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return cuda_status(e, "cudaGetDeviceCount") == DOE_CUDA_ERROR ? DOE_NO_DEVICE : DOE_NO_DEVICE;
  }
  *count = n;
  return DOE_OK;
}

const char* doe_cuda_op_last_error(void) { return g_op_error; }

uint64_t doe_attention_decode_f32_workspace_bytes(uint32_t num_heads, uint32_t head_dim,
                                                  uint32_t kv_len) {
  return decode_f32_workspace(num_heads, head_dim, kv_len);
}

int doe_attention_decode_f32(const float* q, const float* k_cache, const float* v_cache,
                             float* out, uint32_t num_heads, uint32_t head_dim, uint32_t kv_len,
                             float scale, const doe_launch* launch) {
  if (!q || !k_cache || !v_cache || !out) return invalid("doe_attention_decode_f32: null pointer");
  if (head_dim == 0 || head_dim > 256)
    return invalid("doe_attention_decode_f32: head_dim must be 1..256 (got %u)", head_dim);
  if (num_heads == 0) return DOE_OK;
  if (kv_len == 0) return invalid("doe_attention_decode_f32: kv_len must be positive");
  return launch_decode_f32(q, k_cache, v_cache, out, num_heads, head_dim, kv_len, scale,
                           launch_or_default(launch));
}

int doe_attention_online(const doe_attn_uniforms* u, const float* q, const void* k,
                         const void* v, uint32_t kv_elem, float* out,
                         const uint32_t* kv_len_buffer, const uint32_t* page_table,
                         const doe_launch* launch) {
  if (!u || !q || !k || !v || !out) return invalid("doe_attention_online: null pointer");
  if (u->num_kv_heads == 0 || u->num_heads % u->num_kv_heads != 0)
    return invalid("doe_attention_online: num_heads %u is not a multiple of num_kv_heads %u",
                   u->num_heads, u->num_kv_heads);
  if (u->head_dim == 0 || u->head_dim > 512)
    return invalid("doe_attention_online: head_dim must be 1..512 (got %u)", u->head_dim);
  if (u->kv_layout > 2) return invalid("doe_attention_online: kv_layout %u", u->kv_layout);
  if (u->kv_layout == 2 && (!page_table || u->page_size == 0))
    return invalid("doe_attention_online: paged layout needs page_table and page_size");
  if (u->kv_len_source != 0 && !kv_len_buffer)
    return invalid("doe_attention_online: kv_len_source needs kv_len_buffer");
  if (kv_elem > 1) return invalid("doe_attention_online: kv_elem must be 0 (f16) or 1 (f32)");
  const doe_launch* l = launch_or_default(launch);
  GenericAttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.u = *u;
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.kv_len_buffer = kv_len_buffer;
  a.page_table = page_table;
  a.q_pos_stride = (int64_t)u->num_heads * u->head_dim;
  a.q_head_stride = u->head_dim;
  a.kv_pos_stride = (int64_t)u->num_kv_heads * u->head_dim;
  a.kv_head_stride = u->head_dim;
  a.status = l->status;
  return launch_attn_generic(a, kv_elem == 1, static_cast<cudaStream_t>(l->stream));
}

int doe_attention_prefill_wgsl_f32(const float* q, const float* k, const float* v, float* out,
                                   uint32_t seq_len, uint32_t head_dim, uint32_t num_heads,
                                   float scale, const doe_launch* launch) {
  if (!q || !k || !v || !out) return invalid("doe_attention_prefill_wgsl_f32: null pointer");
  if (head_dim == 0 || head_dim > 512)
    return invalid("doe_attention_prefill_wgsl_f32: head_dim must be 1..512");
  const doe_launch* l = launch_or_default(launch);
  GenericAttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.u.num_heads = num_heads;
  a.u.num_kv_heads = num_heads;
  a.u.head_dim = head_dim;
  a.u.seq_len = seq_len;
  a.u.query_len = seq_len;
  a.u.scale = scale;
  a.u.is_causal = 1;
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  // [H, S, D]: position stride D, head stride S*D
  a.q_pos_stride = head_dim;
  a.q_head_stride = (int64_t)seq_len * head_dim;
  a.kv_pos_stride = head_dim;
  a.kv_head_stride = (int64_t)seq_len * head_dim;
  a.kv_rows = seq_len;
  a.status = l->status;
  return launch_attn_generic(a, true, static_cast<cudaStream_t>(l->stream));
}

int doe_attention_prefill_f16(const void* q, const void* k, const void* v, float* out,
                              uint32_t seq_len, uint32_t num_heads, uint32_t num_kv_heads,
                              uint32_t head_dim, float scale, uint32_t causal,
                              const doe_paged_kv* cache, uint32_t cache_seq, uint32_t cache_start,
                              const doe_launch* launch) {
  if (!q || !k || !v || !out) return invalid("doe_attention_prefill_f16: null pointer");
  if (head_dim != 128) {
    set_op_error("doe_attention_prefill_f16: the tcgen05 prefill kernel is built for head_dim 128 (got %u)",
                 head_dim);
    return DOE_UNSUPPORTED;
  }
  if (num_kv_heads == 0 || num_heads == 0 || num_heads % num_kv_heads != 0)
    return invalid("doe_attention_prefill_f16: num_heads %u is not a multiple of num_kv_heads %u",
                   num_heads, num_kv_heads);
  if (seq_len == 0) return DOE_OK;
  if ((uint64_t)num_heads * ((seq_len + 127) / 128) > 0x7fffffffull)
    return invalid("doe_attention_prefill_f16: grid too large");
  if (cache != nullptr) {
    int rc = check_paged_kv(cache, "doe_attention_prefill_f16");
    if (rc != DOE_OK) return rc;
    if (cache->kv_dtype != DOE_KV_F16 || cache->head_dim != 128 || cache->num_kv_heads != num_kv_heads)
      return invalid("doe_attention_prefill_f16: the cache must be f16 with the same kv heads and head_dim 128");
    if (!causal || seq_len % 16 != 0 || cache_start % 16 != 0) {
      set_op_error("doe_attention_prefill_f16: the fused cache write needs a causal prefill with "
                   "seq_len and cache_start multiples of 16 (use doe_paged_append otherwise)");
      return DOE_UNSUPPORTED;
    }
  }
  return launch_prefill_f16(q, k, v, out, seq_len, num_heads, num_kv_heads, scale, causal, cache,
                            cache_seq, cache_start, launch_or_default(launch));
}

int doe_attention_stitch_f32(const float* partials, uint32_t rows, uint32_t num_shards,
                             uint32_t head_dim, float* out, const doe_launch* launch) {
  if (!partials || !out) return invalid("doe_attention_stitch_f32: null pointer");
  if (num_shards == 0 || head_dim == 0)
    return invalid("doe_attention_stitch_f32: num_shards and head_dim must be positive");
  return launch_stitch(partials, rows, num_shards, head_dim, out, launch_or_default(launch));
}

uint64_t doe_paged_decode_workspace_bytes(const doe_paged_kv* kv, uint32_t num_seqs,
                                          uint32_t num_heads, uint32_t split_pages) {
  if (check_paged_kv(kv, "doe_paged_decode_workspace_bytes") != DOE_OK) return 0;
  if (num_heads % kv->num_kv_heads != 0) return 0;
  uint64_t ws = 0;
  launch_paged_decode(kv, num_seqs, num_heads, nullptr, nullptr, nullptr, nullptr, 0.0f, nullptr,
                      split_pages, nullptr, &kDefaultLaunch, &ws);
  return ws;
}

namespace {
int check_rope_table(const char* who, const float* freq_cis, uint32_t rope_positions) {
  if (!freq_cis || rope_positions == 0)
    return invalid("%s: freq_cis and a positive rope_positions are required", who);
  if (reinterpret_cast<uintptr_t>(freq_cis) % 16 != 0)
    return invalid("%s: freq_cis must be 16-byte aligned", who);
  return DOE_OK;
}
int paged_decode_common(const char* who, const doe_paged_kv* kv, uint32_t num_seqs, uint32_t num_heads,
                        const void* q, const int32_t* seq_lens, const void* new_k, const void* new_v,
                        float scale, float* out, uint32_t split_pages, const doe_decode_options* opts,
                        const doe_launch* launch) {
  int rc = check_paged_kv(kv, who);
  if (rc != DOE_OK) return rc;
  if (!q || !seq_lens || !out) return invalid("%s: q, seq_lens and out are required", who);
  if ((new_k == nullptr) != (new_v == nullptr)) return invalid("%s: new_k and new_v go together", who);
  if (num_heads == 0 || num_heads % kv->num_kv_heads != 0)
    return invalid("%s: num_heads %u is not a multiple of num_kv_heads %u", who, num_heads,
                   kv->num_kv_heads);
  if (kv->head_dim != 128) {
    set_op_error("%s: the tensor-core decode kernel is built for head_dim 128 (got %u)", who, kv->head_dim);
    return DOE_UNSUPPORTED;
  }
  if (num_seqs == 0) return DOE_OK;
  if (num_seqs > 65535) return invalid("%s: at most 65535 sequences per launch", who);
  if (opts != nullptr) {
    if ((opts->flags & ~(DOE_DECODE_OUT_BF16 | DOE_DECODE_COUNTERS_ZEROED | DOE_DECODE_INPUTS_STABLE)) != 0)
      return invalid("%s: unknown bits in options.flags", who);
    if (opts->freq_cis != nullptr) {
      int rr = check_rope_table(who, opts->freq_cis, opts->rope_positions);
      if (rr != DOE_OK) return rr;
    }
    if (!(opts->attn_softcap >= 0.0f)) return invalid("%s: attn_softcap must be >= 0", who);
  }
  return launch_paged_decode(kv, num_seqs, num_heads, q, seq_lens, new_k, new_v, scale, out, split_pages,
                             opts, launch_or_default(launch), nullptr);
}

}  // namespace

int doe_paged_decode(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t num_heads,
                     const void* q, const int32_t* seq_lens, const void* new_k,
                     const void* new_v, float scale, float* out, uint32_t split_pages,
                     const doe_launch* launch) {
  return paged_decode_common("doe_paged_decode", kv, num_seqs, num_heads, q, seq_lens, new_k, new_v, scale,
                             out, split_pages, nullptr, launch);
}

int doe_paged_decode_ex(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t num_heads,
                        const void* q, const int32_t* seq_lens, const void* new_k,
                        const void* new_v, float scale, float* out, uint32_t split_pages,
                        const doe_decode_options* options, const doe_launch* launch) {
  return paged_decode_common("doe_paged_decode_ex", kv, num_seqs, num_heads, q, seq_lens, new_k, new_v,
                             scale, out, split_pages, options, launch);
}

int doe_paged_decode_rope(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t num_heads,
                          const void* q, const int32_t* seq_lens, const void* new_k,
                          const void* new_v, float scale, float* out, uint32_t split_pages,
                          const float* freq_cis, uint32_t rope_positions, const doe_launch* launch) {
  int rc = check_rope_table("doe_paged_decode_rope", freq_cis, rope_positions);
  if (rc != DOE_OK) return rc;
  doe_decode_options o = {freq_cis, rope_positions, 0, 0.0f, 0};
  return paged_decode_common("doe_paged_decode_rope", kv, num_seqs, num_heads, q, seq_lens, new_k, new_v,
                             scale, out, split_pages, &o, launch);
}

int doe_paged_append(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t n_tokens,
                     const void* new_k, const void* new_v, const int32_t* positions,
                     const doe_launch* launch) {
  int rc = check_paged_kv(kv, "doe_paged_append");
  if (rc != DOE_OK) return rc;
  if (!new_k || !new_v || !positions)
    return invalid("doe_paged_append: new_k, new_v and positions are required");
  if (num_seqs > 65535) return invalid("doe_paged_append: at most 65535 sequences per launch");
  return launch_paged_append(kv, num_seqs, n_tokens, new_k, new_v, positions, nullptr, 0,
                             launch_or_default(launch));
}

int doe_paged_append_rope(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t n_tokens,
                          const void* new_k, const void* new_v, const int32_t* positions,
                          const float* freq_cis, uint32_t rope_positions, const doe_launch* launch) {
  int rc = check_paged_kv(kv, "doe_paged_append_rope");
  if (rc != DOE_OK) return rc;
  rc = check_rope_table("doe_paged_append_rope", freq_cis, rope_positions);
  if (rc != DOE_OK) return rc;
  if (!new_k || !new_v || !positions)
    return invalid("doe_paged_append_rope: new_k, new_v and positions are required");
  if (num_seqs > 65535) return invalid("doe_paged_append_rope: at most 65535 sequences per launch");
  return launch_paged_append(kv, num_seqs, n_tokens, new_k, new_v, positions, freq_cis, rope_positions,
                             launch_or_default(launch));
}

int doe_paged_gather(const doe_paged_kv* kv, uint32_t seq, uint32_t start, uint32_t len,
                     void* k_out, void* v_out, void* k_scale_out, void* v_scale_out,
                     const doe_launch* launch) {
  int rc = check_paged_kv(kv, "doe_paged_gather");
  if (rc != DOE_OK) return rc;
  if (!k_out || !v_out) return invalid("doe_paged_gather: k_out and v_out are required");
  if ((k_scale_out == nullptr) != (v_scale_out == nullptr))
    return invalid("doe_paged_gather: scale outputs go together");
  return launch_paged_gather(kv, seq, start, len, k_out, v_out, k_scale_out, v_scale_out,
                             launch_or_default(launch));
}

int doe_kv_write_dense(const void* k_proj, const void* v_proj, void* k_cache, void* v_cache,
                       const uint32_t* positions, uint32_t num_positions, uint32_t heads,
                       uint32_t max_seq_len, uint32_t head_dim, uint32_t elem_bytes,
                       const doe_launch* launch) {
  if (!k_proj || !v_proj || !k_cache || !v_cache || !positions)
    return invalid("doe_kv_write_dense: null pointer");
  if (elem_bytes != 2 && elem_bytes != 4) return invalid("doe_kv_write_dense: elem_bytes 2 or 4");
  if (num_positions != 1 && num_positions != heads)
    return invalid("doe_kv_write_dense: positions must have 1 or heads (%u) entries", heads);
  return launch_kv_write_dense(k_proj, v_proj, k_cache, v_cache, positions, num_positions, heads,
                               max_seq_len, head_dim, elem_bytes, launch_or_default(launch));
}

int doe_kv_read_dense(const void* k_cache, const void* v_cache, void* k_out, void* v_out,
                      uint32_t heads, uint32_t read_start, uint32_t read_len,
                      uint32_t max_seq_len, uint32_t head_dim, uint32_t elem_bytes,
                      const doe_launch* launch) {
  if (!k_cache || !v_cache || !k_out || !v_out) return invalid("doe_kv_read_dense: null pointer");
  if (elem_bytes != 2 && elem_bytes != 4) return invalid("doe_kv_read_dense: elem_bytes 2 or 4");
  if ((uint64_t)read_start + read_len > max_seq_len) {
    set_op_error("doe_kv_read_dense: rows [%u, %u) exceed max_seq_len %u", read_start,
                 read_start + read_len, max_seq_len);
    return DOE_OUT_OF_RANGE;
  }
  return launch_kv_read_dense(k_cache, v_cache, k_out, v_out, heads, read_start, read_len,
                              max_seq_len, head_dim, elem_bytes, launch_or_default(launch));
}

int doe_rope_f32(float* qk, const float* freq_cis, uint32_t seq_len, uint32_t num_heads,
                 uint32_t head_dim, uint32_t position_offset, const doe_launch* launch) {
  if (!qk || !freq_cis) return invalid("doe_rope_f32: null pointer");
  if (seq_len > 65535) return invalid("doe_rope_f32: at most 65535 positions per launch");
  return launch_rope(qk, freq_cis, seq_len, num_heads, head_dim, position_offset,
                     launch_or_default(launch));
}

int doe_rmsnorm_bf16(const float* x, const void* gamma, float eps, void* out, uint32_t rows, uint32_t cols,
                     const doe_launch* launch) {
  if (!x || !gamma || !out) return invalid("doe_rmsnorm_bf16: null pointer");
  if (cols == 0 || cols % 4 != 0) return invalid("doe_rmsnorm_bf16: cols must be a positive multiple of 4");
  if (rows > 2147483647u) return invalid("doe_rmsnorm_bf16: too many rows");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(gamma) % 8 ||
      reinterpret_cast<uintptr_t>(out) % 8)
    return invalid("doe_rmsnorm_bf16: x must be 16-byte aligned, gamma and out 8-byte aligned");
  if (!(eps >= 0.0f)) return invalid("doe_rmsnorm_bf16: eps must be >= 0");
  if (rows == 0) return DOE_OK;
  return launch_rmsnorm(x, gamma, eps, out, rows, cols, launch_or_default(launch));
}

// ---- ORT plugin EP basic operators (doe_ort_ep.cc:1899-2401) -------------
namespace {

bool overlaps(const void* p, uint64_t p_bytes, const void* q, uint64_t q_bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p), b = reinterpret_cast<uintptr_t>(q);
  return p_bytes != 0 && q_bytes != 0 && a < b + q_bytes && b < a + p_bytes;
}

constexpr uint64_t kMaxElems = 1ull << 40;  // a sanity bound on element counts (4 TiB of f32)

}  // namespace

int doe_ep_unary_f32(uint32_t op, const float* x, float* y, uint64_t n, const doe_launch* launch) {
  if (op > DOE_EP_GELU) return invalid("doe_ep_unary_f32: unknown op %u", op);
  if (n == 0) return DOE_OK;
  if (!x || !y) return invalid("doe_ep_unary_f32: null pointer");
  if (n > kMaxElems) return invalid("doe_ep_unary_f32: n too large");
  if (x != y && overlaps(x, n * 4, y, n * 4)) return invalid("doe_ep_unary_f32: x and y partly overlap");
  return launch_ep_unary(op, x, y, n, launch_or_default(launch));
}

int doe_ep_binary_f32(uint32_t op, const float* a, const float* b, float* y, uint64_t n,
                      const doe_launch* launch) {
  if (op > DOE_EP_ADD_RELU) return invalid("doe_ep_binary_f32: unknown op %u", op);
  if (n == 0) return DOE_OK;
  if (!a || !b || !y) return invalid("doe_ep_binary_f32: null pointer");
  if (n > kMaxElems) return invalid("doe_ep_binary_f32: n too large");
  if ((a != y && overlaps(a, n * 4, y, n * 4)) || (b != y && overlaps(b, n * 4, y, n * 4)))
    return invalid("doe_ep_binary_f32: an input partly overlaps y");
  return launch_ep_binary(op, a, b, y, n, launch_or_default(launch));
}

int doe_ep_softmax_f32(const float* x, float* y, uint64_t rows, uint32_t cols, const doe_launch* launch) {
  if (rows == 0 || cols == 0) return DOE_OK;  // ExecuteSoftmax returns early for an empty axis
  if (!x || !y) return invalid("doe_ep_softmax_f32: null pointer");
  if (rows > kMaxElems / cols) return invalid("doe_ep_softmax_f32: too many elements");
  if (x != y && overlaps(x, rows * cols * 4, y, rows * cols * 4))
    return invalid("doe_ep_softmax_f32: x and y partly overlap");
  return launch_ep_softmax(x, y, rows, cols, launch_or_default(launch));
}

int doe_ep_layernorm_f32(const float* x, const float* scale, float epsilon, float* y, uint64_t rows,
                         uint32_t cols, const doe_launch* launch) {
  if (rows == 0 || cols == 0) return DOE_OK;
  if (!x || !scale || !y) return invalid("doe_ep_layernorm_f32: null pointer");
  if (!(epsilon >= 0.0f)) return invalid("doe_ep_layernorm_f32: epsilon must be >= 0");
  if (rows > kMaxElems / cols) return invalid("doe_ep_layernorm_f32: too many elements");
  if (x != y && overlaps(x, rows * cols * 4, y, rows * cols * 4))
    return invalid("doe_ep_layernorm_f32: x and y partly overlap");
  if (overlaps(scale, (uint64_t)cols * 4, y, rows * cols * 4))
    return invalid("doe_ep_layernorm_f32: scale overlaps y");
  return launch_ep_layernorm(x, scale, epsilon, y, rows, cols, launch_or_default(launch));
}

int doe_ep_concat_f32(const float* a, const float* b, float* y, uint64_t outer, uint64_t a_axis, uint64_t b_axis,
                      uint64_t inner, const doe_launch* launch) {
  if (a_axis > kMaxElems || b_axis > kMaxElems || inner > kMaxElems || outer > kMaxElems)
    return invalid("doe_ep_concat_f32: dimension too large");
  const uint64_t a_run = a_axis * inner, b_run = b_axis * inner;
  if (a_run > kMaxElems || b_run > kMaxElems) return invalid("doe_ep_concat_f32: too many elements");
  if (outer == 0 || a_run + b_run == 0) return DOE_OK;
  if (outer > kMaxElems / (a_run + b_run)) return invalid("doe_ep_concat_f32: too many elements");
  if (!y || (a_run && !a) || (b_run && !b)) return invalid("doe_ep_concat_f32: null pointer");
  const uint64_t yb = outer * (a_run + b_run) * 4;
  if (overlaps(a, outer * a_run * 4, y, yb) || overlaps(b, outer * b_run * 4, y, yb))
    return invalid("doe_ep_concat_f32: y overlaps an input");
  return launch_ep_concat(a, b, y, outer, a_run, b_run, launch_or_default(launch));
}

int doe_ep_matmul_f32(const float* a, const float* b, const float* addend, float* y, uint32_t m, uint32_t k,
                      uint32_t n, uint32_t flags, const doe_launch* launch) {
  if (flags & ~DOE_EP_MATMUL_RELU) return invalid("doe_ep_matmul_f32: unknown flags %#x", flags);
  if (m > 0x7fffffffu || k > 0x7fffffffu || n > 0x7fffffffu)
    return invalid("doe_ep_matmul_f32: m, k and n must be below 2^31");
  if (m == 0 || n == 0) return DOE_OK;
  if ((m + 127u) / 128u > 65535u) return invalid("doe_ep_matmul_f32: m above 65535 * 128");
  if (!y || (k && (!a || !b))) return invalid("doe_ep_matmul_f32: null pointer");
  if ((uint64_t)m > (1ull << 62) / ((uint64_t)n * 4)) return invalid("doe_ep_matmul_f32: output too large");
  const uint64_t yb = (uint64_t)m * n * 4;
  if (overlaps(a, (uint64_t)m * k * 4, y, yb) || overlaps(b, (uint64_t)k * n * 4, y, yb))
    return invalid("doe_ep_matmul_f32: y overlaps a or b");
  if (addend && addend != y && overlaps(addend, yb, y, yb))
    return invalid("doe_ep_matmul_f32: addend partly overlaps y");
  return launch_ep_matmul(a, b, addend, y, m, k, n, (flags & DOE_EP_MATMUL_RELU) != 0, launch_or_default(launch));
}

uint64_t doe_ep_gemm_relu_gemm_workspace_bytes(uint32_t batch, uint32_t hidden) {
  return ((uint64_t)batch * hidden * 4 + 255) & ~uint64_t(255);
}

int doe_ep_gemm_relu_gemm_f32(const float* x, const float* w1, const float* b1, const float* w2, const float* b2,
                              float* y, uint32_t batch, uint32_t in_dim, uint32_t hidden, uint32_t out_dim,
                              const doe_launch* launch) {
  const doe_launch* l = launch_or_default(launch);
  if (batch == 0 || out_dim == 0) return DOE_OK;
  if (!b2 || !y || (hidden && (!b1 || !w2)) || (hidden && in_dim && (!x || !w1)))
    return invalid("doe_ep_gemm_relu_gemm_f32: null pointer");
  const uint64_t need = doe_ep_gemm_relu_gemm_workspace_bytes(batch, hidden);
  if (hidden && (!l->workspace || l->workspace_bytes < need))
    return invalid("doe_ep_gemm_relu_gemm_f32: the hidden activations need a workspace of %llu bytes",
                   (unsigned long long)need);
  float* h = static_cast<float*>(l->workspace);
  int rc = DOE_OK;
  if (hidden) rc = doe_ep_matmul_f32(x, w1, b1, h, batch, in_dim, hidden, DOE_EP_MATMUL_RELU, l);
  if (rc == DOE_OK) rc = doe_ep_matmul_f32(h, w2, b2, y, batch, hidden, out_dim, 0, l);
  return rc;
}

uint64_t doe_linear_workspace_bytes(uint32_t n_out, uint32_t k) { return linear_workspace(n_out, k); }

uint64_t doe_tp_buffer_bytes(uint32_t rows, uint32_t cols) { return tp_buffer_bytes(rows, cols); }

float* doe_tp_slot_ptr(void* buffer, uint32_t slot, uint32_t rows, uint32_t cols) {
  return buffer ? tp_slot_ptr(buffer, slot, rows, cols) : nullptr;
}

int doe_peer_buffer_create(uint64_t bytes, void** dev_ptr, void* ipc_handle_out) {
  if (!dev_ptr || !ipc_handle_out || bytes == 0) return invalid("doe_peer_buffer_create: bad arguments");
  void* p = nullptr;
  int rc = cuda_status(cudaMalloc(&p, bytes), "cudaMalloc(peer buffer)");
  if (rc != DOE_OK) return rc;
  rc = cuda_status(cudaMemset(p, 0, bytes), "cudaMemset(peer buffer)");
  cudaIpcMemHandle_t h;
  if (rc == DOE_OK) rc = cuda_status(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  if (rc != DOE_OK) {
    cudaFree(p);
    return rc;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return DOE_OK;
}

int doe_peer_buffer_open(const void* ipc_handle, void** dev_ptr) {
  if (!ipc_handle || !dev_ptr) return invalid("doe_peer_buffer_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int doe_peer_buffer_close(void* dev_ptr) {
  if (!dev_ptr) return DOE_OK;
  return cuda_status(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

int doe_peer_buffer_free(void* dev_ptr) {
  if (!dev_ptr) return DOE_OK;
  return cuda_status(cudaFree(dev_ptr), "cudaFree(peer buffer)");
}

int doe_tp_reduce_rmsnorm(const doe_tp_peers* peers, uint32_t slot, const void* gamma, float eps, float* h_out,
                          void* xn_out, uint32_t rows, uint32_t cols, const doe_launch* launch) {
  const char* who = "doe_tp_reduce_rmsnorm";
  if (!peers || !h_out) return invalid("%s: peers and h_out are required", who);
  if (peers->world == 0 || peers->world > DOE_TP_MAX_RANKS || peers->rank >= peers->world)
    return invalid("%s: rank %u of world %u", who, peers->rank, peers->world);
  for (uint32_t i = 0; i < peers->world; ++i)
    if (!peers->buffers[i] || reinterpret_cast<uintptr_t>(peers->buffers[i]) % 256)
      return invalid("%s: buffer %u is null or not 256-byte aligned", who, i);
  if (slot > 1) return invalid("%s: slot must be 0 or 1", who);
  if (cols == 0 || cols % 4) return invalid("%s: cols must be a positive multiple of 4", who);
  if (gamma && !xn_out) return invalid("%s: gamma needs xn_out", who);
  if (reinterpret_cast<uintptr_t>(h_out) % 16 || (gamma && (reinterpret_cast<uintptr_t>(gamma) % 8 ||
                                                            reinterpret_cast<uintptr_t>(xn_out) % 8)))
    return invalid("%s: h_out must be 16-byte aligned, gamma and xn_out 8-byte aligned", who);
  if (!(eps >= 0.0f)) return invalid("%s: eps must be >= 0", who);
  if (rows == 0) return DOE_OK;
  if (rows > 2147483647u) return invalid("%s: too many rows", who);
  return launch_tp_reduce_rmsnorm(peers, slot, gamma, eps, h_out, xn_out, rows, cols, launch_or_default(launch));
}

static int linear_checked(const char* who, const void* x, const void* w, uint32_t batch, uint32_t n_out,
                          uint32_t k, const doe_linear_out* out, const doe_linear_norm* norm,
                          const doe_launch* launch) {
  if (!x || !w || !out) return invalid("%s: x, w and out are required", who);
  if (batch == 0) return DOE_OK;
  if (batch > 32) {
    set_op_error("%s: batch %u > 32 (the kernel's MMA N)", who, batch);
    return DOE_UNSUPPORTED;
  }
  if (n_out == 0 || n_out % 128 != 0) return invalid("%s: n_out %u must be a positive multiple of 128", who, n_out);
  if (k == 0 || k % 64 != 0) return invalid("%s: k %u must be a positive multiple of 64", who, k);
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16)
    return invalid("%s: x and w must be 16-byte aligned", who);
  for (int i = 0; i < 3; ++i)
    if (reinterpret_cast<uintptr_t>(out->out[i]) % 16) return invalid("%s: outputs must be 16-byte aligned", who);
  if (out->dtype > DOE_DTYPE_F32) return invalid("%s: unknown dtype %u", who, out->dtype);
  if (out->epilogue == DOE_LINEAR_SWIGLU) {
    if (!out->out[0] || out->residual) return invalid("%s: SwiGLU writes out[0] only, without residual", who);
  } else if (out->epilogue == DOE_LINEAR_STORE) {
    uint32_t total = 0;
    bool gap = false;
    for (int i = 0; i < 3; ++i) {
      if (out->width[i] == 0) {
        gap = true;
        continue;
      }
      if (gap || out->width[i] % 128 != 0 || !out->out[i])
        return invalid("%s: segments must be leading, non-null, multiples of 128 wide", who);
      total += out->width[i];
    }
    if (total != n_out) return invalid("%s: segment widths sum to %u, n_out is %u", who, total, n_out);
    if (out->residual && (out->dtype != DOE_DTYPE_F32 || out->width[1] != 0))
      return invalid("%s: a residual needs f32 output and a single segment", who);
  } else {
    return invalid("%s: unknown epilogue %u", who, out->epilogue);
  }
  if (norm && norm->gamma) {
    if (out->epilogue != DOE_LINEAR_STORE || out->dtype != DOE_DTYPE_F32 || out->width[1] != 0)
      return invalid("%s: the norm's producer side needs a STORE product with f32 output and one segment", who);
    if (!norm->normed_out || !norm->ssq_out) return invalid("%s: gamma needs normed_out and ssq_out", who);
    if (reinterpret_cast<uintptr_t>(norm->gamma) % 16 || reinterpret_cast<uintptr_t>(norm->normed_out) % 16 ||
        reinterpret_cast<uintptr_t>(norm->ssq_out) % 4)
      return invalid("%s: gamma and normed_out must be 16-byte aligned, ssq_out 4-byte aligned", who);
  }
  if (norm && norm->ssq_in) {
    if (reinterpret_cast<uintptr_t>(norm->ssq_in) % 4) return invalid("%s: ssq_in must be 4-byte aligned", who);
    if (!(norm->eps >= 0.0f)) return invalid("%s: eps must be >= 0", who);
  }
  return launch_linear(x, w, batch, n_out, k, out, norm, launch_or_default(launch));
}

int doe_linear_bf16(const void* x, const void* w, uint32_t batch, uint32_t n_out, uint32_t k,
                    const doe_linear_out* out, const doe_launch* launch) {
  return linear_checked("doe_linear_bf16", x, w, batch, n_out, k, out, nullptr, launch);
}

int doe_linear_bf16_norm(const void* x, const void* w, uint32_t batch, uint32_t n_out, uint32_t k,
                         const doe_linear_out* out, const doe_linear_norm* norm, const doe_launch* launch) {
  return linear_checked("doe_linear_bf16_norm", x, w, batch, n_out, k, out, norm, launch);
}

}  // extern "C"
