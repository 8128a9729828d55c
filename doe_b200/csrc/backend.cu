// backend.cu -- the backend surface of include/doe_cuda.h: one device, one
// stream, a handle -> device buffer map, pinned upload staging and dispatch
// of Doe kernel_dispatch commands by kernel / op name.
//
// Mirrors a Doe device backend (runtime/zig/src/backend/backend_iface.zig:13-31,
// the Vulkan one in runtime/zig/src/backend/vulkan/): buffers are keyed by the
// caller's u64 handle, created on first use and grown when a larger size is
// bound (vk_resources.zig:143-171); uploads are staged (native_runtime.zig:270-375);
// capture copies device bytes back into caller memory (vk_resources.zig:378);
// an unknown kernel is an explicit `unsupported` result, never a host
// fallback (backend_execute.zig:286-297).  Single-threaded per context, like
// the reference backends.
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

using namespace doe;

namespace {

struct DevBuffer {
  void* ptr = nullptr;
  uint64_t bytes = 0;
  std::vector<uint8_t> shadow;  // host copy of small buffers (uniforms)
  bool shadow_valid = false;
  // Writes run on the upload stream, captures on the download stream and
  // kernels on the compute stream; these events order them per buffer:
  // a write waits for the last kernel that bound the buffer (ev_used) and
  // for a capture still reading it (ev_read); a kernel waits for the writes
  // and captures before it; a capture waits for the last kernel and for a
  // write queued after it.
  cudaEvent_t ev_written = nullptr, ev_used = nullptr, ev_read = nullptr;
  bool write_pending = false, used = false, read_pending = false;
};

constexpr uint64_t kShadowMax = 64 * 1024;

uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

}  // namespace

struct doe_cuda_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;  // kernels
  cudaStream_t copy = nullptr;    // buffer writes (uploads)
  cudaStream_t down = nullptr;    // captures (downloads)
  std::unordered_map<uint64_t, DevBuffer> buffers;
  uint8_t* staging = nullptr;  // pinned host
  uint64_t staging_bytes = 0;
  uint64_t staging_used = 0;
  void* workspace = nullptr;
  uint64_t workspace_bytes = 0;
  int32_t* status_dev = nullptr;
  int32_t* status_host = nullptr;  // pinned
  bool per_command_sync = false;
  bool timestamps = false;
  // set_upload_behavior: the queue is flushed after every `submit_every`
  // buffer writes (UINT32_MAX: never, the reference's lazy default)
  int upload_mode = 0;
  int queue_wait_mode = 0;  // set_queue_wait_mode: 0 process_events, 1 wait_any
  uint32_t upload_submit_every = UINT32_MAX;
  uint32_t pending_uploads = 0;
  cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
  bool timing_open = false;
  std::string last_error;
};

namespace {

int fail(doe_cuda_ctx* ctx, int code, const char* fmt, ...) {
  char buf[768];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (ctx) ctx->last_error = buf;
  return code;
}

int cu(doe_cuda_ctx* ctx, cudaError_t e, const char* where) {
  if (e == cudaSuccess) return DOE_OK;
  return fail(ctx, DOE_CUDA_ERROR, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

int bind_device(doe_cuda_ctx* ctx) { return cu(ctx, cudaSetDevice(ctx->device), "cudaSetDevice"); }

int sync_stream(doe_cuda_ctx* ctx) {
  int rc = cu(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  if (rc == DOE_OK) rc = cu(ctx, cudaStreamSynchronize(ctx->copy), "cudaStreamSynchronize(upload)");
  if (rc == DOE_OK) rc = cu(ctx, cudaStreamSynchronize(ctx->down), "cudaStreamSynchronize(download)");
  if (rc == DOE_OK) ctx->staging_used = 0;
  return rc;
}

// A write of `b` on the upload stream waits for the last kernel that bound it
// and for a capture still reading it.
int upload_after_uses(doe_cuda_ctx* ctx, DevBuffer& b) {
  int rc = DOE_OK;
  if (b.used) rc = cu(ctx, cudaStreamWaitEvent(ctx->copy, b.ev_used, 0), "cudaStreamWaitEvent(upload)");
  if (rc == DOE_OK && b.read_pending) {
    rc = cu(ctx, cudaStreamWaitEvent(ctx->copy, b.ev_read, 0), "cudaStreamWaitEvent(upload)");
    b.read_pending = false;  // what follows this write is ordered after it
  }
  return rc;
}
// A capture of `b` on the download stream waits for the last kernel that bound
// it and for a write queued since.
int download_after_writes(doe_cuda_ctx* ctx, DevBuffer& b) {
  int rc = DOE_OK;
  if (b.used) rc = cu(ctx, cudaStreamWaitEvent(ctx->down, b.ev_used, 0), "cudaStreamWaitEvent(download)");
  if (rc == DOE_OK && b.write_pending)
    rc = cu(ctx, cudaStreamWaitEvent(ctx->down, b.ev_written, 0), "cudaStreamWaitEvent(download)");
  return rc;
}

int ensure_buffer(doe_cuda_ctx* ctx, uint64_t handle, uint64_t bytes, DevBuffer** out) {
  auto it = ctx->buffers.find(handle);
  if (it != ctx->buffers.end() && it->second.bytes >= bytes) {
    *out = &it->second;
    return DOE_OK;
  }
  void* p = nullptr;
  const uint64_t alloc = bytes < 256 ? 256 : (bytes + 255) / 256 * 256;
  int rc = cu(ctx, cudaMalloc(&p, alloc), "cudaMalloc");
  if (rc != DOE_OK) return rc;
  rc = cu(ctx, cudaMemsetAsync(p, 0, alloc, ctx->stream), "cudaMemsetAsync");
  if (rc != DOE_OK) {
    cudaFree(p);
    return rc;
  }
  DevBuffer& b = ctx->buffers[handle];
  if (!b.ev_written) {
    rc = cu(ctx, cudaEventCreateWithFlags(&b.ev_written, cudaEventDisableTiming), "cudaEventCreate");
    if (rc == DOE_OK) rc = cu(ctx, cudaEventCreateWithFlags(&b.ev_used, cudaEventDisableTiming), "cudaEventCreate");
    if (rc == DOE_OK) rc = cu(ctx, cudaEventCreateWithFlags(&b.ev_read, cudaEventDisableTiming), "cudaEventCreate");
    if (rc != DOE_OK) {
      cudaFree(p);
      return rc;
    }
  }
  if (b.ptr) {  // grow: keep the old contents (after every queued copy and kernel)
    rc = sync_stream(ctx);
    if (rc == DOE_OK)
      rc = cu(ctx, cudaMemcpyAsync(p, b.ptr, b.bytes, cudaMemcpyDeviceToDevice, ctx->stream),
              "cudaMemcpyAsync(grow)");
    if (rc == DOE_OK) rc = sync_stream(ctx);
    cudaFree(b.ptr);
    if (rc != DOE_OK) {
      b.ptr = nullptr;
      b.bytes = 0;
      cudaFree(p);
      return rc;
    }
  }
  const bool fresh = b.ptr == nullptr;
  b.ptr = p;
  b.bytes = alloc;
  // The host shadow mirrors small buffers whose every byte came from the
  // zero fill or from buffer_write; a storage binding ends that (resolve()).
  if ((fresh || b.shadow_valid) && alloc <= kShadowMax) {
    b.shadow.resize(alloc, 0);
    b.shadow_valid = true;
  } else {
    b.shadow.clear();
    b.shadow_valid = false;
  }
  // the zero fill (and any grow copy) ran on the compute stream: copies wait for it
  rc = cu(ctx, cudaEventRecord(b.ev_used, ctx->stream), "cudaEventRecord");
  if (rc != DOE_OK) return rc;
  b.used = true;
  *out = &b;
  return DOE_OK;
}

// One more buffer write was queued: flush the queue when set_upload_behavior's
// submit_every writes have accumulated (runtime/zig/src/backend/vulkan/
// backend_execute.zig:51-55).
int upload_submitted(doe_cuda_ctx* ctx) {
  if (ctx->upload_submit_every == UINT32_MAX) return DOE_OK;
  if (++ctx->pending_uploads < ctx->upload_submit_every) return DOE_OK;
  ctx->pending_uploads = 0;
  return sync_stream(ctx);
}

int ensure_staging(doe_cuda_ctx* ctx, uint64_t bytes) {
  if (ctx->staging_used + bytes <= ctx->staging_bytes) return DOE_OK;
  int rc = sync_stream(ctx);  // every staged copy has landed; reuse from the start
  if (rc != DOE_OK) return rc;
  if (bytes <= ctx->staging_bytes) return DOE_OK;
  if (ctx->staging) cudaFreeHost(ctx->staging);
  ctx->staging = nullptr;
  ctx->staging_bytes = 0;
  uint64_t want = 64ull << 20;
  while (want < bytes) want *= 2;
  rc = cu(ctx, cudaHostAlloc((void**)&ctx->staging, want, cudaHostAllocDefault), "cudaHostAlloc");
  if (rc != DOE_OK) return rc;
  ctx->staging_bytes = want;
  return DOE_OK;
}

int ensure_workspace(doe_cuda_ctx* ctx, uint64_t bytes) {
  if (bytes <= ctx->workspace_bytes) return DOE_OK;
  int rc = sync_stream(ctx);
  if (rc != DOE_OK) return rc;
  if (ctx->workspace) cudaFree(ctx->workspace);
  ctx->workspace = nullptr;
  ctx->workspace_bytes = 0;
  rc = cu(ctx, cudaMalloc(&ctx->workspace, bytes), "cudaMalloc(workspace)");
  if (rc != DOE_OK) return rc;
  ctx->workspace_bytes = bytes;
  return DOE_OK;
}

// ---- dispatch ---------------------------------------------------------------
struct Bound {
  uint8_t* ptr = nullptr;
  uint64_t size = 0;
  DevBuffer* buf = nullptr;
};

struct DispatchCtx {
  doe_cuda_ctx* ctx;
  const doe_binding* b;
  uint32_t n;
  const char* kernel;
  const char* entry_point;  // null or "" = "main"
  uint32_t x, y, z;         // workgroup counts of the command
};

const doe_binding* find_binding(const DispatchCtx& d, uint32_t binding) {
  for (uint32_t i = 0; i < d.n; ++i)
    if (d.b[i].binding == binding && d.b[i].group == 0) return &d.b[i];
  return nullptr;
}

int resolve(const DispatchCtx& d, uint32_t binding, bool required, Bound* out) {
  const doe_binding* bd = find_binding(d, binding);
  if (!bd) {
    if (!required) return DOE_OK;
    return fail(d.ctx, DOE_INVALID_ARGUMENT, "%s: binding %u is missing", d.kernel, binding);
  }
  const bool whole = bd->size == 0 || bd->size == UINT64_MAX;
  auto it = d.ctx->buffers.find(bd->handle);
  DevBuffer* buf = nullptr;
  if (it == d.ctx->buffers.end()) {
    if (whole)
      return fail(d.ctx, DOE_NOT_FOUND, "%s: binding %u names unknown handle %llu", d.kernel,
                  binding, (unsigned long long)bd->handle);
    int rc = ensure_buffer(d.ctx, bd->handle, bd->offset + bd->size, &buf);
    if (rc != DOE_OK) return rc;
  } else {
    buf = &it->second;
    if (!whole && bd->offset + bd->size > buf->bytes) {
      int rc = ensure_buffer(d.ctx, bd->handle, bd->offset + bd->size, &buf);
      if (rc != DOE_OK) return rc;
    }
  }
  if (bd->offset > buf->bytes)
    return fail(d.ctx, DOE_OUT_OF_RANGE, "%s: binding %u offset beyond its buffer", d.kernel, binding);
  buf->shadow_valid = false;  // a kernel may write a storage binding
  out->ptr = static_cast<uint8_t*>(buf->ptr) + bd->offset;
  out->size = whole ? buf->bytes - bd->offset : bd->size;
  out->buf = buf;
  return DOE_OK;
}

// Reads `n` bytes of a uniform binding from the host shadow (or the device).
int read_uniform(const DispatchCtx& d, uint32_t binding, void* dst, uint64_t n) {
  const doe_binding* bd = find_binding(d, binding);
  if (!bd) return fail(d.ctx, DOE_INVALID_ARGUMENT, "%s: uniform binding %u is missing", d.kernel, binding);
  auto it = d.ctx->buffers.find(bd->handle);
  if (it == d.ctx->buffers.end())
    return fail(d.ctx, DOE_NOT_FOUND, "%s: uniform handle %llu was never written", d.kernel,
                (unsigned long long)bd->handle);
  DevBuffer& b = it->second;
  std::memset(dst, 0, n);
  const uint64_t avail = b.bytes > bd->offset ? b.bytes - bd->offset : 0;
  const uint64_t take = n < avail ? n : avail;
  if (b.shadow_valid && bd->offset + take <= b.shadow.size()) {
    std::memcpy(dst, b.shadow.data() + bd->offset, take);
    return DOE_OK;
  }
  int rc = sync_stream(d.ctx);
  if (rc != DOE_OK) return rc;
  return cu(d.ctx, cudaMemcpy(dst, static_cast<uint8_t*>(b.ptr) + bd->offset, take,
                              cudaMemcpyDeviceToHost),
            "cudaMemcpy(uniform)");
}

int op_result(doe_cuda_ctx* ctx, int rc) {
  if (rc != DOE_OK) ctx->last_error = doe_cuda_op_last_error();
  return rc;
}

doe_launch make_launch(doe_cuda_ctx* ctx) {
  doe_launch l;
  l.stream = ctx->stream;
  l.workspace = ctx->workspace;
  l.workspace_bytes = ctx->workspace_bytes;
  l.status = ctx->status_dev;
  return l;
}

int need(const DispatchCtx& d, const Bound& b, uint64_t bytes, const char* what) {
  if (b.size < bytes)
    return fail(d.ctx, DOE_INVALID_ARGUMENT, "%s: %s binding holds %llu bytes, %llu needed",
                d.kernel, what, (unsigned long long)b.size, (unsigned long long)bytes);
  return DOE_OK;
}

#define DOE_TRY(x)                \
  do {                            \
    int _rc = (x);                \
    if (_rc != DOE_OK) return _rc; \
  } while (0)

// attention-decode.wgsl: {num_heads, head_dim, kv_len, scale}; q, k, v, out.
int run_attention_decode(const DispatchCtx& d) {
  uint32_t u[4];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  float scale;
  std::memcpy(&scale, &u[3], 4);
  const uint64_t H = u[0], D = u[1], L = u[2];
  Bound q, k, v, o;
  DOE_TRY(resolve(d, 1, true, &q));
  DOE_TRY(resolve(d, 2, true, &k));
  DOE_TRY(resolve(d, 3, true, &v));
  DOE_TRY(resolve(d, 4, true, &o));
  DOE_TRY(need(d, q, H * D * 4, "q"));
  DOE_TRY(need(d, k, H * L * D * 4, "k_cache"));
  DOE_TRY(need(d, v, H * L * D * 4, "v_cache"));
  DOE_TRY(need(d, o, H * D * 4, "output"));
  DOE_TRY(ensure_workspace(d.ctx, doe_attention_decode_f32_workspace_bytes(u[0], u[1], u[2])));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_attention_decode_f32((const float*)q.ptr, (const float*)k.ptr,
                                                   (const float*)v.ptr, (float*)o.ptr, u[0], u[1],
                                                   u[2], scale, &l));
}

// attention-prefill.wgsl: {seq_len, head_dim, num_heads, scale}; q, k, v, out [H,S,D].
int run_attention_prefill_wgsl(const DispatchCtx& d) {
  uint32_t u[4];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  float scale;
  std::memcpy(&scale, &u[3], 4);
  const uint64_t S = u[0], D = u[1], H = u[2];
  Bound q, k, v, o;
  DOE_TRY(resolve(d, 1, true, &q));
  DOE_TRY(resolve(d, 2, true, &k));
  DOE_TRY(resolve(d, 3, true, &v));
  DOE_TRY(resolve(d, 4, true, &o));
  for (const Bound* b : {&q, &k, &v, &o}) DOE_TRY(need(d, *b, H * S * D * 4, "q/k/v/output"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_attention_prefill_wgsl_f32((const float*)q.ptr, (const float*)k.ptr,
                                                         (const float*)v.ptr, (float*)o.ptr, u[0],
                                                         u[1], u[2], scale, &l));
}

// Rounds f32 query rows to f16 (nearest even), the operand type of the
// tcgen05 prefill; four elements per thread.
__global__ void query_to_f16_kernel(const float4* __restrict__ x, uint2* __restrict__ y, uint64_t n4) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = __ldcs(x + i);
    const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&lo);
    o.y = *reinterpret_cast<const uint32_t*>(&hi);
    y[i] = o;
  }
}

// The exec-v1 prefill ops in the form the tensor-core prefill computes: every
// query row of a prompt against the same prompt's keys, head_dim 128, dense
// [pos, Hkv, D] K/V from position 0, no softcap, window or kv_len buffer.
bool prefill_shape(const doe_attn_uniforms& u) {
  return u.head_dim == 128 && u.query_len == u.seq_len && u.seq_len > 0 && u.start_pos == 0 &&
         u.kv_start == 0 && u.kv_layout == 0 && u.kv_len_source == 0 && u.attn_softcap == 0.0f &&
         u.sliding_window == 0 && u.num_kv_heads != 0 && u.num_heads % u.num_kv_heads == 0;
}

// attention_prefill / attention_prefill_kv_axis_sharded on the tcgen05 prefill:
// Q is rounded to f16 into the context workspace (the kernel's operands are
// f16; K and V already are), then the prefill writes the f32 output rows.
int run_prefill_tc(const DispatchCtx& d, const doe_attn_uniforms& u, const Bound& q, const Bound& k,
                   const Bound& v, const Bound& o) {
  const uint64_t S = u.seq_len, H = u.num_heads, Hkv = u.num_kv_heads, D = u.head_dim;
  DOE_TRY(need(d, k, S * Hkv * D * 2, "K"));
  DOE_TRY(need(d, v, S * Hkv * D * 2, "V"));
  const uint64_t n = S * H * D;
  DOE_TRY(ensure_workspace(d.ctx, n * 2));
  const int threads = 256;
  const uint64_t want = (n / 4 + threads - 1) / threads;
  const unsigned blocks = (unsigned)(want < 4096 ? want : 4096);
  query_to_f16_kernel<<<blocks, threads, 0, d.ctx->stream>>>(reinterpret_cast<const float4*>(q.ptr),
                                                            static_cast<uint2*>(d.ctx->workspace), n / 4);
  DOE_TRY(cu(d.ctx, cudaGetLastError(), "query_to_f16_kernel"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_attention_prefill_f16(d.ctx->workspace, k.ptr, v.ptr, (float*)o.ptr, u.seq_len,
                                                    u.num_heads, u.num_kv_heads, u.head_dim, u.scale,
                                                    u.is_causal ? 1u : 0u, nullptr, 0, 0, &l));
}

bool aligned16(const Bound& b) { return (reinterpret_cast<uintptr_t>(b.ptr) & 15) == 0; }

// attention_head{256,512}_f16kv.wgsl and exec-v1 attention ops: the 15-word
// uniform; Q f32, K f16, V f16, output f32, kv_len_buffer, page_table.
// `prefill`: the exec-v1 prefill names, which take the tcgen05 prefill when
// the uniform is a whole-prompt prefill it computes (prefill_shape) and the
// bindings are 16-byte aligned; other uniforms run the head256 kernel.
int run_attention_online(const DispatchCtx& d, uint32_t fixed_head_dim, bool prefill = false) {
  doe_attn_uniforms u;
  DOE_TRY(read_uniform(d, 0, &u, 60));
  u.pad = 0;
  if (fixed_head_dim && u.head_dim != fixed_head_dim)
    return fail(d.ctx, DOE_INVALID_ARGUMENT, "%s: head_dim %u does not match the kernel's %u",
                d.kernel, u.head_dim, fixed_head_dim);
  Bound q, k, v, o, klb, pt;
  DOE_TRY(resolve(d, 1, true, &q));
  DOE_TRY(resolve(d, 2, true, &k));
  DOE_TRY(resolve(d, 3, true, &v));
  DOE_TRY(resolve(d, 4, true, &o));
  DOE_TRY(resolve(d, 5, u.kv_len_source != 0, &klb));
  DOE_TRY(resolve(d, 6, u.kv_layout == 2, &pt));
  const uint64_t qbytes = (uint64_t)u.query_len * u.num_heads * u.head_dim * 4;
  DOE_TRY(need(d, q, qbytes, "Q"));
  DOE_TRY(need(d, o, qbytes, "output"));
  if (u.kv_len_source != 0) DOE_TRY(need(d, klb, 4, "kv_len_buffer"));
  if (u.num_kv_heads == 0 || u.num_heads % u.num_kv_heads != 0 || u.head_dim == 0 ||
      u.head_dim > 512 || u.kv_layout > 2)
    return fail(d.ctx, DOE_INVALID_ARGUMENT, "%s: inconsistent uniform block", d.kernel);
  if (prefill && prefill_shape(u) && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o))
    return run_prefill_tc(d, u, q, k, v, o);
  doe_launch l = make_launch(d.ctx);
  GenericAttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.u = u;
  a.q = (const float*)q.ptr;
  a.k = k.ptr;
  a.v = v.ptr;
  a.out = (float*)o.ptr;
  a.kv_len_buffer = (const uint32_t*)klb.ptr;
  a.page_table = (const uint32_t*)pt.ptr;
  a.page_table_len = pt.ptr ? pt.size / 4 : 0;
  const uint64_t row_bytes = (uint64_t)u.num_kv_heads * u.head_dim * 2;
  a.kv_rows = (k.size < v.size ? k.size : v.size) / row_bytes;
  if (a.kv_rows == 0) return fail(d.ctx, DOE_INVALID_ARGUMENT, "%s: empty K/V bindings", d.kernel);
  a.q_pos_stride = (int64_t)u.num_heads * u.head_dim;
  a.q_head_stride = u.head_dim;
  a.kv_pos_stride = (int64_t)u.num_kv_heads * u.head_dim;
  a.kv_head_stride = u.head_dim;
  a.status = l.status;
  return op_result(d.ctx, launch_attn_generic(a, false, d.ctx->stream));
}

// kv_write / kv_write_shared: {heads, max_seq_len, head_dim, elem_bytes};
// k_proj, v_proj, k_cache, v_cache, positions (u32, 1 or `heads` entries).
int run_kv_write(const DispatchCtx& d) {
  uint32_t u[4];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  const uint64_t heads = u[0], max_len = u[1], D = u[2], eb = u[3];
  if (eb != 2 && eb != 4) return fail(d.ctx, DOE_INVALID_ARGUMENT, "%s: elem_bytes must be 2 or 4", d.kernel);
  Bound kp, vp, kc, vc, pos;
  DOE_TRY(resolve(d, 1, true, &kp));
  DOE_TRY(resolve(d, 2, true, &vp));
  DOE_TRY(resolve(d, 3, true, &kc));
  DOE_TRY(resolve(d, 4, true, &vc));
  DOE_TRY(resolve(d, 5, true, &pos));
  DOE_TRY(need(d, kp, heads * D * eb, "key_projection"));
  DOE_TRY(need(d, vp, heads * D * eb, "value_projection"));
  DOE_TRY(need(d, kc, heads * max_len * D * eb, "key_cache"));
  DOE_TRY(need(d, vc, heads * max_len * D * eb, "value_cache"));
  const uint32_t npos = pos.size / 4 >= heads && heads > 1 ? (uint32_t)heads : 1;
  DOE_TRY(need(d, pos, (uint64_t)npos * 4, "decode_position"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_kv_write_dense(kp.ptr, vp.ptr, kc.ptr, vc.ptr, (const uint32_t*)pos.ptr,
                                             npos, u[0], u[1], u[2], u[3], &l));
}

// kv_read: {heads, max_seq_len, head_dim, elem_bytes, read_start, read_len};
// k_cache, v_cache, k_out, v_out.
int run_kv_read(const DispatchCtx& d) {
  uint32_t u[6];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  const uint64_t heads = u[0], max_len = u[1], D = u[2], eb = u[3], len = u[5];
  Bound kc, vc, ko, vo;
  DOE_TRY(resolve(d, 1, true, &kc));
  DOE_TRY(resolve(d, 2, true, &vc));
  DOE_TRY(resolve(d, 3, true, &ko));
  DOE_TRY(resolve(d, 4, true, &vo));
  DOE_TRY(need(d, kc, heads * max_len * D * eb, "key_cache"));
  DOE_TRY(need(d, vc, heads * max_len * D * eb, "value_cache"));
  DOE_TRY(need(d, ko, heads * len * D * eb, "key_output"));
  DOE_TRY(need(d, vo, heads * len * D * eb, "value_output"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_kv_read_dense(kc.ptr, vc.ptr, ko.ptr, vo.ptr, u[0], u[4], u[5], u[1],
                                            u[2], u[3], &l));
}

// rope.wgsl / rope: {seq_len, head_dim, num_heads, position_offset}; qk (rw), freq_cis.
int run_rope(const DispatchCtx& d) {
  uint32_t u[4];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  Bound qk, fc;
  DOE_TRY(resolve(d, 1, true, &qk));
  DOE_TRY(resolve(d, 2, true, &fc));
  DOE_TRY(need(d, qk, (uint64_t)u[0] * u[2] * u[1] * 4, "qk"));
  DOE_TRY(need(d, fc, ((uint64_t)u[0] + u[3]) * (u[1] / 2) * 8, "freq_cis"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_rope_f32((float*)qk.ptr, (const float*)fc.ptr, u[0], u[2], u[1], u[3], &l));
}

// attention_paged_decode: {num_seqs, num_heads, num_kv_heads, head_dim,
// page_size, num_pages, max_pages_per_seq, kv_dtype, scale, split_pages};
// q, k_pool, v_pool, block_table, seq_lens, out, [new_k, new_v], [k_scale, v_scale].
int run_paged_decode(const DispatchCtx& d) {
  uint32_t u[10];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  float scale;
  std::memcpy(&scale, &u[8], 4);
  Bound q, kp, vp, bt, sl, o, nk, nv, ks, vs;
  DOE_TRY(resolve(d, 1, true, &q));
  DOE_TRY(resolve(d, 2, true, &kp));
  DOE_TRY(resolve(d, 3, true, &vp));
  DOE_TRY(resolve(d, 4, true, &bt));
  DOE_TRY(resolve(d, 5, true, &sl));
  DOE_TRY(resolve(d, 6, true, &o));
  DOE_TRY(resolve(d, 7, false, &nk));
  DOE_TRY(resolve(d, 8, false, &nv));
  DOE_TRY(resolve(d, 9, u[7] == DOE_KV_INT8, &ks));
  DOE_TRY(resolve(d, 10, u[7] == DOE_KV_INT8, &vs));
  const uint64_t B = u[0], H = u[1], Hkv = u[2], D = u[3], page = u[4], np = u[5], mp = u[6];
  const uint64_t eb = u[7] == DOE_KV_INT8 ? 1 : 2;
  DOE_TRY(need(d, q, B * H * D * 2, "q"));
  DOE_TRY(need(d, kp, np * page * Hkv * D * eb, "k_pool"));
  DOE_TRY(need(d, vp, np * page * Hkv * D * eb, "v_pool"));
  DOE_TRY(need(d, bt, B * mp * 4, "block_table"));
  DOE_TRY(need(d, sl, B * 4, "seq_lens"));
  DOE_TRY(need(d, o, B * H * D * 4, "out"));
  if (nk.ptr) DOE_TRY(need(d, nk, B * Hkv * D * 2, "new_k"));
  if (nv.ptr) DOE_TRY(need(d, nv, B * Hkv * D * 2, "new_v"));
  if (ks.ptr) DOE_TRY(need(d, ks, np * Hkv * page * 2, "k_scale"));
  if (vs.ptr) DOE_TRY(need(d, vs, np * Hkv * page * 2, "v_scale"));
  doe_paged_kv kv;
  kv.k_pool = kp.ptr;
  kv.v_pool = vp.ptr;
  kv.k_scale = ks.ptr;
  kv.v_scale = vs.ptr;
  kv.kv_dtype = u[7];
  kv.num_pages = u[5];
  kv.page_size = u[4];
  kv.num_kv_heads = u[2];
  kv.head_dim = u[3];
  kv.max_pages_per_seq = u[6];
  kv.block_table = (const int32_t*)bt.ptr;
  DOE_TRY(ensure_workspace(d.ctx, doe_paged_decode_workspace_bytes(&kv, u[0], u[1], u[9])));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_paged_decode(&kv, u[0], u[1], q.ptr, (const int32_t*)sl.ptr, nk.ptr,
                                           nv.ptr, scale, (float*)o.ptr, u[9], &l));
}

// kv_append_paged: {num_seqs, n_tokens, num_kv_heads, head_dim, page_size,
// num_pages, max_pages_per_seq, kv_dtype}; new_k, new_v, k_pool, v_pool,
// block_table, positions, [k_scale, v_scale].
int run_paged_append(const DispatchCtx& d) {
  uint32_t u[8];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  Bound nk, nv, kp, vp, bt, pos, ks, vs;
  DOE_TRY(resolve(d, 1, true, &nk));
  DOE_TRY(resolve(d, 2, true, &nv));
  DOE_TRY(resolve(d, 3, true, &kp));
  DOE_TRY(resolve(d, 4, true, &vp));
  DOE_TRY(resolve(d, 5, true, &bt));
  DOE_TRY(resolve(d, 6, true, &pos));
  DOE_TRY(resolve(d, 7, u[7] == DOE_KV_INT8, &ks));
  DOE_TRY(resolve(d, 8, u[7] == DOE_KV_INT8, &vs));
  const uint64_t B = u[0], T = u[1], Hkv = u[2], D = u[3], page = u[4], np = u[5], mp = u[6];
  const uint64_t eb = u[7] == DOE_KV_INT8 ? 1 : 2;
  DOE_TRY(need(d, nk, B * T * Hkv * D * 2, "new_k"));
  DOE_TRY(need(d, nv, B * T * Hkv * D * 2, "new_v"));
  DOE_TRY(need(d, kp, np * page * Hkv * D * eb, "k_pool"));
  DOE_TRY(need(d, vp, np * page * Hkv * D * eb, "v_pool"));
  DOE_TRY(need(d, bt, B * mp * 4, "block_table"));
  DOE_TRY(need(d, pos, B * 4, "positions"));
  doe_paged_kv kv;
  kv.k_pool = kp.ptr;
  kv.v_pool = vp.ptr;
  kv.k_scale = ks.ptr;
  kv.v_scale = vs.ptr;
  kv.kv_dtype = u[7];
  kv.num_pages = u[5];
  kv.page_size = u[4];
  kv.num_kv_heads = u[2];
  kv.head_dim = u[3];
  kv.max_pages_per_seq = u[6];
  kv.block_table = (const int32_t*)bt.ptr;
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_paged_append(&kv, u[0], u[1], nk.ptr, nv.ptr,
                                           (const int32_t*)pos.ptr, &l));
}

// attention_stitch: {rows, num_shards, head_dim}; partials, out.
int run_stitch(const DispatchCtx& d) {
  uint32_t u[3];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  Bound p, o;
  DOE_TRY(resolve(d, 1, true, &p));
  DOE_TRY(resolve(d, 2, true, &o));
  DOE_TRY(need(d, p, (uint64_t)u[0] * u[1] * (u[2] + 2) * 4, "partials"));
  DOE_TRY(need(d, o, (uint64_t)u[0] * u[2] * 4, "out"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_attention_stitch_f32((const float*)p.ptr, u[0], u[1], u[2],
                                                   (float*)o.ptr, &l));
}

// ---- the other kernels of the Gemma command streams -------------------------
// Element counts follow the dispatch: a 256-thread workgroup kernel with no
// bounds check of its own (gelu.wgsl, residual.wgsl) covers x * 256
// elements, clamped to its bindings' sizes.
uint64_t min3(uint64_t a, uint64_t b, uint64_t c) { return a < b ? (a < c ? a : c) : (b < c ? b : c); }

bool entry_is(const DispatchCtx& d, const char* name) {
  return d.entry_point != nullptr && std::strcmp(d.entry_point, name) == 0;
}

// rmsnorm.wgsl: {size, eps}; input, weight, output; one row per workgroup.
int run_rmsnorm(const DispatchCtx& d) {
  uint32_t u[2];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  float eps;
  std::memcpy(&eps, &u[1], 4);
  const bool offset = entry_is(d, "main_weight_offset");
  if (d.entry_point && d.entry_point[0] && !offset && !entry_is(d, "main"))
    return fail(d.ctx, DOE_UNSUPPORTED, "%s: entry point '%s' is not implemented", d.kernel, d.entry_point);
  Bound in, w, out;
  DOE_TRY(resolve(d, 1, true, &in));
  DOE_TRY(resolve(d, 2, true, &w));
  DOE_TRY(resolve(d, 3, true, &out));
  const uint64_t rows = d.x, size = u[0];
  DOE_TRY(need(d, in, rows * size * 4, "input"));
  DOE_TRY(need(d, w, size * 4, "weight"));
  DOE_TRY(need(d, out, rows * size * 4, "output"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_rmsnorm_f32((const float*)in.ptr, (const float*)w.ptr, (float*)out.ptr, d.x, u[0],
                                          eps, offset ? 1u : 0u, &l));
}

// matmul-gemv.wgsl: {rows, cols}; matrix, vector, output; row r < x.
int run_gemv(const DispatchCtx& d) {
  uint32_t u[2];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  Bound m, v, out;
  DOE_TRY(resolve(d, 1, true, &m));
  DOE_TRY(resolve(d, 2, true, &v));
  DOE_TRY(resolve(d, 3, true, &out));
  const uint64_t rows = u[0] < d.x ? u[0] : d.x, cols = u[1];
  DOE_TRY(need(d, m, rows * cols * 4, "matrix"));
  DOE_TRY(need(d, v, cols * 4, "vector"));
  DOE_TRY(need(d, out, rows * 4, "output"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_gemv_f32((const float*)m.ptr, (const float*)v.ptr, (float*)out.ptr, (uint32_t)rows,
                                       u[1], &l));
}

// matmul-tiled.wgsl: a, b, c, {M, K, N} at binding 3; C = A B row-major.
int run_matmul_tiled(const DispatchCtx& d) {
  uint32_t u[3];
  DOE_TRY(read_uniform(d, 3, u, sizeof(u)));
  Bound a, b, c;
  DOE_TRY(resolve(d, 0, true, &a));
  DOE_TRY(resolve(d, 1, true, &b));
  DOE_TRY(resolve(d, 2, true, &c));
  const uint64_t M = u[0], K = u[1], N = u[2];
  DOE_TRY(need(d, a, M * K * 4, "a"));
  DOE_TRY(need(d, b, K * N * 4, "b"));
  DOE_TRY(need(d, c, M * N * 4, "c"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_ep_matmul_f32((const float*)a.ptr, (const float*)b.ptr, nullptr, (float*)c.ptr, u[0],
                                            u[1], u[2], 0, &l));
}

// gelu.wgsl: input, output.
int run_gelu(const DispatchCtx& d) {
  Bound in, out;
  DOE_TRY(resolve(d, 0, true, &in));
  DOE_TRY(resolve(d, 1, true, &out));
  const uint64_t n = min3((uint64_t)d.x * 256, in.size / 4, out.size / 4);
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_gelu_tanh_f32((const float*)in.ptr, (float*)out.ptr, n, &l));
}

// residual.wgsl: a, b, out.
int run_residual(const DispatchCtx& d) {
  Bound a, b, out;
  DOE_TRY(resolve(d, 0, true, &a));
  DOE_TRY(resolve(d, 1, true, &b));
  DOE_TRY(resolve(d, 2, true, &out));
  const uint64_t n = min3((uint64_t)d.x * 256, a.size / 4, min3(b.size / 4, out.size / 4, UINT64_MAX));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_ep_binary_f32(DOE_EP_ADD, (const float*)a.ptr, (const float*)b.ptr, (float*)out.ptr,
                                            n, &l));
}

// sample.wgsl: {vocab_size}; logits, output_token.
int run_sample(const DispatchCtx& d) {
  uint32_t u[1];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  Bound lg, tok;
  DOE_TRY(resolve(d, 1, true, &lg));
  DOE_TRY(resolve(d, 2, true, &tok));
  DOE_TRY(need(d, lg, (uint64_t)u[0] * 4, "logits"));
  DOE_TRY(need(d, tok, 4, "output_token"));
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_argmax_f32((const float*)lg.ptr, u[0], (uint32_t*)tok.ptr, &l));
}

// gather.wgsl: {seq_len, embed_dim}; token_ids, embed_table, output.
int run_gather(const DispatchCtx& d) {
  uint32_t u[2];
  DOE_TRY(read_uniform(d, 0, u, sizeof(u)));
  Bound ids, table, out;
  DOE_TRY(resolve(d, 1, true, &ids));
  DOE_TRY(resolve(d, 2, true, &table));
  DOE_TRY(resolve(d, 3, true, &out));
  const uint64_t S = u[0], D = u[1];
  DOE_TRY(need(d, ids, S * 4, "token_ids"));
  DOE_TRY(need(d, out, S * D * 4, "output"));
  if (D == 0) return DOE_OK;
  doe_launch l = make_launch(d.ctx);
  return op_result(d.ctx, doe_gather_rows_f32((const uint32_t*)ids.ptr, (const float*)table.ptr, table.size / 4 / D,
                                              (float*)out.ptr, u[0], u[1], &l));
}

enum class Op {
  kNone,
  kDecodeWgsl,
  kPrefillWgsl,
  kOnline,
  kPrefill,
  kOnline256,
  kOnline512,
  kKvWrite,
  kKvRead,
  kRope,
  kPagedDecode,
  kPagedAppend,
  kStitch,
  kRmsNorm,
  kGemv,
  kMatmulTiled,
  kGelu,
  kResidual,
  kSample,
  kGather
};

Op lookup(const char* k) {
  if (!k) return Op::kNone;
  struct Entry {
    const char* name;
    Op op;
  };
  // WGSL kernel names of Doe's command streams and the exec-v1 op names of
  // runtime/zig/src/doe_wgsl/emit_csl_exec_v1.zig:113-180 that belong to the
  // attention / KV path; attention_paged_decode, kv_append_paged and
  // attention_stitch are this backend's batched forms.
  static const Entry table[] = {
      {"attention-decode.wgsl", Op::kDecodeWgsl},
      {"complex_attention_decode.wgsl", Op::kDecodeWgsl},
      {"attention-prefill.wgsl", Op::kPrefillWgsl},
      {"attention_head256_f16kv.wgsl", Op::kOnline256},
      {"attention_head512_f16kv.wgsl", Op::kOnline512},
      {"attention", Op::kOnline},
      {"attention_sliding", Op::kOnline},
      {"attention_prefill", Op::kPrefill},
      {"attention_prefill_kv_axis_sharded", Op::kPrefill},
      {"kv_write", Op::kKvWrite},
      {"kv_write_shared", Op::kKvWrite},
      {"kv_read", Op::kKvRead},
      {"rope.wgsl", Op::kRope},
      {"rope", Op::kRope},
      {"attention_paged_decode", Op::kPagedDecode},
      {"kv_append_paged", Op::kPagedAppend},
      {"attention_stitch", Op::kStitch},
      // the other kernels of the Gemma command streams
      {"rmsnorm.wgsl", Op::kRmsNorm},
      {"matmul-gemv.wgsl", Op::kGemv},
      {"matmul-tiled.wgsl", Op::kMatmulTiled},
      {"gelu.wgsl", Op::kGelu},
      {"residual.wgsl", Op::kResidual},
      {"sample.wgsl", Op::kSample},
      {"gather.wgsl", Op::kGather},
  };
  for (const Entry& e : table)
    if (std::strcmp(e.name, k) == 0) return e.op;
  return Op::kNone;
}

}  // namespace

extern "C" {

int doe_cuda_open(int ordinal, doe_cuda_ctx** out) {
  if (!out) return DOE_INVALID_ARGUMENT;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    set_op_error("doe_cuda_open: no CUDA device");
    return DOE_NO_DEVICE;
  }
  if (ordinal < 0 || ordinal >= n) {
    set_op_error("doe_cuda_open: ordinal %d out of range (%d devices)", ordinal, n);
    return DOE_NO_DEVICE;
  }
  doe_cuda_ctx* ctx = new doe_cuda_ctx();
  ctx->device = ordinal;
  int rc = bind_device(ctx);
  if (rc == DOE_OK) rc = cu(ctx, cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  if (rc == DOE_OK) rc = cu(ctx, cudaStreamCreateWithFlags(&ctx->copy, cudaStreamNonBlocking), "cudaStreamCreate(upload)");
  if (rc == DOE_OK) rc = cu(ctx, cudaStreamCreateWithFlags(&ctx->down, cudaStreamNonBlocking), "cudaStreamCreate(download)");
  if (rc == DOE_OK) rc = cu(ctx, cudaMalloc(&ctx->status_dev, sizeof(int32_t)), "cudaMalloc(status)");
  if (rc == DOE_OK) rc = cu(ctx, cudaMemset(ctx->status_dev, 0, sizeof(int32_t)), "cudaMemset(status)");
  if (rc == DOE_OK) rc = cu(ctx, cudaHostAlloc((void**)&ctx->status_host, sizeof(int32_t), cudaHostAllocDefault), "cudaHostAlloc(status)");
  if (rc == DOE_OK) rc = cu(ctx, cudaEventCreate(&ctx->ev_begin), "cudaEventCreate");
  if (rc == DOE_OK) rc = cu(ctx, cudaEventCreate(&ctx->ev_end), "cudaEventCreate");
  if (rc != DOE_OK) {
    set_op_error("%s", ctx->last_error.c_str());
    doe_cuda_close(ctx);
    return rc;
  }
  *out = ctx;
  return DOE_OK;
}

int doe_cuda_close(doe_cuda_ctx* ctx) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->copy) cudaStreamSynchronize(ctx->copy);
  if (ctx->down) cudaStreamSynchronize(ctx->down);
  for (auto& kv : ctx->buffers) {
    if (kv.second.ptr) cudaFree(kv.second.ptr);
    if (kv.second.ev_written) cudaEventDestroy(kv.second.ev_written);
    if (kv.second.ev_used) cudaEventDestroy(kv.second.ev_used);
    if (kv.second.ev_read) cudaEventDestroy(kv.second.ev_read);
  }
  if (ctx->staging) cudaFreeHost(ctx->staging);
  if (ctx->workspace) cudaFree(ctx->workspace);
  if (ctx->status_dev) cudaFree(ctx->status_dev);
  if (ctx->status_host) cudaFreeHost(ctx->status_host);
  if (ctx->ev_begin) cudaEventDestroy(ctx->ev_begin);
  if (ctx->ev_end) cudaEventDestroy(ctx->ev_end);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (ctx->copy) cudaStreamDestroy(ctx->copy);
  if (ctx->down) cudaStreamDestroy(ctx->down);
  delete ctx;
  return DOE_OK;
}

const char* doe_cuda_last_error(const doe_cuda_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : doe_cuda_op_last_error();
}

void* doe_cuda_stream(doe_cuda_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int doe_cuda_buffer_ensure(doe_cuda_ctx* ctx, uint64_t handle, uint64_t bytes) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  DOE_TRY(bind_device(ctx));
  DevBuffer* b;
  return ensure_buffer(ctx, handle, bytes, &b);
}

int doe_cuda_buffer_write(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset, const void* data,
                          uint64_t size) {
  if (!ctx || (!data && size)) return DOE_INVALID_ARGUMENT;
  DOE_TRY(bind_device(ctx));
  DevBuffer* b;
  DOE_TRY(ensure_buffer(ctx, handle, offset + size, &b));
  if (size == 0) return DOE_OK;
  if (b->shadow_valid) std::memcpy(b->shadow.data() + offset, data, size);
  DOE_TRY(ensure_staging(ctx, size));
  std::memcpy(ctx->staging + ctx->staging_used, data, size);
  DOE_TRY(upload_after_uses(ctx, *b));
  int rc = cu(ctx, cudaMemcpyAsync(static_cast<uint8_t*>(b->ptr) + offset,
                                   ctx->staging + ctx->staging_used, size, cudaMemcpyHostToDevice,
                                   ctx->copy),
              "cudaMemcpyAsync(H2D)");
  ctx->staging_used += (size + 255) / 256 * 256;
  if (rc == DOE_OK) rc = cu(ctx, cudaEventRecord(b->ev_written, ctx->copy), "cudaEventRecord");
  if (rc == DOE_OK) b->write_pending = true;
  if (rc == DOE_OK) rc = upload_submitted(ctx);
  return rc;
}

int doe_cuda_buffer_write_async(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset, const void* data,
                                uint64_t size) {
  if (!ctx || (!data && size)) return DOE_INVALID_ARGUMENT;
  DOE_TRY(bind_device(ctx));
  cudaPointerAttributes pa;
  if (size && (cudaPointerGetAttributes(&pa, data) != cudaSuccess || pa.type != cudaMemoryTypeHost)) {
    cudaGetLastError();
    return fail(ctx, DOE_INVALID_ARGUMENT, "deferred write: the source must be page-locked host memory");
  }
  DevBuffer* b;
  DOE_TRY(ensure_buffer(ctx, handle, offset + size, &b));
  if (size == 0) return DOE_OK;
  if (b->shadow_valid) std::memcpy(b->shadow.data() + offset, data, size);
  DOE_TRY(upload_after_uses(ctx, *b));
  DOE_TRY(cu(ctx, cudaMemcpyAsync(static_cast<uint8_t*>(b->ptr) + offset, data, size, cudaMemcpyHostToDevice,
                                  ctx->copy),
             "cudaMemcpyAsync(H2D)"));
  DOE_TRY(cu(ctx, cudaEventRecord(b->ev_written, ctx->copy), "cudaEventRecord"));
  b->write_pending = true;
  return upload_submitted(ctx);
}

int doe_cuda_set_queue_wait_mode(doe_cuda_ctx* ctx, int mode) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  if (mode != DOE_QUEUE_WAIT_PROCESS_EVENTS && mode != DOE_QUEUE_WAIT_ANY)
    return fail(ctx, DOE_INVALID_ARGUMENT, "set_queue_wait_mode: unknown mode %d", mode);
  ctx->queue_wait_mode = mode;
  return DOE_OK;
}

int doe_cuda_set_upload_behavior(doe_cuda_ctx* ctx, int mode, uint32_t submit_every) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  if (mode != DOE_UPLOAD_COPY_DST_COPY_SRC && mode != DOE_UPLOAD_COPY_DST)
    return fail(ctx, DOE_INVALID_ARGUMENT, "set_upload_behavior: unknown usage mode %d", mode);
  ctx->upload_mode = mode;
  ctx->upload_submit_every = submit_every > 0 ? submit_every : 1;
  if (ctx->pending_uploads >= ctx->upload_submit_every) {
    ctx->pending_uploads = 0;
    DOE_TRY(bind_device(ctx));
    return sync_stream(ctx);
  }
  return DOE_OK;
}

int doe_cuda_buffer_read(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset, void* dst,
                         uint64_t size) {
  if (!ctx || (!dst && size)) return DOE_INVALID_ARGUMENT;
  auto it = ctx->buffers.find(handle);
  if (it == ctx->buffers.end())
    return fail(ctx, DOE_NOT_FOUND, "capture: unknown handle %llu", (unsigned long long)handle);
  if (offset + size > it->second.bytes)
    return fail(ctx, DOE_OUT_OF_RANGE, "capture: [%llu, %llu) beyond %llu bytes",
                (unsigned long long)offset, (unsigned long long)(offset + size),
                (unsigned long long)it->second.bytes);
  if (size == 0) return DOE_OK;
  DOE_TRY(bind_device(ctx));
  // The read waits for the copy before returning, so a page-locked
  // destination can take the DMA directly (no staging hop).  Copies run on
  // the copy stream after the writes queued there and the last kernel that
  // bound the buffer.
  DOE_TRY(download_after_writes(ctx, it->second));
  cudaPointerAttributes pa;
  if (cudaPointerGetAttributes(&pa, dst) == cudaSuccess && pa.type == cudaMemoryTypeHost) {
    DOE_TRY(cu(ctx, cudaMemcpyAsync(dst, static_cast<uint8_t*>(it->second.ptr) + offset, size,
                                    cudaMemcpyDeviceToHost, ctx->down),
               "cudaMemcpyAsync(D2H)"));
    DOE_TRY(cu(ctx, cudaStreamSynchronize(ctx->down), "cudaStreamSynchronize(download)"));
    return DOE_OK;
  }
  cudaGetLastError();  // a pageable pointer is not an error
  DOE_TRY(ensure_staging(ctx, size));
  const uint64_t at = ctx->staging_used;
  ctx->staging_used += (size + 255) / 256 * 256;  // the staged uploads queued before stay intact
  DOE_TRY(cu(ctx, cudaMemcpyAsync(ctx->staging + at, static_cast<uint8_t*>(it->second.ptr) + offset, size,
                                  cudaMemcpyDeviceToHost, ctx->down),
             "cudaMemcpyAsync(D2H)"));
  DOE_TRY(cu(ctx, cudaStreamSynchronize(ctx->down), "cudaStreamSynchronize(download)"));
  std::memcpy(dst, ctx->staging + at, size);
  return DOE_OK;
}

int doe_cuda_buffer_read_async(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset, void* dst,
                               uint64_t size) {
  if (!ctx || (!dst && size)) return DOE_INVALID_ARGUMENT;
  auto it = ctx->buffers.find(handle);
  if (it == ctx->buffers.end())
    return fail(ctx, DOE_NOT_FOUND, "capture: unknown handle %llu", (unsigned long long)handle);
  if (offset + size > it->second.bytes)
    return fail(ctx, DOE_OUT_OF_RANGE, "capture: [%llu, %llu) beyond %llu bytes",
                (unsigned long long)offset, (unsigned long long)(offset + size),
                (unsigned long long)it->second.bytes);
  if (size == 0) return DOE_OK;
  DOE_TRY(bind_device(ctx));
  cudaPointerAttributes pa;
  if (cudaPointerGetAttributes(&pa, dst) != cudaSuccess || pa.type != cudaMemoryTypeHost) {
    cudaGetLastError();
    return fail(ctx, DOE_INVALID_ARGUMENT, "deferred capture: the destination must be page-locked host memory");
  }
  DOE_TRY(download_after_writes(ctx, it->second));
  DOE_TRY(cu(ctx, cudaMemcpyAsync(dst, static_cast<uint8_t*>(it->second.ptr) + offset, size, cudaMemcpyDeviceToHost,
                                  ctx->down),
             "cudaMemcpyAsync(D2H)"));
  // a later write or kernel must not change the bytes before the copy has read them
  DOE_TRY(cu(ctx, cudaEventRecord(it->second.ev_read, ctx->down), "cudaEventRecord"));
  it->second.read_pending = true;
  return DOE_OK;
}

int doe_cuda_buffer_release(doe_cuda_ctx* ctx, uint64_t handle) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  auto it = ctx->buffers.find(handle);
  if (it == ctx->buffers.end())
    return fail(ctx, DOE_NOT_FOUND, "release: unknown handle %llu", (unsigned long long)handle);
  DOE_TRY(bind_device(ctx));
  DOE_TRY(sync_stream(ctx));
  cudaFree(it->second.ptr);
  if (it->second.ev_written) cudaEventDestroy(it->second.ev_written);
  if (it->second.ev_used) cudaEventDestroy(it->second.ev_used);
  if (it->second.ev_read) cudaEventDestroy(it->second.ev_read);
  ctx->buffers.erase(it);
  return DOE_OK;
}

int doe_cuda_buffer_size(doe_cuda_ctx* ctx, uint64_t handle, uint64_t* bytes) {
  if (!ctx || !bytes) return DOE_INVALID_ARGUMENT;
  auto it = ctx->buffers.find(handle);
  if (it == ctx->buffers.end()) return DOE_NOT_FOUND;
  *bytes = it->second.bytes;
  return DOE_OK;
}

int doe_cuda_buffer_device_ptr(doe_cuda_ctx* ctx, uint64_t handle, void** out) {
  if (!ctx || !out) return DOE_INVALID_ARGUMENT;
  auto it = ctx->buffers.find(handle);
  if (it == ctx->buffers.end()) return DOE_NOT_FOUND;
  *out = it->second.ptr;
  return DOE_OK;
}

int doe_cuda_kernel_supported(const char* kernel) { return lookup(kernel) != Op::kNone; }

int doe_cuda_prewarm_kernel(doe_cuda_ctx* ctx, const char* kernel) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  if (lookup(kernel) == Op::kNone)
    return fail(ctx, DOE_UNSUPPORTED, "prewarm: kernel '%s' is not implemented by doe_cuda",
                kernel ? kernel : "(null)");
  return DOE_OK;  // kernels are compiled into the library: nothing to build
}

int doe_cuda_prewarm_upload(doe_cuda_ctx* ctx, uint64_t max_upload_bytes) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  DOE_TRY(bind_device(ctx));
  return ensure_staging(ctx, max_upload_bytes);
}

int doe_cuda_set_queue_sync_mode(doe_cuda_ctx* ctx, int per_command) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  ctx->per_command_sync = per_command != 0;
  return DOE_OK;
}

int doe_cuda_set_gpu_timestamp_mode(doe_cuda_ctx* ctx, int on) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  ctx->timestamps = on != 0;
  return DOE_OK;
}

int doe_cuda_dispatch(doe_cuda_ctx* ctx, const char* kernel, const char* entry_point, uint32_t x,
                      uint32_t y, uint32_t z, const doe_binding* bindings, uint32_t num_bindings,
                      doe_exec_result* result) {
  // The attention / KV kernels size their grids from the uniforms; x, the
  // workgroup count, sets the rows of rmsnorm.wgsl and matmul-gemv.wgsl and
  // the element count of gelu.wgsl and residual.wgsl, as in the WGSL.
  if (!ctx || (!bindings && num_bindings)) return DOE_INVALID_ARGUMENT;
  doe_exec_result res;
  std::memset(&res, 0, sizeof(res));
  const uint64_t t0 = now_ns();
  const Op op = lookup(kernel);
  const bool other_entry = entry_point && entry_point[0] && std::strcmp(entry_point, "main") != 0;
  if (other_entry && op != Op::kNone && std::strstr(kernel, ".wgsl") != nullptr &&
      !(op == Op::kRmsNorm && std::strcmp(entry_point, "main_weight_offset") == 0)) {
    res.status = DOE_UNSUPPORTED;
    if (result) *result = res;
    return fail(ctx, DOE_UNSUPPORTED, "dispatch: entry point '%s' of %s is not implemented",
                entry_point, kernel);
  }
  if (op == Op::kNone) {
    res.status = DOE_UNSUPPORTED;
    if (result) *result = res;
    return fail(ctx, DOE_UNSUPPORTED, "dispatch: kernel '%s' is not implemented by doe_cuda",
                kernel ? kernel : "(null)");
  }
  int rc = bind_device(ctx);
  DispatchCtx d{ctx, bindings, num_bindings, kernel, entry_point, x, y, z};
  // the kernel runs after the writes and captures queued for its buffers
  for (uint32_t i = 0; i < num_bindings && rc == DOE_OK && bindings; ++i) {
    auto bit = ctx->buffers.find(bindings[i].handle);
    if (bit == ctx->buffers.end()) continue;
    if (bit->second.write_pending) {
      rc = cu(ctx, cudaStreamWaitEvent(ctx->stream, bit->second.ev_written, 0), "cudaStreamWaitEvent");
      bit->second.write_pending = false;
    }
    if (rc == DOE_OK && bit->second.read_pending) {  // the kernel may overwrite bytes a capture reads
      rc = cu(ctx, cudaStreamWaitEvent(ctx->stream, bit->second.ev_read, 0), "cudaStreamWaitEvent");
      bit->second.read_pending = false;
    }
  }
  const bool timed = ctx->timestamps;
  if (rc == DOE_OK && timed) rc = cu(ctx, cudaEventRecord(ctx->ev_begin, ctx->stream), "cudaEventRecord");
  const uint64_t t1 = now_ns();
  if (rc == DOE_OK) {
    switch (op) {
      case Op::kDecodeWgsl: rc = run_attention_decode(d); break;
      case Op::kPrefillWgsl: rc = run_attention_prefill_wgsl(d); break;
      case Op::kOnline: rc = run_attention_online(d, 0); break;
      case Op::kPrefill: rc = run_attention_online(d, 0, true); break;
      case Op::kOnline256: rc = run_attention_online(d, 256); break;
      case Op::kOnline512: rc = run_attention_online(d, 512); break;
      case Op::kKvWrite: rc = run_kv_write(d); break;
      case Op::kKvRead: rc = run_kv_read(d); break;
      case Op::kRope: rc = run_rope(d); break;
      case Op::kPagedDecode: rc = run_paged_decode(d); break;
      case Op::kPagedAppend: rc = run_paged_append(d); break;
      case Op::kStitch: rc = run_stitch(d); break;
      case Op::kRmsNorm: rc = run_rmsnorm(d); break;
      case Op::kGemv: rc = run_gemv(d); break;
      case Op::kMatmulTiled: rc = run_matmul_tiled(d); break;
      case Op::kGelu: rc = run_gelu(d); break;
      case Op::kResidual: rc = run_residual(d); break;
      case Op::kSample: rc = run_sample(d); break;
      case Op::kGather: rc = run_gather(d); break;
      default: rc = DOE_UNSUPPORTED; break;
    }
  }
  if (rc == DOE_OK && timed) rc = cu(ctx, cudaEventRecord(ctx->ev_end, ctx->stream), "cudaEventRecord");
  // later writes and captures of the bound buffers wait for this kernel
  for (uint32_t i = 0; i < num_bindings && rc == DOE_OK && bindings; ++i) {
    auto bit = ctx->buffers.find(bindings[i].handle);
    if (bit != ctx->buffers.end()) {
      rc = cu(ctx, cudaEventRecord(bit->second.ev_used, ctx->stream), "cudaEventRecord");
      bit->second.used = true;
    }
  }
  const uint64_t t2 = now_ns();
  res.setup_ns = t1 - t0;
  res.encode_ns = t2 - t1;
  res.dispatch_count = rc == DOE_OK ? 1 : 0;
  res.gpu_timestamp_attempted = timed ? 1 : 0;
  if (rc == DOE_OK && ctx->per_command_sync) {
    uint64_t wait = 0;
    rc = doe_cuda_flush(ctx, &wait);
    res.submit_wait_ns = wait;
    if (rc == DOE_OK && timed) {
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, ctx->ev_begin, ctx->ev_end) == cudaSuccess) {
        res.gpu_timestamp_ns = (uint64_t)(ms * 1.0e6);
        res.gpu_timestamp_valid = 1;
      }
    }
  }
  res.status = rc == DOE_OK ? DOE_OK : (rc == DOE_UNSUPPORTED ? DOE_UNSUPPORTED : DOE_ERROR);
  if (result) *result = res;
  return rc;
}

int doe_cuda_flush(doe_cuda_ctx* ctx, uint64_t* wait_ns) {
  if (!ctx) return DOE_INVALID_ARGUMENT;
  DOE_TRY(bind_device(ctx));
  const uint64_t t0 = now_ns();
  DOE_TRY(cu(ctx, cudaMemcpyAsync(ctx->status_host, ctx->status_dev, sizeof(int32_t),
                                  cudaMemcpyDeviceToHost, ctx->stream),
             "cudaMemcpyAsync(status)"));
  DOE_TRY(sync_stream(ctx));
  if (wait_ns) *wait_ns = now_ns() - t0;
  const int32_t bits = *ctx->status_host;
  if (bits != 0) {
    DOE_TRY(cu(ctx, cudaMemsetAsync(ctx->status_dev, 0, sizeof(int32_t), ctx->stream),
               "cudaMemsetAsync(status)"));
    return fail(ctx, DOE_OUT_OF_RANGE,
                "device reported error bits 0x%x (1 page outside the pool, 2 position >= "
                "capacity, 4 sequence longer than its block table)",
                bits);
  }
  return DOE_OK;
}

}  // extern "C"
