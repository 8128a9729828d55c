/*
 * doe_cuda.h -- C ABI of libdoe_cuda.so, the sm_100a attention / KV-cache
 * backend for Doe (doerun/doe).
 *
 * Plain C types only: pointers, sizes and integer status codes.  Device
 * pointers are CUDA global-memory addresses; `stream` is a cudaStream_t
 * passed as void*.  Every entry point returns a doe_status; none of them
 * falls back to the host when a kernel cannot run.
 *
 * Two surfaces share the same kernels:
 *   1. the backend surface (doe_cuda_open ... doe_cuda_flush): a device,
 *      a stream and a handle -> buffer map driven by Doe's command model;
 *   2. the operator surface (doe_attention_*, doe_paged_*, doe_kv_*): direct
 *      launches on caller-owned device memory, which is what an ONNX Runtime
 *      plugin EP's Compute callback binds to.
 *
 * Reference citations are paths inside the doerun/doe tree.
 */
#ifndef DOE_CUDA_H
#define DOE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DOE_CUDA_ABI_VERSION 1

/* Status codes.  OK/UNSUPPORTED/ERROR mirror NativeExecutionStatus
 * (runtime/zig/src/core/abi/wgpu_execution_types.zig:1-5); the rest refine
 * ERROR the way the Zig backends return distinct error-union members.      */
typedef enum doe_status {
  DOE_OK = 0,
  DOE_UNSUPPORTED = 1,      /* unknown kernel / op, or unsupported shape   */
  DOE_ERROR = 2,            /* generic failure                              */
  DOE_INVALID_ARGUMENT = 3, /* null pointer, size mismatch, bad uniform     */
  DOE_OUT_OF_RANGE = 4,     /* position / page outside the cache            */
  DOE_NOT_FOUND = 5,        /* unknown buffer handle                        */
  DOE_CUDA_ERROR = 6,       /* a CUDA runtime call failed                   */
  DOE_NO_DEVICE = 7         /* no CUDA device (or ordinal out of range)     */
} doe_status;

/* Device-side error bits that kernels OR into a launch's status word.      */
#define DOE_DEVICE_ERR_PAGE 0x1     /* block-table entry outside the pool   */
#define DOE_DEVICE_ERR_POSITION 0x2 /* write position >= cache capacity     */
#define DOE_DEVICE_ERR_LENGTH 0x4   /* sequence longer than its block table */
#define DOE_DEVICE_ERR_TIMEOUT 0x8  /* a bounded in-kernel wait gave up     */

/* KV element types of a paged cache.                                       */
#define DOE_KV_F16 0u
#define DOE_KV_INT8 1u /* int8 symmetric + f16 scale per (token, kv head)   */

/* Launch context of the operator surface.  `workspace` is device scratch
 * of at least the op's *_workspace_bytes(); `status` is an optional device
 * int32 that kernels OR DOE_DEVICE_ERR_* bits into (read it after the stream
 * has finished).                                                           */
typedef struct doe_launch {
  void* stream;
  void* workspace;
  uint64_t workspace_bytes;
  int32_t* status;
} doe_launch;

/* ======================================================================== */
/* Library                                                                  */
/* ======================================================================== */
int doe_cuda_abi_version(void);
int doe_cuda_device_count(int* count);
/* Last error text of the calling thread for the operator surface.          */
const char* doe_cuda_op_last_error(void);

/* ======================================================================== */
/* Backend surface -- replaces the BackendVTable slots of a device backend  */
/* (runtime/zig/src/backend/backend_iface.zig:13-31).                       */
/* ======================================================================== */
typedef struct doe_cuda_ctx doe_cuda_ctx;

/* Buffer binding of a kernel_dispatch command
 * (runtime/zig/src/model_compute_types.zig:19-35 KernelBinding).           */
typedef struct doe_binding {
  uint32_t binding;
  uint32_t group;
  uint64_t handle;
  uint64_t offset;
  uint64_t size; /* 0 or UINT64_MAX = whole buffer from offset */
  uint32_t buffer_type;
  uint32_t reserved;
} doe_binding;

/* NativeExecutionResult (runtime/zig/src/core/abi/wgpu_execution_types.zig:7-17). */
typedef struct doe_exec_result {
  int32_t status;
  uint32_t dispatch_count;
  uint64_t setup_ns;
  uint64_t encode_ns;
  uint64_t submit_wait_ns;
  uint64_t gpu_timestamp_ns;
  uint32_t gpu_timestamp_attempted;
  uint32_t gpu_timestamp_valid;
} doe_exec_result;

/* init_backend arm (runtime/zig/src/backend/backend_registry.zig:12-43).   */
int doe_cuda_open(int ordinal, doe_cuda_ctx** out);
/* deinit (backend_iface.zig:14).                                           */
int doe_cuda_close(doe_cuda_ctx* ctx);
const char* doe_cuda_last_error(const doe_cuda_ctx* ctx);
/* The backend's stream (cudaStream_t), for callers that time or order work. */
void* doe_cuda_stream(doe_cuda_ctx* ctx);

/* Handle -> device buffer map (runtime/zig/src/backend/vulkan/vk_resources.zig:143-171):
 * buffers are created on first use and grown (contents kept) when a larger
 * size is requested.                                                       */
int doe_cuda_buffer_ensure(doe_cuda_ctx* ctx, uint64_t handle, uint64_t bytes);
/* execute_buffer_write_bytes (backend_iface.zig:16): host bytes go through
 * a pinned staging area and an async copy on the backend stream.           */
int doe_cuda_buffer_write(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset,
                          const void* data, uint64_t size);
/* capture_buffer (backend_iface.zig:30): waits for the stream, then copies
 * device bytes into caller memory.                                         */
int doe_cuda_buffer_read(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset,
                         void* dst, uint64_t size);
/* capture_buffer in the deferred queue mode (set_queue_wait_mode,
 * backend_iface.zig:18): the device-to-host copy is queued on the backend
 * stream after the work already queued, and the call returns at once.  `dst`
 * must be page-locked host memory (cudaHostAlloc / cudaHostRegister); its
 * bytes are valid after the next doe_cuda_flush.  A serving loop queues step
 * i + 1 while step i still runs.                                           */
int doe_cuda_buffer_read_async(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset,
                               void* dst, uint64_t size);
/* execute_buffer_write_bytes in the deferred mode: `data` must be page-locked
 * host memory, copied by DMA on the backend's copy stream after the call
 * returns (no staging copy); the caller keeps it unchanged until the next
 * doe_cuda_flush.  Ordered like doe_cuda_buffer_write.                     */
int doe_cuda_buffer_write_async(doe_cuda_ctx* ctx, uint64_t handle, uint64_t offset,
                                const void* data, uint64_t size);
int doe_cuda_buffer_release(doe_cuda_ctx* ctx, uint64_t handle);
int doe_cuda_buffer_size(doe_cuda_ctx* ctx, uint64_t handle, uint64_t* bytes);
int doe_cuda_buffer_device_ptr(doe_cuda_ctx* ctx, uint64_t handle, void** out);

/* execute_command(kernel_dispatch) (backend_iface.zig:15;
 * runtime/zig/src/backend/vulkan/backend_execute.zig:281-317).  `kernel` is a
 * WGSL kernel file name Doe's command streams use ("attention-decode.wgsl",
 * "attention-prefill.wgsl", "attention_head256_f16kv.wgsl",
 * "attention_head512_f16kv.wgsl", "rope.wgsl") or an exec-v1 op name
 * (runtime/zig/src/doe_wgsl/emit_csl_exec_v1.zig:113-180: "attention",
 * "attention_sliding", "attention_prefill", "attention_prefill_kv_axis_sharded",
 * "kv_write", "kv_write_shared", "kv_read", "rope") -- and the other kernels
 * of the Gemma command streams: "rmsnorm.wgsl" (entry points "main" and
 * "main_weight_offset"), "matmul-gemv.wgsl", "matmul-tiled.wgsl",
 * "gelu.wgsl", "residual.wgsl", "sample.wgsl", "gather.wgsl", with the
 * bindings and uniforms of bench/inference-pipeline/kernels/<name>.  Unknown names return
 * DOE_UNSUPPORTED with a message; nothing runs on the host instead.
 * The two prefill op names take the tcgen05 prefill (doe_attention_prefill_f16,
 * Q rounded to f16 first) when the 15-word uniform describes a whole prompt:
 * head_dim 128, query_len == seq_len, start_pos == kv_start == 0, dense
 * layout, kv_len from the uniform, no softcap and no window, with 16-byte
 * aligned bindings.  Other uniforms run the head256 kernel.  The kv-axis
 * sharded form's per-shard partials and host stitch (a Cerebras PE layout,
 * runtime/zig/src/doe_wgsl/emit_csl_semantic_ops.zig:560-600) collapse into
 * the one kernel, which writes the stitched output rows.                  */
int doe_cuda_dispatch(doe_cuda_ctx* ctx, const char* kernel,
                      const char* entry_point, uint32_t x, uint32_t y,
                      uint32_t z, const doe_binding* bindings,
                      uint32_t num_bindings, doe_exec_result* result);
/* 1 if `kernel` names a dispatchable kernel / op, else 0.                  */
int doe_cuda_kernel_supported(const char* kernel);
/* prewarm_kernel_dispatch (backend_iface.zig:23-29).                       */
int doe_cuda_prewarm_kernel(doe_cuda_ctx* ctx, const char* kernel);
/* prewarm_upload_path (backend_iface.zig:22): sizes the pinned staging area. */
int doe_cuda_prewarm_upload(doe_cuda_ctx* ctx, uint64_t max_upload_bytes);
/* set_upload_behavior (backend_iface.zig:17; the Vulkan backend's
 * runtime/zig/src/backend/vulkan/backend_execute.zig:514-519, used at :51-55):
 * after every `submit_every` buffer writes (doe_cuda_buffer_write and
 * doe_cuda_buffer_write_async) the queue is flushed and waited for, like
 * flush_queue; 0 counts as 1, UINT32_MAX never flushes (the default, the
 * reference's lazy batching).  `mode` is the upload buffer usage
 * (UploadBufferUsageMode, runtime/zig/src/backend/runtime_types.zig:6-9);
 * device buffers here are always copy sources and destinations, so it is
 * validated and kept but changes nothing.                                  */
#define DOE_UPLOAD_COPY_DST_COPY_SRC 0
#define DOE_UPLOAD_COPY_DST 1
int doe_cuda_set_upload_behavior(doe_cuda_ctx* ctx, int mode, uint32_t submit_every);
/* set_queue_wait_mode (backend_iface.zig:18; QueueWaitMode,
 * runtime/zig/src/backend/runtime_types.zig:11-14): how flush_queue waits.
 * As in the Vulkan backend (vulkan/native_runtime.zig:360-369) both modes
 * wait for every queued copy and kernel; the mode is validated and kept.
 * Host copies that do not wait are the separate deferred calls
 * doe_cuda_buffer_write_async / doe_cuda_buffer_read_async.              */
#define DOE_QUEUE_WAIT_PROCESS_EVENTS 0
#define DOE_QUEUE_WAIT_ANY 1
int doe_cuda_set_queue_wait_mode(doe_cuda_ctx* ctx, int mode);
/* set_queue_sync_mode (backend_iface.zig:19): 0 deferred, 1 per command.   */
int doe_cuda_set_queue_sync_mode(doe_cuda_ctx* ctx, int per_command);
/* set_gpu_timestamp_mode (backend_iface.zig:20): 0 off, 1 on.              */
int doe_cuda_set_gpu_timestamp_mode(doe_cuda_ctx* ctx, int on);
/* flush_queue (backend_iface.zig:21): waits for the stream; returns the
 * wait in ns and turns device-side error bits into a status.               */
int doe_cuda_flush(doe_cuda_ctx* ctx, uint64_t* wait_ns);

/* ======================================================================== */
/* Operator surface                                                          */
/* ======================================================================== */

/* attention-decode.wgsl (bench/inference-pipeline/kernels/attention-decode.wgsl:46-136):
 * q [H,D] f32, k_cache/v_cache [H,kv_len,D] f32, out [H,D] f32.  Split-K over
 * kv_len with a combine kernel; no kv_len limit (the WGSL kernel stops at
 * 2048, its workgroup score array).                                         */
uint64_t doe_attention_decode_f32_workspace_bytes(uint32_t num_heads,
                                                  uint32_t head_dim,
                                                  uint32_t kv_len);
int doe_attention_decode_f32(const float* q, const float* k_cache,
                             const float* v_cache, float* out,
                             uint32_t num_heads, uint32_t head_dim,
                             uint32_t kv_len, float scale,
                             const doe_launch* launch);

/* Uniform block of attention_head256_f16kv.wgsl
 * (runtime/zig/tests/tsir/real/attention_head256_f16kv/attention_head256_f16kv.wgsl:14-30). */
typedef struct doe_attn_uniforms {
  uint32_t num_heads;
  uint32_t num_kv_heads;
  uint32_t head_dim;
  uint32_t seq_len;
  uint32_t query_len;
  float scale;
  uint32_t is_causal;
  uint32_t start_pos;
  float attn_softcap;
  uint32_t sliding_window;
  uint32_t kv_len_source; /* 0: seq_len from the uniform, else kv_len_buffer[0] */
  uint32_t kv_start;
  uint32_t page_size;
  uint32_t kv_layout; /* 0 dense, 1 sliding ring, 2 paged through page_table */
  uint32_t pad;
} doe_attn_uniforms;

/* attention_head256_f16kv.wgsl main (…:72-269) for any head_dim <= 512:
 * q/out [query_len, H, D] f32, k/v [pos, Hkv, D] of `kv_elem` (0 = f16,
 * 1 = f32), optional kv_len_buffer / page_table device arrays.             */
int doe_attention_online(const doe_attn_uniforms* u, const float* q,
                         const void* k, const void* v, uint32_t kv_elem,
                         float* out, const uint32_t* kv_len_buffer,
                         const uint32_t* page_table, const doe_launch* launch);

/* attention-prefill.wgsl (bench/inference-pipeline/kernels/attention-prefill.wgsl:19-112):
 * causal, q/k/v/out [H,S,D] f32.                                            */
int doe_attention_prefill_wgsl_f32(const float* q, const float* k,
                                   const float* v, float* out, uint32_t seq_len,
                                   uint32_t head_dim, uint32_t num_heads,
                                   float scale, const doe_launch* launch);

/* Causal prefill on the tcgen05 tensor cores: the head256 online softmax with
 * query_len = seq_len, is_causal, start_pos = kv_start = 0
 * (attention_head256_f16kv.wgsl:113-136, 181-268), f16 q [S,H,D] and k/v
 * [S,Hkv,D] (the [B,S,H,D] layout with B = 1), f32 out [S,H,D], f32
 * accumulation, head_dim 128.  When `cache` is given (causal only, seq_len and
 * cache_start multiples of 16, f16 pools) the prompt's K/V rows are also
 * written into the paged cache at positions cache_start.. of block-table row
 * `cache_seq` (kv_write, runtime/zig/src/tsir/emit_kernel_body.zig:620-690).
 * Pointers must be 16-byte aligned.                                         */
int doe_attention_prefill_f16(const void* q, const void* k, const void* v,
                              float* out, uint32_t seq_len, uint32_t num_heads,
                              uint32_t num_kv_heads, uint32_t head_dim,
                              float scale, uint32_t causal,
                              const struct doe_paged_kv* cache,
                              uint32_t cache_seq, uint32_t cache_start,
                              const doe_launch* launch);

/* stitch_kv_axis_sharded_partials (bench/tools/attention_kv_axis_sharded_stitch.py:46-90):
 * partials [rows, num_shards, D+2] f32 rows [O_unnorm[D], local_max,
 * local_sum] -> out [rows, D].                                             */
int doe_attention_stitch_f32(const float* partials, uint32_t rows,
                             uint32_t num_shards, uint32_t head_dim, float* out,
                             const doe_launch* launch);

/* A paged KV cache: pools [num_pages * page_size, num_kv_heads, head_dim]
 * (attention_head256_f16kv.wgsl:51-63 kv_layout 2, row = page_table[p /
 * page] * page + p % page), one block-table row per sequence.  int8 pools
 * carry f16 scales laid out [num_pages, num_kv_heads, page_size].          */
typedef struct doe_paged_kv {
  void* k_pool;
  void* v_pool;
  void* k_scale;
  void* v_scale;
  uint32_t kv_dtype; /* DOE_KV_F16 or DOE_KV_INT8 */
  uint32_t num_pages;
  uint32_t page_size; /* a multiple of 16 */
  uint32_t num_kv_heads;
  uint32_t head_dim;
  uint32_t max_pages_per_seq;
  const int32_t* block_table; /* [num_seqs, max_pages_per_seq] device int32 */
} doe_paged_kv;

/* Batched GQA decode over a paged cache (the head256 online softmax with one
 * query per sequence, generalised to per-sequence block tables).  q [B,H,D]
 * f16, seq_lens [B] device int32 = tokens to attend (after the append),
 * out [B,H,D] f32.  When new_k/new_v ([B,Hkv,D] f16) are given, the kernel
 * first writes them at position seq_lens[b] - 1 (quantising for int8 pools):
 * the fused append + attend step.  split_pages = 0 picks a split size.     */
uint64_t doe_paged_decode_workspace_bytes(const doe_paged_kv* kv,
                                          uint32_t num_seqs, uint32_t num_heads,
                                          uint32_t split_pages);
int doe_paged_decode(const doe_paged_kv* kv, uint32_t num_seqs,
                     uint32_t num_heads, const void* q, const int32_t* seq_lens,
                     const void* new_k, const void* new_v, float scale,
                     float* out, uint32_t split_pages, const doe_launch* launch);

/* kv_write generalised to the paged cache (runtime/zig/src/tsir/emit_kernel_body.zig:620-690;
 * runtime/zig/src/tsir/emit_kernel_body_kv.zig:30-102): new_k/new_v
 * [B, n_tokens, Hkv, D] f16 written at positions[b] + t.  int8 pools are
 * quantised per (token, kv head): scale = f16(absmax/127),
 * q = clamp(rint(x/scale), -127, 127).  Unmapped pages set
 * DOE_DEVICE_ERR_PAGE and skip the row.                                    */
int doe_paged_append(const doe_paged_kv* kv, uint32_t num_seqs,
                     uint32_t n_tokens, const void* new_k, const void* new_v,
                     const int32_t* positions, const doe_launch* launch);

/* RoPE fused into the paged append and the paged decode (rope.wgsl:12-35,
 * bench/inference-pipeline/kernels/): before K rows are written -- and, in the
 * decode, before the query is used -- each is rotated at its absolute
 * position pos (positions[b] + t for the append, seq_lens[b] - 1 for the
 * decode's new token and query): pairs (i, i + D/2) become
 * x0' = x0 cos - x1 sin, x1' = x0 sin + x1 cos in f32 (each product and sum
 * rounded), with cos, sin = freq_cis[(pos * D/2 + i) * 2 + {0, 1}] (device
 * f32, rope_positions rows, 16-byte aligned), then rounded to f16 (and
 * quantised for int8 pools).  V rows are written as given.  A position
 * >= rope_positions sets DOE_DEVICE_ERR_POSITION and leaves that row
 * unrotated.  head_dim 128 (append: 1, 2, 4 or 8 kv heads).  The decode's
 * workspace is doe_paged_decode_workspace_bytes.                           */
int doe_paged_append_rope(const doe_paged_kv* kv, uint32_t num_seqs,
                          uint32_t n_tokens, const void* new_k, const void* new_v,
                          const int32_t* positions, const float* freq_cis,
                          uint32_t rope_positions, const doe_launch* launch);
int doe_paged_decode_rope(const doe_paged_kv* kv, uint32_t num_seqs,
                          uint32_t num_heads, const void* q, const int32_t* seq_lens,
                          const void* new_k, const void* new_v, float scale,
                          float* out, uint32_t split_pages, const float* freq_cis,
                          uint32_t rope_positions, const doe_launch* launch);

/* Options of the batched paged decode (doe_paged_decode_ex), the head256
 * kernel's remaining uniform words for query_len 1:
 *   freq_cis / rope_positions  RoPE of the query and the new K row, exactly as
 *                              doe_paged_decode_rope (null: none);
 *   sliding_window             0: every key; w: only the last w keys, i.e.
 *                              key positions >= seq_len - w
 *                              (attention_head256_f16kv.wgsl:129-135);
 *   attn_softcap               0: off; c: each scaled score s becomes
 *                              c * tanh(s / c) (…wgsl:197-199);
 *   flags                      DOE_DECODE_OUT_BF16: `out` is bf16 storage
 *                              [B, H, D] (each f32 result rounded to
 *                              nearest even), the input of a bf16 o_proj;
 *                              DOE_DECODE_COUNTERS_ZEROED: the workspace's
 *                              split counters are already zero (the workspace
 *                              serves paged decodes only, the first of them
 *                              on zeroed memory; every decode that sets no
 *                              DOE_DEVICE_ERR_TIMEOUT leaves them zero), so
 *                              the per-call clear is skipped;
 *                              DOE_DECODE_INPUTS_STABLE: seq_lens, the block
 *                              table and every pool row other than the rows
 *                              this call appends hold their final values
 *                              before the call is enqueued (no kernel that
 *                              may still run writes them), so the kernel
 *                              reads them and starts its first copies before
 *                              waiting for the preceding kernel (programmatic
 *                              dependent launch); q, new_k, new_v and the
 *                              RoPE table may still come from that kernel;
 *                              other bits must be 0.                       */
#define DOE_DECODE_OUT_BF16 0x1u
#define DOE_DECODE_COUNTERS_ZEROED 0x2u
#define DOE_DECODE_INPUTS_STABLE 0x4u
typedef struct doe_decode_options {
  const float* freq_cis;
  uint32_t rope_positions;
  uint32_t sliding_window;
  float attn_softcap;
  uint32_t flags;
} doe_decode_options;
int doe_paged_decode_ex(const doe_paged_kv* kv, uint32_t num_seqs,
                        uint32_t num_heads, const void* q, const int32_t* seq_lens,
                        const void* new_k, const void* new_v, float scale,
                        float* out, uint32_t split_pages,
                        const doe_decode_options* options, const doe_launch* launch);

/* kv_read over the paged cache (runtime/zig/src/tsir/emit_kernel_body.zig:692-760):
 * copies tokens [start, start+len) of sequence `seq` into k_out/v_out
 * [len, Hkv, D] (element type of the pool); int8 pools also copy scales into
 * k_scale_out/v_scale_out [len, Hkv] when given.                           */
int doe_paged_gather(const doe_paged_kv* kv, uint32_t seq, uint32_t start,
                     uint32_t len, void* k_out, void* v_out, void* k_scale_out,
                     void* v_scale_out, const doe_launch* launch);

/* Dense per-head kv_write / kv_read, the reference's own form
 * (emit_kernel_body.zig:620-760; CPU semantics
 * bench/tools/run_csl_webgpu_emulator.mjs:615-644).  proj [heads, D],
 * caches [heads, max_seq_len, D], elem_bytes 2 or 4.  positions is a device
 * u32 array of 1 (shared) or `heads` entries; position >= max_seq_len sets
 * DOE_DEVICE_ERR_POSITION and writes nothing for that head.              */
int doe_kv_write_dense(const void* k_proj, const void* v_proj, void* k_cache,
                       void* v_cache, const uint32_t* positions,
                       uint32_t num_positions, uint32_t heads,
                       uint32_t max_seq_len, uint32_t head_dim,
                       uint32_t elem_bytes, const doe_launch* launch);
int doe_kv_read_dense(const void* k_cache, const void* v_cache, void* k_out,
                      void* v_out, uint32_t heads, uint32_t read_start,
                      uint32_t read_len, uint32_t max_seq_len,
                      uint32_t head_dim, uint32_t elem_bytes,
                      const doe_launch* launch);

/* rope.wgsl (bench/inference-pipeline/kernels/rope.wgsl:12-35): qk [S,H,D]
 * f32 rotated in place with freq_cis [(pos*D/2 + i)*2 + {cos, sin}].        */
int doe_rope_f32(float* qk, const float* freq_cis, uint32_t seq_len,
                 uint32_t num_heads, uint32_t head_dim,
                 uint32_t position_offset, const doe_launch* launch);

/* ======================================================================== */
/* Decoder-block operators (a Llama-style ONNX decoder through the ORT EP). */
/* The EP's Compute for the f32 basic ops (MatMul, MatMul+Add, LayerNorm:  */
/* runtime/bridge/onnxruntime-ep/src/doe_ort_ep.cc:2165, :2302, :2062)     */
/* becomes, for bf16 decode graphs: SimplifiedLayerNormalization ->        */
/* doe_rmsnorm_bf16; MatMul with its fused Split / SwiGLU / residual Add ->  */
/* doe_linear_bf16; GroupQueryAttention with rotary -> doe_paged_decode_ex   */
/* (DOE_DECODE_OUT_BF16); the tensor-parallel AllReduce -> NCCL.            */
/* ======================================================================== */

/* out[r, c] = bf16(x[r, c] * (1 / sqrt(mean_c(x[r, :]^2) + eps)) * gamma[c])
 * x [rows, cols] f32 (the residual stream), gamma [cols] bf16, out [rows,
 * cols] bf16; cols a multiple of 4; 16-byte aligned.                       */
int doe_rmsnorm_bf16(const float* x, const void* gamma, float eps, void* out,
                     uint32_t rows, uint32_t cols, const doe_launch* launch);

/* Linear layer for decode-sized batches, y[b, n] = sum_k x[b, k] w[n, k]
 * with f32 accumulation on the tensor cores; the weights stream from HBM
 * once.  x [batch, k] bf16 with batch <= 32; w [n_out, k] bf16 (output
 * features as rows: an ONNX MatMul initializer [k, n] is transposed once at
 * load); n_out a multiple of 128, k a multiple of 64; x, w and the outputs
 * 16-byte aligned.
 * Epilogues (doe_linear_out.epilogue):
 *   DOE_LINEAR_STORE   y split into up to 3 consecutive column segments of
 *                      widths width[i] (multiples of 128, summing to n_out),
 *                      segment i written to out[i] as [batch, width[i]] in
 *                      `dtype` (a plain MatMul: one segment; the fused QKV
 *                      projection: q | k | v).  With `residual` ([batch,
 *                      n_out] f32; dtype f32; one segment) the result is
 *                      residual + y: the Add after o_proj / down_proj
 *                      (residual may alias out[0]).
 *   DOE_LINEAR_SWIGLU  w rows come in 128-row blocks of 64 gate rows then the
 *                      64 matching up rows; out[0] [batch, n_out / 2] =
 *                      silu(gate) * up in `dtype` (silu(g) = g / (1 + e^-g)).
 * n_out at most 2^21.
 * Workspace: at least doe_linear_workspace_bytes(n_out, k) bytes (the same
 * for every shape).  It starts with per-tile arrival counters that must be
 * zero before the first call on that workspace; every call that sets no
 * DOE_DEVICE_ERR_TIMEOUT leaves them zero again, so one zeroed workspace
 * serves any number of calls, of any shapes, that run one after another on
 * a stream.                                                                */
#define DOE_LINEAR_STORE 0u
#define DOE_LINEAR_SWIGLU 1u
#define DOE_DTYPE_BF16 0u
#define DOE_DTYPE_F16 1u
#define DOE_DTYPE_F32 2u
typedef struct doe_linear_out {
  void* out[3];
  uint32_t width[3];       /* 0 = segment unused                           */
  uint32_t dtype;          /* DOE_DTYPE_*                                   */
  uint32_t epilogue;       /* DOE_LINEAR_*                                  */
  const float* residual;   /* DOE_LINEAR_STORE with dtype f32, or null      */
} doe_linear_out;
uint64_t doe_linear_workspace_bytes(uint32_t n_out, uint32_t k);
int doe_linear_bf16(const void* x, const void* w, uint32_t batch, uint32_t n_out,
                    uint32_t k, const doe_linear_out* out, const doe_launch* launch);

/* doe_linear_bf16 with an RMSNorm split over the two products around it, in
 * place of the SimplifiedLayerNormalization between them (doe_rmsnorm_bf16)
 * when no tensor-parallel reduction sits in between.  It has no counterpart
 * of its own in the reference, whose graph runs the norm as its own node.
 *   producer (gamma set): a DOE_LINEAR_STORE product with dtype f32 and one
 *     segment (the o_proj / down_proj writing the residual stream h) also
 *     writes normed_out [batch, n_out] bf16 = bf16(h * gamma) and ssq_out
 *     [n_out / 32][32] f32, the sum of h^2 over each 32 columns for each
 *     batch row (0 for rows past batch);
 *   consumer (ssq_in set): a product whose x is such a normed_out and ssq_in
 *     its ssq_out (k = the producer's n_out) multiplies row b of its result
 *     by 1 / sqrt(sum_i ssq_in[i][b] / k + eps) before its epilogue, so y =
 *     W (rmsnorm(h) * gamma) with the norm's scale applied after the product
 *     instead of before the bf16 rounding of x.  The blocks are summed in a
 *     fixed order: results do not depend on timing.
 * Either side may be absent; norm null is doe_linear_bf16.                 */
typedef struct doe_linear_norm {
  const void* gamma;      /* producer: bf16 [n_out], or null; 16-byte aligned */
  void* normed_out;       /* producer: bf16 [batch, n_out]; 16-byte aligned */
  float* ssq_out;         /* producer: f32 [n_out / 32][32]                 */
  const float* ssq_in;    /* consumer: f32 [k / 32][32], or null            */
  float eps;              /* consumer: >= 0                                 */
} doe_linear_norm;
int doe_linear_bf16_norm(const void* x, const void* w, uint32_t batch, uint32_t n_out,
                         uint32_t k, const doe_linear_out* out, const doe_linear_norm* norm,
                         const doe_launch* launch);

/* Tensor-parallel reduction fused into the RMSNorm that consumes it (the
 * AllReduce after o_proj / down_proj, one process per GPU of one node).
 * Every rank owns one peer buffer of doe_tp_buffer_bytes(rows, cols) bytes,
 * created by doe_peer_buffer_create and mapped into the other ranks by
 * doe_peer_buffer_open on the exported IPC handle (64 bytes).  Layout:
 * 8 u64 arrival flags (written by the peers), this rank's epoch and exit
 * counters, then 2 slots of [rows, cols] f32 partial sums.  A linear layer
 * writes its partial product into slot s of its own buffer
 * (doe_tp_slot_ptr); doe_tp_reduce_rmsnorm then, on every rank:
 *   - tells every peer that its slot is complete (a system-scope release
 *     store of the call's epoch into the peer's flag for this rank);
 *   - waits (bounded; DOE_DEVICE_ERR_TIMEOUT on expiry) for every peer's flag;
 *   - sums the world partials of slot s row by row in rank order over
 *     NVLink, so every rank gets bit-identical sums, writes them to h_out
 *     [rows, cols] f32, and, with gamma, writes
 *     xn_out = bf16(h * (1 / sqrt(mean(h^2) + eps)) * gamma) like
 *     doe_rmsnorm_bf16.
 * All ranks make the same sequence of calls.  Two slots suffice when the
 * calls alternate them: a rank overwrites slot s only after a later reduce
 * saw every peer's flag, which peers raise after reading slot s.  Buffers
 * start zeroed; cols a multiple of 4; world <= 8.
 * After a call that set DOE_DEVICE_ERR_TIMEOUT, its h_out / xn_out are not
 * valid (a late peer's slot may have been read before it was complete) and
 * the ranks' epochs no longer agree: the peer buffers must be freed and
 * created again, zeroed, on every rank before the next reduction.          */
#define DOE_TP_MAX_RANKS 8
typedef struct doe_tp_peers {
  uint32_t rank;
  uint32_t world;
  void* buffers[DOE_TP_MAX_RANKS]; /* every rank's buffer, mapped here; [rank] = own */
} doe_tp_peers;
uint64_t doe_tp_buffer_bytes(uint32_t rows, uint32_t cols);
float* doe_tp_slot_ptr(void* buffer, uint32_t slot, uint32_t rows, uint32_t cols);
int doe_peer_buffer_create(uint64_t bytes, void** dev_ptr, void* ipc_handle_out);
int doe_peer_buffer_open(const void* ipc_handle, void** dev_ptr);
int doe_peer_buffer_close(void* dev_ptr);
int doe_peer_buffer_free(void* dev_ptr);
int doe_tp_reduce_rmsnorm(const doe_tp_peers* peers, uint32_t slot, const void* gamma,
                          float eps, float* h_out, void* xn_out, uint32_t rows,
                          uint32_t cols, const doe_launch* launch);

/* ======================================================================== */
/* Allocation-free f32 decode.  This entry point has no counterpart in the   */
/* reference; it exists for callers that cannot allocate device memory.      */
/* ======================================================================== */

/* Bytes of the scratch array compiled into the library (one per device).   */
#define DOE_NOALLOC_SCRATCH_BYTES (1u << 18)

/* doe_attention_decode_f32 without a workspace argument, for embedders that
 * cannot hand the library scratch memory and must not have it allocate any
 * (a plugin callback with no allocator for temporaries, a serving loop whose
 * device memory is fixed up front).  The split partials live in a 256 KiB
 * array inside the library, held on every device that loads it until the
 * process exits.  The call allocates nothing: no cudaMalloc / cudaFree.
 *   - Problems whose partials exceed DOE_NOALLOC_SCRATCH_BYTES (num_heads x
 *     splits x (head_dim + 2) floats, as doe_attention_decode_f32_workspace_bytes
 *     counts them) return DOE_INVALID_ARGUMENT.  The limit applies to every
 *     problem, also to those whose splits fit one thread-block cluster and
 *     keep their partials in shared memory, so whether a size is accepted
 *     does not depend on the device.
 *   - The first call on a device looks up the array's device address; make
 *     it before any stream capture on that device.  The address is kept for
 *     the life of the process: the library must not be used on a device
 *     after cudaDeviceReset (or any reset of its primary context).
 *   - All calls share the array: calls whose kernels may overlap on the GPU
 *     race and must be ordered by the caller.
 * `stream` is a cudaStream_t (NULL = legacy default stream).               */
int doe_attention_decode_f32_noalloc(const float* q, const float* k_cache,
                                     const float* v_cache, float* out,
                                     uint32_t num_heads, uint32_t head_dim,
                                     uint32_t kv_len, float scale, void* stream);

/* ======================================================================== */
/* ONNX Runtime plugin EP basic operators (f32), on device tensors.  Each    */
/* replaces one of the EP's host compute kernels                            */
/* (runtime/bridge/onnxruntime-ep/src/doe_ort_ep.cc), with the same         */
/* arithmetic in f32; reductions may sum in another order (agreement with   */
/* the host loops is within 1e-5 * max(|ref|, 1)).  Tensors are dense and    */
/* row-major; element-wise and row ops may run in place (y == x).  Shape    */
/* rules the EP checks before Compute (ValidateSameRuntimeShape,           */
/* ValidateRuntimeMatMulShape, doe_ort_ep.cc:1864-1897) are the caller's;   */
/* sizes that cannot be valid are rejected with DOE_INVALID_ARGUMENT.       */
/* ======================================================================== */
#define DOE_EP_IDENTITY 0u /* ExecuteIdentity  :1919  y = x                 */
#define DOE_EP_RELU 1u     /* ExecuteRelu      :1955  y = x < 0 ? 0 : x     */
#define DOE_EP_SIGMOID 2u  /* ExecuteSigmoid   :1971  y = 1 / (1 + e^-x)    */
#define DOE_EP_TANH 3u     /* ExecuteTanh      :1987  y = tanh(x)           */
#define DOE_EP_GELU 4u     /* ExecuteGelu      :2003  0.5x(1 + erf(x/sqrt2)) */
#define DOE_EP_ADD 0u      /* ExecuteAdd       :1933  y = a + b             */
#define DOE_EP_ADD_RELU 1u /* ExecuteAddRelu   :2380  y = relu(a + b)       */
#define DOE_EP_MATMUL_RELU 0x1u /* doe_ep_matmul_f32 flag: relu(. + addend) */

/* y[i] = op(x[i]) for i < n (op: DOE_EP_IDENTITY .. DOE_EP_GELU).          */
int doe_ep_unary_f32(uint32_t op, const float* x, float* y, uint64_t n,
                     const doe_launch* launch);
/* y[i] = op(a[i], b[i]) (op: DOE_EP_ADD, DOE_EP_ADD_RELU).                 */
int doe_ep_binary_f32(uint32_t op, const float* a, const float* b, float* y,
                      uint64_t n, const doe_launch* launch);
/* ExecuteSoftmax :2021: each of `rows` rows of `cols`:
 * y = exp(x - max) * (sum != 0 ? 1 / sum : 0).  cols == 0 is a no-op.     */
int doe_ep_softmax_f32(const float* x, float* y, uint64_t rows, uint32_t cols,
                       const doe_launch* launch);
/* ExecuteLayerNorm :2062 (scale only; the EP uses epsilon 1e-5):
 * y = (x - mean) * (1 / sqrt(var + epsilon)) * scale[c], var the mean
 * squared deviation, per row of `cols`; scale [cols].                      */
int doe_ep_layernorm_f32(const float* x, const float* scale, float epsilon,
                         float* y, uint64_t rows, uint32_t cols,
                         const doe_launch* launch);
/* ExecuteConcat :2110: a [outer, a_axis, inner] and b [outer, b_axis,
 * inner] -> y [outer, a_axis + b_axis, inner] (a first).  y must not
 * overlap a or b.                                                          */
int doe_ep_concat_f32(const float* a, const float* b, float* y, uint64_t outer,
                      uint64_t a_axis, uint64_t b_axis, uint64_t inner,
                      const doe_launch* launch);
/* ExecuteMatMul :2165, ExecuteGemm :2197, ExecuteMatMulAdd :2302,
 * ExecuteMatMulAddRelu :2341: y[m, n] = sum_k a[m, k] b[k, n]
 * (+ addend[m, n] when addend != NULL) (then relu with DOE_EP_MATMUL_RELU).
 * a [m, k], b [k, n], addend and y [m, n]; y must not overlap a or b;
 * m, k and n below 2^31.                                                  */
int doe_ep_matmul_f32(const float* a, const float* b, const float* addend,
                      float* y, uint32_t m, uint32_t k, uint32_t n,
                      uint32_t flags, const doe_launch* launch);
/* ExecuteGemmReluGemm :2236: h = relu(x w1 + b1), y = h w2 + b2 with x
 * [batch, in], w1 [in, hidden], b1 [batch, hidden], w2 [hidden, out], b2
 * and y [batch, out].  h lives in launch->workspace, which must hold
 * doe_ep_gemm_relu_gemm_workspace_bytes(batch, hidden) bytes.              */
uint64_t doe_ep_gemm_relu_gemm_workspace_bytes(uint32_t batch, uint32_t hidden);
int doe_ep_gemm_relu_gemm_f32(const float* x, const float* w1, const float* b1,
                              const float* w2, const float* b2, float* y,
                              uint32_t batch, uint32_t in_dim, uint32_t hidden,
                              uint32_t out_dim, const doe_launch* launch);

/* ======================================================================== */
/* The other kernels of Doe's Gemma inference command streams              */
/* (examples/inference_gemma3_*_commands.json), so every kernel_dispatch of */
/* a stream runs on this backend.  Each restates one WGSL kernel of         */
/* bench/inference-pipeline/kernels/ in f32; reductions may sum in another  */
/* order (agreement within 1e-5 * max(|ref|, 1)).  residual.wgsl is         */
/* doe_ep_binary_f32(DOE_EP_ADD) and matmul-tiled.wgsl is                    */
/* doe_ep_matmul_f32 (C = A B, row-major).                                   */
/* ======================================================================== */

/* rmsnorm.wgsl main (:14-52) / main_weight_offset (:54-90): for each of
 * `rows` rows of `size` floats, out = x * (1 / sqrt(sum(x^2) / size + eps))
 * * g with g = weight[i] (weight_offset 0) or 1 + weight[i] (1).          */
int doe_rmsnorm_f32(const float* x, const float* weight, float* out, uint32_t rows,
                    uint32_t size, float eps, uint32_t weight_offset,
                    const doe_launch* launch);
/* matmul-gemv.wgsl (:1-74): out[r] = sum_c matrix[r * cols + c] * vector[c]
 * for r < rows.                                                            */
int doe_gemv_f32(const float* matrix, const float* vector, float* out, uint32_t rows,
                 uint32_t cols, const doe_launch* launch);
/* gelu.wgsl (:1-12): y = 0.5 x (1 + tanh(clamp(0.7978845608 (x + 0.044715
 * x^3), -15, 15))).                                                        */
int doe_gelu_tanh_f32(const float* x, float* y, uint64_t n, const doe_launch* launch);
/* sample.wgsl main (:1-52): token[0] = argmax of logits[0, n).  A logit
 * counts only if it is greater than -1e30; among equal maxima the one with
 * the smallest index mod 256, then the smallest index, wins (the kernel's
 * 256-thread strided scan and left-leaning tree); with none, 0.             */
int doe_argmax_f32(const float* logits, uint32_t n, uint32_t* token, const doe_launch* launch);
/* gather.wgsl (:1-24): out[s, d] = table[ids[s] * dim + d] for s < seq_len,
 * d < dim; an id >= table_rows sets DOE_DEVICE_ERR_PAGE and writes zeros.   */
int doe_gather_rows_f32(const uint32_t* ids, const float* table, uint64_t table_rows,
                        float* out, uint32_t seq_len, uint32_t dim,
                        const doe_launch* launch);

/* ======================================================================== */
/* Host KV page pool -- hands out physical pages and keeps the per-sequence  */
/* block tables that the paged kernels read (the reference takes one         */
/* page_table binding per dispatch, attention_head256_f16kv.wgsl:38).       */
/* ======================================================================== */
typedef struct doe_kv_pool doe_kv_pool;
int doe_kv_pool_create(uint32_t num_pages, uint32_t page_size,
                       uint32_t max_seqs, uint32_t max_pages_per_seq,
                       doe_kv_pool** out);
int doe_kv_pool_destroy(doe_kv_pool* pool);
/* Make sequence `seq` able to hold `tokens` tokens (allocates pages).      */
int doe_kv_pool_reserve(doe_kv_pool* pool, uint32_t seq, uint32_t tokens);
int doe_kv_pool_release(doe_kv_pool* pool, uint32_t seq);
int doe_kv_pool_free_pages(const doe_kv_pool* pool, uint32_t* out);
int doe_kv_pool_seq_pages(const doe_kv_pool* pool, uint32_t seq, uint32_t* out);
/* Writes the [max_seqs, max_pages_per_seq] int32 table (-1 = unmapped).    */
int doe_kv_pool_block_table(const doe_kv_pool* pool, int32_t* out,
                            uint64_t out_entries);

#ifdef __cplusplus
}
#endif

#endif /* DOE_CUDA_H */
