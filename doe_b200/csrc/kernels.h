// kernels.h -- internal launch entry points shared by the translation units
// of libdoe_cuda.so (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/doe_cuda.h"

namespace doe {

// Launch `kernel` with programmatic stream serialization: it may start while
// the previous kernel on `st` finishes (it must call pdl_wait first).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

void set_op_error(const char* fmt, ...);

// Per-device state of the host launchers (function attributes, occupancy
// answers) is kept for ordinals below kMaxDevices.
constexpr int kMaxDevices = 64;
// The current device's ordinal, or -1 (with the op error set) when there is
// none or it is not below kMaxDevices.
int current_device();
// Runs `set` (returning a doe status) once per device for one call site's
// flags; a failure is returned and the next call tries again.
template <typename F>
int once_per_device(std::atomic<bool> (&done)[kMaxDevices], F&& set) {
  const int dev = current_device();
  if (dev < 0) return DOE_CUDA_ERROR;
  if (done[dev].load(std::memory_order_acquire)) return DOE_OK;
  const int rc = set();
  if (rc == DOE_OK) done[dev].store(true, std::memory_order_release);
  return rc;
}
int cuda_status(cudaError_t err, const char* where);

// Arguments of the head256-semantics online-softmax kernel (attn_generic.cu).
struct GenericAttnArgs {
  doe_attn_uniforms u;
  const float* q;
  const void* k;
  const void* v;
  float* out;
  const uint32_t* kv_len_buffer;
  const uint32_t* page_table;
  uint64_t page_table_len;  // entries; 0 = unchecked
  uint64_t kv_rows;         // rows in K/V; 0 = unchecked
  int64_t q_pos_stride, q_head_stride;    // elements of q / out
  int64_t kv_pos_stride, kv_head_stride;  // elements of k / v
  int32_t* status;
};

int launch_attn_generic(const GenericAttnArgs& a, bool kv_f32, cudaStream_t st);

uint64_t decode_f32_workspace(uint32_t num_heads, uint32_t head_dim, uint32_t kv_len);
int launch_decode_f32(const float* q, const float* k, const float* v, float* out,
                      uint32_t num_heads, uint32_t head_dim, uint32_t kv_len, float scale,
                      const doe_launch* launch);
int launch_combine_natural(const float* part_o, const float* part_ml, float* out, int rows,
                           int fixed_len, int split_tokens, int max_splits, int head_dim,
                           cudaStream_t st);
int launch_paged_decode(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t num_heads,
                        const void* q, const int32_t* seq_lens, const void* new_k,
                        const void* new_v, float scale, float* out, uint32_t split_pages,
                        const doe_decode_options* opts, const doe_launch* launch,
                        uint64_t* ws_needed_out);
int launch_paged_append(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t n_tokens,
                        const void* new_k, const void* new_v, const int32_t* positions,
                        const float* freq_cis, uint32_t rope_positions, const doe_launch* launch);
int launch_paged_gather(const doe_paged_kv* kv, uint32_t seq, uint32_t start, uint32_t len,
                        void* k_out, void* v_out, void* ks_out, void* vs_out,
                        const doe_launch* launch);
int launch_kv_write_dense(const void* k_proj, const void* v_proj, void* k_cache, void* v_cache,
                          const uint32_t* positions, uint32_t num_positions, uint32_t heads,
                          uint32_t max_seq_len, uint32_t head_dim, uint32_t elem_bytes,
                          const doe_launch* launch);
int launch_kv_read_dense(const void* k_cache, const void* v_cache, void* k_out, void* v_out,
                         uint32_t heads, uint32_t read_start, uint32_t read_len,
                         uint32_t max_seq_len, uint32_t head_dim, uint32_t elem_bytes,
                         const doe_launch* launch);
int launch_stitch(const float* partials, uint32_t rows, uint32_t num_shards, uint32_t head_dim,
                  float* out, const doe_launch* launch);
int launch_prefill_f16(const void* q, const void* k, const void* v, float* out, uint32_t seq_len,
                       uint32_t num_heads, uint32_t num_kv_heads, float scale, uint32_t causal,
                       const doe_paged_kv* cache, uint32_t cache_seq, uint32_t cache_start,
                       const doe_launch* launch);
uint64_t linear_workspace(uint32_t n_out, uint32_t k);
int launch_linear(const void* x, const void* w, uint32_t batch, uint32_t n_out, uint32_t k,
                  const doe_linear_out* out, const doe_linear_norm* norm, const doe_launch* launch);
int launch_rmsnorm(const float* x, const void* gamma, float eps, void* out, uint32_t rows, uint32_t cols,
                   const doe_launch* launch);
int num_sms();  // of the current device, cached per device

// ORT plugin EP basic operators (ep_ops.cu)
int launch_ep_unary(uint32_t op, const float* x, float* y, uint64_t n, const doe_launch* launch);
int launch_ep_binary(uint32_t op, const float* a, const float* b, float* y, uint64_t n, const doe_launch* launch);
int launch_ep_softmax(const float* x, float* y, uint64_t rows, uint32_t cols, const doe_launch* launch);
int launch_ep_layernorm(const float* x, const float* scale, float eps, float* y, uint64_t rows, uint32_t cols,
                        const doe_launch* launch);
int launch_ep_concat(const float* a, const float* b, float* y, uint64_t outer, uint64_t a_run, uint64_t b_run,
                     const doe_launch* launch);
int launch_ep_matmul(const float* a, const float* b, const float* addend, float* y, uint32_t m, uint32_t k,
                     uint32_t n, bool relu, const doe_launch* launch);
uint64_t tp_buffer_bytes(uint32_t rows, uint32_t cols);
float* tp_slot_ptr(void* buffer, uint32_t slot, uint32_t rows, uint32_t cols);
int launch_tp_reduce_rmsnorm(const doe_tp_peers* p, uint32_t slot, const void* gamma, float eps, float* h_out,
                             void* xn_out, uint32_t rows, uint32_t cols, const doe_launch* launch);
int launch_rope(float* qk, const float* freq_cis, uint32_t seq_len, uint32_t num_heads,
                uint32_t head_dim, uint32_t position_offset, const doe_launch* launch);

}  // namespace doe
