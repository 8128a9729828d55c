// no_alloc.cu -- doe_attention_decode_f32_noalloc: the attention-decode.wgsl
// kernel for callers that cannot allocate device memory.
//
// Some embedders of this library have no way to hand it scratch memory and
// must not have it allocate any: a plugin callback whose host exposes no
// allocator for temporary buffers, a serving loop whose device memory is
// partitioned up front and must not grow mid-request, or code that records
// its launches for later replay, where an allocation in the middle would not
// be replayed.  For them this entry point runs the same split-K decode as
// doe_attention_decode_f32 but keeps its split partials in a fixed array
// compiled into the library, so the call allocates nothing.
//
// Rules of use:
//   * The scratch array is kDoeNoAllocScratchBytes (256 KiB) per device and
//     lives until the process exits on every device that loads the library.
//     A problem whose partials would not fit (num_heads x splits x
//     (head_dim + 2) floats > 256 KiB) is rejected with DOE_INVALID_ARGUMENT.
//     The limit is checked with the workspace count of the split path for
//     every problem, also for those whose splits would fit one thread-block
//     cluster and never touch the array, so the sizes accepted do not depend
//     on which launch form a device can schedule.
//   * The first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current and caches it; make that
//     first call before any stream capture on the device.  The cached address
//     lives as long as the process: after cudaDeviceReset (or a reset of the
//     device's primary context by an embedder) it is stale, so the library
//     must not be used on that device again.
//   * Every call shares the one array and leaves the previous call's partials
//     in it.  Calls whose kernels overlap on the GPU (different streams with
//     no ordering between them) race on the array and must be serialised by
//     the caller.  Nothing in the array needs to start at zero: every split
//     writes its partial row before the combine kernel reads it.
#include <mutex>

#include "common.cuh"

namespace {

constexpr uint64_t kDoeNoAllocScratchBytes = 1u << 18;
constexpr int kMaxDevices = 64;

// The scratch: split partials ([H * splits, D] outputs, then [H * splits, 2]
// (max, sum) pairs) of the decode kernels.
static __device__ __align__(256) float g_noalloc_scratch[kDoeNoAllocScratchBytes / sizeof(float)];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (set-up once per
// device, with that device current).
int scratch_address(void** out) {
  int dev = -1;
  int rc = doe::cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != DOE_OK) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    doe::set_op_error("doe_attention_decode_f32_noalloc: device ordinal %d beyond %d", dev,
                      kMaxDevices);
    return DOE_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    rc = doe::cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress");
    if (rc != DOE_OK) return rc;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DOE_OK;
}

}  // namespace

extern "C" int doe_attention_decode_f32_noalloc(const float* q, const float* k_cache,
                                                const float* v_cache, float* out,
                                                uint32_t num_heads, uint32_t head_dim,
                                                uint32_t kv_len, float scale, void* stream) {
  if (!q || !k_cache || !v_cache || !out) {
    doe::set_op_error("doe_attention_decode_f32_noalloc: null pointer");
    return DOE_INVALID_ARGUMENT;
  }
  if (head_dim == 0 || head_dim > 256) {
    doe::set_op_error("doe_attention_decode_f32_noalloc: head_dim must be 1..256 (got %u)", head_dim);
    return DOE_INVALID_ARGUMENT;
  }
  if (num_heads == 0) return DOE_OK;
  if (kv_len == 0) {
    doe::set_op_error("doe_attention_decode_f32_noalloc: kv_len must be positive");
    return DOE_INVALID_ARGUMENT;
  }
  const uint64_t need = doe::decode_f32_workspace(num_heads, head_dim, kv_len);
  if (need > kDoeNoAllocScratchBytes) {
    doe::set_op_error(
        "doe_attention_decode_f32_noalloc: %u heads x head_dim %u x kv_len %u need %llu bytes of "
        "split partials; the built-in scratch holds %llu",
        num_heads, head_dim, kv_len, (unsigned long long)need,
        (unsigned long long)kDoeNoAllocScratchBytes);
    return DOE_INVALID_ARGUMENT;
  }
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != DOE_OK) return rc;
  doe_launch l;
  l.stream = stream;
  l.workspace = scratch;
  l.workspace_bytes = kDoeNoAllocScratchBytes;
  l.status = nullptr;
  return doe::launch_decode_f32(q, k_cache, v_cache, out, num_heads, head_dim, kv_len, scale, &l);
}
