// pipeline_ops.cu -- the non-attention kernels of Doe's Gemma inference
// command streams (examples/inference_gemma3_*_commands.json), so a whole
// stream's kernel_dispatch commands run on this backend:
//   rmsnorm.wgsl      RMSNorm over rows of f32 (plus the 1 + w weight form)
//   matmul-gemv.wgsl  out[r] = dot(matrix[r, :], vector), f32
//   gelu.wgsl         tanh-form GELU with the inner argument clamped to +-15
//   sample.wgsl       argmax over the logits, with the reference's tie order
//   gather.wgsl       embedding rows of token ids
// (residual.wgsl and matmul-tiled.wgsl are the EP's Add and f32 MatMul.)
// Sources: bench/inference-pipeline/kernels/<name>.wgsl.  These are f32
// HBM- or latency-bound kernels; none is GEMM-shaped enough for the tensor
// cores at f32 parity (the f32 bar is 1e-5, TF32 keeps 10 mantissa bits).
#include "common.cuh"

namespace doe {
namespace pl {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (int)(blockDim.x >> 5) ? red[l] : 0.0f;
    v = warp_sum(v);
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// rmsnorm.wgsl main / main_weight_offset: one CTA per row,
// out = x * (1 / sqrt(mean(x^2) + eps)) * (w or 1 + w).
template <bool OFFSET>
__global__ void __launch_bounds__(kThreads) rmsnorm_f32_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               float* __restrict__ out, uint32_t size, float eps) {
  __shared__ float red[32];
  const size_t base = (size_t)blockIdx.x * size;
  float s = 0.0f;
  for (uint32_t i = threadIdx.x; i < size; i += kThreads) {
    const float v = x[base + i];
    s = fmaf(v, v, s);
  }
  const float total = block_sum(s, red);
  const float rms = 1.0f / sqrtf(total / (float)size + eps);
  for (uint32_t i = threadIdx.x; i < size; i += kThreads) {
    const float g = OFFSET ? 1.0f + w[i] : w[i];
    out[base + i] = x[base + i] * rms * g;
  }
}

// matmul-gemv.wgsl: one warp per matrix row, float4 loads (four in flight
// per lane) when rows are 16-byte aligned, a shuffle reduction.
template <bool VEC>
__global__ void __launch_bounds__(kThreads) gemv_f32_kernel(const float* __restrict__ m, const float* __restrict__ v,
                                                            float* __restrict__ out, uint32_t rows, uint32_t cols) {
  const uint32_t row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* mr = m + (size_t)row * cols;
  float acc = 0.0f;
  if (VEC) {
    const float4* m4 = reinterpret_cast<const float4*>(mr);
    const float4* v4 = reinterpret_cast<const float4*>(v);
    const uint32_t n4 = cols / 4;
    uint32_t c = lane;
    for (; c + 96 < n4; c += 128) {
      float4 a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = __ldcs(m4 + c + 32 * u);
        b[u] = __ldg(v4 + c + 32 * u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) acc += a[u].x * b[u].x + a[u].y * b[u].y + a[u].z * b[u].z + a[u].w * b[u].w;
    }
    for (; c < n4; c += 32) {
      const float4 a = __ldcs(m4 + c), b = __ldg(v4 + c);
      acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
    }
    for (uint32_t t = n4 * 4 + lane; t < cols; t += 32) acc += mr[t] * v[t];
  } else {
    for (uint32_t t = lane; t < cols; t += 32) acc += mr[t] * __ldg(v + t);
  }
  acc = warp_sum(acc);
  if (lane == 0) out[row] = acc;
}

// gelu.wgsl: 0.5 x (1 + tanh(clamp(0.7978845608 (x + 0.044715 x^3), -15, 15))).
__global__ void __launch_bounds__(kThreads) gelu_tanh_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                             uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    const float inner = 0.7978845608f * (v + 0.044715f * v * v * v);
    y[i] = 0.5f * v * (1.0f + tanhf(fminf(fmaxf(inner, -15.0f), 15.0f)));
  }
}

// sample.wgsl's argmax: a logit counts only if it is > -1e30 (NaN never);
// among equal maxima the reference's 256-thread strided scan and left-leaning
// tree keep the smallest (index mod 256), then the smallest index; with no
// counted logit the token is 0.  (value, order key) pairs reduce with that
// rule in any grouping, so the result matches for any thread layout.
struct Best {
  float v;
  uint32_t i;
};
__device__ __forceinline__ bool better(const Best& a, const Best& b) {
  if (a.v != b.v) return a.v > b.v;
  const uint32_t ka = a.i & 255u, kb = b.i & 255u;
  return ka != kb ? ka < kb : a.i < b.i;
}
constexpr int kArgmaxThreads = 1024;
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ logits, uint32_t n,
                                                                uint32_t* __restrict__ token) {
  __shared__ Best red[32];
  Best b{-1e30f, 0u};
  bool any = false;
  for (uint32_t i = threadIdx.x; i < n; i += kArgmaxThreads) {
    const Best c{logits[i], i};
    if (c.v > -1e30f && (!any || better(c, b))) {
      b = c;
      any = true;
    }
  }
  if (!any) b = Best{-INFINITY, 0xFFFFFFFFu};  // nothing counted here
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best c;
    c.v = __shfl_down_sync(0xffffffffu, b.v, o);
    c.i = __shfl_down_sync(0xffffffffu, b.i, o);
    if (c.i != 0xFFFFFFFFu && (b.i == 0xFFFFFFFFu || better(c, b))) b = c;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = b;
  __syncthreads();
  if (w == 0) {
    b = red[l];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best c;
      c.v = __shfl_down_sync(0xffffffffu, b.v, o);
      c.i = __shfl_down_sync(0xffffffffu, b.i, o);
      if (c.i != 0xFFFFFFFFu && (b.i == 0xFFFFFFFFu || better(c, b))) b = c;
    }
    if (l == 0) token[0] = b.i == 0xFFFFFFFFu ? 0u : b.i;
  }
}

// gather.wgsl: out[s, d] = table[ids[s], d] for s < seq_len, d < dim; an id
// beyond the table's rows sets DOE_DEVICE_ERR_PAGE and leaves its row zero.
__global__ void __launch_bounds__(kThreads) gather_rows_kernel(const uint32_t* __restrict__ ids,
                                                               const float* __restrict__ table,
                                                               float* __restrict__ out, uint32_t seq_len,
                                                               uint32_t dim, uint64_t table_rows,
                                                               int32_t* status) {
  const uint32_t s = blockIdx.y;
  if (s >= seq_len) return;
  const uint32_t id = ids[s];
  float* o = out + (size_t)s * dim;
  if ((uint64_t)id >= table_rows) {
    for (uint32_t d = blockIdx.x * kThreads + threadIdx.x; d < dim; d += gridDim.x * kThreads) o[d] = 0.0f;
    if (threadIdx.x == 0 && blockIdx.x == 0) report(status, DOE_DEVICE_ERR_PAGE);
    return;
  }
  const float* t = table + (size_t)id * dim;
  for (uint32_t d = blockIdx.x * kThreads + threadIdx.x; d < dim; d += gridDim.x * kThreads) o[d] = t[d];
}

}  // namespace pl
}  // namespace doe

using namespace doe;

namespace {
int invalid_arg(const char* msg) {
  set_op_error("%s", msg);
  return DOE_INVALID_ARGUMENT;
}
cudaStream_t stream_of(const doe_launch* l) { return l ? static_cast<cudaStream_t>(l->stream) : nullptr; }
}  // namespace

extern "C" {

int doe_rmsnorm_f32(const float* x, const float* weight, float* out, uint32_t rows, uint32_t size, float eps,
                    uint32_t weight_offset, const doe_launch* launch) {
  if (!x || !weight || !out) return invalid_arg("doe_rmsnorm_f32: null pointer");
  if (rows == 0 || size == 0) return DOE_OK;
  if (rows > 0x7FFFFFFFu) return invalid_arg("doe_rmsnorm_f32: too many rows");
  if (weight_offset) pl::rmsnorm_f32_kernel<true><<<rows, pl::kThreads, 0, stream_of(launch)>>>(x, weight, out, size, eps);
  else pl::rmsnorm_f32_kernel<false><<<rows, pl::kThreads, 0, stream_of(launch)>>>(x, weight, out, size, eps);
  return cuda_status(cudaGetLastError(), "rmsnorm_f32_kernel");
}

int doe_gemv_f32(const float* matrix, const float* vector, float* out, uint32_t rows, uint32_t cols,
                 const doe_launch* launch) {
  if (!matrix || !vector || !out) return invalid_arg("doe_gemv_f32: null pointer");
  if (rows == 0) return DOE_OK;
  const unsigned grid = (rows + pl::kThreads / 32 - 1) / (pl::kThreads / 32);
  const bool vec = cols % 4 == 0 && (reinterpret_cast<uintptr_t>(matrix) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(vector) & 15) == 0;
  if (vec) pl::gemv_f32_kernel<true><<<grid, pl::kThreads, 0, stream_of(launch)>>>(matrix, vector, out, rows, cols);
  else pl::gemv_f32_kernel<false><<<grid, pl::kThreads, 0, stream_of(launch)>>>(matrix, vector, out, rows, cols);
  return cuda_status(cudaGetLastError(), "gemv_f32_kernel");
}

int doe_gelu_tanh_f32(const float* x, float* y, uint64_t n, const doe_launch* launch) {
  if (!x || !y) return invalid_arg("doe_gelu_tanh_f32: null pointer");
  if (n == 0) return DOE_OK;
  const uint64_t want = (n + pl::kThreads - 1) / pl::kThreads;
  const unsigned grid = (unsigned)(want < (uint64_t)num_sms() * 8 ? want : (uint64_t)num_sms() * 8);
  pl::gelu_tanh_kernel<<<grid, pl::kThreads, 0, stream_of(launch)>>>(x, y, n);
  return cuda_status(cudaGetLastError(), "gelu_tanh_kernel");
}

int doe_argmax_f32(const float* logits, uint32_t n, uint32_t* token, const doe_launch* launch) {
  if (!logits || !token) return invalid_arg("doe_argmax_f32: null pointer");
  pl::argmax_kernel<<<1, pl::kArgmaxThreads, 0, stream_of(launch)>>>(logits, n, token);
  return cuda_status(cudaGetLastError(), "argmax_kernel");
}

int doe_gather_rows_f32(const uint32_t* ids, const float* table, uint64_t table_rows, float* out,
                        uint32_t seq_len, uint32_t dim, const doe_launch* launch) {
  if (!ids || !table || !out) return invalid_arg("doe_gather_rows_f32: null pointer");
  if (seq_len == 0 || dim == 0) return DOE_OK;
  if (seq_len > 65535) return invalid_arg("doe_gather_rows_f32: seq_len above 65535");
  const dim3 grid((dim + pl::kThreads - 1) / pl::kThreads, seq_len);
  pl::gather_rows_kernel<<<grid, pl::kThreads, 0, stream_of(launch)>>>(ids, table, out, seq_len, dim, table_rows,
                                                                      launch ? launch->status : nullptr);
  return cuda_status(cudaGetLastError(), "gather_rows_kernel");
}

}  // extern "C"
