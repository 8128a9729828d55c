// ep_ops.cu -- the ONNX Runtime plugin EP's basic f32 operators on the GPU.
//
// The reference EP computes these on the host, one node at a time
// (runtime/bridge/onnxruntime-ep/src/doe_ort_ep.cc:1899-2401).  Here each is a
// kernel on device tensors, so an ONNX graph whose nodes the EP claims stays
// in HBM between nodes:
//   element-wise  Identity, Relu, Sigmoid, Tanh, Gelu (erf form)   :1899-2017
//                 Add, AddRelu                                      :1933,2380
//   rows          Softmax over the last axis (max-shifted exp, then
//                 multiply by 1 / sum; sum 0 -> 0)                  :2019-2058
//                 LayerNormalization over the last axis, scale only
//                 ((x - mean) * 1/sqrt(var + eps) * scale)          :2060-2106
//   Concat        two inputs along one axis                         :2108-2163
//   MatMul        rank-2 f32 [M,K] x [K,N], optionally + an addend of
//                 the output's shape (Gemm, MatMulAdd) and Relu
//                 (MatMulAddRelu); GemmReluGemm is two of them       :2165-2378
// Everything is f32 with f32 accumulation.  The matrix product runs on the
// FP32 pipe: the tensor cores' f32-input form (TF32) keeps 10 mantissa bits,
// which misses the 1e-5 relative agreement the reference's f32 loops define.
// Sums are reduced in a different order than the reference's left folds
// (tree reductions, FMA in the product), within that tolerance.
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"

namespace doe {
namespace ep {

constexpr int kThreads = 256;

template <int OP>
__device__ __forceinline__ float unary(float v) {
  if constexpr (OP == DOE_EP_RELU) return v < 0.0f ? 0.0f : v;
  else if constexpr (OP == DOE_EP_SIGMOID) return 1.0f / (1.0f + expf(-v));
  else if constexpr (OP == DOE_EP_TANH) return tanhf(v);
  else if constexpr (OP == DOE_EP_GELU) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
  else return v;  // Identity
}

template <int OP>
__device__ __forceinline__ float binary(float a, float b) {
  const float s = a + b;
  if constexpr (OP == DOE_EP_ADD_RELU) return s < 0.0f ? 0.0f : s;
  else return s;
}

// y[i] = f(x[i]).  VEC: float4 over the first n / 4 * 4 elements (all
// pointers 16-byte aligned), kUnroll float4 loads in flight per thread before
// their stores; the scalar tail (n % 4) by the first threads.
constexpr int kUnroll = 4;

template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads) unary_kernel(const float* x, float* y, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t i = t;
  if constexpr (VEC) {
    const uint64_t n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* y4 = reinterpret_cast<float4*>(y);
    for (uint64_t base = t; base < n4; base += stride * kUnroll) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (base + u * stride < n4) v[u] = x4[base + u * stride];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (base + u * stride < n4)
          __stcs(y4 + base + u * stride,
                 make_float4(unary<OP>(v[u].x), unary<OP>(v[u].y), unary<OP>(v[u].z), unary<OP>(v[u].w)));
    }
    i = n4 * 4 + t;
  }
  for (; i < n; i += stride) y[i] = unary<OP>(x[i]);
}

template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads) binary_kernel(const float* a, const float* b, float* y, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t i = t;
  if constexpr (VEC) {
    const uint64_t n4 = n / 4;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    float4* y4 = reinterpret_cast<float4*>(y);
    for (uint64_t base = t; base < n4; base += stride * kUnroll) {
      float4 p[kUnroll], q[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (base + u * stride < n4) {
          p[u] = a4[base + u * stride];
          q[u] = b4[base + u * stride];
        }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (base + u * stride < n4)
          __stcs(y4 + base + u * stride, make_float4(binary<OP>(p[u].x, q[u].x), binary<OP>(p[u].y, q[u].y),
                                                     binary<OP>(p[u].z, q[u].z), binary<OP>(p[u].w, q[u].w)));
    }
    i = n4 * 4 + t;
  }
  for (; i < n; i += stride) y[i] = binary<OP>(a[i], b[i]);
}


// Block-wide reduction of one value per thread (sum or max); every thread
// gets the result.  `red` holds kThreads / 32 partials; the leading barrier
// lets a caller reuse it back to back.
template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) v = MAX ? fmaxf(v, red[w]) : v + red[w];
  return v;
}

// One CTA per row (grid-stride over rows).  CACHE: the row is read from HBM
// once into shared memory (cols floats); otherwise each pass re-reads it.
// VEC: rows are read and written as float4 (cols % 4 == 0, x, y and scale
// 16-byte aligned), kUnroll loads in flight per thread.
// SOFTMAX: y = exp(x - max) * (sum != 0 ? 1 / sum : 0)
// else:    y = (x - mean) * (1 / sqrt(var + eps)) * scale, var = mean((x - mean)^2)
template <bool SOFTMAX, bool CACHE, bool VEC>
__global__ void __launch_bounds__(kThreads)
    rows_kernel(const float* x, const float* __restrict__ scale, float eps, float* y, uint64_t rows, uint32_t cols) {
  extern __shared__ float4 srow4[];
  float* srow = reinterpret_cast<float*>(srow4);
  __shared__ float red[kThreads / 32];
  const float inv_cols = 1.0f / (float)cols;
  constexpr uint32_t W = VEC ? 4 : 1;  // floats per access
  const uint32_t units = cols / W;
  for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    auto load = [&](uint32_t u) -> float4 {
      if constexpr (VEC) return reinterpret_cast<const float4*>(xr)[u];
      else return make_float4(xr[u], 0.0f, 0.0f, 0.0f);
    };
    auto cached = [&](uint32_t u) -> float4 {
      if constexpr (!CACHE) return load(u);
      else if constexpr (VEC) return srow4[u];
      else return make_float4(srow[u], 0.0f, 0.0f, 0.0f);
    };
    // combine the W live lanes of a unit into acc
    auto fold = [&](float acc, float4 v, auto&& f) {
      acc = f(acc, v.x);
      if constexpr (VEC) {
        acc = f(acc, v.y);
        acc = f(acc, v.z);
        acc = f(acc, v.w);
      }
      return acc;
    };
    auto mx = [](float a, float v) { return fmaxf(a, v); };
    auto sum = [](float a, float v) { return a + v; };
    // pass 1: max (softmax) or sum (layer norm), caching the row
    float acc = SOFTMAX ? -INFINITY : 0.0f;
    for (uint32_t base = threadIdx.x; base < units; base += kThreads * kUnroll) {
      float4 v[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k)
        if (base + k * kThreads < units) v[k] = load(base + k * kThreads);
#pragma unroll
      for (int k = 0; k < kUnroll; ++k)
        if (base + k * kThreads < units) {
          const uint32_t u = base + k * kThreads;
          if constexpr (CACHE) {
            if constexpr (VEC) srow4[u] = v[k];
            else srow[u] = v[k].x;
          }
          acc = SOFTMAX ? fold(acc, v[k], mx) : fold(acc, v[k], sum);
        }
    }
    const float first = block_reduce<SOFTMAX>(acc, red);
    // pass 2: sum of exp (softmax) or of squared deviations (layer norm)
    const float mean = SOFTMAX ? 0.0f : first * inv_cols;
    auto second_term = [&](float a, float v) {
      if constexpr (SOFTMAX) return a + expf(v - first);
      else {
        const float d = v - mean;
        return a + d * d;
      }
    };
    acc = 0.0f;
    for (uint32_t u = threadIdx.x; u < units; u += kThreads) acc = fold(acc, cached(u), second_term);
    const float second = block_reduce<false>(acc, red);
    // pass 3: the output row
    const float inv = SOFTMAX ? (second != 0.0f ? 1.0f / second : 0.0f) : 1.0f / sqrtf(second * inv_cols + eps);
    for (uint32_t u = threadIdx.x; u < units; u += kThreads) {
      const float4 v = cached(u);
      if constexpr (SOFTMAX) {
        if constexpr (VEC)
          __stcs(reinterpret_cast<float4*>(yr) + u, make_float4(expf(v.x - first) * inv, expf(v.y - first) * inv,
                                                                expf(v.z - first) * inv, expf(v.w - first) * inv));
        else yr[u] = expf(v.x - first) * inv;
      } else {
        if constexpr (VEC) {
          const float4 s = reinterpret_cast<const float4*>(scale)[u];
          __stcs(reinterpret_cast<float4*>(yr) + u,
                 make_float4((v.x - mean) * inv * s.x, (v.y - mean) * inv * s.y, (v.z - mean) * inv * s.z,
                             (v.w - mean) * inv * s.w));
        } else {
          yr[u] = (v.x - mean) * inv * scale[u];
        }
      }
    }
    __syncthreads();  // the cached row is rewritten by the next row
  }
}


// Rows of at most kThreads * kUnroll float4 (4096 floats), read and written as
// float4: each thread keeps its part of the row in registers, and the CTA's
// next row is loaded while this one is reduced and written (rows belong to
// CTAs by row % gridDim.x, so in place the prefetched row is never one being
// written).  Same arithmetic as rows_kernel; softmax keeps exp(x - max) from
// the sum pass for the output pass.
template <bool SOFTMAX>
__global__ void __launch_bounds__(kThreads)
    rows_reg_kernel(const float* x, const float* __restrict__ scale, float eps, float* y, uint64_t rows,
                    uint32_t cols) {
  __shared__ float red[kThreads / 32];
  const uint32_t units = cols / 4;
  const float inv_cols = 1.0f / (float)cols;
  float4 cur[kUnroll], nxt[kUnroll];
  auto load_row = [&](uint64_t row, float4 (&v)[kUnroll]) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * cols);
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const uint32_t u = threadIdx.x + k * kThreads;
      if (u < units) v[k] = xr[u];
    }
  };
  uint64_t row = blockIdx.x;
  if (row < rows) load_row(row, cur);
  for (; row < rows; row += gridDim.x) {
    const uint64_t next = row + gridDim.x;
    if (next < rows) load_row(next, nxt);
    float acc = SOFTMAX ? -INFINITY : 0.0f;
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
      if (threadIdx.x + k * kThreads < units) {
        const float4 v = cur[k];
        acc = SOFTMAX ? fmaxf(fmaxf(acc, v.x), fmaxf(fmaxf(v.y, v.z), v.w)) : acc + v.x + v.y + v.z + v.w;
      }
    const float first = block_reduce<SOFTMAX>(acc, red);
    const float mean = SOFTMAX ? 0.0f : first * inv_cols;
    acc = 0.0f;
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
      if (threadIdx.x + k * kThreads < units) {
        float4& v = cur[k];
        if (SOFTMAX) {
          v = make_float4(expf(v.x - first), expf(v.y - first), expf(v.z - first), expf(v.w - first));
          acc += v.x + v.y + v.z + v.w;
        } else {
          const float dx = v.x - mean, dy = v.y - mean, dz = v.z - mean, dw = v.w - mean;
          acc += dx * dx + dy * dy + dz * dz + dw * dw;
        }
      }
    const float second = block_reduce<false>(acc, red);
    const float inv = SOFTMAX ? (second != 0.0f ? 1.0f / second : 0.0f) : 1.0f / sqrtf(second * inv_cols + eps);
    float4* yr = reinterpret_cast<float4*>(y + row * cols);
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const uint32_t u = threadIdx.x + k * kThreads;
      if (u < units) {
        const float4 v = cur[k];
        if (SOFTMAX) {
          __stcs(yr + u, make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv));
        } else {
          const float4 sc = reinterpret_cast<const float4*>(scale)[u];
          __stcs(yr + u, make_float4((v.x - mean) * inv * sc.x, (v.y - mean) * inv * sc.y,
                                     (v.z - mean) * inv * sc.z, (v.w - mean) * inv * sc.w));
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) cur[k] = nxt[k];
  }
}

// y[o, 0:a_axis*inner] = a[o, :], y[o, a_axis*inner:] = b[o, :]
__global__ void __launch_bounds__(kThreads)
    concat_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y, uint64_t outer,
                  uint64_t a_run, uint64_t b_run) {
  const uint64_t run = a_run + b_run, total = outer * run;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint64_t o = i / run, r = i - o * run;
    y[i] = r < a_run ? a[o * a_run + r] : b[o * b_run + (r - a_run)];
  }
}

// C[M,N] = A[M,K] B[K,N] (+ addend[M,N]) (then Relu), all row-major f32.
// 128 x 128 output tile per CTA, 256 threads with 8 x 8 outputs each, K
// steps of 8 through two shared-memory stages (A stored k-major so both
// operands are read as float4 rows).  Loads outside the matrices read 0;
// each output is one FMA chain over k in order.
constexpr int TM = 128, TN = 128, TK = 8;

__global__ void __launch_bounds__(kThreads)
    matmul_kernel(const float* __restrict__ A, const float* __restrict__ B, const float* __restrict__ addend,
                  float* __restrict__ C, int M, int K, int N, int relu) {
  __shared__ __align__(16) float As[2][TK][TM];
  __shared__ __align__(16) float Bs[2][TK][TN];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, 8 x 8 outputs each
  // loader mapping: A tile 128 x 8 -> each thread 4 elements of one row;
  // B tile 8 x 128 -> each thread 4 consecutive columns of one k row
  const int a_row = tid / 2, a_k = (tid % 2) * 4;
  const int b_k = tid / 32, b_col = (tid % 32) * 4;
  float ra[4], rb[4];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gm = m0 + a_row, gk = k0 + a_k + i;
      ra[i] = (gm < M && gk < K) ? A[(size_t)gm * K + gk] : 0.0f;
      const int gk2 = k0 + b_k, gn = n0 + b_col + i;
      rb[i] = (gk2 < K && gn < N) ? B[(size_t)gk2 * N + gn] : 0.0f;
    }
  };
  auto stash = [&](int s) {
#pragma unroll
    for (int i = 0; i < 4; ++i) As[s][a_k + i][a_row] = ra[i];
    *reinterpret_cast<float4*>(&Bs[s][b_k][b_col]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  const int steps = (K + TK - 1) / TK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int s = 0; s < steps; ++s) {
    const int cur = s & 1;
    if (s + 1 < steps) fetch((s + 1) * TK);  // global loads in flight during the math
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      // rows tr*4 .. +3 and 64 + tr*4 .. +3; columns tc*4 .. +3 and 64 + tc*4 .. +3
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][tr * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][kk][64 + tr * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tc * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][64 + tc * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (s + 1 < steps) {
      stash(cur ^ 1);  // the other stage was last read before the previous barrier
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? tr * 4 + i : 64 + tr * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tc * 4 + j : 64 + tc * 4 + (j - 4));
      if (gn >= N) continue;
      const size_t o = (size_t)gm * N + gn;
      float v = acc[i][j];
      if (addend != nullptr) v += addend[o];
      if (relu) v = v < 0.0f ? 0.0f : v;
      C[o] = v;
    }
  }
}

// matmul_kernel for aligned shapes (k and n multiples of 4, A and B 16-byte
// aligned): K steps of 16 and float4 loads of both operands, so half the
// barriers and a quarter of the load instructions per FMA.  Same tiles, same
// per-output FMA chain over k in order.
constexpr int TK2 = 16;

__global__ void __launch_bounds__(kThreads, 2)
    matmul_vec_kernel(const float* __restrict__ A, const float* __restrict__ B, const float* __restrict__ addend,
                      float* __restrict__ C, int M, int K, int N, int relu) {
  __shared__ __align__(16) float As[2][TK2][TM];
  __shared__ __align__(16) float Bs[2][TK2][TN];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, 8 x 8 outputs each
  // A tile 128 x 16: row tid / 2, k (tid % 2) * 8 .. + 8 as two float4;
  // B tile 16 x 128: k rows tid / 32 and tid / 32 + 8, columns (tid % 32) * 4 .. + 4
  const int a_row = tid >> 1, a_k = (tid & 1) * 8;
  const int b_k = tid >> 5, b_col = (tid & 31) * 4;
  const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float4 ra[2], rb[2];
  auto fetch = [&](int k0) {
    const int gm = m0 + a_row;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int gk = k0 + a_k + 4 * i;  // k % 4 == 0: all four in range when gk is
      ra[i] = (gm < M && gk < K) ? *reinterpret_cast<const float4*>(A + (size_t)gm * K + gk) : zero;
      const int gk2 = k0 + b_k + 8 * i, gn = n0 + b_col;  // n % 4 == 0 likewise
      rb[i] = (gk2 < K && gn < N) ? *reinterpret_cast<const float4*>(B + (size_t)gk2 * N + gn) : zero;
    }
  };
  auto stash = [&](int s) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      As[s][a_k + 4 * i + 0][a_row] = ra[i].x;
      As[s][a_k + 4 * i + 1][a_row] = ra[i].y;
      As[s][a_k + 4 * i + 2][a_row] = ra[i].z;
      As[s][a_k + 4 * i + 3][a_row] = ra[i].w;
      *reinterpret_cast<float4*>(&Bs[s][b_k + 8 * i][b_col]) = rb[i];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  const int steps = (K + TK2 - 1) / TK2;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int s = 0; s < steps; ++s) {
    const int cur = s & 1;
    if (s + 1 < steps) fetch((s + 1) * TK2);  // global loads in flight during the math
#pragma unroll
    for (int kk = 0; kk < TK2; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][tr * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][kk][64 + tr * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tc * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][64 + tc * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (s + 1 < steps) {
      stash(cur ^ 1);  // the other stage was last read before the previous barrier
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? tr * 4 + i : 64 + tr * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tc * 4 + j : 64 + tc * 4 + (j - 4));
      if (gn >= N) continue;
      const size_t o = (size_t)gm * N + gn;
      float v = acc[i][j];
      if (addend != nullptr) v += addend[o];
      if (relu) v = v < 0.0f ? 0.0f : v;
      C[o] = v;
    }
  }
}

// A grid-stride kernel's grid: one wave of the CTAs that fit on the SMs at
// once (registers and shared memory permitting), or fewer when there is
// less work.  A second, partial wave would leave SMs idle at the end.
// The occupancy query is cached per (kernel, device, shared-memory bytes).
template <typename Kernel>
unsigned resident_grid(Kernel kernel, size_t smem, uint64_t work, int per_block) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) cudaGetLastError();
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), dev, smem);
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) per_sm = it->second;
  }
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem) != cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = per_sm;
  }
  const uint64_t want = (work + per_block - 1) / per_block;
  const uint64_t cap = (uint64_t)num_sms() * per_sm;
  return (unsigned)(want < 1 ? 1 : (want < cap ? want : cap));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int OP>
int launch_unary_op(const float* x, float* y, uint64_t n, cudaStream_t s) {
  if (aligned16(x) && aligned16(y)) {
    const unsigned g = resident_grid(unary_kernel<OP, true>, 0, (n / 4 + kUnroll - 1) / kUnroll, kThreads);
    unary_kernel<OP, true><<<g, kThreads, 0, s>>>(x, y, n);
  } else {
    unary_kernel<OP, false><<<resident_grid(unary_kernel<OP, false>, 0, n, kThreads), kThreads, 0, s>>>(x, y, n);
  }
  return cuda_status(cudaGetLastError(), "ep unary_kernel");
}

template <int OP>
int launch_binary_op(const float* a, const float* b, float* y, uint64_t n, cudaStream_t s) {
  if (aligned16(a) && aligned16(b) && aligned16(y)) {
    const unsigned g = resident_grid(binary_kernel<OP, true>, 0, (n / 4 + kUnroll - 1) / kUnroll, kThreads);
    binary_kernel<OP, true><<<g, kThreads, 0, s>>>(a, b, y, n);
  } else {
    const unsigned g = resident_grid(binary_kernel<OP, false>, 0, n, kThreads);
    binary_kernel<OP, false><<<g, kThreads, 0, s>>>(a, b, y, n);
  }
  return cuda_status(cudaGetLastError(), "ep binary_kernel");
}

// Rows up to this many floats are cached in shared memory (one read of x).
constexpr uint32_t kMaxCachedCols = 48 * 1024 / 4;

template <bool SOFTMAX>
int launch_rows(const float* x, const float* scale, float eps, float* y, uint64_t rows, uint32_t cols,
                cudaStream_t s) {
  const bool vec = cols % 4 == 0 && aligned16(x) && aligned16(y) && (scale == nullptr || aligned16(scale));
  const size_t smem = cols * sizeof(float);
  auto go = [&](auto kernel, size_t bytes) {
    kernel<<<resident_grid(kernel, bytes, rows, 1), kThreads, bytes, s>>>(x, scale, eps, y, rows, cols);
  };
  if (vec && cols <= (uint32_t)(kThreads * kUnroll * 4)) {
    go(rows_reg_kernel<SOFTMAX>, 0);
  } else if (cols <= kMaxCachedCols) {
    if (vec) go(rows_kernel<SOFTMAX, true, true>, smem);
    else go(rows_kernel<SOFTMAX, true, false>, smem);
  } else {
    if (vec) go(rows_kernel<SOFTMAX, false, true>, 0);
    else go(rows_kernel<SOFTMAX, false, false>, 0);
  }
  return cuda_status(cudaGetLastError(), SOFTMAX ? "ep softmax rows_kernel" : "ep layernorm rows_kernel");
}

}  // namespace ep

int launch_ep_unary(uint32_t op, const float* x, float* y, uint64_t n, const doe_launch* l) {
  const cudaStream_t s = static_cast<cudaStream_t>(l->stream);
  switch (op) {
    case DOE_EP_IDENTITY: return ep::launch_unary_op<DOE_EP_IDENTITY>(x, y, n, s);
    case DOE_EP_RELU: return ep::launch_unary_op<DOE_EP_RELU>(x, y, n, s);
    case DOE_EP_SIGMOID: return ep::launch_unary_op<DOE_EP_SIGMOID>(x, y, n, s);
    case DOE_EP_TANH: return ep::launch_unary_op<DOE_EP_TANH>(x, y, n, s);
    case DOE_EP_GELU: return ep::launch_unary_op<DOE_EP_GELU>(x, y, n, s);
    default: return DOE_INVALID_ARGUMENT;
  }
}

int launch_ep_binary(uint32_t op, const float* a, const float* b, float* y, uint64_t n, const doe_launch* l) {
  const cudaStream_t s = static_cast<cudaStream_t>(l->stream);
  switch (op) {
    case DOE_EP_ADD: return ep::launch_binary_op<DOE_EP_ADD>(a, b, y, n, s);
    case DOE_EP_ADD_RELU: return ep::launch_binary_op<DOE_EP_ADD_RELU>(a, b, y, n, s);
    default: return DOE_INVALID_ARGUMENT;
  }
}

int launch_ep_softmax(const float* x, float* y, uint64_t rows, uint32_t cols, const doe_launch* l) {
  return ep::launch_rows<true>(x, nullptr, 0.0f, y, rows, cols, static_cast<cudaStream_t>(l->stream));
}

int launch_ep_layernorm(const float* x, const float* scale, float eps, float* y, uint64_t rows, uint32_t cols,
                        const doe_launch* l) {
  return ep::launch_rows<false>(x, scale, eps, y, rows, cols, static_cast<cudaStream_t>(l->stream));
}

int launch_ep_concat(const float* a, const float* b, float* y, uint64_t outer, uint64_t a_run, uint64_t b_run,
                     const doe_launch* l) {
  const unsigned g = ep::resident_grid(ep::concat_kernel, 0, outer * (a_run + b_run), ep::kThreads);
  ep::concat_kernel<<<g, ep::kThreads, 0, static_cast<cudaStream_t>(l->stream)>>>(a, b, y, outer, a_run, b_run);
  return cuda_status(cudaGetLastError(), "ep concat_kernel");
}

int launch_ep_matmul(const float* a, const float* b, const float* addend, float* y, uint32_t m, uint32_t k,
                     uint32_t n, bool relu, const doe_launch* l) {
  const dim3 grid((n + ep::TN - 1) / ep::TN, (m + ep::TM - 1) / ep::TM);
  const cudaStream_t s = static_cast<cudaStream_t>(l->stream);
  if (k % 4 == 0 && n % 4 == 0 && ep::aligned16(a) && ep::aligned16(b)) {
    ep::matmul_vec_kernel<<<grid, ep::kThreads, 0, s>>>(a, b, addend, y, (int)m, (int)k, (int)n, relu ? 1 : 0);
    return cuda_status(cudaGetLastError(), "ep matmul_vec_kernel");
  }
  ep::matmul_kernel<<<grid, ep::kThreads, 0, s>>>(a, b, addend, y, (int)m, (int)k, (int)n, relu ? 1 : 0);
  return cuda_status(cudaGetLastError(), "ep matmul_kernel");
}

}  // namespace doe
