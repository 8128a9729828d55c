// decode_f32.cu -- attention-decode.wgsl on sm_100a: single-query f32
// attention, q [H,D], K/V [H,L,D], out [H,D]
// (bench/inference-pipeline/kernels/attention-decode.wgsl:46-136).
//
// The WGSL kernel runs one 64-lane workgroup per head and holds every score
// in workgroup memory (kv_len <= 2048).  Here the KV length is split across
// CTAs (split-K) so all SMs stream K/V; each warp keeps an online softmax
// over its tokens, the CTA merges its warps, and combine_splits_kernel
// stitches the splits (the LSE recipe of
// bench/tools/attention_kv_axis_sharded_stitch.py:46-90).
//
// Numerics: f32 throughout, natural-exp softmax.  The reference clamps
// s - max to [-30, 30] before exp (…wgsl:90); only the lower bound can bind
// (s - max <= 0), where it lifts a weight below e^-30 = 9.4e-14 up to
// 9.4e-14.  This kernel uses the exact weight, so each such key differs by
// less than 9.4e-14 * |v| in the numerator.
#include "common.cuh"

namespace doe {

struct DecodeF32Args {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  float* part_o;   // [H * max_splits, D]
  float* part_ml;  // [H * max_splits, 2]
  int num_heads, head_dim, kv_len, split_tokens, max_splits;
  float scale;
};

constexpr int kF32Warps = 4;
constexpr int kF32MaxPerLane = 8;  // head_dim <= 256

template <int PER_LANE>
__global__ void __launch_bounds__(kF32Warps * 32) decode_f32_split_kernel(const DecodeF32Args a) {
  const int split = blockIdx.x, head = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = a.head_dim;
  const int t_begin = split * a.split_tokens;
  const int t_end = min(a.kv_len, t_begin + a.split_tokens);
  const float* qh = a.q + (size_t)head * D;
  const float* kh = a.k + (size_t)head * D * a.kv_len;
  const float* vh = a.v + (size_t)head * D * a.kv_len;

  float qr[PER_LANE], acc[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int d = lane + 32 * i;
    qr[i] = d < D ? qh[d] : 0.0f;
    acc[i] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;

  // TOK tokens per warp step (all their K/V loads issued together), one
  // rescale per step; TOK * PER_LANE = 16 keeps 32 loaded floats per lane
  constexpr int TOK = 16 / PER_LANE;
  for (int t0 = t_begin + TOK * warp; t0 < t_end; t0 += TOK * kF32Warps) {
    float kv_k[TOK][PER_LANE], kv_v[TOK][PER_LANE];
#pragma unroll
    for (int j = 0; j < TOK; ++j) {
      const int t = t0 + j;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int d = lane + 32 * i;
        const bool ok = t < t_end && d < D;
        kv_k[j][i] = ok ? __ldcg(kh + (size_t)t * D + d) : 0.0f;
        kv_v[j][i] = ok ? __ldcg(vh + (size_t)t * D + d) : 0.0f;
      }
    }
    float s[TOK];
#pragma unroll
    for (int j = 0; j < TOK; ++j) {
      float part = 0.0f;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) part = fmaf(qr[i], kv_k[j][i], part);
      s[j] = part;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < TOK; ++j) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
    float smax = -INFINITY;
#pragma unroll
    for (int j = 0; j < TOK; ++j) {
      s[j] = (t0 + j < t_end) ? s[j] * a.scale : -INFINITY;
      smax = fmaxf(smax, s[j]);
    }
    const float m_new = fmaxf(m, smax);
    const float corr = expf(m - m_new);
    float p[TOK];
    float psum = 0.0f;
#pragma unroll
    for (int j = 0; j < TOK; ++j) {
      p[j] = expf(s[j] - m_new);
      psum += p[j];
    }
    l = l * corr + psum;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      float x = acc[i] * corr;
#pragma unroll
      for (int j = 0; j < TOK; ++j) x = fmaf(p[j], kv_v[j][i], x);
      acc[i] = x;
    }
    m = m_new;
  }

  __shared__ float sm_m[kF32Warps], sm_l[kF32Warps];
  __shared__ float sm_o[kF32Warps][32 * kF32MaxPerLane];
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) sm_o[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kF32Warps; ++w) M = fmaxf(M, sm_m[w]);
  float f[kF32Warps], L = 0.0f;
#pragma unroll
  for (int w = 0; w < kF32Warps; ++w) {
    f[w] = M == -INFINITY ? 0.0f : expf(sm_m[w] - M);
    L += f[w] * sm_l[w];
  }
  const int nsplits = (a.kv_len + a.split_tokens - 1) / a.split_tokens;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < kF32Warps; ++w) O += f[w] * sm_o[w][d];
    if (nsplits == 1) {
      a.out[(size_t)head * D + d] = L > 0.0f ? O / L : 0.0f;
    } else {
      const size_t prow = (size_t)head * a.max_splits + split;
      a.part_o[prow * D + d] = O;
      if (d == 0) {
        a.part_ml[prow * 2] = M;
        a.part_ml[prow * 2 + 1] = L;
      }
    }
  }
}

static void decode_f32_plan(uint32_t num_heads, uint32_t head_dim, uint32_t kv_len,
                            int* split_tokens, int* max_splits) {
  // aim for ~2 CTAs per SM over all heads; a split is a whole number of
  // 4-warp steps (TOK = 16 / per-lane dims tokens per warp step)
  const uint32_t per_lane = head_dim <= 64 ? 2 : (head_dim <= 128 ? 4 : 8);
  const uint32_t chunk = kF32Warps * (16 / per_lane);
  const uint32_t want = num_heads == 0 ? 1 : (296 + num_heads - 1) / num_heads;
  uint32_t st = (kv_len + want - 1) / (want ? want : 1);
  st = (st + chunk - 1) / chunk * chunk;
  if (st < chunk) st = chunk;
  *split_tokens = (int)st;
  *max_splits = (int)((kv_len + st - 1) / st);
  if (*max_splits < 1) *max_splits = 1;
}

uint64_t decode_f32_workspace(uint32_t num_heads, uint32_t head_dim, uint32_t kv_len) {
  int st, ms;
  decode_f32_plan(num_heads, head_dim, kv_len, &st, &ms);
  if (ms <= 1) return 0;
  return (uint64_t)num_heads * ms * (head_dim + 2) * sizeof(float);
}

int launch_decode_f32(const float* q, const float* k, const float* v, float* out,
                      uint32_t num_heads, uint32_t head_dim, uint32_t kv_len, float scale,
                      const doe_launch* launch) {
  int st, ms;
  decode_f32_plan(num_heads, head_dim, kv_len, &st, &ms);
  const uint64_t ws = decode_f32_workspace(num_heads, head_dim, kv_len);
  if (ws > 0 && (launch->workspace == nullptr || launch->workspace_bytes < ws)) {
    set_op_error("doe_attention_decode_f32: workspace of %llu bytes required, %llu given",
                 (unsigned long long)ws, (unsigned long long)launch->workspace_bytes);
    return DOE_INVALID_ARGUMENT;
  }
  DecodeF32Args a;
  a.q = q; a.k = k; a.v = v; a.out = out;
  a.part_o = static_cast<float*>(launch->workspace);
  a.part_ml = a.part_o ? a.part_o + (size_t)num_heads * ms * head_dim : nullptr;
  a.num_heads = (int)num_heads;
  a.head_dim = (int)head_dim;
  a.kv_len = (int)kv_len;
  a.split_tokens = st;
  a.max_splits = ms;
  a.scale = scale;
  cudaStream_t s = static_cast<cudaStream_t>(launch->stream);
  dim3 grid(ms, num_heads), block(kF32Warps * 32);
  const int per_lane = (int)((head_dim + 31) / 32);
  if (per_lane <= 2) decode_f32_split_kernel<2><<<grid, block, 0, s>>>(a);
  else if (per_lane <= 4) decode_f32_split_kernel<4><<<grid, block, 0, s>>>(a);
  else decode_f32_split_kernel<8><<<grid, block, 0, s>>>(a);
  int rc = cuda_status(cudaGetLastError(), "decode_f32_split_kernel");
  if (rc != DOE_OK || ms <= 1) return rc;
  return launch_combine_natural(a.part_o, a.part_ml, out, (int)num_heads, (int)kv_len, st, ms,
                                (int)head_dim, s);
}

}  // namespace doe
