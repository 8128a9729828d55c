// decode_f32.cu -- attention-decode.wgsl on sm_100a: single-query f32
// attention, q [H,D], K/V [H,L,D], out [H,D]
// (bench/inference-pipeline/kernels/attention-decode.wgsl:46-136).
//
// The WGSL kernel runs one 64-lane workgroup per head and holds every score
// in workgroup memory (kv_len <= 2048).  Here the KV length is split across
// CTAs (split-K) so all SMs stream K/V; each warp keeps an online softmax
// over its tokens and the CTA merges its warps.  The splits of one head form
// a thread-block cluster (up to 16 CTAs): each writes its partial into the
// first CTA's shared memory and, after one cluster barrier, that CTA
// stitches them with the LSE recipe of
// bench/tools/attention_kv_axis_sharded_stitch.py:46-90 -- one launch, no
// workspace.  Heads needing more than 16 splits fall back to partials in the
// workspace and combine_splits_kernel.
//
// Numerics: f32 throughout, natural-exp softmax.  The reference clamps
// s - max to [-30, 30] before exp (…wgsl:90); only the lower bound can bind
// (s - max <= 0), where it lifts a weight below e^-30 = 9.4e-14 up to
// 9.4e-14.  This kernel uses the exact weight, so each such key differs by
// less than 9.4e-14 * |v| in the numerator.
#include <cooperative_groups.h>

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

constexpr int kF32MaxCluster = 16;

// One CTA's split of one head: online softmax over tokens
// [split * split_tokens, ...) per warp, then the warps merged.  Leaves the
// CTA's un-normalised O in o_sm[0..D) and returns its (max, sum).
template <int PER_LANE>
__device__ __forceinline__ void decode_f32_cta(const DecodeF32Args& a, int split, int head, float* o_sm,
                                               float& M_out, float& L_out) {
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
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < kF32Warps; ++w) O += f[w] * sm_o[w][d];
    o_sm[d] = O;
  }
  M_out = M;
  L_out = L;
}

// Splits as partials in the workspace (stitched by combine_splits_kernel).
template <int PER_LANE>
__global__ void __launch_bounds__(kF32Warps * 32) decode_f32_split_kernel(const DecodeF32Args a) {
  const int split = blockIdx.x, head = blockIdx.y;
  const int D = a.head_dim;
  __shared__ float o_sm[32 * kF32MaxPerLane];
  float M, L;
  decode_f32_cta<PER_LANE>(a, split, head, o_sm, M, L);
  __syncthreads();
  const int nsplits = (a.kv_len + a.split_tokens - 1) / a.split_tokens;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float O = o_sm[d];
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

// The splits of one head as one cluster (gridDim.x == cluster size): each
// CTA stores (O, max, sum) into the first CTA's shared memory, which
// stitches them after the cluster barrier.
template <int PER_LANE>
__global__ void __launch_bounds__(kF32Warps * 32) decode_f32_cluster_kernel(const DecodeF32Args a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int split = blockIdx.x, head = blockIdx.y;
  const int D = a.head_dim;
  __shared__ float o_sm[32 * kF32MaxPerLane];
  __shared__ float part_o[kF32MaxCluster][32 * kF32MaxPerLane];
  __shared__ float part_ml[kF32MaxCluster][2];
  float M, L;
  decode_f32_cta<PER_LANE>(a, split, head, o_sm, M, L);
  __syncthreads();
  float* lead_o = cluster.map_shared_rank(&part_o[split][0], 0);
  for (int d = threadIdx.x; d < D; d += blockDim.x) lead_o[d] = o_sm[d];
  if (threadIdx.x == 0) {
    float* lead_ml = cluster.map_shared_rank(&part_ml[split][0], 0);
    lead_ml[0] = M;
    lead_ml[1] = L;
  }
  cluster.sync();  // every partial is in the first CTA's shared memory
  if (split != 0) return;
  const int n = (int)gridDim.x;
  float MM = -INFINITY;
  for (int sp = 0; sp < n; ++sp) MM = fmaxf(MM, part_ml[sp][0]);
  float LL = 0.0f;
  for (int sp = 0; sp < n; ++sp) LL += (MM == -INFINITY ? 0.0f : expf(part_ml[sp][0] - MM)) * part_ml[sp][1];
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float O = 0.0f;
    for (int sp = 0; sp < n; ++sp) O += (MM == -INFINITY ? 0.0f : expf(part_ml[sp][0] - MM)) * part_o[sp][d];
    a.out[(size_t)head * D + d] = LL > 0.0f ? O / LL : 0.0f;
  }
}

// One cluster of `max_splits` CTAs per head; DOE_UNSUPPORTED when the device
// will not run a cluster that large (the caller then uses the workspace path).
template <int PER_LANE>
static int launch_cluster_one(const DecodeF32Args& a, cudaStream_t s) {
  static std::atomic<bool> attr[kMaxDevices];
  int rc = once_per_device(attr, [] {
    cudaFuncSetAttribute(decode_f32_cluster_kernel<PER_LANE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaGetLastError();  // a device that refuses non-portable sizes leaves an error to clear
    return (int)DOE_OK;
  });
  if (rc != DOE_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.max_splits, a.num_heads);
  cfg.blockDim = dim3(kF32Warps * 32);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = a.max_splits;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // whether the device runs a cluster of this size, asked once per device and size
  static std::atomic<int> runs[kMaxDevices][kF32MaxCluster + 1];  // 0 unknown, 1 yes, -1 no
  const int dev = current_device();
  if (dev < 0) return DOE_CUDA_ERROR;
  int known = runs[dev][a.max_splits].load();
  if (known == 0) {
    int clusters = 0;
    known = (cudaOccupancyMaxActiveClusters(&clusters, decode_f32_cluster_kernel<PER_LANE>, &cfg) ==
                 cudaSuccess && clusters >= 1) ? 1 : -1;
    cudaGetLastError();
    runs[dev][a.max_splits].store(known);
  }
  if (known < 0) return DOE_UNSUPPORTED;
  return cuda_status(cudaLaunchKernelEx(&cfg, decode_f32_cluster_kernel<PER_LANE>, a),
                     "decode_f32_cluster_kernel");
}

static int launch_decode_f32_cluster(const DecodeF32Args& a, int per_lane, cudaStream_t s) {
  if (per_lane <= 2) return launch_cluster_one<2>(a, s);
  if (per_lane <= 4) return launch_cluster_one<4>(a, s);
  return launch_cluster_one<8>(a, s);
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
  if (ms > 1 && ms <= kF32MaxCluster && num_heads <= 65535) {
    int rc = launch_decode_f32_cluster(a, per_lane, s);
    if (rc != DOE_UNSUPPORTED) return rc;  // else: the workspace path below
  }
  if (per_lane <= 2) decode_f32_split_kernel<2><<<grid, block, 0, s>>>(a);
  else if (per_lane <= 4) decode_f32_split_kernel<4><<<grid, block, 0, s>>>(a);
  else decode_f32_split_kernel<8><<<grid, block, 0, s>>>(a);
  int rc = cuda_status(cudaGetLastError(), "decode_f32_split_kernel");
  if (rc != DOE_OK || ms <= 1) return rc;
  return launch_combine_natural(a.part_o, a.part_ml, out, (int)num_heads, (int)kv_len, st, ms,
                                (int)head_dim, s);
}

}  // namespace doe
