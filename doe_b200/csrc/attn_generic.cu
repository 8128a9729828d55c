// attn_generic.cu -- the Doppler online-softmax attention kernel
// (runtime/zig/tests/tsir/real/attention_head256_f16kv/attention_head256_f16kv.wgsl:72-269)
// for any uniform block: query_len >= 1, GQA, causal / sliding-window key
// bounds, tanh softcap, dense / ring / paged KV, kv length from the uniform or
// a buffer, f16 or f32 K/V, head_dim up to 512.
//
// This is the compatibility path of the dispatch surface, not the throughput
// path (the batched paged decode and the tcgen05 prefill are).  It keeps the
// reference's arithmetic order per query row: 32-key blocks, vec4 dot
// products summed left to right, block max, correction exp(m_i - m_new),
// l_i += p in key order, acc += p * v in key order, out = acc * (1 / l).
// Products and sums use __fmul_rn / __fadd_rn so nothing is contracted into
// an FMA; only exp / tanh come from CUDA's math library.
//
// Mapping: one warp per (query, head) row.  Lane j scores key 32*blk + j (its
// own K row); V is read coalesced, each lane owning head dims lane + 32*i.
#include "common.cuh"

namespace doe {

constexpr int kGenWarps = 4;
constexpr int kGenMaxDim = 512;

template <typename KT>
__device__ __forceinline__ float ldkv(const KT* p);
template <>
__device__ __forceinline__ float ldkv<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ldkv<float>(const float* p) { return *p; }

template <typename KT, int PER_LANE>
__global__ void __launch_bounds__(kGenWarps * 32) attn_online_generic_kernel(const GenericAttnArgs a) {
  const doe_attn_uniforms& u = a.u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t row = (uint64_t)blockIdx.x * kGenWarps + warp;
  const uint32_t H = u.num_heads, D = u.head_dim;
  __shared__ float q_sm[kGenWarps][kGenMaxDim];
  if (row >= (uint64_t)u.query_len * H) return;
  const uint32_t qp = (uint32_t)(row / H), h = (uint32_t)(row % H);
  const uint32_t kvh = h / (H / u.num_kv_heads);
  const uint32_t seq_len = u.kv_len_source == 0 ? u.seq_len : a.kv_len_buffer[0];
  const float* qrow = a.q + qp * a.q_pos_stride + h * a.q_head_stride;
  for (uint32_t d = lane; d < D; d += 32) q_sm[warp][d] = qrow[d];
  __syncwarp();

  const uint32_t abs_q = qp + u.start_pos;
  uint32_t min_key = 0, max_key = seq_len;
  if (u.is_causal) {
    if (abs_q < u.kv_start) max_key = 0;
    else max_key = min(seq_len, abs_q - u.kv_start + 1);
  }
  if (u.sliding_window > 0 && abs_q >= u.sliding_window) {
    const uint32_t min_abs = abs_q - u.sliding_window + 1;
    if (min_abs > u.kv_start) min_key = min_abs - u.kv_start;
    min_key = min(min_key, seq_len);
  }

  const KT* K = static_cast<const KT*>(a.k);
  const KT* V = static_cast<const KT*>(a.v);
  float acc[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) acc[i] = 0.0f;
  float m_i = -3.402823e+38f, l_i = 0.0f;
  const uint32_t vec_dim = D & ~3u;
  const uint32_t nblocks = (seq_len + 31) / 32;

  for (uint32_t blk = 0; blk < nblocks; ++blk) {
    const uint32_t kp = blk * 32 + lane;
    bool active = kp < seq_len && kp >= min_key && kp < max_key;
    uint64_t phys = 0;
    if (active) {
      const uint32_t abs_key = u.kv_start + kp;
      if (u.kv_layout == 1 && u.sliding_window > 0) {
        phys = abs_key % u.sliding_window;
      } else if (u.kv_layout == 2) {
        const uint32_t pidx = abs_key / u.page_size;
        if (a.page_table_len && pidx >= a.page_table_len) {
          report(a.status, DOE_DEVICE_ERR_PAGE);
          active = false;
        } else {
          phys = (uint64_t)a.page_table[pidx] * u.page_size + (abs_key - pidx * u.page_size);
        }
      } else {
        phys = abs_key;
      }
      if (active && a.kv_rows && phys >= a.kv_rows) {
        report(a.status, DOE_DEVICE_ERR_PAGE);
        active = false;
      }
    }
    float s = 0.0f;
    if (active) {
      const KT* krow = K + phys * a.kv_pos_stride + kvh * a.kv_head_stride;
      float dot = 0.0f;
      for (uint32_t d = 0; d < vec_dim; d += 4) {
        float dp = __fmul_rn(q_sm[warp][d], ldkv(krow + d));
        dp = __fadd_rn(dp, __fmul_rn(q_sm[warp][d + 1], ldkv(krow + d + 1)));
        dp = __fadd_rn(dp, __fmul_rn(q_sm[warp][d + 2], ldkv(krow + d + 2)));
        dp = __fadd_rn(dp, __fmul_rn(q_sm[warp][d + 3], ldkv(krow + d + 3)));
        dot = __fadd_rn(dot, dp);
      }
      for (uint32_t d = vec_dim; d < D; ++d) dot = __fadd_rn(dot, __fmul_rn(q_sm[warp][d], ldkv(krow + d)));
      s = __fmul_rn(dot, u.scale);
      if (u.attn_softcap > 0.0f) s = __fmul_rn(tanhf(s / u.attn_softcap), u.attn_softcap);
    }
    const float block_max = warp_max(active ? s : -3.402823e+38f);
    const float m_new = fmaxf(m_i, block_max);
    const float corr = expf(m_i - m_new);
    l_i = __fmul_rn(l_i, corr);
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) acc[i] = __fmul_rn(acc[i], corr);
    const float p = active ? expf(s - m_new) : 0.0f;
    for (int j = 0; j < 32; ++j) {
      const float pj = __shfl_sync(0xffffffffu, p, j);
      l_i = __fadd_rn(l_i, pj);
      if (pj == 0.0f) continue;  // warp-uniform
      const uint64_t pphys = __shfl_sync(0xffffffffu, phys, j);
      const KT* vrow = V + pphys * a.kv_pos_stride + kvh * a.kv_head_stride;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const uint32_t d = lane + 32 * i;
        if (d < D) acc[i] = __fadd_rn(acc[i], __fmul_rn(pj, ldkv(vrow + d)));
      }
    }
    m_i = m_new;
  }
  const float inv = l_i > 0.0f ? 1.0f / l_i : 0.0f;
  float* orow = a.out + qp * a.q_pos_stride + h * a.q_head_stride;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const uint32_t d = lane + 32 * i;
    if (d < D) orow[d] = __fmul_rn(acc[i], inv);
  }
}

int launch_attn_generic(const GenericAttnArgs& a, bool kv_f32, cudaStream_t st) {
  const uint64_t rows = (uint64_t)a.u.query_len * a.u.num_heads;
  if (rows == 0) return DOE_OK;
  const uint64_t blocks = (rows + kGenWarps - 1) / kGenWarps;
  if (blocks > 0x7fffffffull) {
    set_op_error("attention: %llu query rows exceed the grid limit", (unsigned long long)rows);
    return DOE_UNSUPPORTED;
  }
  const int per_lane = (int)((a.u.head_dim + 31) / 32);
  dim3 grid((unsigned)blocks), block(kGenWarps * 32);
#define DOE_GEN(KT, PL) attn_online_generic_kernel<KT, PL><<<grid, block, 0, st>>>(a)
  if (kv_f32) {
    if (per_lane <= 2) DOE_GEN(float, 2);
    else if (per_lane <= 4) DOE_GEN(float, 4);
    else if (per_lane <= 8) DOE_GEN(float, 8);
    else DOE_GEN(float, 16);
  } else {
    if (per_lane <= 2) DOE_GEN(__half, 2);
    else if (per_lane <= 4) DOE_GEN(__half, 4);
    else if (per_lane <= 8) DOE_GEN(__half, 8);
    else DOE_GEN(__half, 16);
  }
#undef DOE_GEN
  return cuda_status(cudaGetLastError(), "attn_online_generic_kernel");
}

}  // namespace doe
