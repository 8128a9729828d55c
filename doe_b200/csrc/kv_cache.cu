// kv_cache.cu -- KV-cache writes and reads, the stitch op and rope.
//
//   paged append  : kv_write (runtime/zig/src/tsir/emit_kernel_body.zig:620-690,
//                   emit_kernel_body_kv.zig:30-102) over a paged pool, with
//                   per-(token, kv head) int8 quantisation for int8 pools
//   paged gather  : kv_read (emit_kernel_body.zig:692-760) through a block table
//   dense write / read : the reference's per-head form, position checked
//                   against max_seq_len (run_csl_webgpu_emulator.mjs:615-644)
//   stitch        : bench/tools/attention_kv_axis_sharded_stitch.py:46-90
//   rope          : bench/inference-pipeline/kernels/rope.wgsl:12-35
//
// All copies are bit-exact.  The int8 quantiser (quantize_s8, div127 in
// common.cuh) forms its quotients from correctly rounded reciprocals and one
// exact residual correction, and rounds half to even, so it gives the CPU
// definition's IEEE-division results bit for bit.
#include "common.cuh"

namespace doe {

// ---- paged append ----------------------------------------------------------
struct PagedAppendArgs {
  const __half* new_k;  // [B, T, Hkv, D]
  const __half* new_v;
  uint8_t* k_pool;
  uint8_t* v_pool;
  __half* k_scale;      // [num_pages, Hkv, page_size]
  __half* v_scale;
  const int32_t* block_table;
  const int32_t* positions;
  int32_t* status;
  const float* freq_cis;  // RoPE table [rope_positions, D/2, {cos, sin}] or null
  int n_tokens, num_kv_heads, head_dim, page_size, num_pages, max_pages;
  int rope_positions;
  int page_shift;  // log2(page_size) when it is a power of two, else -1
};

// One warp per (sequence, token, kv head); lane owns head_dim/32 elements
// (an even count, so they load as half2 pairs).
template <bool INT8, int EPL>
__global__ void __launch_bounds__(256) paged_append_kernel(const PagedAppendArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x, b = blockIdx.y;
  const int Hkv = a.num_kv_heads, D = a.head_dim;
  const int pos0 = a.positions[b];
  const long long pos = (long long)pos0 + t;
  const long long pidx = pos / a.page_size;
  int page = -1;
  if (pos0 >= 0 && pidx < a.max_pages) page = a.block_table[(size_t)b * a.max_pages + pidx];
  if ((unsigned)page >= (unsigned)a.num_pages) {
    if (threadIdx.x == 0) report(a.status, DOE_DEVICE_ERR_PAGE);
    return;
  }
  const int in_page = (int)(pos - pidx * a.page_size);
  const size_t row = (size_t)page * a.page_size + in_page;
  for (int h = warp; h < Hkv; h += 8) {
    const size_t src_off = (((size_t)b * a.n_tokens + t) * Hkv + h) * D + (size_t)lane * EPL;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const __half* src = (kv ? a.new_v : a.new_k) + src_off;
      __half2 x2[EPL / 2];
#pragma unroll
      for (int i = 0; i < EPL / 2; ++i) x2[i] = reinterpret_cast<const __half2*>(src)[i];
      if (!INT8) {
        __half2* dst = reinterpret_cast<__half2*>((kv ? a.v_pool : a.k_pool) +
                                                  ((row * Hkv + h) * D + (size_t)lane * EPL) * 2);
#pragma unroll
        for (int i = 0; i < EPL / 2; ++i) dst[i] = x2[i];
      } else {
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < EPL / 2; ++i)
          amax = fmaxf(amax, fmaxf(fabsf(__low2float(x2[i])), fabsf(__high2float(x2[i]))));
        amax = warp_max(amax);
        const __half sh = __float2half_rn(div127(amax));
        const float sf = __half2float(sh);
        const float rs = sf != 0.0f ? __frcp_rn(sf) : 0.0f;
        int8_t* dst = reinterpret_cast<int8_t*>(kv ? a.v_pool : a.k_pool) + (row * Hkv + h) * D +
                      (size_t)lane * EPL;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float xv = (i & 1) ? __high2float(x2[i / 2]) : __low2float(x2[i / 2]);
          dst[i] = (int8_t)(uint8_t)(sf != 0.0f ? quantize_s8(xv, sf, rs) & 0xff : 0);
        }
        if (lane == 0) (kv ? a.v_scale : a.k_scale)[((size_t)page * Hkv + h) * a.page_size + in_page] = sh;
      }
    }
  }
}

// head_dim 128 fast path: one warp per (sequence, token); each half-warp owns
// a (K or V, kv head) row per step, 16 lanes x 16 bytes.  All of the token's
// rows are loaded before any is written, so a warp keeps Hkv x 512 bytes in
// flight.  Same arithmetic as paged_append_kernel.
template <bool INT8, int HKV>
__global__ void __launch_bounds__(128) paged_append_d128_kernel(const PagedAppendArgs a) {
  constexpr int D = 128;
  constexpr int ROWS = 2 * HKV;          // K and V rows of one token
  constexpr int PER = (ROWS + 1) / 2;    // rows per half-warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hw = lane >> 4, l16 = lane & 15;
  const int t = blockIdx.x * 4 + warp, b = blockIdx.y;
  if (t >= a.n_tokens) return;
  const int pos0 = a.positions[b];
  const long long pos = (long long)pos0 + t;
  const long long pidx = pos / a.page_size;
  int page = -1;
  if (pos0 >= 0 && pidx < a.max_pages) page = a.block_table[(size_t)b * a.max_pages + pidx];
  if ((unsigned)page >= (unsigned)a.num_pages) {
    if (lane == 0) report(a.status, DOE_DEVICE_ERR_PAGE);
    return;
  }
  const int in_page = (int)(pos - pidx * a.page_size);
  const size_t row = (size_t)page * a.page_size + in_page;
  const size_t src_tok = ((size_t)b * a.n_tokens + t) * HKV * D;
  // RoPE (rope.wgsl:12-35): lane l16 holds dims [8 l16, 8 l16 + 8); dim d < 64
  // pairs with d + 64, held by lane l16 ^ 8.  Both lanes of a pair need the
  // table entries of pair index 8 (l16 & 7) + e at this token's position.
  const bool rope = a.freq_cis != nullptr;
  float rc[8], rsn[8];
  if (rope)
    rope_table<4>(a.freq_cis, a.rope_positions, D / 2, pos, 8 * (l16 & 7), a.status, lane == 0, rc, rsn);
  uint4 x[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int rr = 2 * i + hw;  // 0..HKV-1: K heads, HKV..: V heads
    if (rr < ROWS) {
      const __half* src = (rr < HKV ? a.new_k : a.new_v) + src_tok + (size_t)(rr % HKV) * D + 8 * l16;
      x[i] = *reinterpret_cast<const uint4*>(src);
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int rr = 2 * i + hw;
    if (rope) {
      // every lane takes part in the exchange; only K rows are rotated
      uint4 px;
      px.x = __shfl_xor_sync(0xffffffffu, x[i].x, 8);
      px.y = __shfl_xor_sync(0xffffffffu, x[i].y, 8);
      px.z = __shfl_xor_sync(0xffffffffu, x[i].z, 8);
      px.w = __shfl_xor_sync(0xffffffffu, x[i].w, 8);
      if (rr < HKV) rope_rotate<4>(reinterpret_cast<const uint32_t*>(&x[i]),
                                  reinterpret_cast<const uint32_t*>(&px), l16 < 8, rc, rsn,
                                  reinterpret_cast<uint32_t*>(&x[i]));
    }
    if (rr >= ROWS) continue;  // uniform per half-warp; shuffles below stay inside it
    const int h = rr % HKV;
    uint8_t* pool = rr < HKV ? a.k_pool : a.v_pool;
    if (!INT8) {
      *reinterpret_cast<uint4*>(pool + ((row * HKV + h) * D + 8 * l16) * 2) = x[i];
      continue;
    }
    const __half2* hx = reinterpret_cast<const __half2*>(&x[i]);
    // |x| max in f16x2 (exact), then across the half-warp
    __half2 m2 = __hmax2(__habs2(hx[0]), __habs2(hx[1]));
    m2 = __hmax2(m2, __hmax2(__habs2(hx[2]), __habs2(hx[3])));
    float amax = fmaxf(__low2float(m2), __high2float(m2));
    // both half-warps run this together (ROWS is even); offsets <= 8 stay in a half
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const __half sh = __float2half_rn(div127(amax));
    const float sf = __half2float(sh);
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (sf >= 0x1p-14f && sf <= 65504.0f) {  // normal scale: packed, no clamp needed
      const float rs = __frcp_rn(sf);
#pragma unroll
      for (int e = 0; e < 4; ++e) quantize_s8x2_normal(__half22float2(hx[e]), sf, rs, q[2 * e], q[2 * e + 1]);
    } else if (sf != 0.0f) {
      const float rs = __frcp_rn(sf);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        q[2 * e] = quantize_s8(__low2float(hx[e]), sf, rs);
        q[2 * e + 1] = quantize_s8(__high2float(hx[e]), sf, rs);
      }
    }
    const uint32_t lo = pack_s8x4(q[0], q[1], q[2], q[3]), hi = pack_s8x4(q[4], q[5], q[6], q[7]);
    *reinterpret_cast<uint2*>(pool + (row * HKV + h) * D + 8 * l16) = make_uint2(lo, hi);
    if (l16 == 0) (rr < HKV ? a.k_scale : a.v_scale)[((size_t)page * HKV + h) * a.page_size + in_page] = sh;
  }
}

// head_dim 128 int8 quantise-append without RoPE: four lanes per row, each
// with 32 consecutive elements (64 bytes in, 32 bytes out), so one warp
// instruction works on 8 rows and the per-row work (the |x| max exchange,
// the scale's quotient and reciprocal, the page lookup, the scale store) is
// shared by 4 lanes instead of 16.  A warp covers 16 rows: one token of 8 kv
// heads (K then V), or 16 / (2 HKV) tokens of fewer heads; it loads all of
// them before it quantises any.  The page of each of the warp's tokens is
// looked up once, by lane j for its j-th token, and passed by shuffle.
// Same arithmetic, same bytes as paged_append_d128_kernel<true, HKV>.
template <int HKV>
__global__ void __launch_bounds__(128) paged_append_int8_d128_kernel(const PagedAppendArgs a) {
  constexpr int D = 128, ROWS = 2 * HKV, TPW = 16 / ROWS;  // tokens per warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, l4 = lane & 3;
  const int b = blockIdx.y;
  const int t0 = (blockIdx.x * 4 + warp) * TPW;
  const __half* in_k = a.new_k + ((size_t)b * a.n_tokens) * HKV * D + 32 * l4;
  const __half* in_v = a.new_v + ((size_t)b * a.n_tokens) * HKV * D + 32 * l4;
  uint4 x[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int fr = 8 * i + (lane >> 2), t = t0 + fr / ROWS, rr = fr % ROWS;
    if (t < a.n_tokens) {
      const uint4* src = reinterpret_cast<const uint4*>((rr < HKV ? in_k : in_v) +
                                                        ((size_t)t * HKV + rr % HKV) * D);
#pragma unroll
      for (int j = 0; j < 4; ++j) x[i][j] = __ldcs(src + j);  // read once: evict first
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) x[i][j] = make_uint4(0, 0, 0, 0);
    }
  }
  // lane j < TPW: the page row of token t0 + j (-1 when outside the chunk)
  long long my_row = -1;
  int my_in_page = 0, my_page = 0;
  {
    const int t = t0 + lane;
    const int pos0 = a.positions[b];
    if (lane < TPW && t < a.n_tokens) {
      const unsigned pos = (unsigned)pos0 + (unsigned)t;  // < 2^32: pos0 >= 0, t < 2^31
      const unsigned pidx = a.page_shift >= 0 ? pos >> a.page_shift : pos / (unsigned)a.page_size;
      int page = -1;
      if (pos0 >= 0 && pidx < (unsigned)a.max_pages) page = a.block_table[(size_t)b * a.max_pages + pidx];
      if ((unsigned)page < (unsigned)a.num_pages) {
        my_page = page;
        my_in_page = (int)(pos - pidx * (unsigned)a.page_size);
        my_row = (long long)page * a.page_size + my_in_page;
      } else {
        report(a.status, DOE_DEVICE_ERR_PAGE);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int fr = 8 * i + (lane >> 2), tt = fr / ROWS, rr = fr % ROWS, h = rr % HKV;
    const long long row = __shfl_sync(0xffffffffu, my_row, tt);
    const int page = __shfl_sync(0xffffffffu, my_page, tt);
    const int in_page = __shfl_sync(0xffffffffu, my_in_page, tt);
    const __half2* hx = reinterpret_cast<const __half2*>(&x[i][0]);
    __half2 m2 = __habs2(hx[0]);
#pragma unroll
    for (int e = 1; e < 16; ++e) m2 = __hmax2(m2, __habs2(hx[e]));
    float amax = fmaxf(__low2float(m2), __high2float(m2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const __half sh = __float2half_rn(div127(amax));
    const float sf = __half2float(sh);
    uint32_t w[8];
    if (sf >= 0x1p-14f && sf <= 65504.0f) {  // normal scale: packed, no clamp needed
      const float rs = __frcp_rn(sf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int q0, q1, q2, q3;
        quantize_s8x2_normal(__half22float2(hx[2 * e]), sf, rs, q0, q1);
        quantize_s8x2_normal(__half22float2(hx[2 * e + 1]), sf, rs, q2, q3);
        w[e] = pack_s8x4(q0, q1, q2, q3);
      }
    } else if (sf != 0.0f) {
      const float rs = __frcp_rn(sf);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        w[e] = pack_s8x4(quantize_s8(__low2float(hx[2 * e]), sf, rs), quantize_s8(__high2float(hx[2 * e]), sf, rs),
                         quantize_s8(__low2float(hx[2 * e + 1]), sf, rs),
                         quantize_s8(__high2float(hx[2 * e + 1]), sf, rs));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = 0;
    }
    if (row < 0) continue;  // outside the chunk, or a bad page (reported above)
    uint8_t* pool = rr < HKV ? a.k_pool : a.v_pool;
    uint4* dst = reinterpret_cast<uint4*>(pool + ((size_t)row * HKV + h) * D + 32 * l4);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    if (l4 == 0) (rr < HKV ? a.k_scale : a.v_scale)[((size_t)page * HKV + h) * a.page_size + in_page] = sh;
  }
}

int launch_paged_append(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t n_tokens,
                        const void* new_k, const void* new_v, const int32_t* positions,
                        const float* freq_cis, uint32_t rope_positions, const doe_launch* launch) {
  if (num_seqs == 0 || n_tokens == 0) return DOE_OK;
  const bool d128 = kv->head_dim == 128 && (kv->num_kv_heads == 8 || kv->num_kv_heads == 4 ||
                                            kv->num_kv_heads == 2 || kv->num_kv_heads == 1);
  if (freq_cis != nullptr && !d128) {
    set_op_error("doe_paged_append_rope: built for head_dim 128 with 1, 2, 4 or 8 kv heads "
                 "(got head_dim %u, %u kv heads)", kv->head_dim, kv->num_kv_heads);
    return DOE_UNSUPPORTED;
  }
  if (kv->head_dim % 64 != 0 || kv->head_dim > 512) {
    set_op_error("doe_paged_append: head_dim must be a multiple of 64 up to 512 (got %u)",
                 kv->head_dim);
    return DOE_UNSUPPORTED;
  }
  PagedAppendArgs a;
  a.new_k = static_cast<const __half*>(new_k);
  a.new_v = static_cast<const __half*>(new_v);
  a.k_pool = static_cast<uint8_t*>(kv->k_pool);
  a.v_pool = static_cast<uint8_t*>(kv->v_pool);
  a.k_scale = static_cast<__half*>(kv->k_scale);
  a.v_scale = static_cast<__half*>(kv->v_scale);
  a.block_table = kv->block_table;
  a.positions = positions;
  a.status = launch->status;
  a.n_tokens = (int)n_tokens;
  a.num_kv_heads = (int)kv->num_kv_heads;
  a.head_dim = (int)kv->head_dim;
  a.page_size = (int)kv->page_size;
  a.num_pages = (int)kv->num_pages;
  a.max_pages = (int)kv->max_pages_per_seq;
  a.freq_cis = freq_cis;
  a.rope_positions = (int)rope_positions;
  a.page_shift = -1;
  for (int s = 0; s < 31; ++s)
    if (kv->page_size == (1u << s)) a.page_shift = s;
  cudaStream_t st = static_cast<cudaStream_t>(launch->stream);
  const bool int8 = kv->kv_dtype == DOE_KV_INT8;
  if (d128 && int8 && freq_cis == nullptr) {
    const unsigned tok_per_cta = 4 * (8 / kv->num_kv_heads);
    dim3 g4((n_tokens + tok_per_cta - 1) / tok_per_cta, num_seqs);
    switch (kv->num_kv_heads) {
      case 8: paged_append_int8_d128_kernel<8><<<g4, 128, 0, st>>>(a); break;
      case 4: paged_append_int8_d128_kernel<4><<<g4, 128, 0, st>>>(a); break;
      case 2: paged_append_int8_d128_kernel<2><<<g4, 128, 0, st>>>(a); break;
      default: paged_append_int8_d128_kernel<1><<<g4, 128, 0, st>>>(a); break;
    }
    return cuda_status(cudaGetLastError(), "paged_append_int8_d128_kernel");
  }
  if (d128) {
    dim3 g2((n_tokens + 3) / 4, num_seqs);
#define DOE_PA2(H) \
  (int8 ? paged_append_d128_kernel<true, H><<<g2, 128, 0, st>>>(a) \
        : paged_append_d128_kernel<false, H><<<g2, 128, 0, st>>>(a))
    switch (kv->num_kv_heads) {
      case 8: DOE_PA2(8); break;
      case 4: DOE_PA2(4); break;
      case 2: DOE_PA2(2); break;
      default: DOE_PA2(1); break;
    }
#undef DOE_PA2
    return cuda_status(cudaGetLastError(), "paged_append_d128_kernel");
  }
  dim3 grid(n_tokens, num_seqs), block(256);
  const int epl = (int)kv->head_dim / 32;
#define DOE_PA(E) \
  (int8 ? paged_append_kernel<true, E><<<grid, block, 0, st>>>(a) \
        : paged_append_kernel<false, E><<<grid, block, 0, st>>>(a))
  switch (epl) {
    case 2: DOE_PA(2); break;
    case 4: DOE_PA(4); break;
    case 6: DOE_PA(6); break;
    case 8: DOE_PA(8); break;
    case 10: DOE_PA(10); break;
    case 12: DOE_PA(12); break;
    case 14: DOE_PA(14); break;
    default: DOE_PA(16); break;
  }
#undef DOE_PA
  return cuda_status(cudaGetLastError(), "paged_append_kernel");
}

// ---- paged gather (kv_read) ------------------------------------------------
struct PagedGatherArgs {
  const uint8_t* k_pool;
  const uint8_t* v_pool;
  const __half* k_scale;
  const __half* v_scale;
  uint8_t* k_out;
  uint8_t* v_out;
  __half* ks_out;
  __half* vs_out;
  const int32_t* table_row;
  int32_t* status;
  int start, len, num_kv_heads, row_bytes, page_size, num_pages, max_pages;
};

__global__ void paged_gather_kernel(const PagedGatherArgs a) {
  const int i = blockIdx.x;  // output token
  const long long pos = (long long)a.start + i;
  const long long pidx = pos / a.page_size;
  const int page = pidx < a.max_pages ? a.table_row[pidx] : -1;
  if ((unsigned)page >= (unsigned)a.num_pages) {
    if (threadIdx.x == 0) report(a.status, DOE_DEVICE_ERR_PAGE);
    return;
  }
  const int in_page = (int)(pos - pidx * a.page_size);
  const size_t row = (size_t)page * a.page_size + in_page;
  const int n16 = a.row_bytes / 16;
  for (int j = threadIdx.x; j < n16; j += blockDim.x) {
    reinterpret_cast<uint4*>(a.k_out + (size_t)i * a.row_bytes)[j] =
        reinterpret_cast<const uint4*>(a.k_pool + row * a.row_bytes)[j];
    reinterpret_cast<uint4*>(a.v_out + (size_t)i * a.row_bytes)[j] =
        reinterpret_cast<const uint4*>(a.v_pool + row * a.row_bytes)[j];
  }
  if (a.ks_out && a.k_scale) {
    for (int h = threadIdx.x; h < a.num_kv_heads; h += blockDim.x) {
      const size_t si = ((size_t)page * a.num_kv_heads + h) * a.page_size + in_page;
      a.ks_out[(size_t)i * a.num_kv_heads + h] = a.k_scale[si];
      a.vs_out[(size_t)i * a.num_kv_heads + h] = a.v_scale[si];
    }
  }
}

int launch_paged_gather(const doe_paged_kv* kv, uint32_t seq, uint32_t start, uint32_t len,
                        void* k_out, void* v_out, void* ks_out, void* vs_out,
                        const doe_launch* launch) {
  if (len == 0) return DOE_OK;
  const uint32_t elem = kv->kv_dtype == DOE_KV_INT8 ? 1 : 2;
  const uint64_t row_bytes = (uint64_t)kv->num_kv_heads * kv->head_dim * elem;
  if (row_bytes % 16 != 0) {
    set_op_error("doe_paged_gather: row of %llu bytes is not a multiple of 16",
                 (unsigned long long)row_bytes);
    return DOE_UNSUPPORTED;
  }
  PagedGatherArgs a;
  a.k_pool = static_cast<const uint8_t*>(kv->k_pool);
  a.v_pool = static_cast<const uint8_t*>(kv->v_pool);
  a.k_scale = static_cast<const __half*>(kv->k_scale);
  a.v_scale = static_cast<const __half*>(kv->v_scale);
  a.k_out = static_cast<uint8_t*>(k_out);
  a.v_out = static_cast<uint8_t*>(v_out);
  a.ks_out = static_cast<__half*>(ks_out);
  a.vs_out = static_cast<__half*>(vs_out);
  a.table_row = kv->block_table + (size_t)seq * kv->max_pages_per_seq;
  a.status = launch->status;
  a.start = (int)start;
  a.len = (int)len;
  a.num_kv_heads = (int)kv->num_kv_heads;
  a.row_bytes = (int)row_bytes;
  a.page_size = (int)kv->page_size;
  a.num_pages = (int)kv->num_pages;
  a.max_pages = (int)kv->max_pages_per_seq;
  paged_gather_kernel<<<len, 128, 0, static_cast<cudaStream_t>(launch->stream)>>>(a);
  return cuda_status(cudaGetLastError(), "paged_gather_kernel");
}

// ---- dense per-head kv_write / kv_read --------------------------------------
__global__ void kv_write_dense_kernel(const uint8_t* k_proj, const uint8_t* v_proj,
                                      uint8_t* k_cache, uint8_t* v_cache,
                                      const uint32_t* positions, uint32_t num_positions,
                                      uint32_t max_seq_len, uint32_t row_bytes,
                                      int32_t* status) {
  const uint32_t head = blockIdx.x;
  const uint32_t pos = positions[num_positions == 1 ? 0 : head];
  if (pos >= max_seq_len) {
    if (threadIdx.x == 0) report(status, DOE_DEVICE_ERR_POSITION);
    return;
  }
  const size_t src = (size_t)head * row_bytes;
  const size_t dst = ((size_t)head * max_seq_len + pos) * row_bytes;
  for (uint32_t j = threadIdx.x; j < row_bytes; j += blockDim.x) {
    k_cache[dst + j] = k_proj[src + j];
    v_cache[dst + j] = v_proj[src + j];
  }
}

__global__ void kv_read_dense_kernel(const uint8_t* k_cache, const uint8_t* v_cache,
                                     uint8_t* k_out, uint8_t* v_out, uint32_t read_start,
                                     uint32_t read_len, uint32_t max_seq_len,
                                     uint32_t row_bytes) {
  const uint32_t i = blockIdx.x, head = blockIdx.y;
  const size_t src = ((size_t)head * max_seq_len + read_start + i) * row_bytes;
  const size_t dst = ((size_t)head * read_len + i) * row_bytes;
  for (uint32_t j = threadIdx.x; j < row_bytes; j += blockDim.x) {
    k_out[dst + j] = k_cache[src + j];
    v_out[dst + j] = v_cache[src + j];
  }
}

int launch_kv_write_dense(const void* k_proj, const void* v_proj, void* k_cache, void* v_cache,
                          const uint32_t* positions, uint32_t num_positions, uint32_t heads,
                          uint32_t max_seq_len, uint32_t head_dim, uint32_t elem_bytes,
                          const doe_launch* launch) {
  if (heads == 0) return DOE_OK;
  kv_write_dense_kernel<<<heads, 128, 0, static_cast<cudaStream_t>(launch->stream)>>>(
      static_cast<const uint8_t*>(k_proj), static_cast<const uint8_t*>(v_proj),
      static_cast<uint8_t*>(k_cache), static_cast<uint8_t*>(v_cache), positions, num_positions,
      max_seq_len, head_dim * elem_bytes, launch->status);
  return cuda_status(cudaGetLastError(), "kv_write_dense_kernel");
}

int launch_kv_read_dense(const void* k_cache, const void* v_cache, void* k_out, void* v_out,
                         uint32_t heads, uint32_t read_start, uint32_t read_len,
                         uint32_t max_seq_len, uint32_t head_dim, uint32_t elem_bytes,
                         const doe_launch* launch) {
  if (heads == 0 || read_len == 0) return DOE_OK;
  kv_read_dense_kernel<<<dim3(read_len, heads), 128, 0, static_cast<cudaStream_t>(launch->stream)>>>(
      static_cast<const uint8_t*>(k_cache), static_cast<const uint8_t*>(v_cache),
      static_cast<uint8_t*>(k_out), static_cast<uint8_t*>(v_out), read_start, read_len,
      max_seq_len, head_dim * elem_bytes);
  return cuda_status(cudaGetLastError(), "kv_read_dense_kernel");
}

// ---- stitch (natural-domain partials rows [O[D], max, sum]) -----------------
__global__ void stitch_kernel(const float* partials, uint32_t num_shards, uint32_t head_dim,
                              float* out) {
  const uint32_t row = blockIdx.x;
  const uint32_t w = head_dim + 2;
  const float* p = partials + (size_t)row * num_shards * w;
  float gmax = p[head_dim];
  for (uint32_t i = 1; i < num_shards; ++i) gmax = fmaxf(gmax, p[(size_t)i * w + head_dim]);
  float gsum = 0.0f;
  for (uint32_t i = 0; i < num_shards; ++i)
    gsum += expf(p[(size_t)i * w + head_dim] - gmax) * p[(size_t)i * w + head_dim + 1];
  for (uint32_t d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.0f;
    if (gsum != 0.0f)
      for (uint32_t i = 0; i < num_shards; ++i)
        acc += expf(p[(size_t)i * w + head_dim] - gmax) * p[(size_t)i * w + d];
    out[(size_t)row * head_dim + d] = gsum == 0.0f ? 0.0f : acc / gsum;
  }
}

int launch_stitch(const float* partials, uint32_t rows, uint32_t num_shards, uint32_t head_dim,
                  float* out, const doe_launch* launch) {
  if (rows == 0) return DOE_OK;
  const uint32_t threads = head_dim >= 256 ? 256 : ((head_dim + 31) / 32) * 32;
  stitch_kernel<<<rows, threads, 0, static_cast<cudaStream_t>(launch->stream)>>>(
      partials, num_shards, head_dim, out);
  return cuda_status(cudaGetLastError(), "stitch_kernel");
}

// ---- rope --------------------------------------------------------------------
__global__ void rope_kernel(float* qk, const float* freq_cis, uint32_t seq_len,
                            uint32_t num_heads, uint32_t head_dim, uint32_t position_offset) {
  const uint32_t half = head_dim / 2;
  const uint32_t pair = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t head = blockIdx.y, s = blockIdx.z;
  if (pair >= half || head >= num_heads || s >= seq_len) return;
  const uint64_t pos = (uint64_t)s + position_offset;
  float* base = qk + ((size_t)s * num_heads + head) * head_dim;
  const float x0 = base[pair], x1 = base[pair + half];
  const uint64_t f = pos * half + pair;
  const float c = freq_cis[f * 2], sn = freq_cis[f * 2 + 1];
  base[pair] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
  base[pair + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
}

int launch_rope(float* qk, const float* freq_cis, uint32_t seq_len, uint32_t num_heads,
                uint32_t head_dim, uint32_t position_offset, const doe_launch* launch) {
  if (seq_len == 0 || num_heads == 0 || head_dim < 2) return DOE_OK;
  const uint32_t half = head_dim / 2;
  dim3 grid((half + 63) / 64, num_heads, seq_len);
  rope_kernel<<<grid, 64, 0, static_cast<cudaStream_t>(launch->stream)>>>(
      qk, freq_cis, seq_len, num_heads, head_dim, position_offset);
  return cuda_status(cudaGetLastError(), "rope_kernel");
}

}  // namespace doe
