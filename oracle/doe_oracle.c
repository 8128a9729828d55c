/*
 * doe_oracle.c -- CPU restatement of Doe's attention / KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 * Nothing in the shipped library (doe_b200/libdoe_cuda.so) links, loads or
 * calls this file.  Built with -O2 -ffp-contract=off so every sum below runs
 * in the order written (no fused multiply-add), as the WGSL/Zig sources
 * state it.  Reference paths are relative to the doerun/doe source tree.
 */
#include "doe_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
  else omp_set_num_threads(omp_get_num_procs());
#else
  (void)threads;
#endif
}

/* ------------------------------------------------------------------------ */
/* binary16 <-> binary32, round to nearest even (IEEE 754-2008 conversion). */
/* ------------------------------------------------------------------------ */
float doe_oracle_h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t ex = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (ex == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      /* subnormal: man * 2^-24, exactly representable in binary32 */
      float f = (float)man * (1.0f / 16777216.0f);
      memcpy(&bits, &f, 4);
      bits |= sign;
    }
  } else if (ex == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((ex + 112u) << 23) | (man << 13);
  }
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

uint16_t doe_oracle_f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) /* inf / nan */
    return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
  if (ax >= 0x477ff000u) /* >= 65520 rounds to infinity */
    return (uint16_t)(sign | 0x7c00u);
  if (ax < 0x38800000u) { /* below 2^-14: binary16 subnormal or zero */
    if (ax <= 0x33000000u) return sign; /* <= 2^-25 rounds to zero (tie -> even) */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126u - e; /* value * 2^24 = m * 2^(e-126) */
    uint32_t r = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (r & 1u))) r++;
    return (uint16_t)(sign | r);
  }
  uint32_t h = (ax - (112u << 23)) >> 13;
  uint32_t rest = ax & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

void doe_oracle_h2f_array(const uint16_t* src, float* dst, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) dst[i] = doe_oracle_h2f(src[i]);
}

void doe_oracle_f2h_array(const float* src, uint16_t* dst, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) dst[i] = doe_oracle_f2h(src[i]);
}

/* ------------------------------------------------------------------------ */
/* attention-decode.wgsl (bench/inference-pipeline/kernels/attention-decode.wgsl:1-136)
 *
 * One workgroup of 64 lanes per head:
 *   scores[t] = dot_qk(head, t) * scale, dot_qk = vec4 dots then tail (18-44)
 *   lane max over t = lane, lane+64, ... then tree 32..1 (66-83)
 *   e_t = exp(clamp(s_t - max, -30, 30)); lane sums; tree 32..1 (86-105)
 *   p_t = e_t / total (108-113); o_d = sum_t p_t * v[t,d], serial in t (116-135)
 * The f64 twin follows the same order; it pins the attention-slice KAT whose
 * exact logits were computed in higher precision.
 */
#define DOE_DECODE_WGSL_BODY(T, EXPF)                                          \
  if (!q || !k || !v || !out || head_dim == 0 || kv_len == 0)                  \
    return DOE_ORACLE_EINVAL;                                                  \
  T* scores = (T*)malloc(sizeof(T) * kv_len);                                  \
  if (!scores) return DOE_ORACLE_EINVAL;                                       \
  for (uint32_t head = 0; head < num_heads; ++head) {                          \
    const T* qh = q + (uint64_t)head * head_dim;                               \
    const T* kh = k + (uint64_t)head * head_dim * kv_len;                      \
    const T* vh = v + (uint64_t)head * head_dim * kv_len;                      \
    uint32_t vec_dim = head_dim & ~3u;                                         \
    for (uint32_t t = 0; t < kv_len; ++t) {                                    \
      const T* kt = kh + (uint64_t)t * head_dim;                               \
      T acc = 0;                                                               \
      for (uint32_t d = 0; d < vec_dim; d += 4) {                              \
        T dp = qh[d] * kt[d];                                                  \
        dp = dp + qh[d + 1] * kt[d + 1];                                       \
        dp = dp + qh[d + 2] * kt[d + 2];                                       \
        dp = dp + qh[d + 3] * kt[d + 3];                                       \
        acc = acc + dp;                                                        \
      }                                                                        \
      for (uint32_t d = vec_dim; d < head_dim; ++d) acc = acc + qh[d] * kt[d]; \
      scores[t] = acc * scale;                                                 \
    }                                                                          \
    T lane[64];                                                                \
    for (uint32_t tid = 0; tid < 64; ++tid) {                                  \
      T lm = (T)-1e30;                                                         \
      for (uint32_t s2 = tid; s2 < kv_len; s2 += 64)                           \
        lm = scores[s2] > lm ? scores[s2] : lm;                                \
      lane[tid] = lm;                                                          \
    }                                                                          \
    for (uint32_t st = 32; st > 0; st /= 2)                                    \
      for (uint32_t tid = 0; tid < st; ++tid)                                  \
        lane[tid] = lane[tid + st] > lane[tid] ? lane[tid + st] : lane[tid];   \
    T rm = lane[0];                                                            \
    for (uint32_t tid = 0; tid < 64; ++tid) {                                  \
      T ls = 0;                                                                \
      for (uint32_t s3 = tid; s3 < kv_len; s3 += 64) {                         \
        T x = scores[s3] - rm;                                                 \
        x = x < (T)-30 ? (T)-30 : (x > (T)30 ? (T)30 : x);                     \
        T e = EXPF(x);                                                         \
        scores[s3] = e;                                                        \
        ls = ls + e;                                                           \
      }                                                                        \
      lane[tid] = ls;                                                          \
    }                                                                          \
    for (uint32_t st = 32; st > 0; st /= 2)                                    \
      for (uint32_t tid = 0; tid < st; ++tid) lane[tid] = lane[tid] + lane[tid + st]; \
    T total = lane[0];                                                         \
    for (uint32_t t = 0; t < kv_len; ++t) scores[t] = scores[t] / total;       \
    for (uint32_t d = 0; d < head_dim; ++d) {                                  \
      T acc = 0;                                                               \
      for (uint32_t t = 0; t < kv_len; ++t)                                    \
        acc = acc + scores[t] * vh[(uint64_t)t * head_dim + d];                \
      out[(uint64_t)head * head_dim + d] = acc;                                \
    }                                                                          \
  }                                                                            \
  free(scores);                                                                \
  return DOE_ORACLE_OK;

int doe_oracle_attention_decode_wgsl_f32(const float* q, const float* k,
                                         const float* v, float* out,
                                         uint32_t num_heads, uint32_t head_dim,
                                         uint32_t kv_len, float scale) {
  DOE_DECODE_WGSL_BODY(float, expf)
}

int doe_oracle_attention_decode_wgsl_f64(const double* q, const double* k,
                                         const double* v, double* out,
                                         uint32_t num_heads, uint32_t head_dim,
                                         uint32_t kv_len, double scale) {
  DOE_DECODE_WGSL_BODY(double, exp)
}

/* ------------------------------------------------------------------------ */
/* attention-prefill.wgsl (bench/inference-pipeline/kernels/attention-prefill.wgsl:19-112)
 * Causal: col > row -> -1e30 (39-40); scalar dot in d order (43-47); 64-lane
 * strided max/sum combined serially by lane 0 (61-91); p = e/total; o serial.
 * Layout [H, S, D].
 */
int doe_oracle_attention_prefill_wgsl_f32(const float* q, const float* k,
                                          const float* v, float* out,
                                          uint32_t seq_len, uint32_t head_dim,
                                          uint32_t num_heads, float scale) {
  if (!q || !k || !v || !out || seq_len == 0 || head_dim == 0) return DOE_ORACLE_EINVAL;
  float* scores = (float*)malloc(sizeof(float) * seq_len);
  if (!scores) return DOE_ORACLE_EINVAL;
  for (uint32_t head = 0; head < num_heads; ++head) {
    uint64_t ho = (uint64_t)head * seq_len * head_dim;
    for (uint32_t row = 0; row < seq_len; ++row) {
      const float* qr = q + ho + (uint64_t)row * head_dim;
      for (uint32_t col = 0; col < seq_len; ++col) {
        if (col > row) {
          scores[col] = -1e30f;
        } else {
          const float* kc = k + ho + (uint64_t)col * head_dim;
          float dot = 0.0f;
          for (uint32_t d = 0; d < head_dim; ++d) dot = dot + qr[d] * kc[d];
          scores[col] = dot * scale;
        }
      }
      float lane[64];
      for (uint32_t tid = 0; tid < 64; ++tid) {
        float m = -1e30f;
        for (uint32_t i = tid; i < seq_len; i += 64) m = fmaxf(m, scores[i]);
        lane[tid] = m;
      }
      float row_max = lane[0];
      for (uint32_t j = 1; j < 64; ++j) row_max = fmaxf(row_max, lane[j]);
      for (uint32_t tid = 0; tid < 64; ++tid) {
        float s = 0.0f;
        for (uint32_t i = tid; i < seq_len; i += 64) {
          float x = scores[i] - row_max;
          x = x < -30.0f ? -30.0f : (x > 30.0f ? 30.0f : x);
          float e = expf(x);
          scores[i] = e;
          s = s + e;
        }
        lane[tid] = s;
      }
      float total = 0.0f;
      for (uint32_t j = 0; j < 64; ++j) total = total + lane[j];
      for (uint32_t i = 0; i < seq_len; ++i) scores[i] = scores[i] / total;
      for (uint32_t d = 0; d < head_dim; ++d) {
        float acc = 0.0f;
        for (uint32_t t = 0; t < seq_len; ++t)
          acc = acc + scores[t] * v[ho + (uint64_t)t * head_dim + d];
        out[ho + (uint64_t)row * head_dim + d] = acc;
      }
    }
  }
  free(scores);
  return DOE_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* reference_interpreter.zig tryAttentionScores
 * (runtime/zig/src/tsir/reference_interpreter.zig:1095-1289):
 *   pass 1: dot (d order) * scale, masked keys -> -1e30, running max from -inf
 *   pass 2: w = exp(s - max), sum (k order); sum == 0 -> no result
 *   out[d] = sum_k v[k,d] * (w[k] / sum)  (division inside the loop, 1271-1280)
 */
int doe_oracle_attention_two_pass_f32(const float* q, const float* k,
                                      const float* v, float* out,
                                      uint32_t head_dim, uint32_t kv_len,
                                      float scale, uint32_t causal_mode,
                                      uint32_t window) {
  if (!q || !k || !v || !out || head_dim == 0 || kv_len == 0) return DOE_ORACLE_EINVAL;
  if (causal_mode == 2 && window == 0) return DOE_ORACLE_EINVAL;
  float* scores = (float*)malloc(sizeof(float) * kv_len);
  if (!scores) return DOE_ORACLE_EINVAL;
  const float sentinel = -1.0e30f;
  uint32_t sliding_start = 0;
  if (causal_mode == 2 && kv_len > window) sliding_start = kv_len - window;
  float max_score = -INFINITY;
  for (uint32_t t = 0; t < kv_len; ++t) {
    float dot = 0.0f;
    for (uint32_t d = 0; d < head_dim; ++d) dot += q[d] * k[(uint64_t)t * head_dim + d];
    float sc = dot * scale;
    if (causal_mode == 1 && t > kv_len - 1) sc = sentinel; /* single-Q: never */
    if (causal_mode == 2 && t < sliding_start) sc = sentinel;
    scores[t] = sc;
    if (sc > max_score) max_score = sc;
  }
  float sum_exp = 0.0f;
  for (uint32_t t = 0; t < kv_len; ++t) {
    float e = expf(scores[t] - max_score);
    scores[t] = e;
    sum_exp += e;
  }
  if (sum_exp == 0.0f) {
    free(scores);
    return DOE_ORACLE_EZERO;
  }
  for (uint32_t d = 0; d < head_dim; ++d) {
    float acc = 0.0f;
    for (uint32_t t = 0; t < kv_len; ++t)
      acc += v[(uint64_t)t * head_dim + d] * (scores[t] / sum_exp);
    out[d] = acc;
  }
  free(scores);
  return DOE_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* emit_local_partials / stitch_kv_axis_sharded_partials
 * (bench/tools/attention_kv_axis_sharded_stitch.py:46-90, 93-174;
 *  runtime/zig/src/tsir/emit_kernel_body_attention.zig:279-443)
 * A shard's row is [sum_k w_k v_k (unnormalised), local_max, local_sum];
 * tail slots (slot_base + k >= kv_len) are held at the -1e30 sentinel.
 */
int doe_oracle_emit_local_partials_f32(const float* q, const float* k_local,
                                       const float* v_local, float* out_row,
                                       uint32_t head_dim, uint32_t slots,
                                       uint32_t slot_base, uint32_t kv_len,
                                       float scale) {
  if (!q || !out_row || head_dim == 0) return DOE_ORACLE_EINVAL;
  const float sentinel = -1.0e30f;
  float* scores = (float*)malloc(sizeof(float) * (slots ? slots : 1));
  if (!scores) return DOE_ORACLE_EINVAL;
  float local_max = sentinel;
  for (uint32_t t = 0; t < slots; ++t) {
    scores[t] = sentinel;
    if (slot_base + t >= kv_len) continue;
    float dot = 0.0f;
    for (uint32_t d = 0; d < head_dim; ++d) dot += q[d] * k_local[(uint64_t)t * head_dim + d];
    float sc = dot * scale;
    scores[t] = sc;
    if (sc > local_max) local_max = sc;
  }
  float local_sum = 0.0f;
  for (uint32_t t = 0; t < slots; ++t) {
    float e = expf(scores[t] - local_max);
    scores[t] = e;
    local_sum += e;
  }
  for (uint32_t d = 0; d < head_dim; ++d) {
    float acc = 0.0f;
    for (uint32_t t = 0; t < slots; ++t) acc += v_local[(uint64_t)t * head_dim + d] * scores[t];
    out_row[d] = acc;
  }
  out_row[head_dim] = local_max;
  out_row[head_dim + 1] = local_sum;
  free(scores);
  return DOE_ORACLE_OK;
}

int doe_oracle_stitch_partials_f32(const float* partials, uint32_t num_shards,
                                   uint32_t head_dim, float* out) {
  if (!partials || !out || num_shards == 0 || head_dim == 0) return DOE_ORACLE_EINVAL;
  const uint32_t row = head_dim + 2;
  float gmax = partials[head_dim];
  for (uint32_t i = 1; i < num_shards; ++i) {
    float m = partials[(uint64_t)i * row + head_dim];
    if (m > gmax) gmax = m;
  }
  float gsum = 0.0f;
  for (uint32_t i = 0; i < num_shards; ++i) {
    const float* p = partials + (uint64_t)i * row;
    gsum += expf(p[head_dim] - gmax) * p[head_dim + 1];
  }
  if (gsum == 0.0f) {
    memset(out, 0, sizeof(float) * head_dim);
    return DOE_ORACLE_OK;
  }
  for (uint32_t d = 0; d < head_dim; ++d) {
    float acc = 0.0f;
    for (uint32_t i = 0; i < num_shards; ++i) {
      const float* p = partials + (uint64_t)i * row;
      acc += expf(p[head_dim] - gmax) * p[d];
    }
    out[d] = acc / gsum;
  }
  return DOE_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* attention_head256_f16kv.wgsl, generalised to any head_dim
 * (runtime/zig/tests/tsir/real/attention_head256_f16kv/attention_head256_f16kv.wgsl:14-269)
 *   kv head = h / (H / Hkv)                                          (46-49)
 *   get_kv_pos: dense / ring (abs % window) / paged table            (51-63)
 *   kv length from the uniform or kv_len_buffer[0]                   (65-70)
 *   key bounds: causal limit abs_q - kv_start + 1, window lower bound (113-136)
 *   32-key blocks: scores (vec4 dots), optional tanh softcap, block max,
 *   correction exp(m_i - m_new), p = exp(s - m_new), acc += p v     (138-255)
 *   out = acc * (l > 0 ? 1/l : 0)                                    (257-268)
 */
typedef struct kv_rows {
  uint32_t dtype; /* 0 f16, 1 int8 with per-(row, head) f16 scale */
  const void* base;
  const uint16_t* scale; /* [num_pages, num_kv_heads, page_size] */
  uint32_t num_kv_heads;
  uint32_t head_dim;
  uint32_t page_size;
} kv_rows;

/* Scale of physical row `phys`, kv head `kvh`: page-blocked so the 16 (or
 * page_size) tokens of one page and head sit next to each other.          */
static uint64_t scale_index(uint64_t phys, uint32_t kvh, uint32_t num_kv_heads,
                            uint32_t page_size) {
  uint64_t page = phys / page_size, in_page = phys % page_size;
  return (page * num_kv_heads + kvh) * page_size + in_page;
}

static void load_row(const kv_rows* s, uint64_t phys, uint32_t kvh, float* dst) {
  uint64_t off = (phys * s->num_kv_heads + kvh) * s->head_dim;
  if (s->dtype == 0) {
    const uint16_t* src = (const uint16_t*)s->base + off;
    for (uint32_t d = 0; d < s->head_dim; ++d) dst[d] = doe_oracle_h2f(src[d]);
  } else {
    const int8_t* src = (const int8_t*)s->base + off;
    float sc = doe_oracle_h2f(s->scale[scale_index(phys, kvh, s->num_kv_heads, s->page_size)]);
    for (uint32_t d = 0; d < s->head_dim; ++d) dst[d] = (float)src[d] * sc;
  }
}

/* One query row of the online-softmax kernel.  `phys_of(ctx, key_pos)` maps
 * a logical key position to a physical cache row (or UINT64_MAX: rejected). */
typedef uint64_t (*phys_fn)(const void* ctx, uint32_t key_pos);

static int online_row(const float* qrow, uint32_t head_dim, uint32_t seq_len,
                      uint32_t min_key_pos, uint32_t max_key_pos, float scale,
                      float softcap, const kv_rows* ks, const kv_rows* vs,
                      uint32_t kvh, phys_fn phys_of, const void* pctx,
                      float* outrow) {
  enum { BLOCK = 32 };
  float* acc = (float*)calloc(head_dim, sizeof(float));
  float* krow = (float*)malloc(sizeof(float) * head_dim);
  float* vrow = (float*)malloc(sizeof(float) * head_dim);
  if (!acc || !krow || !vrow) {
    free(acc); free(krow); free(vrow);
    return DOE_ORACLE_EINVAL;
  }
  float m_i = -3.402823e+38f;
  float l_i = 0.0f;
  uint32_t vec_dim = head_dim & ~3u;
  uint32_t nblocks = (seq_len + BLOCK - 1) / BLOCK;
  int rc = DOE_ORACLE_OK;
  for (uint32_t blk = 0; blk < nblocks && rc == DOE_ORACLE_OK; ++blk) {
    uint32_t start = blk * BLOCK;
    float scores[BLOCK], probs[BLOCK];
    int active[BLOCK];
    float block_max = -3.402823e+38f;
    for (uint32_t j = 0; j < BLOCK; ++j) {
      uint32_t kp = start + j;
      scores[j] = 0.0f;
      probs[j] = 0.0f;
      active[j] = (kp < seq_len && kp >= min_key_pos && kp < max_key_pos);
      if (!active[j]) continue;
      uint64_t phys = phys_of(pctx, kp);
      if (phys == UINT64_MAX) { rc = DOE_ORACLE_ERANGE; break; }
      load_row(ks, phys, kvh, krow);
      float dotp = 0.0f;
      for (uint32_t d = 0; d < vec_dim; d += 4) {
        float dp = qrow[d] * krow[d];
        dp = dp + qrow[d + 1] * krow[d + 1];
        dp = dp + qrow[d + 2] * krow[d + 2];
        dp = dp + qrow[d + 3] * krow[d + 3];
        dotp = dotp + dp;
      }
      for (uint32_t d = vec_dim; d < head_dim; ++d) dotp = dotp + qrow[d] * krow[d];
      float s = dotp * scale;
      if (softcap > 0.0f) s = tanhf(s / softcap) * softcap;
      scores[j] = s;
      block_max = fmaxf(block_max, s);
    }
    if (rc != DOE_ORACLE_OK) break;
    float m_new = fmaxf(m_i, block_max);
    float corr = expf(m_i - m_new);
    l_i = l_i * corr;
    for (uint32_t d = 0; d < head_dim; ++d) acc[d] = acc[d] * corr;
    for (uint32_t j = 0; j < BLOCK; ++j) {
      if (!active[j]) continue;
      float p = expf(scores[j] - m_new);
      probs[j] = p;
      l_i = l_i + p;
    }
    for (uint32_t j = 0; j < BLOCK; ++j) {
      float p = probs[j];
      if (p == 0.0f) continue;
      uint64_t phys = phys_of(pctx, start + j);
      load_row(vs, phys, kvh, vrow);
      for (uint32_t d = 0; d < head_dim; ++d) acc[d] = acc[d] + p * vrow[d];
    }
    m_i = m_new;
  }
  if (rc == DOE_ORACLE_OK) {
    float inv = l_i > 0.0f ? 1.0f / l_i : 0.0f;
    for (uint32_t d = 0; d < head_dim; ++d) outrow[d] = acc[d] * inv;
  }
  free(acc); free(krow); free(vrow);
  return rc;
}

typedef struct single_table_ctx {
  const doe_oracle_attn_uniforms* u;
  const uint32_t* page_table;
} single_table_ctx;

static uint64_t phys_single(const void* vctx, uint32_t key_pos) {
  const single_table_ctx* c = (const single_table_ctx*)vctx;
  const doe_oracle_attn_uniforms* u = c->u;
  uint32_t abs_key = u->kv_start + key_pos;
  if (u->kv_layout == 1 && u->sliding_window > 0) return abs_key % u->sliding_window;
  if (u->kv_layout == 2) {
    uint32_t page_idx = abs_key / u->page_size;
    uint32_t in_page = abs_key - page_idx * u->page_size;
    return (uint64_t)c->page_table[page_idx] * u->page_size + in_page;
  }
  return abs_key;
}

int doe_oracle_attention_online_f16kv(const doe_oracle_attn_uniforms* u,
                                      const float* q, const uint16_t* k,
                                      const uint16_t* v, float* out,
                                      const uint32_t* kv_len_buffer,
                                      const uint32_t* page_table, int threads) {
  if (!u || !q || !k || !v || !out) return DOE_ORACLE_EINVAL;
  if (u->num_kv_heads == 0 || u->num_heads % u->num_kv_heads != 0 || u->head_dim == 0)
    return DOE_ORACLE_EINVAL;
  if (u->kv_layout == 2 && (!page_table || u->page_size == 0)) return DOE_ORACLE_EINVAL;
  if (u->kv_len_source != 0 && !kv_len_buffer) return DOE_ORACLE_EINVAL;
  const uint32_t H = u->num_heads, D = u->head_dim;
  const uint32_t heads_per_kv = u->num_heads / u->num_kv_heads;
  const uint32_t seq_len = u->kv_len_source == 0 ? u->seq_len : kv_len_buffer[0];
  kv_rows ks = {0, k, NULL, u->num_kv_heads, D, 1};
  kv_rows vs = {0, v, NULL, u->num_kv_heads, D, 1};
  single_table_ctx pctx = {u, page_table};
  int rc = DOE_ORACLE_OK;
  set_threads(threads);
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (uint32_t qp = 0; qp < u->query_len; ++qp) {
    for (uint32_t h = 0; h < H; ++h) {
      uint32_t abs_q = qp + u->start_pos;
      uint32_t min_key = 0, max_key = seq_len;
      if (u->is_causal) {
        if (abs_q < u->kv_start) max_key = 0;
        else {
          uint32_t lim = abs_q - u->kv_start + 1;
          max_key = seq_len < lim ? seq_len : lim;
        }
      }
      if (u->sliding_window > 0 && abs_q >= u->sliding_window) {
        uint32_t min_abs = abs_q - u->sliding_window + 1;
        if (min_abs > u->kv_start) min_key = min_abs - u->kv_start;
        if (min_key > seq_len) min_key = seq_len;
      }
      uint64_t off = ((uint64_t)qp * H + h) * D;
      int r = online_row(q + off, D, seq_len, min_key, max_key, u->scale,
                         u->attn_softcap, &ks, &vs, h / heads_per_kv, phys_single,
                         &pctx, out + off);
      if (r != DOE_ORACLE_OK) {
#pragma omp atomic write
        rc = r;
      }
    }
  }
  return rc;
}

/* ------------------------------------------------------------------------ */
/* Batched paged decode: the head256 semantics with query_len = 1, causal at
 * abs_q = kv_len - 1 (so every key 0..kv_len-1 is active), kv_start = 0 and a
 * per-sequence row of the block table in place of the single page_table.
 * int8 pools dequantise as q * float(scale[row, head]).                   */
typedef struct batched_ctx {
  const int32_t* row;
  uint32_t max_pages;
  uint32_t page_size;
  uint32_t num_pages;
} batched_ctx;

static uint64_t phys_batched(const void* vctx, uint32_t key_pos) {
  const batched_ctx* c = (const batched_ctx*)vctx;
  uint32_t page_idx = key_pos / c->page_size;
  if (page_idx >= c->max_pages) return UINT64_MAX;
  int32_t page = c->row[page_idx];
  if (page < 0 || (uint32_t)page >= c->num_pages) return UINT64_MAX;
  return (uint64_t)page * c->page_size + (key_pos - page_idx * c->page_size);
}

/* With a sliding window (attention_head256_f16kv.wgsl:129-135 at abs_q =
 * kv_len - 1, kv_start = 0) only the last `sliding_window` keys are active;
 * with a softcap (…wgsl:197-199) each scaled score becomes
 * tanh(s / softcap) * softcap.                                              */
int doe_oracle_paged_decode_ex(uint32_t num_seqs, uint32_t num_heads,
                               uint32_t num_kv_heads, uint32_t head_dim,
                               uint32_t page_size, uint32_t num_pages,
                               uint32_t max_pages_per_seq, const uint16_t* q,
                               const void* k_pool, const void* v_pool,
                               const uint16_t* k_scale, const uint16_t* v_scale,
                               uint32_t kv_dtype, const int32_t* block_table,
                               const int32_t* kv_lens, float scale,
                               uint32_t sliding_window, float softcap, float* out,
                               int threads) {
  if (!q || !k_pool || !v_pool || !block_table || !kv_lens || !out) return DOE_ORACLE_EINVAL;
  if (num_kv_heads == 0 || num_heads % num_kv_heads || head_dim == 0 || page_size == 0)
    return DOE_ORACLE_EINVAL;
  if (kv_dtype > 1 || (kv_dtype == 1 && (!k_scale || !v_scale))) return DOE_ORACLE_EINVAL;
  const uint32_t H = num_heads, D = head_dim, group = num_heads / num_kv_heads;
  kv_rows ks = {kv_dtype, k_pool, k_scale, num_kv_heads, D, page_size};
  kv_rows vs = {kv_dtype, v_pool, v_scale, num_kv_heads, D, page_size};
  int rc = DOE_ORACLE_OK;
  set_threads(threads);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (uint32_t b = 0; b < num_seqs; ++b) {
    for (uint32_t h = 0; h < H; ++h) {
      float qrow[512];
      uint64_t off = ((uint64_t)b * H + h) * D;
      for (uint32_t d = 0; d < D && d < 512; ++d) qrow[d] = doe_oracle_h2f(q[off + d]);
      int32_t len = kv_lens[b];
      int r;
      if (len < 0 || D > 512) {
        r = DOE_ORACLE_EINVAL;
      } else {
        batched_ctx pctx = {block_table + (uint64_t)b * max_pages_per_seq,
                            max_pages_per_seq, page_size, num_pages};
        uint32_t min_key = 0;
        if (sliding_window > 0 && (uint32_t)len > sliding_window)
          min_key = (uint32_t)len - sliding_window;  /* abs_q - window + 1 */
        r = online_row(qrow, D, (uint32_t)len, min_key, (uint32_t)len, scale, softcap,
                       &ks, &vs, h / group, phys_batched, &pctx, out + off);
      }
      if (r != DOE_ORACLE_OK) {
#pragma omp atomic write
        rc = r;
      }
    }
  }
  return rc;
}

int doe_oracle_paged_decode(uint32_t num_seqs, uint32_t num_heads,
                            uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t page_size, uint32_t num_pages,
                            uint32_t max_pages_per_seq, const uint16_t* q,
                            const void* k_pool, const void* v_pool,
                            const uint16_t* k_scale, const uint16_t* v_scale,
                            uint32_t kv_dtype, const int32_t* block_table,
                            const int32_t* kv_lens, float scale, float* out,
                            int threads) {
  return doe_oracle_paged_decode_ex(num_seqs, num_heads, num_kv_heads, head_dim, page_size,
                                    num_pages, max_pages_per_seq, q, k_pool, v_pool, k_scale,
                                    v_scale, kv_dtype, block_table, kv_lens, scale, 0, 0.0f, out,
                                    threads);
}

/* ------------------------------------------------------------------------ */
/* kv_write / kv_read, dense single-head form
 * (runtime/zig/src/tsir/emit_kernel_body.zig:620-690 kv_write, 692-760 kv_read;
 *  CPU semantics bench/tools/run_csl_webgpu_emulator.mjs:615-644: position >=
 *  max_seq_len is an error; the copy is exact and touches no other row).  */
int doe_oracle_kv_write_dense(const float* k_proj, const float* v_proj,
                              float* k_cache, float* v_cache, uint32_t position,
                              uint32_t max_seq_len, uint32_t head_dim) {
  if (!k_proj || !v_proj || !k_cache || !v_cache) return DOE_ORACLE_EINVAL;
  if (position >= max_seq_len) return DOE_ORACLE_ERANGE;
  uint64_t base = (uint64_t)position * head_dim;
  memcpy(k_cache + base, k_proj, sizeof(float) * head_dim);
  memcpy(v_cache + base, v_proj, sizeof(float) * head_dim);
  return DOE_ORACLE_OK;
}

int doe_oracle_kv_read_dense(const float* k_cache, const float* v_cache,
                             float* k_out, float* v_out, uint32_t read_start,
                             uint32_t read_len, uint32_t max_seq_len,
                             uint32_t head_dim) {
  if (!k_cache || !v_cache || !k_out || !v_out) return DOE_ORACLE_EINVAL;
  if ((uint64_t)read_start + read_len > max_seq_len) return DOE_ORACLE_ERANGE;
  uint64_t base = (uint64_t)read_start * head_dim;
  memcpy(k_out, k_cache + base, sizeof(float) * head_dim * read_len);
  memcpy(v_out, v_cache + base, sizeof(float) * head_dim * read_len);
  return DOE_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* int8 symmetric per-row quantisation.  The reference has no int8 KV; this
 * follows the stated definition: scale = f16(absmax / 127),
 * q = clamp(rint(x / float(scale)), -127, 127), absmax == 0 -> scale 0, q 0.
 * A scale that rounds to zero in f16 also stores q = 0.                    */
void doe_oracle_quantize_rows_int8(const uint16_t* x, uint64_t rows,
                                   uint32_t head_dim, int8_t* q,
                                   uint16_t* scale) {
  for (uint64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * head_dim;
    float amax = 0.0f;
    for (uint32_t d = 0; d < head_dim; ++d) {
      float a = fabsf(doe_oracle_h2f(xr[d]));
      if (a > amax) amax = a;
    }
    uint16_t sh = doe_oracle_f2h(amax / 127.0f);
    float sf = doe_oracle_h2f(sh);
    scale[r] = sh;
    for (uint32_t d = 0; d < head_dim; ++d) {
      if (sf == 0.0f) {
        q[r * head_dim + d] = 0;
        continue;
      }
      float t = rintf(doe_oracle_h2f(xr[d]) / sf);
      if (t > 127.0f) t = 127.0f;
      if (t < -127.0f) t = -127.0f;
      q[r * head_dim + d] = (int8_t)t;
    }
  }
}

/* Paged append: the kv_write copy generalised to a [token, Hkv, D] pool
 * addressed through a per-sequence block table row (head256 get_kv_pos,
 * kv_layout 2: phys = table[p / page] * page + p % page).  A position whose
 * page is unmapped or outside the pool is rejected before anything is
 * written for that sequence.                                              */
int doe_oracle_paged_append(uint32_t num_seqs, uint32_t n_tokens,
                            uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t page_size, uint32_t num_pages,
                            uint32_t max_pages_per_seq,
                            const uint16_t* new_k, const uint16_t* new_v,
                            void* k_pool, void* v_pool, uint16_t* k_scale,
                            uint16_t* v_scale, uint32_t kv_dtype,
                            const int32_t* block_table,
                            const int32_t* positions, int threads) {
  if (!new_k || !new_v || !k_pool || !v_pool || !block_table || !positions)
    return DOE_ORACLE_EINVAL;
  if (page_size == 0 || head_dim == 0 || num_kv_heads == 0 || kv_dtype > 1)
    return DOE_ORACLE_EINVAL;
  if (kv_dtype == 1 && (!k_scale || !v_scale)) return DOE_ORACLE_EINVAL;
  const uint64_t row = (uint64_t)num_kv_heads * head_dim;
  int rc = DOE_ORACLE_OK;
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (uint32_t b = 0; b < num_seqs; ++b) {
    const int32_t* trow = block_table + (uint64_t)b * max_pages_per_seq;
    int ok = positions[b] >= 0;
    for (uint32_t t = 0; ok && t < n_tokens; ++t) {
      uint64_t p = (uint64_t)positions[b] + t;
      uint64_t pi = p / page_size;
      if (pi >= max_pages_per_seq || trow[pi] < 0 || (uint32_t)trow[pi] >= num_pages) ok = 0;
    }
    if (!ok) {
#pragma omp atomic write
      rc = DOE_ORACLE_ERANGE;
      continue;
    }
    for (uint32_t t = 0; t < n_tokens; ++t) {
      uint64_t p = (uint64_t)positions[b] + t;
      uint64_t phys = (uint64_t)trow[p / page_size] * page_size + p % page_size;
      const uint16_t* sk = new_k + ((uint64_t)b * n_tokens + t) * row;
      const uint16_t* sv = new_v + ((uint64_t)b * n_tokens + t) * row;
      if (kv_dtype == 0) {
        memcpy((uint16_t*)k_pool + phys * row, sk, row * 2);
        memcpy((uint16_t*)v_pool + phys * row, sv, row * 2);
      } else {
        for (uint32_t h = 0; h < num_kv_heads; ++h) {
          uint64_t si = scale_index(phys, h, num_kv_heads, page_size);
          doe_oracle_quantize_rows_int8(sk + (uint64_t)h * head_dim, 1, head_dim,
                                        (int8_t*)k_pool + phys * row + (uint64_t)h * head_dim,
                                        k_scale + si);
          doe_oracle_quantize_rows_int8(sv + (uint64_t)h * head_dim, 1, head_dim,
                                        (int8_t*)v_pool + phys * row + (uint64_t)h * head_dim,
                                        v_scale + si);
        }
      }
    }
  }
  return rc;
}

int doe_oracle_paged_gather(uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t page_size, uint32_t num_pages,
                            const int32_t* block_row, uint32_t max_pages,
                            uint32_t len, uint32_t elem_bytes,
                            const void* pool, void* out) {
  if (!block_row || !pool || !out || page_size == 0) return DOE_ORACLE_EINVAL;
  const uint64_t rowb = (uint64_t)num_kv_heads * head_dim * elem_bytes;
  for (uint32_t p = 0; p < len; ++p) {
    uint32_t pi = p / page_size;
    if (pi >= max_pages || block_row[pi] < 0 || (uint32_t)block_row[pi] >= num_pages)
      return DOE_ORACLE_ERANGE;
    uint64_t phys = (uint64_t)block_row[pi] * page_size + p % page_size;
    memcpy((char*)out + (uint64_t)p * rowb, (const char*)pool + phys * rowb, rowb);
  }
  return DOE_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* rope.wgsl (bench/inference-pipeline/kernels/rope.wgsl:12-35): pairs
 * (i, i + D/2) rotate by freq_cis[(pos * D/2 + i) * 2 + {0: cos, 1: sin}],
 * pos = seq_idx + position_offset, layout [S, H, D], in place.            */
int doe_oracle_rope_f32(float* qk, const float* freq_cis, uint32_t seq_len,
                        uint32_t num_heads, uint32_t head_dim,
                        uint32_t position_offset) {
  if (!qk || !freq_cis || head_dim < 2) return DOE_ORACLE_EINVAL;
  uint32_t half = head_dim / 2;
  for (uint32_t s = 0; s < seq_len; ++s) {
    uint64_t pos = (uint64_t)s + position_offset;
    for (uint32_t h = 0; h < num_heads; ++h) {
      float* base = qk + ((uint64_t)s * num_heads + h) * head_dim;
      for (uint32_t i = 0; i < half; ++i) {
        float x0 = base[i], x1 = base[i + half];
        uint64_t f = pos * half + i;
        float c = freq_cis[f * 2], sn = freq_cis[f * 2 + 1];
        base[i] = x0 * c - x1 * sn;
        base[i + half] = x0 * sn + x1 * c;
      }
    }
  }
  return DOE_ORACLE_OK;
}
