/* cpu_baseline.c -- the timed CPU baseline of the batched paged GQA decode.
 *
 * TEST / BENCHMARK INFRASTRUCTURE ONLY: bench.py times this as the CPU leg
 * (cpu_baseline and --impl reference).  It computes exactly what the parity
 * oracle's doe_oracle_paged_decode_ex (doe_oracle.c) computes -- the head256
 * online softmax of attention_head256_f16kv.wgsl:72-269 with query_len 1 over
 * a per-sequence block table: 32-key blocks, vec4 partial dot products,
 * block max, correction expf(m_i - m_new), p = expf(s - m_new),
 * acc = acc * corr then acc + p * v in key order, out = acc / l -- in the
 * same float32 operation order (built with -ffp-contract=off and without
 * fast-math, so every product and sum is rounded where the oracle rounds it),
 * and tests/test_cpu_baseline.py holds it to the oracle bit for bit.
 *
 * It is organised for a CPU instead of for readability: one task per
 * (sequence, kv head) unit handles all the query heads of that kv head, so
 * each K and V row is read and converted once per unit (f16 via F16C, int8
 * times its scale) instead of once per query head; the score dot products
 * run with the heads in SIMD lanes (each lane keeps the oracle's scalar
 * order); pages are looked up once per 32-key block; nothing is allocated
 * per row.  OpenMP spreads the units over the host's cores.
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

#include "doe_oracle.h"

#define BLOCK 32
#define MAX_GROUP 16
#define MAX_D 256

static inline void load_f16_row(const uint16_t* src, uint32_t D, float* dst) {
  uint32_t d = 0;
  for (; d + 8 <= D; d += 8)
    _mm256_storeu_ps(dst + d, _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(src + d))));
  for (; d < D; ++d) dst[d] = _cvtsh_ss(src[d]);
}

static inline float h2f_scalar(uint16_t h) { return _cvtsh_ss(h); }

static int unit(uint32_t b, uint32_t g, uint32_t G, uint32_t H, uint32_t Hkv, uint32_t D, uint32_t page_size,
                uint32_t num_pages, uint32_t max_pages, const uint16_t* q, const void* k_pool,
                const void* v_pool, const uint16_t* k_scale, const uint16_t* v_scale, uint32_t int8,
                const int32_t* row, int32_t len, float scale, uint32_t window, float softcap, float* out) {
  float qT[MAX_D * MAX_GROUP];         /* [d][head]: the heads of one d side by side */
  float acc[MAX_GROUP][MAX_D];
  float m_i[MAX_GROUP], l_i[MAX_GROUP];
  float krow[MAX_D], vrow[MAX_D];
  float scores[BLOCK][MAX_GROUP], probs[BLOCK][MAX_GROUP];
  uint64_t phys[BLOCK];
  int active[BLOCK];
  for (uint32_t gi = 0; gi < G; ++gi) {
    const uint16_t* qh = q + ((uint64_t)b * H + (uint64_t)g * G + gi) * D;
    for (uint32_t d = 0; d < D; ++d) qT[d * G + gi] = h2f_scalar(qh[d]);
    for (uint32_t d = 0; d < D; ++d) acc[gi][d] = 0.0f;
    m_i[gi] = -3.402823e+38f;
    l_i[gi] = 0.0f;
  }
  const uint32_t seq_len = (uint32_t)len;
  const uint32_t min_key = (window > 0 && seq_len > window) ? seq_len - window : 0;
  const uint32_t vec_dim = D & ~3u;
  const uint32_t nblocks = (seq_len + BLOCK - 1) / BLOCK;
  for (uint32_t blk = 0; blk < nblocks; ++blk) {
    const uint32_t start = blk * BLOCK;
    float block_max[MAX_GROUP];
    for (uint32_t gi = 0; gi < G; ++gi) block_max[gi] = -3.402823e+38f;
    for (uint32_t j = 0; j < BLOCK; ++j) {
      const uint32_t kp = start + j;
      for (uint32_t gi = 0; gi < G; ++gi) scores[j][gi] = probs[j][gi] = 0.0f;
      active[j] = kp < seq_len && kp >= min_key;
      if (!active[j]) continue;
      const uint32_t pidx = kp / page_size;
      if (pidx >= max_pages || row[pidx] < 0 || (uint32_t)row[pidx] >= num_pages) return DOE_ORACLE_ERANGE;
      phys[j] = (uint64_t)row[pidx] * page_size + (kp - pidx * page_size);
      const uint64_t off = (phys[j] * Hkv + g) * D;
      if (!int8) {
        load_f16_row((const uint16_t*)k_pool + off, D, krow);
      } else {
        const int8_t* src = (const int8_t*)k_pool + off;
        const uint64_t si = ((phys[j] / page_size) * Hkv + g) * page_size + phys[j] % page_size;
        const float sc = h2f_scalar(k_scale[si]);
        for (uint32_t d = 0; d < D; ++d) krow[d] = (float)src[d] * sc;
      }
      float dot[MAX_GROUP];
      for (uint32_t gi = 0; gi < G; ++gi) dot[gi] = 0.0f;
      for (uint32_t d = 0; d < vec_dim; d += 4) {
        const float* q0 = qT + d * G;
        for (uint32_t gi = 0; gi < G; ++gi) {  /* heads in SIMD lanes, oracle order per lane */
          float dp = q0[gi] * krow[d];
          dp = dp + q0[G + gi] * krow[d + 1];
          dp = dp + q0[2 * G + gi] * krow[d + 2];
          dp = dp + q0[3 * G + gi] * krow[d + 3];
          dot[gi] = dot[gi] + dp;
        }
      }
      for (uint32_t d = vec_dim; d < D; ++d)
        for (uint32_t gi = 0; gi < G; ++gi) dot[gi] = dot[gi] + qT[d * G + gi] * krow[d];
      for (uint32_t gi = 0; gi < G; ++gi) {
        float s = dot[gi] * scale;
        if (softcap > 0.0f) s = tanhf(s / softcap) * softcap;
        scores[j][gi] = s;
        block_max[gi] = fmaxf(block_max[gi], s);
      }
    }
    for (uint32_t gi = 0; gi < G; ++gi) {
      const float m_new = fmaxf(m_i[gi], block_max[gi]);
      const float corr = expf(m_i[gi] - m_new);
      l_i[gi] = l_i[gi] * corr;
      for (uint32_t d = 0; d < D; ++d) acc[gi][d] = acc[gi][d] * corr;
      for (uint32_t j = 0; j < BLOCK; ++j) {
        if (!active[j]) continue;
        const float p = expf(scores[j][gi] - m_new);
        probs[j][gi] = p;
        l_i[gi] = l_i[gi] + p;
      }
      m_i[gi] = m_new;
    }
    for (uint32_t j = 0; j < BLOCK; ++j) {
      if (!active[j]) continue;
      int any = 0;
      for (uint32_t gi = 0; gi < G; ++gi) any |= probs[j][gi] != 0.0f;
      if (!any) continue;
      const uint64_t off = (phys[j] * Hkv + g) * D;
      if (!int8) {
        load_f16_row((const uint16_t*)v_pool + off, D, vrow);
      } else {
        const int8_t* src = (const int8_t*)v_pool + off;
        const uint64_t si = ((phys[j] / page_size) * Hkv + g) * page_size + phys[j] % page_size;
        const float sc = h2f_scalar(v_scale[si]);
        for (uint32_t d = 0; d < D; ++d) vrow[d] = (float)src[d] * sc;
      }
      for (uint32_t gi = 0; gi < G; ++gi) {
        const float p = probs[j][gi];
        if (p == 0.0f) continue;
        float* a = acc[gi];
        for (uint32_t d = 0; d < D; ++d) a[d] = a[d] + p * vrow[d];
      }
    }
  }
  for (uint32_t gi = 0; gi < G; ++gi) {
    const float inv = l_i[gi] > 0.0f ? 1.0f / l_i[gi] : 0.0f;
    float* o = out + ((uint64_t)b * H + (uint64_t)g * G + gi) * D;
    for (uint32_t d = 0; d < D; ++d) o[d] = acc[gi][d] * inv;
  }
  return DOE_ORACLE_OK;
}

int doe_cpu_paged_decode(uint32_t num_seqs, uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim,
                         uint32_t page_size, uint32_t num_pages, uint32_t max_pages_per_seq,
                         const uint16_t* q, const void* k_pool, const void* v_pool, const uint16_t* k_scale,
                         const uint16_t* v_scale, uint32_t kv_dtype, const int32_t* block_table,
                         const int32_t* kv_lens, float scale, uint32_t sliding_window, float softcap,
                         float* out, int threads) {
  if (!q || !k_pool || !v_pool || !block_table || !kv_lens || !out) return DOE_ORACLE_EINVAL;
  if (num_kv_heads == 0 || num_heads % num_kv_heads || head_dim == 0 || head_dim > MAX_D || page_size == 0)
    return DOE_ORACLE_EINVAL;
  const uint32_t G = num_heads / num_kv_heads;
  if (G > MAX_GROUP || kv_dtype > 1 || (kv_dtype == 1 && (!k_scale || !v_scale))) return DOE_ORACLE_EINVAL;
  int rc = DOE_ORACLE_OK;
  if (threads > 0) omp_set_num_threads(threads);
  const int64_t units = (int64_t)num_seqs * num_kv_heads;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t u = 0; u < units; ++u) {
    const uint32_t b = (uint32_t)(u / num_kv_heads), g = (uint32_t)(u % num_kv_heads);
    int r = kv_lens[b] < 0 ? DOE_ORACLE_EINVAL
                           : unit(b, g, G, num_heads, num_kv_heads, head_dim, page_size, num_pages,
                                  max_pages_per_seq, q, k_pool, v_pool, k_scale, v_scale, kv_dtype,
                                  block_table + (uint64_t)b * max_pages_per_seq, kv_lens[b], scale,
                                  sliding_window, softcap, out);
    if (r != DOE_ORACLE_OK) {
#pragma omp atomic write
      rc = r;
    }
  }
  return rc;
}
