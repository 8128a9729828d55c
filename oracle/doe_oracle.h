/*
 * doe_oracle.h -- CPU restatement of Doe's attention / KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels in doe_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg (and its `--impl reference` arm) may load
 * it.  The product path (libdoe_cuda.so) never links or calls it.
 *
 * Every function names the reference file:line whose arithmetic it follows
 * (paths are relative to the doerun/doe source tree).
 *
 * Conventions
 *   - f16 values travel as raw uint16_t bit patterns (IEEE binary16).
 *   - Functions return 0 on success and a negative DOE_ORACLE_E* code on a
 *     rejected input, mirroring the reference's explicit error results.
 *   - `threads` <= 0 means "all OpenMP threads"; 1 means scalar.
 */
#ifndef DOE_ORACLE_H
#define DOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DOE_ORACLE_OK 0
#define DOE_ORACLE_EINVAL (-1)
#define DOE_ORACLE_ERANGE (-2)  /* position / page outside the cache      */
#define DOE_ORACLE_EZERO (-3)   /* softmax denominator is zero (two-pass)  */

/* ---- binary16 helpers (round-to-nearest-even) ------------------------- */
float doe_oracle_h2f(uint16_t h);
uint16_t doe_oracle_f2h(float f);
void doe_oracle_h2f_array(const uint16_t* src, float* dst, uint64_t n);
void doe_oracle_f2h_array(const float* src, uint16_t* dst, uint64_t n);

/* ---- attention-decode.wgsl (bench/inference-pipeline/kernels/) -------- */
/* q [H,D], k/v [H,L,D], out [H,D]; f32 (and an f64 twin for exact KATs). */
int doe_oracle_attention_decode_wgsl_f32(const float* q, const float* k,
                                         const float* v, float* out,
                                         uint32_t num_heads, uint32_t head_dim,
                                         uint32_t kv_len, float scale);
int doe_oracle_attention_decode_wgsl_f64(const double* q, const double* k,
                                         const double* v, double* out,
                                         uint32_t num_heads, uint32_t head_dim,
                                         uint32_t kv_len, double scale);

/* ---- attention-prefill.wgsl: causal, [H,S,D] f32 ----------------------- */
int doe_oracle_attention_prefill_wgsl_f32(const float* q, const float* k,
                                          const float* v, float* out,
                                          uint32_t seq_len, uint32_t head_dim,
                                          uint32_t num_heads, float scale);

/* ---- reference_interpreter.zig tryAttentionScores (two-pass, single Q) - */
/* causal_mode: 0 none, 1 causal, 2 sliding window (window > 0).          */
int doe_oracle_attention_two_pass_f32(const float* q, const float* k,
                                      const float* v, float* out,
                                      uint32_t head_dim, uint32_t kv_len,
                                      float scale, uint32_t causal_mode,
                                      uint32_t window);

/* ---- kv-axis-sharded partials + LSE stitch ----------------------------- */
/* partials row layout: [O_unnormalised[D], local_max, local_sum_exp].      */
int doe_oracle_emit_local_partials_f32(const float* q, const float* k_local,
                                       const float* v_local, float* out_row,
                                       uint32_t head_dim, uint32_t slots,
                                       uint32_t slot_base, uint32_t kv_len,
                                       float scale);
int doe_oracle_stitch_partials_f32(const float* partials, uint32_t num_shards,
                                   uint32_t head_dim, float* out);

/* ---- attention_head256_f16kv.wgsl generalised (online softmax) -------- */
/* The 15-word uniform block of the reference kernel (minus _pad).          */
typedef struct doe_oracle_attn_uniforms {
  uint32_t num_heads;
  uint32_t num_kv_heads;
  uint32_t head_dim;
  uint32_t seq_len;
  uint32_t query_len;
  float scale;
  uint32_t is_causal;
  uint32_t start_pos;
  float attn_softcap;
  uint32_t sliding_window;
  uint32_t kv_len_source;
  uint32_t kv_start;
  uint32_t page_size;
  uint32_t kv_layout; /* 0 dense, 1 sliding ring, 2 paged */
} doe_oracle_attn_uniforms;

/* Q/out [query_len, H, D] f32; K/V [pos, Hkv, D] f16.                      */
int doe_oracle_attention_online_f16kv(const doe_oracle_attn_uniforms* u,
                                      const float* q, const uint16_t* k,
                                      const uint16_t* v, float* out,
                                      const uint32_t* kv_len_buffer,
                                      const uint32_t* page_table, int threads);

/* ---- batched paged decode (per-sequence block tables) ------------------ */
/* Q [B,H,D] f16; pools [num_pages*page_size, Hkv, D]; block_table [B,max_pages]
 * int32; kv_lens [B] = tokens to attend; out [B,H,D] f32.  kv_dtype 0 = f16
 * pools (scales ignored), 1 = int8 pools with f16 scales laid out
 * [num_pages, Hkv, page_size] (page-blocked per token and kv head).          */
int doe_oracle_paged_decode(uint32_t num_seqs, uint32_t num_heads,
                            uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t page_size, uint32_t num_pages,
                            uint32_t max_pages_per_seq, const uint16_t* q,
                            const void* k_pool, const void* v_pool,
                            const uint16_t* k_scale, const uint16_t* v_scale,
                            uint32_t kv_dtype, const int32_t* block_table,
                            const int32_t* kv_lens, float scale, float* out,
                            int threads);
/* The same with a sliding window (last `sliding_window` keys; 0 = all) and a
 * score softcap (s = tanh(s / softcap) * softcap; 0 = off).               */
int doe_oracle_paged_decode_ex(uint32_t num_seqs, uint32_t num_heads,
                               uint32_t num_kv_heads, uint32_t head_dim,
                               uint32_t page_size, uint32_t num_pages,
                               uint32_t max_pages_per_seq, const uint16_t* q,
                               const void* k_pool, const void* v_pool,
                               const uint16_t* k_scale, const uint16_t* v_scale,
                               uint32_t kv_dtype, const int32_t* block_table,
                               const int32_t* kv_lens, float scale,
                               uint32_t sliding_window, float softcap, float* out,
                               int threads);

/* ---- KV append / read (kv_write, kv_read) ------------------------------ */
/* Dense single-head form of emit_kernel_body.zig kv_write: cache[pos*D+d]. */
int doe_oracle_kv_write_dense(const float* k_proj, const float* v_proj,
                              float* k_cache, float* v_cache, uint32_t position,
                              uint32_t max_seq_len, uint32_t head_dim);
int doe_oracle_kv_read_dense(const float* k_cache, const float* v_cache,
                             float* k_out, float* v_out, uint32_t read_start,
                             uint32_t read_len, uint32_t max_seq_len,
                             uint32_t head_dim);

/* Paged append of n_tokens per sequence starting at positions[b].
 * new_k/new_v [B, n_tokens, Hkv, D] f16.  kv_dtype 0 copies f16 bits;
 * kv_dtype 1 quantises to int8 + f16 scale per (token, kv head).          */
int doe_oracle_paged_append(uint32_t num_seqs, uint32_t n_tokens,
                            uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t page_size, uint32_t num_pages,
                            uint32_t max_pages_per_seq,
                            const uint16_t* new_k, const uint16_t* new_v,
                            void* k_pool, void* v_pool, uint16_t* k_scale,
                            uint16_t* v_scale, uint32_t kv_dtype,
                            const int32_t* block_table,
                            const int32_t* positions, int threads);

/* Paged gather of one sequence's first `len` tokens into [len, Hkv, D].   */
int doe_oracle_paged_gather(uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t page_size, uint32_t num_pages,
                            const int32_t* block_row, uint32_t max_pages,
                            uint32_t len, uint32_t elem_bytes,
                            const void* pool, void* out);

/* int8 symmetric quantisation of rows of D f16 values (per token per head). */
void doe_oracle_quantize_rows_int8(const uint16_t* x, uint64_t rows,
                                   uint32_t head_dim, int8_t* q,
                                   uint16_t* scale);

/* ---- rope.wgsl: rotate-half with a [pos][pair]{cos,sin} table ---------- */
int doe_oracle_rope_f32(float* qk, const float* freq_cis, uint32_t seq_len,
                        uint32_t num_heads, uint32_t head_dim,
                        uint32_t position_offset);

#ifdef __cplusplus
}
#endif

#endif /* DOE_ORACLE_H */
