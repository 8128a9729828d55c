// kv_pool.cpp -- host-side page allocator for the paged KV cache.
//
// The reference binds one page_table per dispatch
// (runtime/zig/tests/tsir/real/attention_head256_f16kv/attention_head256_f16kv.wgsl:38,
// consumed by get_kv_pos, :51-63) and leaves its contents to the caller.  This
// pool is that caller for the batched kernels: it owns the free list of
// physical pages and the per-sequence rows of the block table
// ([max_seqs, max_pages_per_seq] int32, -1 = unmapped).  Pure host code.
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/doe_cuda.h"

struct doe_kv_pool {
  uint32_t num_pages = 0;
  uint32_t page_size = 0;
  uint32_t max_seqs = 0;
  uint32_t max_pages = 0;
  std::vector<int32_t> free_list;           // LIFO stack of free pages
  std::vector<std::vector<int32_t>> pages;  // per sequence, logical order
  std::mutex mu;
};

extern "C" {

int doe_kv_pool_create(uint32_t num_pages, uint32_t page_size, uint32_t max_seqs,
                       uint32_t max_pages_per_seq, doe_kv_pool** out) {
  if (!out) return DOE_INVALID_ARGUMENT;
  *out = nullptr;
  if (num_pages == 0 || page_size == 0 || max_seqs == 0 || max_pages_per_seq == 0)
    return DOE_INVALID_ARGUMENT;
  if (num_pages > 0x7fffffffu) return DOE_INVALID_ARGUMENT;
  doe_kv_pool* p = new doe_kv_pool();
  p->num_pages = num_pages;
  p->page_size = page_size;
  p->max_seqs = max_seqs;
  p->max_pages = max_pages_per_seq;
  p->free_list.reserve(num_pages);
  for (uint32_t i = num_pages; i > 0; --i) p->free_list.push_back((int32_t)(i - 1));
  p->pages.resize(max_seqs);
  *out = p;
  return DOE_OK;
}

int doe_kv_pool_destroy(doe_kv_pool* pool) {
  if (!pool) return DOE_INVALID_ARGUMENT;
  delete pool;
  return DOE_OK;
}

int doe_kv_pool_reserve(doe_kv_pool* pool, uint32_t seq, uint32_t tokens) {
  if (!pool) return DOE_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(pool->mu);
  if (seq >= pool->max_seqs) return DOE_OUT_OF_RANGE;
  const uint64_t need = ((uint64_t)tokens + pool->page_size - 1) / pool->page_size;
  if (need > pool->max_pages) return DOE_OUT_OF_RANGE;
  std::vector<int32_t>& row = pool->pages[seq];
  if (need <= row.size()) return DOE_OK;
  const uint64_t extra = need - row.size();
  if (extra > pool->free_list.size()) return DOE_OUT_OF_RANGE;  // pool exhausted
  for (uint64_t i = 0; i < extra; ++i) {
    row.push_back(pool->free_list.back());
    pool->free_list.pop_back();
  }
  return DOE_OK;
}

int doe_kv_pool_release(doe_kv_pool* pool, uint32_t seq) {
  if (!pool) return DOE_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(pool->mu);
  if (seq >= pool->max_seqs) return DOE_OUT_OF_RANGE;
  std::vector<int32_t>& row = pool->pages[seq];
  for (auto it = row.rbegin(); it != row.rend(); ++it) pool->free_list.push_back(*it);
  row.clear();
  return DOE_OK;
}

int doe_kv_pool_free_pages(const doe_kv_pool* pool, uint32_t* out) {
  if (!pool || !out) return DOE_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(const_cast<doe_kv_pool*>(pool)->mu);
  *out = (uint32_t)pool->free_list.size();
  return DOE_OK;
}

int doe_kv_pool_seq_pages(const doe_kv_pool* pool, uint32_t seq, uint32_t* out) {
  if (!pool || !out) return DOE_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(const_cast<doe_kv_pool*>(pool)->mu);
  if (seq >= pool->max_seqs) return DOE_OUT_OF_RANGE;
  *out = (uint32_t)pool->pages[seq].size();
  return DOE_OK;
}

int doe_kv_pool_block_table(const doe_kv_pool* pool, int32_t* out, uint64_t out_entries) {
  if (!pool || !out) return DOE_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(const_cast<doe_kv_pool*>(pool)->mu);
  const uint64_t total = (uint64_t)pool->max_seqs * pool->max_pages;
  if (out_entries < total) return DOE_INVALID_ARGUMENT;
  for (uint32_t s = 0; s < pool->max_seqs; ++s) {
    int32_t* row = out + (uint64_t)s * pool->max_pages;
    const std::vector<int32_t>& pg = pool->pages[s];
    for (uint32_t i = 0; i < pool->max_pages; ++i) row[i] = i < pg.size() ? pg[i] : -1;
  }
  return DOE_OK;
}

}  // extern "C"
