// tma.cuh -- TMA tile loads and mbarrier helpers shared by the sm_100a kernels,
// and the host-side encoding of the row-major tensor maps they use.
//
// Every pool and activation on the attention path is a row-major array of
// (row, head, element) with one head's row contiguous; a tensor map over it is
// 3-D {elements, heads, rows} and a box is {inner elements, 1 head, rows}.
// With SWIZZLE_128B a box row is 128 bytes and, when the box starts on a
// 1024-byte boundary, 16-byte chunk x of row R lands at chunk x ^ (R & 7).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace doe {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
// try_wait with a suspend-time hint: a thread whose phase is incomplete sleeps
// in hardware until it completes (or the hint passes) instead of re-polling.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.b32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// Bounded wait (~2 s of SM clocks); false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > 4000000000LL) return false;
  return true;
}

// Box {x.., y, z..} of a 3-D map into shared memory, completing on `bar`.
// x (the innermost coordinate) times the element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
// Contiguous bytes (16-byte aligned, a multiple of 16) into shared memory.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Host: a 3-D map {inner, heads, rows} over a row-major (rows, heads, inner)
// array of `elem_bytes`-byte elements, boxes of {box_inner, 1, box_rows}
// with the 128-byte swizzle.  Returns a doe_status; sets the op error.
int encode_rows_map(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                    uint64_t inner, uint64_t heads, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
                    const char* who);

}  // namespace doe
