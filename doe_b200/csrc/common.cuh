// common.cuh -- shared device helpers for the sm_100a attention / KV kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/doe_cuda.h"
#include "kernels.h"

namespace doe {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void report(int32_t* status, int32_t bits) {
  if (status) atomicOr(status, bits);
}

// Programmatic dependent launch.  pdl_trigger lets the next kernel on the
// stream (launched with launch_pdl) start its prologue while this one runs;
// pdl_wait blocks until the previous kernel on the stream has completed and
// its writes are visible.  A kernel launched with launch_pdl must call
// pdl_wait before it touches memory the previous kernel writes or reads.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// ---- warp mma: D = A(16x16 f16, row) * B(16x8 f16, col) + C (f32) -------
// Fragment layout (PTX ISA, mma.m16n8k16 .f16): lane = 4*g + t.
//   A regs: {(g, 2t..2t+1), (g+8, 2t..), (g, 2t+8..), (g+8, 2t+8..)}
//   B regs: {(k=2t..2t+1, n=g), (k=2t+8.., n=g)}
//   C: c0,c1 = (g, 2t..2t+1), c2,c3 = (g+8, 2t..2t+1)
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                          uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two signed bytes -> f16x2, exactly.  `t` holds byte b_lo in bits 0-7 and
// b_hi in bits 16-23 (other bits ignored).  Each byte, offset by 128 (sign
// bit flipped), is placed in the mantissa of 1024.0h (0x6400): the f16 value
// 1024 + (b + 128) is exact because f16 spacing in [1024, 2048) is 1, and
// subtracting 1152 returns b.
__device__ __forceinline__ uint32_t s8x2_to_f16x2(uint32_t t) {
  uint32_t biased = (t & 0x00ff00ffu) ^ 0x64806480u;
  __half2 h = *reinterpret_cast<__half2*>(&biased);
  const uint32_t k1152 = 0x64806480u;
  h = __hsub2(h, *reinterpret_cast<const __half2*>(&k1152));
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t prmt(uint32_t x, uint32_t y, uint32_t sel) {
  return __byte_perm(x, y, sel);
}

// Two f32 lanes per instruction (sm_100 packed FP32): a * b + c, a + b and
// a * b, each lane rounded as the scalar instruction would round it.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rc, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "mul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// int8 KV quantisation of one element: clamp(rint(x / s), -127, 127) for an
// f16 value x and the row's f16 scale s = f16(absmax / 127) > 0, equal to the
// CPU definition's rint of the f32 IEEE quotient.  The quotient is formed from
// the correctly rounded reciprocal rs and one residual correction (Markstein's
// method): y0 = x rs, y = y0 + (x - y0 s) rs, the residual exact in an FMA.
// For f16 operands x / s is either exactly k + 1/2 or at least 2^-14 from
// every half-integer (2x - (2k+1)s is a multiple of the finer of the two
// operands' ulps), far beyond y's error; y lands on the same side of every
// rounding boundary and is exactly k + 1/2 in the tie case, where rint takes
// the even neighbour as the CPU does.
// The result is a word whose low byte is q (two's complement): y is clamped
// to [-127, 127] in f32 (the same as clamping rint(y)), and adding 1.5 * 2^23
// rounds it to an integer, ties to even, in the low mantissa bits, so the
// sum's bit pattern is 0x4B400000 + q.  Everything stays on the FP32 pipe.
__device__ __forceinline__ int quantize_s8(float x, float s, float rs) {
  const float y0 = x * rs;
  const float y = fmaf(fmaf(-y0, s, x), rs, y0);
  const float c = fminf(fmaxf(y, -127.0f), 127.0f);
  return (int)__float_as_uint(__fadd_rn(c, 12582912.0f));
}
// The row scale's f32 quotient amax / 127 without an IEEE division:
// q0 = amax * RN(1/127), then one residual correction (Markstein's method),
// the residual exact in an FMA.  For every finite f16 amax >= 0 this is the
// correctly rounded quotient (checked exhaustively against exact rational
// arithmetic), so f16(result) equals f16(amax / 127) of the CPU definition.
__device__ __forceinline__ float div127(float amax) {
  constexpr float kInv127 = 0x1.020408p-7f;  // RN_f32(1 / 127)
  const float q0 = amax * kInv127;
  return fmaf(fmaf(-q0, 127.0f, amax), kInv127, q0);
}

// quantize_s8 on two elements with a normal f16 scale (2^-14 <= s <= 65504),
// in sm_100 packed FP32.  With s = f16(amax / 127) normal, |x / s| <=
// 127 / (1 - 2^-11) < 127.07 for |x| <= amax, so rint never leaves
// [-127, 127] and the clamp of quantize_s8 cannot change the result; the
// rest is the same arithmetic (y0 * (-s) is -y0 * s exactly).
__device__ __forceinline__ void quantize_s8x2_normal(float2 x, float s, float rs, int& q0, int& q1) {
  const float2 rs2 = make_float2(rs, rs);
  const float2 y0 = fmul2(x, rs2);
  const float2 y = ffma2(ffma2(y0, make_float2(-s, -s), x), rs2, y0);
  const float2 c = fadd2(y, make_float2(12582912.0f, 12582912.0f));
  q0 = (int)__float_as_uint(c.x);
  q1 = (int)__float_as_uint(c.y);
}

// Low bytes of four words (two's complement int8 values) packed into a word.
__device__ __forceinline__ uint32_t pack_s8x4(int q0, int q1, int q2, int q3) {
  return __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
}

// RoPE on 2W f16 elements of a row (rope.wgsl:12-35): each pair (d, d + D/2)
// becomes x0' = x0 cos - x1 sin, x1' = x0 sin + x1 cos in f32, every product
// and sum rounded separately, and the results are rounded back to f16.
// `mine` holds 2W consecutive dims, `partner` the dims D/2 away; `first` is
// true when mine holds the first halves (x0).  c/sn: the pairs' table entries.
template <int W>
__device__ __forceinline__ void rope_rotate(const uint32_t* mine, const uint32_t* partner, bool first,
                                            const float (&c)[2 * W], const float (&sn)[2 * W],
                                            uint32_t* out) {
#pragma unroll
  for (int e = 0; e < W; ++e) {
    const __half2 m2 = *reinterpret_cast<const __half2*>(&mine[e]);
    const __half2 p2 = *reinterpret_cast<const __half2*>(&partner[e]);
    float r[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float xm = k ? __high2float(m2) : __low2float(m2);
      const float xp = k ? __high2float(p2) : __low2float(p2);
      const float x0 = first ? xm : xp, x1 = first ? xp : xm;
      const int j = 2 * e + k;
      r[k] = first ? __fsub_rn(__fmul_rn(x0, c[j]), __fmul_rn(x1, sn[j]))
                   : __fadd_rn(__fmul_rn(x0, sn[j]), __fmul_rn(x1, c[j]));
    }
    out[e] = pack_half2(r[0], r[1]);
  }
}
// Loads the RoPE table entries of 2W consecutive pairs starting at `pair` for
// position `pos` (freq_cis [positions, half, {cos, sin}]); positions beyond
// the table get the identity and report DOE_DEVICE_ERR_POSITION.
template <int W>
__device__ __forceinline__ void rope_table(const float* freq_cis, int positions, int half, long long pos,
                                           int pair, int32_t* status, bool reporter, float (&c)[2 * W],
                                           float (&sn)[2 * W]) {
  const bool in_table = pos >= 0 && pos < positions;
  if (!in_table && reporter) report(status, DOE_DEVICE_ERR_POSITION);
  const float4* tab = reinterpret_cast<const float4*>(freq_cis + ((size_t)(in_table ? pos : 0) * half + pair) * 2);
#pragma unroll
  for (int q = 0; q < W; ++q) {
    const float4 t4 = in_table ? tab[q] : make_float4(1.0f, 0.0f, 1.0f, 0.0f);
    c[2 * q] = t4.x; sn[2 * q] = t4.y;
    c[2 * q + 1] = t4.z; sn[2 * q + 1] = t4.w;
  }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 128-bit global load that bypasses L1 allocation: KV pages are streamed once.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__host__ __device__ inline uint32_t ceil_div(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

}  // namespace doe
