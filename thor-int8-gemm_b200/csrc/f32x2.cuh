// Packed fp32 / bf16 helpers shared by the row kernels and the GEMM epilogues (the same
// operations in the same order, so both give the same bits).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace t8g {

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Packed fp32 arithmetic (two lanes per instruction), each lane rounded to nearest even.
// A packed multiply that feeds a packed add may be fused into one multiply-add
// (observed: h = t * s + b came out as fma(t, s, b) in a rare cancelling case), so an
// add whose operand is a product that must round separately uses the scalar IEEE add
// (__fadd_rn, never contracted) or the mixed-precision add.rn.f32.bf16.  Products that
// feed only fmas (the quantiser's quotient correction) are unaffected.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t f2_to_bf2(float2 v) { return pack_bf16(v.x, v.y); }

// (p.x + lo(b), p.y + hi(b)) with b a packed bf16 (or fp16) pair, each an IEEE add taking
// the 16-bit operand directly (mixed-precision add, no unpacking); an add with an explicit
// rounding mode is never contracted with the product that feeds it.
__device__ __forceinline__ float2 add_f32_bf16x2(float2 p, uint32_t b) {
  float x, y;
  asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; add.rn.f32.bf16 %0, lo, %3; add.rn.f32.bf16 %1, hi, %4; }"
      : "=f"(x), "=f"(y)
      : "r"(b), "f"(p.x), "f"(p.y));
  return make_float2(x, y);
}
// (lo(a) * lo(b), hi(a) * hi(b)) for two packed bf16 pairs: the product of two bf16 values
// is exact in fp32, formed as fma(a, b, -0) with the 16-bit operands taken directly
// (adding -0 keeps every product, signed zeros included, as the IEEE multiply gives it).
__device__ __forceinline__ float2 mul_bf16x2_exact(uint32_t a, uint32_t b) {
  float x, y;
  asm("{ .reg .b16 alo, ahi, blo, bhi; mov.b32 {alo, ahi}, %2; mov.b32 {blo, bhi}, %3;"
      " fma.rn.f32.bf16 %0, alo, blo, 0f80000000; fma.rn.f32.bf16 %1, ahi, bhi, 0f80000000; }"
      : "=f"(x), "=f"(y)
      : "r"(a), "r"(b));
  return make_float2(x, y);
}
// max(|a|, |b|) lane by lane on packed bf16 pairs (exact; a NaN loses to a number).
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t a, uint32_t b) {
  __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
  __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
  __nv_bfloat162 r = __hmax2(x, __habs2(y));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ float2 add_f32_f16x2(float2 p, uint32_t b) {
  float x, y;
  asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; add.rn.f32.f16 %0, lo, %3; add.rn.f32.f16 %1, hi, %4; }"
      : "=f"(x), "=f"(y)
      : "r"(b), "f"(p.x), "f"(p.y));
  return make_float2(x, y);
}

}  // namespace t8g
