// Packed fp32 / bf16 helpers and the SiLU shared by the row kernels and the GEMM's
// SwiGLU epilogue (the same operations in the same order, so both give the same bits).
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
__device__ __forceinline__ float2 add_f32_f16x2(float2 p, uint32_t b) {
  float x, y;
  asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; add.rn.f32.f16 %0, lo, %3; add.rn.f32.f16 %1, hi, %4; }"
      : "=f"(x), "=f"(y)
      : "r"(b), "f"(p.x), "f"(p.y));
  return make_float2(x, y);
}

// act = (g * sigmoid(g)) * u with sigmoid(g) = 1 / (1 + e^-g), in fp32 with the fast
// hardware exponential and reciprocal (act is compared with the oracle within one bf16
// ulp):
//   e   = 2^(-g * log2(e))              ex2.approx.ftz (the change-of-base identity)
//   d4  = (1 + e) / 4                   one fma: RN(1 + e) scaled exactly by 1/4
//   r4  = approx(1 / d4) = 4 / (1 + e)  rcp.approx.ftz
//   act = ((g / 4) * r4) * u            g / 4 is exact for every bf16 g
// The quarter scaling keeps the reciprocal normal where 1 / (1 + e) itself would be
// subnormal (g < -87.3: 2^-126 < 4 / (1 + e)), so flushing subnormal reciprocals cannot
// change act; (g / 4) * r4 is the same real product as g * (1 / (1 + e)).  For e = inf
// (g < -88.7) r4 = 0 and act is a signed zero, as in fp32 with an IEEE reciprocal.
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

constexpr float kLog2E = 1.44269504088896340736f;

// g4 = g / 4 (exact), u: one packed pair of gate / up values.
__device__ __forceinline__ float2 silu_mul2(float2 g4, float2 u) {
  const float2 t = mul2_rn(g4, make_float2(-4.0f * kLog2E, -4.0f * kLog2E));   // = -g * log2(e), same rounding
  const float2 e = make_float2(ex2_approx(t.x), ex2_approx(t.y));
  const float2 d4 = fma2_rn(e, make_float2(0.25f, 0.25f), make_float2(0.25f, 0.25f));
  const float2 r4 = make_float2(rcp_approx_ftz(d4.x), rcp_approx_ftz(d4.y));
  return mul2_rn(mul2_rn(g4, r4), u);
}

}  // namespace t8g
