// The SwiGLU's sigmoid, exact for bf16 gate values, shared by the SwiGLU row kernels and
// the fc1 GEMM's SwiGLU epilogue (the same table and operations, so both give the same bits).
//
// The reference computes act = (g * sigmoid(g)) * u in float32 with sigmoid(g) =
// 1 / (1 + exp(-g)) (src/ck_fused_mod_norm_quant.py:71).  g is a bf16 value, so
// sigmoid(g) = RN(1 / RN(1 + RN(exp(-g)))) -- exp correctly rounded, the add and divide
// IEEE -- takes one of at most 65536 values, tabulated at build time (csrc/sigmoid_table.c).
// The lookup clamps the magnitude bits of g to [0x32FF, 0x4300]; the ends carry the exact
// constants (|g| < 2^-25: 1/2; |g| >= 128, inf and NaN: 1 for g > 0, 0 for g < 0 -- so
// NaN stays NaN and -inf * 0 gives the reference's NaN), one half of the table per sign:
//     index = sign * 4098 + (clamped - 0x32FF)
// For a packed pair of gate values the clamp is two 16-bit-lane min/max instructions and the
// index one multiply-add, so a pair costs ~9 integer instructions and two shared-memory loads.
// The kernels copy the table (32.8 KB) into shared memory once per CTA.  act is then two IEEE
// multiplies with subnormals kept (for -88.7 < g < -87.3 the sigmoid is subnormal while
// g * sigmoid is a normal number).
#pragma once

#include <stdint.h>

#include "f32x2.cuh"

namespace t8g {

constexpr uint32_t kSigmoidHalf = 4098;                     // entries per sign
constexpr int kSigmoidEntries = 8200;                       // two halves, padded to a multiple of 4
constexpr uint32_t kSigmoidBytes = kSigmoidEntries * 4;
constexpr uint32_t kSigmoidLo = 0x32FFu;                    // clamp floor of the magnitude bits
constexpr uint32_t kSigmoidHi = 0x4300u;                    // clamp ceiling: bf16 bits of 128

__device__ __align__(16) const uint32_t g_sigmoid_table[kSigmoidEntries] = {
#include "sigmoid_table.inc"
};

// Copies the table into shared memory `dst` (16-byte aligned) with threads t, t + n, ...
__device__ __forceinline__ void load_sigmoid_table(uint32_t* dst, int t, int n) {
  const uint4* src = reinterpret_cast<const uint4*>(g_sigmoid_table);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = t; i < kSigmoidEntries / 4; i += n) d[i] = __ldg(src + i);
}

__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// A load from the (constant, already written) table: no side effects, so the compiler may
// schedule it freely after its address is known.
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// (sigmoid(lo(gpair)), sigmoid(hi(gpair))) for a packed bf16 pair; `tab` is the table's
// shared-memory address (cvta'd), offset below by the clamp floor so the clamped value
// indexes it directly.
__device__ __forceinline__ float2 sigmoid_bf16x2(uint32_t gpair, uint32_t tab) {
  const uint32_t mag = gpair & 0x7FFF7FFFu;
  const uint32_t c = min_u16x2(max_u16x2(mag, kSigmoidLo * 0x10001u), kSigmoidHi * 0x10001u);
  const uint32_t sign = (gpair >> 15) & 0x00010001u;
  const uint32_t idx = sign * kSigmoidHalf + c;              // no carry between the halves
  const uint32_t base = tab - kSigmoidLo * 4u;
  return make_float2(lds_f32(base + (idx & 0xFFFFu) * 4u), lds_f32(base + (idx >> 16) * 4u));
}

// (act_lo, act_hi) = ((g * sigmoid(g)) * u) for a packed bf16 gate pair and fp32 up values.
__device__ __forceinline__ float2 silu_mul2(uint32_t gpair, float2 u, uint32_t tab) {
  return mul2_rn(mul2_rn(bf2_to_f2(gpair), sigmoid_bf16x2(gpair, tab)), u);
}

}  // namespace t8g
