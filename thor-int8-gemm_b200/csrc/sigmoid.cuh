// The SwiGLU's sigmoid, exact for bf16 gate values, shared by the SwiGLU row kernel and
// the fc1 GEMM's SwiGLU epilogue (the same table and operations, so both give the same bits).
//
// The reference computes act = (g * sigmoid(g)) * u in float32 with sigmoid(g) =
// 1 / (1 + exp(-g)) (src/ck_fused_mod_norm_quant.py:71).  g is a bf16 value, so
// sigmoid(g) = RN(1 / RN(1 + RN(exp(-g)))) -- exp correctly rounded, the add and divide
// IEEE -- takes one of at most 65536 values.  Those that are not a constant are tabulated
// at build time (csrc/sigmoid_table.c): 2^-25 <= |g| < 128, 8192 entries indexed by the
// sign and the low 12 bits of (|g| bits - 0x3300).  The rest are exact constants:
//   |g| < 2^-25          exp(-g) rounds to 1, sigmoid = 1/2
//   g >= 128, +inf, NaN  exp(-g) rounds to 0, sigmoid = 1 (NaN stays NaN in g * sigmoid)
//   g <= -128, -inf      exp(-g) overflows, sigmoid = 0 (-inf * 0 = NaN, as in the reference)
// The kernels copy the table (32 KB) into shared memory once per CTA.  act is then two
// IEEE multiplies, with subnormals kept (g * sigmoid for g in [-88.7, -87.3), where the
// sigmoid is subnormal, is a normal number).
#pragma once

#include <stdint.h>

#include "f32x2.cuh"

namespace t8g {

constexpr int kSigmoidEntries = 8192;
constexpr uint32_t kSigmoidBytes = kSigmoidEntries * 4;
constexpr uint32_t kSigmoidLo = 0x3300u;   // bf16 magnitude bits of 2^-25

__device__ __align__(16) const uint32_t g_sigmoid_table[kSigmoidEntries] = {
#include "sigmoid_table.inc"
};

// Copies the table into shared memory `dst` (16-byte aligned) with threads t, t + n, ...
__device__ __forceinline__ void load_sigmoid_table(uint32_t* dst, int t, int n) {
  const uint4* src = reinterpret_cast<const uint4*>(g_sigmoid_table);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = t; i < kSigmoidEntries / 4; i += n) d[i] = __ldg(src + i);
}

// sigmoid(g) for the bf16 value whose bits are the low 16 bits of `gb` (upper bits zero).
__device__ __forceinline__ float sigmoid_bf16(uint32_t gb, const uint32_t* tab) {
  const uint32_t mag = gb & 0x7FFFu;
  const uint32_t rel = mag - kSigmoidLo;                        // wraps for |g| < 2^-25
  const bool in = rel < 4096u;
  const uint32_t idx = in ? (rel | ((gb >> 3) & 0x1000u)) : 0u;  // sign -> bit 12
  const float t = __uint_as_float(tab[idx]);
  const float edge = mag < kSigmoidLo ? 0.5f : ((gb & 0x8000u) ? 0.0f : 1.0f);
  return in ? t : edge;
}

// (act_lo, act_hi) = ((g * sigmoid(g)) * u) for a packed bf16 gate pair and fp32 up values.
__device__ __forceinline__ float2 silu_mul2(uint32_t gpair, float2 u, const uint32_t* tab) {
  const float2 s = make_float2(sigmoid_bf16(gpair & 0xFFFFu, tab), sigmoid_bf16(gpair >> 16, tab));
  return mul2_rn(mul2_rn(bf2_to_f2(gpair), s), u);
}

}  // namespace t8g
