// Row kernels (HBM-bound): per-token quantisation, fused RMSNorm + adaLN
// modulation + quantisation, fused SwiGLU + quantisation, and the reference's
// tensorwise two-phase forms.
//
// Data movement: persistent CTAs, one row group of T threads per CTA.  Rows
// stream HBM -> shared memory through a ring of `stages` slots filled by 1-D
// bulk copies (cp.async.bulk, completion on an mbarrier per slot), so many
// rows are in flight per SM without holding registers for them.  Each row is
// read from HBM once and q + one scale (plus optional bf16 outputs) written
// once.  Thread t of the CTA owns the 16-byte vectors c = t, t + T, t + 2T, ...
// of a row.
//
// T is the smallest power of two in [32, 512] that leaves at most kFastVec
// vectors per thread (512 for longer rows; rows are limited by the ring's slot
// size, 96 KB).  Canonical arithmetic, restated
// bit for bit by the CPU oracle:
//   sum of squares: per thread, two FMA accumulators (even / odd element of each
//   bf16 pair) in vector order, combined as even + odd (the squares of bf16 values
//   are exact in fp32); warp butterfly (xor 16, 8, 4, 2, 1); warp partials added
//   left to right;
//   inv = 1 / sqrt(ss / D + eps) with IEEE divide and square root;
//   h = (((x * inv) * w) * s) + b, every product and sum rounded separately;
//   per-token scale = max(amax / qmax, 1e-12) (IEEE divide);
//   q = cvt(RN(v / scale)) (see quant8: a reciprocal multiply with an exact
//   fallback near rounding boundaries), round-half-even (int8, which never
//   needs the +-127 clamp: |v / scale| <= 127 * (1 + 2^-23)) or the saturating
//   RNE e4m3 conversion (fp8).
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

namespace t8g {
namespace rows {

constexpr int kFastVec = 4;        // vectors per thread that set the row-group size T
constexpr float kScaleMin = 1e-12f;   // src/ck_fused_mod_norm_quant.py:141

enum QuantKind : int { kQuantInt8 = 0, kQuantFp8 = 1 };
enum Mode : int { kModeInt8 = 0, kModeFp8 = 1, kModeTensorwise = 2 };

template <int QK>
struct QMax;
template <>
struct QMax<kQuantInt8> {
  static constexpr float v = 127.0f;
};
template <>
struct QMax<kQuantFp8> {
  static constexpr float v = 448.0f;
};


// ---------------------------------------------------------------- bf16 helpers
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x); f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z); f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}
// |a| max |b| on packed bf16 pairs (exact).
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t a, uint32_t b) {
  __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
  __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
  __nv_bfloat162 r = __hmax2(x, __habs2(y));
  return *reinterpret_cast<uint32_t*>(&r);
}
// bf16(1 + s) for a packed pair: a correctly rounded bf16 add, equal to the
// reference's fp32 add then bf16 rounding (src/ck_fused_patch.py:120).
__device__ __forceinline__ uint32_t one_plus_bf16x2(uint32_t s) {
  const __nv_bfloat162 one = __floats2bfloat162_rn(1.0f, 1.0f);
  __nv_bfloat162 r = __hadd2(one, *reinterpret_cast<__nv_bfloat162*>(&s));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ uint4 ld_v4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint4 lds_v4(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Two fp32 values -> two e4m3 codes (RNE, saturating); `lo` lands in the low byte.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// Packed fp32 arithmetic with explicit round-to-nearest-even.  A packed multiply that
// feeds a packed add can still be fused into one multiply-add by the assembler (observed:
// h = t * s + b came out as fma(t, s, b) in a rare cancelling case), so every add whose
// operand is a product uses the scalar IEEE add (__fadd_rn, never contracted) instead.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t f2_to_bf2(float2 v) { return pack_bf16(v.x, v.y); }

// Round-half-even to an integer through the fp32 adder: for |v| < 2^22 the low byte
// of bits(v + 1.5 * 2^23) is rint(v) as a two's-complement int8.
constexpr float kRoundMagic = 12582912.0f;

// Per-row constants of the quantiser.
struct QuantRow {
  float scale;    // max(amax / qmax, 1e-12)
  float2 c_lo;    // RN(RN(1 / scale) * (1 - 2^-21)), both lanes
  float2 c_hi;    // RN(RN(1 / scale) * (1 + 2^-21)), both lanes
};

template <int QK>
__device__ __forceinline__ QuantRow quant_row(float amax) {
  QuantRow r;
  r.scale = fmaxf(__fdiv_rn(amax, QMax<QK>::v), kScaleMin);
  const float rcp = __fdiv_rn(1.0f, r.scale);
  const float lo = __fmul_rn(rcp, 1.0f - 0x1p-21f), hi = __fmul_rn(rcp, 1.0f + 0x1p-21f);
  r.c_lo = make_float2(lo, lo);
  r.c_hi = make_float2(hi, hi);
  return r;
}

// 8 values (4 pairs) -> 8 quantised bytes, bit-identical to cvt(RN(v / scale)) with an
// IEEE divide.  Writing x = v / scale, a = RN(v * c_lo) and b = RN(v * c_hi) bracket
// x within a relative 2^-21 - 2^-23 > 2^-23 of it on either side, so RN(x) lies
// between a and b.  The 8-bit conversion (int8: round half to even; e4m3: RNE with
// saturation) is monotone, so when a and b convert to the same code that code is
// the one RN(x) converts to.  Otherwise (a rounding boundary lies within ~2^-21 of
// x, probability ~2^-17 per value) the lane recomputes its eight values with the
// IEEE divide.  int8 never needs the +-127 clamp: |x| <= 127 * (1 + 2^-23).
template <int QK>
__device__ __forceinline__ uint2 quant8(const float2 (&v)[4], const QuantRow& qr) {
  uint32_t ca[4], cb[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 a = mul2_rn(v[p], qr.c_lo);
    const float2 b = mul2_rn(v[p], qr.c_hi);
    if constexpr (QK == kQuantInt8) {
      const float2 m = make_float2(kRoundMagic, kRoundMagic);
      const float2 ra = add2_rn(a, m), rb = add2_rn(b, m);
      ca[p] = __byte_perm(__float_as_uint(ra.x), __float_as_uint(ra.y), 0x0040);
      cb[p] = __byte_perm(__float_as_uint(rb.x), __float_as_uint(rb.y), 0x0040);
    } else {
      ca[p] = cvt_e4m3x2(a.x, a.y);
      cb[p] = cvt_e4m3x2(b.x, b.y);
    }
  }
  uint32_t w0 = __byte_perm(ca[0], ca[1], 0x5410), w1 = __byte_perm(ca[2], ca[3], 0x5410);
  const uint32_t u0 = __byte_perm(cb[0], cb[1], 0x5410), u1 = __byte_perm(cb[2], cb[3], 0x5410);
  if ((w0 != u0) | (w1 != u1)) {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float qx = __fdiv_rn(v[p].x, qr.scale), qy = __fdiv_rn(v[p].y, qr.scale);
      if constexpr (QK == kQuantInt8)
        ca[p] = __byte_perm(__float_as_uint(__fadd_rn(qx, kRoundMagic)), __float_as_uint(__fadd_rn(qy, kRoundMagic)),
                            0x0040);
      else
        ca[p] = cvt_e4m3x2(qx, qy);
    }
    w0 = __byte_perm(ca[0], ca[1], 0x5410);
    w1 = __byte_perm(ca[2], ca[3], 0x5410);
  }
  return make_uint2(w0, w1);
}

__device__ __forceinline__ void unpack_pairs(const uint4& u, float2 (&v)[4]) {
  v[0] = bf2_to_f2(u.x);
  v[1] = bf2_to_f2(u.y);
  v[2] = bf2_to_f2(u.z);
  v[3] = bf2_to_f2(u.w);
}


// ---------------------------------------------------------------- block reductions
// The CTA is one row group of T threads; `red` holds T/32 floats.
template <int T>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  if constexpr (T == 32) {
    return v;
  } else {
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int i = 1; i < T / 32; ++i) t = __fadd_rn(t, red[i]);
    return t;
  }
}

template <int T>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  if constexpr (T == 32) {
    return v;
  } else {
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int i = 1; i < T / 32; ++i) t = fmaxf(t, red[i]);
    return t;
  }
}

// Non-negative float max via the integer order of its bit pattern.
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

// ---------------------------------------------------------------- row ring
// Shared-memory layout of every row kernel: mbarriers, reduction scratch, then
// `stages` slots of `slot_bytes` (1024-byte aligned).
struct RingGeom {
  int stages;          // slots in the ring (>= 2)
  uint32_t slot_bytes; // bytes of one slot (one row, or gate row + up row)
  uint32_t part_bytes; // bytes of one bulk copy (a row of one operand)
  int parts;           // bulk copies per slot (1, or 2 for gate + up)
};
constexpr int kRingHeader = 1024;   // barriers (<= 16 x 8 B), reductions (2 x 16 floats), flags
constexpr int kMaxStages = 16;

struct RingState {
  uint64_t* full;
  float* red_sum;
  float* red_max;
  uint8_t* slots;
};

__device__ __forceinline__ RingState ring_state(uint8_t* smem) {
  RingState r;
  r.full = reinterpret_cast<uint64_t*>(smem);
  r.red_sum = reinterpret_cast<float*>(smem + 8 * kMaxStages);
  r.red_max = r.red_sum + 16;
  r.slots = smem + kRingHeader;
  return r;
}

// Issue the bulk copies of row `row` into slot `st` (one thread).
__device__ __forceinline__ void ring_issue(const RingState& rs, const RingGeom& g, int st, const void* src0,
                                           const void* src1, uint64_t policy) {
  uint8_t* dst = rs.slots + static_cast<size_t>(st) * g.slot_bytes;
  mbar_arrive_expect_tx(&rs.full[st], g.part_bytes * static_cast<uint32_t>(g.parts));
  bulk_load(dst, src0, g.part_bytes, &rs.full[st], policy);
  if (g.parts == 2) bulk_load(dst + g.part_bytes, src1, g.part_bytes, &rs.full[st], policy);
}

// ---------------------------------------------------------------- kernel arguments
struct QuantRowsArgs {
  const __nv_bfloat16* x;
  int64_t ld_x;
  void* q;
  int64_t ld_q;
  float* q_scale;
  int64_t S;
  int D;
};

struct RmsArgs {
  const __nv_bfloat16* x;
  int64_t ld_x;
  const __nv_bfloat16* w;        // [D] norm weight or nullptr
  const __nv_bfloat16* shift;    // [n_mod, D]
  const __nv_bfloat16* scale;    // [n_mod, D]: adaLN scale, or the multiplier itself
  int64_t ld_mod;
  const int32_t* mod_index;      // [S] modulation row of each token, or nullptr
  int64_t rows_per_mod;          // used when mod_index == nullptr
  int scale_is_multiplier;       // 0: s = bf16(1 + scale); 1: s = scale
  float eps;
  void* q;                       // per-token mode: [S, D] codes
  int64_t ld_q;
  float* q_scale;                // per-token mode: [S]
  __nv_bfloat16* h;              // optional [S, D] bf16 h (required in tensorwise mode)
  int64_t ld_h;
  __nv_bfloat16* res;            // optional [S, D] bf16 h + x
  int64_t ld_res;
  float* amax;                   // tensorwise mode: global max |h| (float32, before rounding)
  int64_t S;
  int D;
};

struct SwigluArgs {
  const __nv_bfloat16* gate;   // [M, F] with row stride ld_in
  const __nv_bfloat16* up;     // [M, F] with row stride ld_in
  int64_t ld_in;
  void* q;
  int64_t ld_q;
  float* q_scale;
  __nv_bfloat16* act;          // optional [M, F] bf16 act (required in tensorwise mode)
  int64_t ld_act;
  float* amax;                 // tensorwise mode
  int64_t M;
  int F;
};

// ---------------------------------------------------------------- common loop
// Runs `body(row, slot_ptr, ring)` for rows blockIdx.x, blockIdx.x + gridDim.x, ...
// with the ring kept `stages - 1` rows ahead.  `src(row, part)` gives the
// global address of a row operand.  Returns after draining in-flight copies.
template <int T, typename Src, typename Body>
__device__ __forceinline__ void row_loop(uint8_t* smem, const RingGeom& g, int64_t nrows, Src src, Body body) {
  RingState rs = ring_state(smem);
  const uint64_t policy = policy_evict_first();
  const int64_t G = gridDim.x;
  if (threadIdx.x == 0) {
    for (int i = 0; i < g.stages; ++i) mbar_init(&rs.full[i], 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  int64_t issued = 0;   // meaningful in thread 0 only
  if (threadIdx.x == 0) {
    for (int i = 0; i < g.stages; ++i) {
      const int64_t r = blockIdx.x + i * G;
      if (r >= nrows) break;
      ring_issue(rs, g, i, src(r, 0), src(r, 1), policy);
      ++issued;
    }
  }
  int64_t k = 0;
  for (int64_t row = blockIdx.x; row < nrows; row += G, ++k) {
    const int st = static_cast<int>(k % g.stages);
    const uint32_t ph = static_cast<uint32_t>((k / g.stages) & 1);
    const bool ok = mbar_wait(&rs.full[st], ph, kStatusTimeoutProducer);
    if (__syncthreads_or(!ok)) break;
    // every thread is past row k-1: refill its slot with row k-1+stages
    if (threadIdx.x == 0 && k > 0) {
      const int64_t r = row - G + static_cast<int64_t>(g.stages) * G;
      if (r < nrows) {
        ring_issue(rs, g, static_cast<int>((k - 1) % g.stages), src(r, 0), src(r, 1), policy);
        ++issued;
      }
    }
    body(row, rs.slots + static_cast<size_t>(st) * g.slot_bytes, rs);
  }
  // teardown: copies still in flight (only after an abort) must land before exit
  if (threadIdx.x == 0) {
    for (int64_t n = k; n < issued; ++n)
      if (!mbar_wait(&rs.full[n % g.stages], static_cast<uint32_t>((n / g.stages) & 1), kStatusTimeoutDrain)) break;
  }
}

// ---------------------------------------------------------------- shared pieces
// Quantise the row held (as bf16) in `src` (shared memory) and store q.
template <int T, int QK>
__device__ __forceinline__ void quant_row_store(const uint8_t* src, int nvec, const QuantRow& qr, uint8_t* qrow) {
  for (int c = threadIdx.x; c < nvec; c += T) {
    float2 v[4];
    unpack_pairs(lds_v4(src + 16 * c), v);
    *reinterpret_cast<uint2*>(qrow + 8 * c) = quant8<QK>(v, qr);
  }
}

__device__ __forceinline__ uint32_t absmax4(uint32_t m2, const uint4& u) {
  m2 = absmax_bf16x2(m2, u.x);
  m2 = absmax_bf16x2(m2, u.y);
  m2 = absmax_bf16x2(m2, u.z);
  return absmax_bf16x2(m2, u.w);
}

// Generic-proxy writes to a ring slot must be ordered before the bulk copy that
// later refills it.
__device__ __forceinline__ void slot_written() { fence_proxy_async_smem(); }

// ---------------------------------------------------------------- per-token quant
template <int T, int QK>
__global__ void __launch_bounds__(T) quant_rows_kernel(const QuantRowsArgs a, const RingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int nvec = a.D >> 3;
  auto src = [&](int64_t r, int) -> const void* { return a.x + r * a.ld_x; };
  row_loop<T>(smem, g, a.S, src, [&](int64_t row, const uint8_t* slot, const RingState& rs) {
    uint32_t m2 = 0;
    for (int c = threadIdx.x; c < nvec; c += T) m2 = absmax4(m2, lds_v4(slot + 16 * c));
    const float amax = block_max<T>(fmaxf(bf_lo(m2), bf_hi(m2)), rs.red_max);
    const QuantRow qr = quant_row<QK>(amax);
    if (threadIdx.x == 0) a.q_scale[row] = qr.scale;
    quant_row_store<T, QK>(slot, nvec, qr, static_cast<uint8_t*>(a.q) + row * a.ld_q);
  });
}

// ---------------------------------------------------------------- RMSNorm + modulation
// Sum of squares: each thread keeps two fp32 accumulators, one for the even and one
// for the odd element of every bf16 pair, adds its vectors' squares in vector order
// with a packed FMA, then combines them as (even + odd) before the row reduction.
template <int T, int MODE>
__global__ void __launch_bounds__(T) rms_mod_kernel(const RmsArgs a, const RingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int nvec = a.D >> 3;
  const float fD = static_cast<float>(a.D);
  auto src = [&](int64_t r, int) -> const void* { return a.x + r * a.ld_x; };
  row_loop<T>(smem, g, a.S, src, [&](int64_t row, uint8_t* slot, const RingState& rs) {
    // pass 1: sum of squares in the canonical order
    float2 acc = make_float2(0.f, 0.f);
    for (int c = threadIdx.x; c < nvec; c += T) {
      float2 v[4];
      unpack_pairs(lds_v4(slot + 16 * c), v);
#pragma unroll
      for (int p = 0; p < 4; ++p) acc = fma2_rn(v[p], v[p], acc);
    }
    const float ss = block_sum<T>(__fadd_rn(acc.x, acc.y), rs.red_sum);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, fD), a.eps)));
    const float2 inv2 = make_float2(inv, inv);

    const int64_t m = a.mod_index ? static_cast<int64_t>(__ldg(a.mod_index + row)) : row / a.rows_per_mod;
    const __nv_bfloat16* shr = a.shift + m * a.ld_mod;
    const __nv_bfloat16* scr = a.scale + m * a.ld_mod;

    // pass 2: h (written back over x in the slot), optional res / h stores, amax
    uint32_t m2 = 0;
    float amax32 = 0.f;
    for (int c = threadIdx.x; c < nvec; c += T) {
      const uint4 xu = lds_v4(slot + 16 * c);
      uint4 su = ld_v4(scr + 8 * c);
      const uint4 bu = ld_v4(shr + 8 * c);
      if (!a.scale_is_multiplier)
        su = make_uint4(one_plus_bf16x2(su.x), one_plus_bf16x2(su.y), one_plus_bf16x2(su.z), one_plus_bf16x2(su.w));
      float2 x[4], sv[4], bv[4], h[4];
      unpack_pairs(xu, x);
      unpack_pairs(su, sv);
      unpack_pairs(bu, bv);
      float2 prod[4];
      if (a.w) {
        float2 wv[4];
        unpack_pairs(ld_v4(a.w + 8 * c), wv);
#pragma unroll
        for (int p = 0; p < 4; ++p) prod[p] = mul2_rn(mul2_rn(mul2_rn(x[p], inv2), wv[p]), sv[p]);
      } else {
#pragma unroll
        for (int p = 0; p < 4; ++p) prod[p] = mul2_rn(mul2_rn(x[p], inv2), sv[p]);
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) h[p] = make_float2(__fadd_rn(prod[p].x, bv[p].x), __fadd_rn(prod[p].y, bv[p].y));
      if (a.res) {
        uint4 ru;
        ru.x = f2_to_bf2(add2_rn(h[0], x[0]));
        ru.y = f2_to_bf2(add2_rn(h[1], x[1]));
        ru.z = f2_to_bf2(add2_rn(h[2], x[2]));
        ru.w = f2_to_bf2(add2_rn(h[3], x[3]));
        *reinterpret_cast<uint4*>(a.res + row * a.ld_res + 8 * c) = ru;
      }
      if constexpr (MODE == kModeTensorwise) {
#pragma unroll
        for (int p = 0; p < 4; ++p) amax32 = fmaxf(amax32, fmaxf(fabsf(h[p].x), fabsf(h[p].y)));
      }
      const uint4 hu = make_uint4(f2_to_bf2(h[0]), f2_to_bf2(h[1]), f2_to_bf2(h[2]), f2_to_bf2(h[3]));
      m2 = absmax4(m2, hu);
      *reinterpret_cast<uint4*>(slot + 16 * c) = hu;
      if (a.h) *reinterpret_cast<uint4*>(a.h + row * a.ld_h + 8 * c) = hu;
    }
    slot_written();
    if constexpr (MODE == kModeTensorwise) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) amax32 = fmaxf(amax32, __shfl_xor_sync(0xFFFFFFFFu, amax32, off));
      if ((threadIdx.x & 31) == 0 && amax32 > 0.f) atomic_max_nonneg(a.amax, amax32);
    } else {
      constexpr int QK = MODE;
      const float amax = block_max<T>(fmaxf(bf_lo(m2), bf_hi(m2)), rs.red_max);   // barrier: h complete
      const QuantRow qr = quant_row<QK>(amax);
      if (threadIdx.x == 0) a.q_scale[row] = qr.scale;
      quant_row_store<T, QK>(slot, nvec, qr, static_cast<uint8_t*>(a.q) + row * a.ld_q);
    }
  });
}

// ---------------------------------------------------------------- SwiGLU
// act = (g * sigmoid(g)) * u with sigmoid(g) = 1 / (1 + e^-g); e^-g and the reciprocal
// use the fast hardware approximations (act is compared with the oracle within one
// bf16 ulp).
// Approximate reciprocal (max 1 ulp), subnormal results kept (no flush to zero).
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float2 silu_mul2(float2 g, float2 u) {
  const float2 e = make_float2(__expf(-g.x), __expf(-g.y));
  const float2 d = add2_rn(make_float2(1.0f, 1.0f), e);
  const float2 r = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  return mul2_rn(mul2_rn(g, r), u);
}

template <int T, int MODE>
__global__ void __launch_bounds__(T) swiglu_kernel(const SwigluArgs a, const RingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int nvec = a.F >> 3;
  auto src = [&](int64_t r, int part) -> const void* { return (part ? a.up : a.gate) + r * a.ld_in; };
  row_loop<T>(smem, g, a.M, src, [&](int64_t row, uint8_t* slot, const RingState& rs) {
    const uint8_t* up = slot + g.part_bytes;
    uint32_t m2 = 0;
    float amax32 = 0.f;
    for (int c = threadIdx.x; c < nvec; c += T) {
      float2 gv[4], uv[4], act[4];
      unpack_pairs(lds_v4(slot + 16 * c), gv);
      unpack_pairs(lds_v4(up + 16 * c), uv);
#pragma unroll
      for (int p = 0; p < 4; ++p) act[p] = silu_mul2(gv[p], uv[p]);
      if constexpr (MODE == kModeTensorwise) {
#pragma unroll
        for (int p = 0; p < 4; ++p) amax32 = fmaxf(amax32, fmaxf(fabsf(act[p].x), fabsf(act[p].y)));
      }
      const uint4 au = make_uint4(f2_to_bf2(act[0]), f2_to_bf2(act[1]), f2_to_bf2(act[2]), f2_to_bf2(act[3]));
      m2 = absmax4(m2, au);
      *reinterpret_cast<uint4*>(slot + 16 * c) = au;   // act replaces the gate row
      if (a.act) *reinterpret_cast<uint4*>(a.act + row * a.ld_act + 8 * c) = au;
    }
    slot_written();
    if constexpr (MODE == kModeTensorwise) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) amax32 = fmaxf(amax32, __shfl_xor_sync(0xFFFFFFFFu, amax32, off));
      if ((threadIdx.x & 31) == 0 && amax32 > 0.f) atomic_max_nonneg(a.amax, amax32);
    } else {
      constexpr int QK = MODE;
      const float amax = block_max<T>(fmaxf(bf_lo(m2), bf_hi(m2)), rs.red_max);   // barrier: act complete
      const QuantRow qr = quant_row<QK>(amax);
      if (threadIdx.x == 0) a.q_scale[row] = qr.scale;
      quant_row_store<T, QK>(slot, nvec, qr, static_cast<uint8_t*>(a.q) + row * a.ld_q);
    }
  });
}

// ---------------------------------------------------------------------------
// tensorwise phase B: q = cvt(RN(h / max(amax / qmax, 1e-12))) from the device amax
// (src/ck_fused_mod_norm_quant.py:92-111); also writes the scale.
// ---------------------------------------------------------------------------
struct QuantGivenArgs {
  const __nv_bfloat16* h;
  int64_t ld_h;
  void* q;
  int64_t ld_q;
  const float* amax;
  float* scale_out;   // optional
  int64_t S;
  int D;
};

template <int QK>
__global__ void __launch_bounds__(256) quant_given_amax_kernel(const QuantGivenArgs a) {
  const QuantRow qr = quant_row<QK>(*a.amax);
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.scale_out) *a.scale_out = qr.scale;
  const int nvec = a.D >> 3;
  const int64_t total = a.S * nvec;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = v / nvec;
    const int c = static_cast<int>(v - row * nvec);
    float2 f[4];
    unpack_pairs(ld_v4(a.h + row * a.ld_h + 8 * c), f);
    *reinterpret_cast<uint2*>(static_cast<uint8_t*>(a.q) + row * a.ld_q + 8 * c) = quant8<QK>(f, qr);
  }
}

// ---------------------------------------------------------------------------
// self-test of the bounded wait: waits on an mbarrier that nothing completes,
// with a short limit, and reports whether the wait gave up (status 0x1FF).
// ---------------------------------------------------------------------------
__global__ void wait_selftest_kernel(uint64_t limit_ns, int* gave_up) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t addr = smem_u32(&bar);
    const uint64_t t0 = globaltimer_ns();
    int result = 0;
    while (!mbar_try_wait(addr, 0)) {
      if (globaltimer_ns() - t0 > limit_ns) {
        record_status(kStatusTimeoutSelfTest);
        result = 1;
        break;
      }
    }
    *gave_up = result;
    mbar_arrive(&bar);   // complete the phase so nothing is left pending
  }
}

}  // namespace rows
}  // namespace t8g
