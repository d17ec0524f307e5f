// Row kernels (HBM-bound): per-token quantisation, fused RMSNorm + adaLN
// modulation + quantisation, fused SwiGLU + quantisation, and the reference's
// tensorwise two-phase forms.
//
// One row (token) is processed by T threads, T the smallest power of two in
// [32, 512] such that each thread holds at most MAX_VEC 16-byte vectors (8
// bf16 values); vector c of the row goes to thread c % T.  The whole row stays
// in registers between the reduction passes, so x (or gate/up) is read from
// HBM exactly once and q + one scale per row are written once.
//
// Canonical arithmetic (restated by the CPU oracle, bit for bit):
//   sum of squares: per-thread FMA accumulation in vector order, warp
//   butterfly (xor 16, 8, 4, 2, 1), then warp partials added left to right;
//   inv = 1 / sqrt(ss / D + eps) with IEEE divide and square root;
//   h = (((x * inv) * w) * s) + b, every product and sum rounded separately;
//   per-token scale = max(amax / qmax, 1e-12); q = cvt(clamp(v / scale)).
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

namespace t8g {
namespace rows {

constexpr int MAX_VEC = 12;
constexpr float kScaleMin = 1e-12f;   // src/ck_fused_mod_norm_quant.py:141

enum QuantKind : int { kQuantInt8 = 0, kQuantFp8 = 1 };

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

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
__device__ __forceinline__ float bf_at(const uint4& v, int j) {
  const uint32_t w = (j < 2) ? v.x : (j < 4) ? v.y : (j < 6) ? v.z : v.w;
  return (j & 1) ? bf_hi(w) : bf_lo(w);
}
__device__ __forceinline__ float round_bf16(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
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

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ld_v4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Two fp32 values -> two e4m3 codes (round to nearest even, saturating);
// `lo` lands in the low byte.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// 8 values -> 8 quantised bytes (IEEE divide by the scale).
template <int QK>
__device__ __forceinline__ uint2 quant8(const float (&f)[8], float scale) {
  uint32_t b[8];
  if constexpr (QK == kQuantInt8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = rintf(__fdiv_rn(f[j], scale));
      v = fminf(fmaxf(v, -127.0f), 127.0f);
      b[j] = static_cast<uint32_t>(static_cast<int>(v)) & 0xFFu;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float v0 = fminf(fmaxf(__fdiv_rn(f[j], scale), -448.0f), 448.0f);
      const float v1 = fminf(fmaxf(__fdiv_rn(f[j + 1], scale), -448.0f), 448.0f);
      const uint32_t p = cvt_e4m3x2(v0, v1);
      b[j] = p & 0xFFu;
      b[j + 1] = p >> 8;
    }
  }
  return make_uint2(b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24), b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24));
}

template <int QK>
__device__ __forceinline__ float scale_from_amax(float amax) {
  return fmaxf(__fdiv_rn(amax, QMax<QK>::v), kScaleMin);
}

// Block geometry: rows of T threads packed into blocks of max(256, T) threads.
template <int T>
struct Geo {
  static constexpr int kBlock = T >= 256 ? T : 256;
  static constexpr int kRows = kBlock / T;
  static constexpr int kWarps = T / 32;
};

// Canonical row sum (see file comment).  `red` holds kWarps floats of this row.
template <int T>
__device__ __forceinline__ float row_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  if constexpr (T == 32) {
    return v;
  } else {
    const int w = (threadIdx.x % T) >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int i = 1; i < T / 32; ++i) t = __fadd_rn(t, red[i]);
    __syncthreads();
    return t;
  }
}

template <int T>
__device__ __forceinline__ float row_max(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  if constexpr (T == 32) {
    return v;
  } else {
    const int w = (threadIdx.x % T) >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int i = 1; i < T / 32; ++i) t = fmaxf(t, red[i]);
    __syncthreads();
    return t;
  }
}

// Non-negative float max via the integer order of its bit pattern.
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

// ---------------------------------------------------------------------------
// per-token quantisation of a bf16 matrix (comfy-kitchen int8_linear input)
// ---------------------------------------------------------------------------
struct QuantRowsArgs {
  const __nv_bfloat16* x;
  int64_t ld_x;
  void* q;
  int64_t ld_q;
  float* q_scale;
  int64_t S;
  int D;
};

template <int T, int QK>
__global__ void __launch_bounds__(Geo<T>::kBlock) quant_rows_kernel(const QuantRowsArgs a) {
  __shared__ float red[Geo<T>::kRows][Geo<T>::kWarps];
  const int tid = threadIdx.x % T;
  const int rloc = threadIdx.x / T;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * Geo<T>::kRows + rloc;
  const bool active = row < a.S;
  const int nvec = a.D >> 3;
  const __nv_bfloat16* xr = a.x + (active ? row : 0) * a.ld_x;
  uint4 xv[MAX_VEC];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAX_VEC; ++i) {
    const int c = tid + T * i;
    xv[i] = (active && c < nvec) ? ld_nc_v4(xr + 8 * c) : make_uint4(0, 0, 0, 0);
    float f[8];
    unpack8(xv[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
  }
  amax = row_max<T>(amax, red[rloc]);
  const float scale = scale_from_amax<QK>(amax);
  if (!active) return;
  if (tid == 0) a.q_scale[row] = scale;
  uint8_t* qr = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll
  for (int i = 0; i < MAX_VEC; ++i) {
    const int c = tid + T * i;
    if (c < nvec) {
      float f[8];
      unpack8(xv[i], f);
      *reinterpret_cast<uint2*>(qr + 8 * c) = quant8<QK>(f, scale);
    }
  }
}

// ---------------------------------------------------------------------------
// RMSNorm + adaLN modulation (+ per-token quant, or tensorwise phase A)
// ---------------------------------------------------------------------------
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
  __nv_bfloat16* h;              // optional [S, D] bf16 h
  int64_t ld_h;
  __nv_bfloat16* res;            // optional [S, D] bf16 h + x
  int64_t ld_res;
  float* amax;                   // tensorwise mode: global max |h| (float32, before rounding)
  int64_t S;
  int D;
};

// MODE 0/1: per-token quant (int8 / fp8); MODE 2: tensorwise phase A.
template <int T, int MODE>
__global__ void __launch_bounds__(Geo<T>::kBlock) rms_mod_kernel(const RmsArgs a) {
  __shared__ float red[Geo<T>::kRows][Geo<T>::kWarps];
  const int tid = threadIdx.x % T;
  const int rloc = threadIdx.x / T;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * Geo<T>::kRows + rloc;
  const bool active = row < a.S;
  const int nvec = a.D >> 3;
  const int64_t r = active ? row : 0;
  const __nv_bfloat16* xr = a.x + r * a.ld_x;

  uint4 xv[MAX_VEC];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAX_VEC; ++i) {
    const int c = tid + T * i;
    xv[i] = (active && c < nvec) ? ld_nc_v4(xr + 8 * c) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int i = 0; i < MAX_VEC; ++i) {
    float f[8];
    unpack8(xv[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = __fmaf_rn(f[j], f[j], ss);
  }
  ss = row_sum<T>(ss, red[rloc]);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(a.D)), a.eps)));

  const int64_t m = a.mod_index ? static_cast<int64_t>(a.mod_index[r]) : r / a.rows_per_mod;
  const __nv_bfloat16* shr = a.shift + m * a.ld_mod;
  const __nv_bfloat16* scr = a.scale + m * a.ld_mod;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAX_VEC; ++i) {
    const int c = tid + T * i;
    if (active && c < nvec) {
      float x[8], b[8], s[8], w[8], h[8];
      unpack8(xv[i], x);
      unpack8(ld_v4(shr + 8 * c), b);
      unpack8(ld_v4(scr + 8 * c), s);
      if (a.w) unpack8(ld_v4(a.w + 8 * c), w);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sj = a.scale_is_multiplier ? s[j] : round_bf16(__fadd_rn(1.0f, s[j]));
        float t = __fmul_rn(x[j], inv);
        if (a.w) t = __fmul_rn(t, w[j]);
        t = __fmul_rn(t, sj);
        h[j] = __fadd_rn(t, b[j]);
      }
      if (a.res) {
        float rs[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) rs[j] = __fadd_rn(h[j], x[j]);
        *reinterpret_cast<uint4*>(a.res + row * a.ld_res + 8 * c) = pack8(rs);
      }
      if constexpr (MODE == 2) {
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(h[j]));
      }
      xv[i] = pack8(h);   // h rounded to bf16 replaces x in registers
      if constexpr (MODE != 2) {
        float hb[8];
        unpack8(xv[i], hb);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(hb[j]));
      }
      if (a.h) *reinterpret_cast<uint4*>(a.h + row * a.ld_h + 8 * c) = xv[i];
    }
  }
  if constexpr (MODE == 2) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
    if ((threadIdx.x & 31) == 0 && amax > 0.f) atomic_max_nonneg(a.amax, amax);
  } else {
    constexpr int QK = MODE;
    amax = row_max<T>(amax, red[rloc]);
    const float scale = scale_from_amax<QK>(amax);
    if (!active) return;
    if (tid == 0) a.q_scale[row] = scale;
    uint8_t* qr = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll
    for (int i = 0; i < MAX_VEC; ++i) {
      const int c = tid + T * i;
      if (c < nvec) {
        float f[8];
        unpack8(xv[i], f);
        *reinterpret_cast<uint2*>(qr + 8 * c) = quant8<QK>(f, scale);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// SwiGLU (+ per-token quant, or tensorwise phase A)
// ---------------------------------------------------------------------------
struct SwigluArgs {
  const __nv_bfloat16* gate;   // [M, F] with row stride ld_in
  const __nv_bfloat16* up;     // [M, F] with row stride ld_in
  int64_t ld_in;
  void* q;
  int64_t ld_q;
  float* q_scale;
  __nv_bfloat16* act;          // optional [M, F] bf16 act
  int64_t ld_act;
  float* amax;                 // tensorwise mode
  int64_t M;
  int F;
};

// act = (g * sigmoid(g)) * u, sigmoid(g) = 1 / (1 + e^-g)
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float sig = __frcp_rn(__fadd_rn(1.0f, __expf(-g)));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

template <int T, int MODE>
__global__ void __launch_bounds__(Geo<T>::kBlock) swiglu_kernel(const SwigluArgs a) {
  __shared__ float red[Geo<T>::kRows][Geo<T>::kWarps];
  const int tid = threadIdx.x % T;
  const int rloc = threadIdx.x / T;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * Geo<T>::kRows + rloc;
  const bool active = row < a.M;
  const int nvec = a.F >> 3;
  const int64_t r = active ? row : 0;
  const __nv_bfloat16* gr = a.gate + r * a.ld_in;
  const __nv_bfloat16* ur = a.up + r * a.ld_in;

  uint4 av[MAX_VEC];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAX_VEC; ++i) {
    const int c = tid + T * i;
    if (active && c < nvec) {
      float g[8], u[8], act[8];
      unpack8(ld_nc_v4(gr + 8 * c), g);
      unpack8(ld_nc_v4(ur + 8 * c), u);
#pragma unroll
      for (int j = 0; j < 8; ++j) act[j] = silu_mul(g[j], u[j]);
      if constexpr (MODE == 2) {
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(act[j]));
      }
      av[i] = pack8(act);
      if constexpr (MODE != 2) {
        float ab[8];
        unpack8(av[i], ab);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(ab[j]));
      }
      if (a.act) *reinterpret_cast<uint4*>(a.act + row * a.ld_act + 8 * c) = av[i];
    } else {
      av[i] = make_uint4(0, 0, 0, 0);
    }
  }
  if constexpr (MODE == 2) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
    if ((threadIdx.x & 31) == 0 && amax > 0.f) atomic_max_nonneg(a.amax, amax);
  } else {
    constexpr int QK = MODE;
    amax = row_max<T>(amax, red[rloc]);
    const float scale = scale_from_amax<QK>(amax);
    if (!active) return;
    if (tid == 0) a.q_scale[row] = scale;
    uint8_t* qr = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll
    for (int i = 0; i < MAX_VEC; ++i) {
      const int c = tid + T * i;
      if (c < nvec) {
        float f[8];
        unpack8(av[i], f);
        *reinterpret_cast<uint2*>(qr + 8 * c) = quant8<QK>(f, scale);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// tensorwise phase B: q = cvt(clamp(h / max(amax / qmax, 1e-12))) from the
// device amax (src/ck_fused_mod_norm_quant.py:92-111); also writes the scale.
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
  const float scale = scale_from_amax<QK>(*a.amax);
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.scale_out) *a.scale_out = scale;
  const int nvec = a.D >> 3;
  const int64_t total = a.S * nvec;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = v / nvec;
    const int c = static_cast<int>(v - row * nvec);
    float f[8];
    unpack8(ld_nc_v4(a.h + row * a.ld_h + 8 * c), f);
    *reinterpret_cast<uint2*>(static_cast<uint8_t*>(a.q) + row * a.ld_q + 8 * c) = quant8<QK>(f, scale);
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
