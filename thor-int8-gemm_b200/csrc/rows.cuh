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
// Row-group shape (host rule, restated by the oracle): V = max(3, ceil(nvec/512))
// vectors per thread, T = 32 * ceil(nvec / (32 V)) threads, nvec = D / 8; rows
// are limited by the ring's slot size (96 KB).  Canonical arithmetic, restated
// bit for bit by the CPU oracle:
//   sum of squares: per thread, two FMA accumulators (even / odd element of each
//   bf16 pair) in vector order, combined as even + odd (the squares of bf16 values
//   are exact in fp32); warp butterfly (xor 16, 8, 4, 2, 1); warp partials added
//   left to right;
//   inv = 1 / sqrt(ss / D + eps) with IEEE divide and square root;
//   h = (((x * inv) * w) * s) + b, every product and sum rounded separately;
//   per-token scale = max(amax / qmax, 1e-12) (IEEE divide);
//   q = cvt(RN(v / scale)) (see quant8: the correctly rounded quotient from a
//   reciprocal multiply and one fma correction), round-half-even (int8, which never
//   needs the +-127 clamp: |v / scale| <= 127) or the saturating RNE e4m3
//   conversion (fp8).
#pragma once

#include <cuda_bf16.h>

#include "f32x2.cuh"
#include "ptx.cuh"
#include "sigmoid.cuh"

namespace t8g {
namespace rows {

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

// Round-half-even to an integer through the fp32 adder: for |v| < 2^22 the low byte
// of bits(v + 1.5 * 2^23) is rint(v) as a two's-complement int8.
constexpr float kRoundMagic = 12582912.0f;

// Per-row constants of the quantiser.
struct QuantRow {
  float scale;    // max(amax / qmax, 1e-12)
  float2 rcp;     // RN(1 / scale) (IEEE divide), both lanes
  float2 scale2;  // scale, both lanes
  float2 nrcp;    // -RN(1 / scale), both lanes
};

template <int QK>
__device__ __forceinline__ QuantRow quant_row(float amax) {
  QuantRow r;
  r.scale = fmaxf(__fdiv_rn(amax, QMax<QK>::v), kScaleMin);
  const float rcp = __fdiv_rn(1.0f, r.scale);
  r.rcp = make_float2(rcp, rcp);
  r.scale2 = make_float2(r.scale, r.scale);
  r.nrcp = make_float2(-rcp, -rcp);
  return r;
}

// 8 values (4 pairs) -> 8 quantised bytes, bit-identical to cvt(RN(v / scale)) with an
// IEEE divide, without a divide and without a branch: the quotient is corrected with
// Markstein's step (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with y = RN(1/s) correctly
// rounded and q = RN(v y) within one ulp of v/s, the remainder r = v - s q is exact in
// fp32 (one fma) and q' = RN(q + r y) (one fma) is the correctly rounded v/s.  The
// remainder can be inexact only when it underflows, which needs |v/s| < 2^-12: there
// q' and RN(v/s) both convert to a zero code (int8: |x| < 0.5; e4m3: |x| < 2^-10).
// The remainder is formed negated, n = RN(q s - v), and q' = RN(n (-y) + q), so that an
// exact zero keeps the sign of v (v = -0 gives q' = -0 + -0 = -0, the IEEE quotient; with
// r = RN(v - s q) it would be +0, and e4m3 has a negative zero code).  The 8-bit
// conversion is then the IEEE one (int8: round half to even through the fp32 adder,
// never needing the +-127 clamp since |v/s| <= 127; e4m3: RNE with saturation).
template <int QK>
__device__ __forceinline__ uint2 quant8(const uint4& packed, const QuantRow& qr) {
  const uint32_t w[4] = {packed.x, packed.y, packed.z, packed.w};
  uint32_t c[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 v = bf2_to_f2(w[p]);
    const float2 q = mul2_rn(v, qr.rcp);
    const float2 n = fma2_rn(q, qr.scale2, make_float2(-v.x, -v.y));
    const float2 qq = fma2_rn(n, qr.nrcp, q);
    if constexpr (QK == kQuantInt8) {
      const float2 rq = add2_rn(qq, make_float2(kRoundMagic, kRoundMagic));
      c[p] = __byte_perm(__float_as_uint(rq.x), __float_as_uint(rq.y), 0x0040);
    } else {
      c[p] = cvt_e4m3x2(qq.x, qq.y);
    }
  }
  return make_uint2(__byte_perm(c[0], c[1], 0x5410), __byte_perm(c[2], c[3], 0x5410));
}

__device__ __forceinline__ void unpack_pairs(const uint4& u, float2 (&v)[4]) {
  v[0] = bf2_to_f2(u.x);
  v[1] = bf2_to_f2(u.y);
  v[2] = bf2_to_f2(u.z);
  v[3] = bf2_to_f2(u.w);
}


// ---------------------------------------------------------------- row groups
// A CTA-per-row kernel runs `count` independent row groups of T threads each (a multiple of
// 32); each group has its own ring and synchronises on its own named barrier (1 + index),
// so two rows are in flight per CTA without a CTA-wide barrier (the SwiGLU kernel shares
// one sigmoid table between its groups this way).
struct RowGroup {
  int index;   // group within the CTA
  int count;   // groups per CTA
  int T;       // threads of the group
  int t;       // this thread's index within the group
};

__device__ __forceinline__ RowGroup row_group(int T) {
  RowGroup g;
  g.T = T;
  g.index = static_cast<int>(threadIdx.x) / T;
  g.count = static_cast<int>(blockDim.x) / T;
  g.t = static_cast<int>(threadIdx.x) - g.index * T;
  return g;
}
__device__ __forceinline__ void group_sync(const RowGroup& g) { named_bar_sync(1 + g.index, g.T); }
__device__ __forceinline__ bool group_any(const RowGroup& g, bool v) { return named_bar_any(1 + g.index, g.T, v); }

// ---------------------------------------------------------------- block reductions
// A row group of T threads; `red` holds one float per warp of the group.  Canonical order:
// butterfly within each warp, then the warp partials added (or maxed) left to right.
__device__ __forceinline__ float block_sum(const RowGroup& grp, float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  const int nw = grp.T >> 5;
  if (nw == 1) return v;
  if ((grp.t & 31) == 0) red[grp.t >> 5] = v;
  group_sync(grp);
  float t = red[0];
  for (int i = 1; i < nw; ++i) t = __fadd_rn(t, red[i]);
  return t;
}

// Max over the warp of non-negative, non-NaN floats (running maxima of |x| that start at
// +0), by the integer order of their bit patterns: one redux instead of a five-step
// butterfly of shuffles and compares.
__device__ __forceinline__ float warp_max_nonneg(float v) {
  uint32_t r;
  asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(__float_as_uint(v)));
  return __uint_as_float(r);
}

// Max of non-negative values over the row group (order-free: every lane of every warp
// folds the warp partials with one more butterfly).
__device__ __forceinline__ float block_max(const RowGroup& grp, float v, float* red) {
  v = warp_max_nonneg(v);
  const int nw = grp.T >> 5;
  if (nw == 1) return v;
  const int lane = grp.t & 31;
  if (lane == 0) red[grp.t >> 5] = v;
  group_sync(grp);
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_max_nonneg(t);
  return t;
}

// Non-negative float max via the integer order of its bit pattern.
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

// Folds each thread's running max of its rows into the tensor's amax word with one atomic
// per warp, after the warp's last row (an atomic per row serialises on the single word).
__device__ __forceinline__ void flush_amax(float* amax, float m) {
  m = warp_max_nonneg(m);
  if ((threadIdx.x & 31) == 0 && m > 0.f) atomic_max_nonneg(amax, m);
}

// ---------------------------------------------------------------- row ring
// Shared-memory layout of a row group: mbarriers, reduction scratch, then `stages` slots of
// `slot_bytes` (1024-byte aligned).
struct RingGeom {
  int stages;          // slots in the ring (>= 2)
  uint32_t slot_bytes; // bytes of one slot (one row, or gate row + up row)
  uint32_t part_bytes; // bytes of one operand row
  int parts;           // operand rows per slot (1, or 2 for gate + up)
  int padded;          // rows copied in 256-byte pieces at kPiecePitch (see below)
};
constexpr int kRingHeader = 1024;   // barriers (<= 16 x 8 B), reductions (2 x 32 floats)
constexpr int kMaxStages = 16;

// Padded row layout: the row is copied in 256-byte pieces (128 bf16 values) placed
// kPiecePitch bytes apart, so that reads of the same offset in 16 consecutive pieces (the
// reference-order reduction's leaf-major pass) fall in distinct banks, while reads of
// consecutive 16-byte vectors (every other pass) stay conflict-free.
constexpr uint32_t kPieceBytes = 256;
constexpr uint32_t kPiecePitch = 272;

__host__ __device__ constexpr uint32_t padded_row_bytes(uint32_t row_bytes) {
  return ((row_bytes + kPieceBytes - 1) / kPieceBytes) * kPiecePitch;
}
// Shared-memory byte offset of 16-byte vector c of a padded row.
__device__ __forceinline__ uint32_t padded_vec(int c) {
  return static_cast<uint32_t>(c >> 4) * kPiecePitch + static_cast<uint32_t>(c & 15) * 16u;
}

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
  r.red_max = r.red_sum + 32;
  r.slots = smem + kRingHeader;
  return r;
}

// Issue the copies of one operand row of `bytes` into `dst` (all lanes of one warp; the
// mbarrier's expected bytes are registered separately): one bulk copy from lane 0, or the
// row's 256-byte pieces spread over the lanes in the padded layout.
__device__ __forceinline__ void issue_row_copies(uint8_t* dst, const void* src, uint32_t bytes, bool padded,
                                                 uint64_t* bar, int lane, uint64_t policy) {
  if (!padded) {
    if (lane == 0) bulk_load(dst, src, bytes, bar, policy);
    return;
  }
  const uint32_t pieces = (bytes + kPieceBytes - 1) / kPieceBytes;
  for (uint32_t p = static_cast<uint32_t>(lane); p < pieces; p += 32) {
    const uint32_t off = p * kPieceBytes;
    const uint32_t n = bytes - off < kPieceBytes ? bytes - off : kPieceBytes;
    bulk_load(dst + p * kPiecePitch, static_cast<const uint8_t*>(src) + off, n, bar, policy);
  }
}

// Issue the copies of row `row` into slot `st` (every lane of the group's first warp).
__device__ __forceinline__ void ring_issue(const RingState& rs, const RingGeom& g, int st, const void* src0,
                                           const void* src1, uint64_t policy, int lane) {
  uint8_t* dst = rs.slots + static_cast<size_t>(st) * g.slot_bytes;
  if (lane == 0) mbar_arrive_expect_tx(&rs.full[st], g.part_bytes * static_cast<uint32_t>(g.parts));
  const uint32_t stride = g.padded ? padded_row_bytes(g.part_bytes) : g.part_bytes;
  issue_row_copies(dst, src0, g.part_bytes, g.padded, &rs.full[st], lane, policy);
  if (g.parts == 2) issue_row_copies(dst + stride, src1, g.part_bytes, g.padded, &rs.full[st], lane, policy);
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
// Runs `body(row, slot_ptr, ring)` for the rows of row group `grp`: rows
// blockIdx.x * count + index, then every gridDim.x * count rows, with the ring kept
// `stages - 1` rows ahead.  `src(row, part)` gives the global address of a row operand.
// `smem` is the group's own region (header + slots).  Returns after draining in-flight
// copies.
template <typename Src, typename Body>
__device__ __forceinline__ void row_loop(uint8_t* smem, const RingGeom& g, const RowGroup& grp, int64_t nrows,
                                         Src src, Body body) {
  RingState rs = ring_state(smem);
  const uint64_t policy = policy_evict_first();
  const int64_t G = static_cast<int64_t>(gridDim.x) * grp.count;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * grp.count + grp.index;
  const bool issuer = grp.t < 32;   // the group's first warp issues the copies
  const int lane = grp.t & 31;
  if (grp.t == 0) {
    for (int i = 0; i < g.stages; ++i) mbar_init(&rs.full[i], 1);
    fence_mbarrier_init();
  }
  group_sync(grp);
  int64_t issued = 0;   // meaningful in the first warp only
  if (issuer) {
    for (int i = 0; i < g.stages; ++i) {
      const int64_t r = first + i * G;
      if (r >= nrows) break;
      ring_issue(rs, g, i, src(r, 0), src(r, 1), policy, lane);
      ++issued;
    }
  }
  // slot and phase of row k advance incrementally (no 64-bit division per row)
  int64_t k = 0;
  int st = 0, prev = g.stages - 1;
  uint32_t ph = 0;
  const int64_t ahead = static_cast<int64_t>(g.stages - 1) * G;   // row k-1+stages = row + ahead
  for (int64_t row = first; row < nrows; row += G, ++k) {
    const bool ok = mbar_wait(&rs.full[st], ph, kStatusTimeoutProducer);
    if (group_any(grp, !ok)) break;
    // every thread of the group is past row k-1: refill its slot with row k-1+stages
    if (issuer && k > 0) {
      const int64_t r = row + ahead;
      if (r < nrows) {
        ring_issue(rs, g, prev, src(r, 0), src(r, 1), policy, lane);
        ++issued;
      }
    }
    body(row, rs.slots + static_cast<size_t>(st) * g.slot_bytes, rs);
    prev = st;
    if (++st == g.stages) {
      st = 0;
      ph ^= 1u;
    }
  }
  // teardown: copies still in flight (only after an abort) must land before exit
  if (grp.t == 0) {
    for (int64_t n = k; n < issued; ++n) {
      if (!mbar_wait(&rs.full[st], ph, kStatusTimeoutDrain)) break;
      if (++st == g.stages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }
}

// ---------------------------------------------------------------- shared pieces
// A row group is blockDim.x = T threads; thread t owns the 16-byte vectors
// c = t + T * i of a row.  Kernels are instantiated for V = 3 or 4 vectors per
// thread (fully unrolled, results kept in registers) and V = 0, the generic form
// for longer rows (runtime loop, results staged in the ring slot).

__device__ __forceinline__ uint32_t absmax4(uint32_t m2, const uint4& u) {
  m2 = absmax_bf16x2(m2, u.x);
  m2 = absmax_bf16x2(m2, u.y);
  m2 = absmax_bf16x2(m2, u.z);
  return absmax_bf16x2(m2, u.w);
}

// Generic-proxy writes to a ring slot must be ordered before the bulk copy that
// later refills it.
__device__ __forceinline__ void slot_written() { fence_proxy_async_smem(); }

__device__ __forceinline__ float pair_max(uint32_t m2) { return fmaxf(bf_lo(m2), bf_hi(m2)); }

template <int QK>
__device__ __forceinline__ void store_q(uint8_t* qrow, int c, const uint4& u, const QuantRow& qr) {
  *reinterpret_cast<uint2*>(qrow + 8 * c) = quant8<QK>(u, qr);
}

// ---------------------------------------------------------------- per-token quant
template <int V, int QK>
__global__ void __launch_bounds__(512) quant_rows_kernel(const QuantRowsArgs a, const RingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int T = blockDim.x;
  const RowGroup grp = row_group(T);
  const int nvec = a.D >> 3;
  auto src = [&](int64_t r, int) -> const void* { return a.x + r * a.ld_x; };
  row_loop(smem, g, grp, a.S, src, [&](int64_t row, const uint8_t* slot, const RingState& rs) {
    uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
    uint32_t m2 = 0;
    if constexpr (V > 0) {
      uint4 xv[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + T * i;
        xv[i] = c < nvec ? lds_v4(slot + 16 * c) : make_uint4(0, 0, 0, 0);
        m2 = absmax4(m2, xv[i]);
      }
      const QuantRow qr = quant_row<QK>(block_max(grp, pair_max(m2), rs.red_max));
      if (threadIdx.x == 0) a.q_scale[row] = qr.scale;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + T * i;
        if (c < nvec) store_q<QK>(qrow, c, xv[i], qr);
      }
    } else {
      for (int c = threadIdx.x; c < nvec; c += T) m2 = absmax4(m2, lds_v4(slot + 16 * c));
      const QuantRow qr = quant_row<QK>(block_max(grp, pair_max(m2), rs.red_max));
      if (threadIdx.x == 0) a.q_scale[row] = qr.scale;
      for (int c = threadIdx.x; c < nvec; c += T) store_q<QK>(qrow, c, lds_v4(slot + 16 * c), qr);
    }
  });
}

// ---------------------------------------------------------------- warp rings
// Rows of at most kWarpRowMaxBytes, reduced only with order-free maxima, run one row
// per warp: every warp has its own ring of `stages` slots (bulk copies issued by its
// lane 0, one mbarrier per slot), folds the row max with shuffles and never waits for
// the other warps of its CTA, so a row costs no CTA barrier and its per-row work
// (reduction, scale, reciprocal) is shared by 32 threads rather than a row group.
constexpr uint32_t kWarpRowMaxBytes = 16 * 1024;
constexpr int kWarpMaxWarps = 32;
constexpr int kWarpMaxStages = 8;
constexpr int kWarpRingHeader = kWarpMaxWarps * kWarpMaxStages * 8;   // mbarriers

struct WarpRingGeom {
  int stages;           // slots per warp (2..kWarpMaxStages)
  uint32_t slot_bytes;  // one row (padded layout: its pieces at kPiecePitch) rounded up to 128 bytes
  uint32_t row_bytes;   // bytes of the row
  int64_t cta_rows;     // > 0: CTA b owns rows [b * cta_rows, (b + 1) * cta_rows), its warps
                        // interleaved; 0: rows are dealt round robin over all warps of the grid
  int padded;           // rows copied in 256-byte pieces at kPiecePitch (all lanes issue)
};

// Issue the copies of one row into `slot` (every lane of the warp): lane 0 registers the
// row's bytes on the slot's mbarrier.
__device__ __forceinline__ void warp_ring_issue(uint64_t* bar, uint8_t* slot, const void* src, const WarpRingGeom& g,
                                                int lane, uint64_t policy) {
  if (lane == 0) mbar_arrive_expect_tx(bar, g.row_bytes);
  issue_row_copies(slot, src, g.row_bytes, g.padded != 0, bar, lane, policy);
}

// Runs `body(row, slot)` for the rows of this warp: blockIdx.x * W + warp, then every
// gridDim.x * W rows (W warps per CTA), each warp `stages - 1` rows ahead.
template <typename Src, typename Body>
__device__ __forceinline__ void warp_row_loop(uint8_t* smem, const WarpRingGeom& g, int64_t nrows, Src src,
                                              Body body) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = blockDim.x >> 5;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem) + warp * kWarpMaxStages;
  uint8_t* slots = smem + kWarpRingHeader + static_cast<size_t>(warp) * g.stages * g.slot_bytes;
  const int64_t GW = static_cast<int64_t>(gridDim.x) * W;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * W + warp;
  const uint64_t policy = policy_evict_first();
  if (lane == 0) {
    for (int i = 0; i < g.stages; ++i) mbar_init(&full[i], 1);
    fence_mbarrier_init();
  }
  __syncwarp();
  int64_t issued = 0;   // the same in every lane
  for (int i = 0; i < g.stages; ++i) {
    const int64_t r = first + i * GW;
    if (r >= nrows) break;
    warp_ring_issue(&full[i], slots + static_cast<size_t>(i) * g.slot_bytes, src(r), g, lane, policy);
    ++issued;
  }
  int st = 0;
  uint32_t ph = 0;
  int64_t k = 0;
  const int64_t ahead = static_cast<int64_t>(g.stages) * GW;
  for (int64_t row = first; row < nrows; row += GW, ++k) {
    const bool ok = mbar_wait(&full[st], ph, kStatusTimeoutProducer);
    if (__any_sync(0xFFFFFFFFu, !ok)) break;
    uint8_t* slot = slots + static_cast<size_t>(st) * g.slot_bytes;
    body(row, slot);
    __syncwarp();
    const int64_t r = row + ahead;
    if (r < nrows) {
      fence_proxy_async_smem();   // the warp's reads of the slot precede the copies that refill it
      warp_ring_issue(&full[st], slot, src(r), g, lane, policy);
      ++issued;
    }
    if (++st == g.stages) {
      st = 0;
      ph ^= 1u;
    }
  }
  // teardown: copies still in flight (only after an abort) must land before exit
  if (lane == 0) {
    for (int64_t n = k; n < issued; ++n) {
      if (!mbar_wait(&full[st], ph, kStatusTimeoutDrain)) break;
      if (++st == g.stages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }
  __syncwarp();
}

// Per-token quantisation, one row per warp (rows of at most kWarpRowMaxBytes).
template <int QK>
__global__ void __launch_bounds__(1024) quant_rows_warp_kernel(const QuantRowsArgs a, const WarpRingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int nvec = a.D >> 3;
  auto src = [&](int64_t r) -> const void* { return a.x + r * a.ld_x; };
  warp_row_loop(smem, g, a.S, src, [&](int64_t row, const uint8_t* slot) {
    uint32_t m2 = 0;
#pragma unroll 4
    for (int c = lane; c < nvec; c += 32) m2 = absmax4(m2, lds_v4(slot + 16 * c));
    float m = pair_max(m2);
    m = warp_max_nonneg(m);
    const QuantRow qr = quant_row<QK>(m);
    if (lane == 0) a.q_scale[row] = qr.scale;
    uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll 4
    for (int c = lane; c < nvec; c += 32) store_q<QK>(qrow, c, lds_v4(slot + 16 * c), qr);
  });
}

// ---------------------------------------------------------------- RMSNorm + modulation
// Sum of squares: each thread keeps two fp32 accumulators, one for the even and one
// for the odd element of every bf16 pair, adds its vectors' squares in vector order
// with a packed FMA, then combines them as (even + odd) before the row reduction.
__device__ __forceinline__ float2 row_sumsq_vec(float2 acc, const uint4& u) {
  float2 v[4];
  unpack_pairs(u, v);
#pragma unroll
  for (int p = 0; p < 4; ++p) acc = fma2_rn(v[p], v[p], acc);
  return acc;
}

// h for one vector: (((x * inv) * w) * s) + b; products packed, the add scalar.
__device__ __forceinline__ void rms_h8(const uint4& xu, float2 inv2, const float2 (&s)[4], const float2 (&b)[4],
                                       const __nv_bfloat16* w, int c, float2 (&x)[4], float2 (&h)[4]) {
  unpack_pairs(xu, x);
  float2 prod[4];
  if (w) {
    float2 wv[4];
    unpack_pairs(ld_v4(w + 8 * c), wv);
#pragma unroll
    for (int p = 0; p < 4; ++p) prod[p] = mul2_rn(mul2_rn(mul2_rn(x[p], inv2), wv[p]), s[p]);
  } else {
#pragma unroll
    for (int p = 0; p < 4; ++p) prod[p] = mul2_rn(mul2_rn(x[p], inv2), s[p]);
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) h[p] = make_float2(__fadd_rn(prod[p].x, b[p].x), __fadd_rn(prod[p].y, b[p].y));
}

// Modulation of one vector of mod row `m`: s = scale (or bf16(1 + scale)), b = shift.
__device__ __forceinline__ void load_mod8(const RmsArgs& a, int64_t m, int c, float2 (&s)[4], float2 (&b)[4]) {
  uint4 su = ld_v4(a.scale + m * a.ld_mod + 8 * c);
  if (!a.scale_is_multiplier)
    su = make_uint4(one_plus_bf16x2(su.x), one_plus_bf16x2(su.y), one_plus_bf16x2(su.z), one_plus_bf16x2(su.w));
  unpack_pairs(su, s);
  unpack_pairs(ld_v4(a.shift + m * a.ld_mod + 8 * c), b);
}

// Stores of one vector of h: res = bf16(h + x), h itself; returns bf16(h).
__device__ __forceinline__ uint4 rms_store8(const RmsArgs& a, int64_t row, int c, const float2 (&x)[4],
                                            const float2 (&h)[4]) {
  if (a.res) {
    uint4 ru;
    ru.x = f2_to_bf2(add2_rn(h[0], x[0]));
    ru.y = f2_to_bf2(add2_rn(h[1], x[1]));
    ru.z = f2_to_bf2(add2_rn(h[2], x[2]));
    ru.w = f2_to_bf2(add2_rn(h[3], x[3]));
    *reinterpret_cast<uint4*>(a.res + row * a.ld_res + 8 * c) = ru;
  }
  const uint4 hu = make_uint4(f2_to_bf2(h[0]), f2_to_bf2(h[1]), f2_to_bf2(h[2]), f2_to_bf2(h[3]));
  if (a.h) *reinterpret_cast<uint4*>(a.h + row * a.ld_h + 8 * c) = hu;
  return hu;
}

__device__ __forceinline__ float absmax_f2x4(float m, const float2 (&h)[4]) {
#pragma unroll
  for (int p = 0; p < 4; ++p) m = fmaxf(m, fmaxf(fabsf(h[p].x), fabsf(h[p].y)));
  return m;
}

// RMSNorm + modulation + per-token quantisation, one CTA (row group) per row, for rows
// longer than a warp ring holds.  The modulation vectors are re-read (from L1/L2) for
// every row: caching them in registers across the rows of one batch element raised
// register use enough to cost more occupancy than the loads it saved (measured at D=3072).
template <int V, int QK>
__global__ void __launch_bounds__(512) rms_mod_kernel(const RmsArgs a, const RingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int T = blockDim.x;
  const RowGroup grp = row_group(T);
  const int nvec = a.D >> 3;
  const float fD = static_cast<float>(a.D);
  int64_t cur_m = -1;
  int64_t seg_end = -1;          // first row past the current batch element (rows_per_mod layout)
  auto src = [&](int64_t r, int) -> const void* { return a.x + r * a.ld_x; };
  row_loop(smem, g, grp, a.S, src, [&](int64_t row, uint8_t* slot, const RingState& rs) {
    // pass 1: sum of squares in the canonical order
    float2 acc = make_float2(0.f, 0.f);
    if constexpr (V > 0) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + T * i;
        if (c < nvec) acc = row_sumsq_vec(acc, lds_v4(slot + 16 * c));
      }
    } else {
      for (int c = threadIdx.x; c < nvec; c += T) acc = row_sumsq_vec(acc, lds_v4(slot + 16 * c));
    }
    const float ss = block_sum(grp, __fadd_rn(acc.x, acc.y), rs.red_sum);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, fD), a.eps)));
    const float2 inv2 = make_float2(inv, inv);
    // each CTA visits rows in increasing order: divide only when a batch element ends
    int64_t m;
    if (a.mod_index) {
      m = static_cast<int64_t>(__ldg(a.mod_index + row));
    } else if (row < seg_end) {
      m = cur_m >= 0 ? cur_m : row / a.rows_per_mod;
    } else {
      m = row / a.rows_per_mod;
      seg_end = (m + 1) * a.rows_per_mod;
    }
    uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
    uint32_t m2 = 0;
    cur_m = m;
    if constexpr (V > 0) {
      uint4 hv[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + T * i;
        hv[i] = make_uint4(0, 0, 0, 0);
        if (c < nvec) {
          float2 x[4], h[4], sm[4], bm[4];
          load_mod8(a, m, c, sm, bm);
          rms_h8(lds_v4(slot + 16 * c), inv2, sm, bm, a.w, c, x, h);
          hv[i] = rms_store8(a, row, c, x, h);
          m2 = absmax4(m2, hv[i]);
        }
      }
      const QuantRow qr = quant_row<QK>(block_max(grp, pair_max(m2), rs.red_max));
      if (threadIdx.x == 0) a.q_scale[row] = qr.scale;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + T * i;
        if (c < nvec) store_q<QK>(qrow, c, hv[i], qr);
      }
    } else {
      for (int c = threadIdx.x; c < nvec; c += T) {
        float2 s[4], b[4], x[4], h[4];
        load_mod8(a, m, c, s, b);
        rms_h8(lds_v4(slot + 16 * c), inv2, s, b, a.w, c, x, h);
        const uint4 hu = rms_store8(a, row, c, x, h);
        m2 = absmax4(m2, hu);
        *reinterpret_cast<uint4*>(slot + 16 * c) = hu;   // h replaces x in the slot
      }
      slot_written();
      const QuantRow qr = quant_row<QK>(block_max(grp, pair_max(m2), rs.red_max));   // barrier: h complete
      if (threadIdx.x == 0) a.q_scale[row] = qr.scale;
      for (int c = threadIdx.x; c < nvec; c += T) store_q<QK>(qrow, c, lds_v4(slot + 16 * c), qr);
    }
  });
}

// RMSNorm + modulation + per-token quantisation, one row per warp (rows of at most
// kWarpRowMaxBytes).  The sum of squares is the canonical row-group tree of
// rms_mod_kernel for a group of T threads: lane l plays thread 32 j + l of every warp
// j < T / 32, so each of those warps' accumulation, butterfly and the left-to-right
// sum of their partials are the same operations in the same order.  h (and the
// optional res) is stored per vector, and bf16(h) replaces x in the slot for the
// quantisation pass.
template <int QK>
__global__ void __launch_bounds__(1024) rms_mod_warp_kernel(const RmsArgs a, const WarpRingGeom g, const int T) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int nvec = a.D >> 3;
  const int nw = T >> 5;
  const float fD = static_cast<float>(a.D);
  int64_t cur_m = -1;
  int64_t seg_end = -1;   // first row past the current batch element (rows_per_mod layout)
  auto src = [&](int64_t r) -> const void* { return a.x + r * a.ld_x; };
  warp_row_loop(smem, g, a.S, src, [&](int64_t row, uint8_t* slot) {
    // pass 1: sum of squares, virtual warp by virtual warp
    float ss = 0.f;
    for (int j = 0; j < nw; ++j) {
      float2 acc = make_float2(0.f, 0.f);
      for (int c = 32 * j + lane; c < nvec; c += T) acc = row_sumsq_vec(acc, lds_v4(slot + 16 * c));
      float v = __fadd_rn(acc.x, acc.y);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
      ss = j == 0 ? v : __fadd_rn(ss, v);
    }
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, fD), a.eps)));
    const float2 inv2 = make_float2(inv, inv);
    int64_t m;
    if (a.mod_index) {
      m = static_cast<int64_t>(__ldg(a.mod_index + row));
    } else if (row < seg_end) {
      m = cur_m;
    } else {
      m = row / a.rows_per_mod;
      seg_end = (m + 1) * a.rows_per_mod;
    }
    cur_m = m;
    // pass 2: h, its stores, the row max; bf16(h) back into the slot
    uint32_t m2 = 0;
#pragma unroll 2
    for (int c = lane; c < nvec; c += 32) {
      float2 s[4], b[4], x[4], h[4];
      load_mod8(a, m, c, s, b);
      rms_h8(lds_v4(slot + 16 * c), inv2, s, b, a.w, c, x, h);
      const uint4 hu = rms_store8(a, row, c, x, h);
      m2 = absmax4(m2, hu);
      *reinterpret_cast<uint4*>(slot + 16 * c) = hu;
    }
    float mx = pair_max(m2);
    mx = warp_max_nonneg(mx);
    const QuantRow qr = quant_row<QK>(mx);
    if (lane == 0) a.q_scale[row] = qr.scale;
    uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll 4
    for (int c = lane; c < nvec; c += 32) store_q<QK>(qrow, c, lds_v4(slot + 16 * c), qr);
  });
}

// ---------------------------------------------------------------- register-resident warp rows
// For rows of exactly 32 * NV vectors (D = 256 NV) a warp copies its row from the slot
// into registers (NV vectors per lane, lane l holding vectors 32 k + l) and refills the
// slot at once, so the next `stages` rows are in flight while it computes; all
// indexing is compile-time.
template <int NV>
struct RowRegs {
  uint4 v[NV];
};

template <typename Src, typename Load, typename Compute>
__device__ __forceinline__ void warp_row_loop_reg(uint8_t* smem, const WarpRingGeom& g, int64_t nrows, Src src,
                                                  Load load, Compute compute) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = blockDim.x >> 5;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem) + warp * kWarpMaxStages;
  uint8_t* slots = smem + kWarpRingHeader + static_cast<size_t>(warp) * g.stages * g.slot_bytes;
  int64_t first, GW, end;
  if (g.cta_rows > 0) {
    first = static_cast<int64_t>(blockIdx.x) * g.cta_rows + warp;
    GW = W;
    end = min(nrows, static_cast<int64_t>(blockIdx.x + 1) * g.cta_rows);
  } else {
    first = static_cast<int64_t>(blockIdx.x) * W + warp;
    GW = static_cast<int64_t>(gridDim.x) * W;
    end = nrows;
  }
  const uint64_t policy = policy_evict_first();
  if (lane == 0) {
    for (int i = 0; i < g.stages; ++i) mbar_init(&full[i], 1);
    fence_mbarrier_init();
  }
  __syncwarp();
  int64_t issued = 0;   // the same in every lane
  for (int i = 0; i < g.stages; ++i) {
    const int64_t r = first + i * GW;
    if (r >= end) break;
    warp_ring_issue(&full[i], slots + static_cast<size_t>(i) * g.slot_bytes, src(r), g, lane, policy);
    ++issued;
  }
  int st = 0;
  uint32_t ph = 0;
  int64_t k = 0;
  const int64_t ahead = static_cast<int64_t>(g.stages) * GW;
  for (int64_t row = first; row < end; row += GW, ++k) {
    const bool ok = mbar_wait(&full[st], ph, kStatusTimeoutProducer);
    if (__any_sync(0xFFFFFFFFu, !ok)) break;
    uint8_t* slot = slots + static_cast<size_t>(st) * g.slot_bytes;
    auto regs = load(slot, row);
    __syncwarp();
    {
      const int64_t r = row + ahead;
      if (r < end) {
        fence_proxy_async_smem();   // the warp's reads of the slot precede the copies that refill it
        warp_ring_issue(&full[st], slot, src(r), g, lane, policy);
        ++issued;
      }
    }
    if (++st == g.stages) {
      st = 0;
      ph ^= 1u;
    }
    compute(row, regs);
  }
  if (lane == 0) {
    for (int64_t n = k; n < issued; ++n) {
      if (!mbar_wait(&full[st], ph, kStatusTimeoutDrain)) break;
      if (++st == g.stages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }
  __syncwarp();
}

template <int NV>
__device__ __forceinline__ RowRegs<NV> load_row_regs(const uint8_t* slot, int lane) {
  RowRegs<NV> r;
#pragma unroll
  for (int k = 0; k < NV; ++k) r.v[k] = lds_v4(slot + 16 * (32 * k + lane));
  return r;
}

// Per-token quantisation, one row of 256 NV elements per warp held in registers (the
// slot refills as soon as the row is loaded).
template <int NV, int QK>
__global__ void __launch_bounds__(512, 1) quant_rows_warp_reg_kernel(const QuantRowsArgs a, const WarpRingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  auto src = [&](int64_t r) -> const void* { return a.x + r * a.ld_x; };
  warp_row_loop_reg(
      smem, g, a.S, src, [&](const uint8_t* slot, int64_t) { return load_row_regs<NV>(slot, lane); },
      [&](int64_t row, const RowRegs<NV>& r) {
        uint32_t m2 = 0;
#pragma unroll
        for (int k = 0; k < NV; ++k) m2 = absmax4(m2, r.v[k]);
        float m = pair_max(m2);
        m = warp_max_nonneg(m);
        const QuantRow qr = quant_row<QK>(m);
        if (lane == 0) a.q_scale[row] = qr.scale;
        uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll
        for (int k = 0; k < NV; ++k) store_q<QK>(qrow, 32 * k + lane, r.v[k], qr);
      });
}

// Mixed-precision helpers: bf16 operands taken straight from the packed pair (no
// unpacking), one rounding each.
// acc.x += lo(u)^2, acc.y += hi(u)^2 (the squares of bf16 values are exact in fp32, so
// this is the packed FMA of the canonical sum of squares).
__device__ __forceinline__ float2 sumsq_bf16x2(float2 acc, uint32_t u) {
  float x, y;
  asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; fma.rn.f32.bf16 %0, lo, lo, %3; fma.rn.f32.bf16 %1, hi, hi, %4; }"
      : "=f"(x), "=f"(y)
      : "r"(u), "f"(acc.x), "f"(acc.y));
  return make_float2(x, y);
}

// The row-group size of the canonical sum for a row of `nvec` vectors (the host rule).
__host__ __device__ constexpr int row_group_threads(int nvec) {
  return 32 * ((nvec + 32 * ((nvec + 511) / 512 < 3 ? 3 : (nvec + 511) / 512) - 1) /
               (32 * ((nvec + 511) / 512 < 3 ? 3 : (nvec + 511) / 512)));
}

// ((p0 + p1) + p2) + ... of NW per-lane partials, each first summed over the warp by the
// canonical butterfly (v + v[lane ^ 16], then ^ 8, 4, 2, 1).  For NW = 2 and 4 the butterflies
// are run as a reduce-scatter: at the xor-16 level (and for NW = 4 the xor-8 level) a lane
// keeps half of the partials and trades the other half with its partner, so every addition
// pairs the same two values as the butterfly (each sum is commutative) with 10 shuffles
// instead of 20 (NW = 4); lane 0 then sums the totals left to right and broadcasts.
template <int NW>
__device__ __forceinline__ float warp_parts_sum(const float (&part)[NW]) {
  const int lane = threadIdx.x & 31;
  if constexpr (NW == 2) {
    const bool hi = lane & 16;
    const float keep = hi ? part[1] : part[0];
    const float give = hi ? part[0] : part[1];
    float m = __fadd_rn(keep, __shfl_xor_sync(0xFFFFFFFFu, give, 16));
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) m = __fadd_rn(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    const float ss = __fadd_rn(m, __shfl_xor_sync(0xFFFFFFFFu, m, 16));   // lane 0: p0 + p1
    return __shfl_sync(0xFFFFFFFFu, ss, 0);
  } else if constexpr (NW == 4) {
    const bool b4 = lane & 16, b3 = lane & 8;
    // xor 16: keep parts 2 b4, 2 b4 + 1
    const float k0 = __fadd_rn(b4 ? part[2] : part[0], __shfl_xor_sync(0xFFFFFFFFu, b4 ? part[0] : part[2], 16));
    const float k1 = __fadd_rn(b4 ? part[3] : part[1], __shfl_xor_sync(0xFFFFFFFFu, b4 ? part[1] : part[3], 16));
    // xor 8: keep part 2 b4 + b3
    float m = __fadd_rn(b3 ? k1 : k0, __shfl_xor_sync(0xFFFFFFFFu, b3 ? k0 : k1, 8));
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) m = __fadd_rn(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    // lane 0 holds p0; lanes 8, 16, 24 hold p1, p2, p3
    const float p1 = __shfl_xor_sync(0xFFFFFFFFu, m, 8);
    const float p2 = __shfl_xor_sync(0xFFFFFFFFu, m, 16);
    const float p3 = __shfl_xor_sync(0xFFFFFFFFu, m, 24);
    const float ss = __fadd_rn(__fadd_rn(__fadd_rn(m, p1), p2), p3);
    return __shfl_sync(0xFFFFFFFFu, ss, 0);
  } else {
    float v[NW];
#pragma unroll
    for (int j = 0; j < NW; ++j) v[j] = part[j];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
      for (int j = 0; j < NW; ++j) v[j] = __fadd_rn(v[j], __shfl_xor_sync(0xFFFFFFFFu, v[j], off));
    }
    float ss = v[0];
#pragma unroll
    for (int j = 1; j < NW; ++j) ss = __fadd_rn(ss, v[j]);
    return ss;
  }
}

// 1 / sqrt(mean(x^2) + eps) of a register-resident row of 256 NV elements, the sum of
// squares in the canonical tree of a row group of T = row_group_threads threads: lane
// l's vector 32 k + l belongs to group warp k mod (T / 32), in ascending k, exactly as
// thread 32 (k mod (T/32)) + l visits it.
template <int NV>
__device__ __forceinline__ float row_inv_reg(const RowRegs<NV>& r, float eps) {
  constexpr int NVEC = 32 * NV;
  constexpr int NW = row_group_threads(NVEC) / 32;
  static_assert(NW >= 1 && NW <= NV, "row group shape");
  float2 acc[NW];
#pragma unroll
  for (int j = 0; j < NW; ++j) acc[j] = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    float2 t = acc[k % NW];
    t = sumsq_bf16x2(t, r.v[k].x);
    t = sumsq_bf16x2(t, r.v[k].y);
    t = sumsq_bf16x2(t, r.v[k].z);
    t = sumsq_bf16x2(t, r.v[k].w);
    acc[k % NW] = t;
  }
  float part[NW];
#pragma unroll
  for (int j = 0; j < NW; ++j) part[j] = __fadd_rn(acc[j].x, acc[j].y);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(warp_parts_sum<NW>(part), static_cast<float>(8 * NVEC)), eps)));
}

// max(m, |a|, |b|) in one three-input max.
__device__ __forceinline__ float max3_abs(float m, float a, float b) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return d;
}

// h for one vector from x, inv, the fp32 multiplier pairs s and the packed bf16 shift:
// h = RN(RN(RN(x * inv) * s) + b); returns bf16(h) and folds |h| into amax.
__device__ __forceinline__ uint4 rms_h_simple8(const uint4& xu, float2 inv2, const float2 (&s)[4], const uint4& bu,
                                               float& amax) {
  const uint32_t xw[4] = {xu.x, xu.y, xu.z, xu.w};
  const uint32_t bw[4] = {bu.x, bu.y, bu.z, bu.w};
  uint32_t hw[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 h = add_f32_bf16x2(mul2_rn(mul2_rn(bf2_to_f2(xw[p]), inv2), s[p]), bw[p]);
    amax = max3_abs(amax, h.x, h.y);
    hw[p] = f2_to_bf2(h);
  }
  return make_uint4(hw[0], hw[1], hw[2], hw[3]);
}

// One vector of the h pass of rms_mod_simple_kernel for a row whose batch element is
// not the CTA's cached one: modulation read from global memory.  Out of line (rare), with
// everything passed by value so that the row stays in registers.
__device__ __noinline__ uint4 rms_h_simple_global8(const __nv_bfloat16* srow, const __nv_bfloat16* brow, int c, uint4 xu,
                                                   float inv, float* amax) {
  const uint4 su = ld_v4(srow + 8 * c);
  float2 sf[4];
  unpack_pairs(make_uint4(one_plus_bf16x2(su.x), one_plus_bf16x2(su.y), one_plus_bf16x2(su.z), one_plus_bf16x2(su.w)),
               sf);
  float m = *amax;
  const uint4 hu = rms_h_simple8(xu, make_float2(inv, inv), sf, ld_v4(brow + 8 * c), m);
  *amax = m;
  return hu;
}

// RMSNorm + adaLN modulation + per-token quantisation in the DiT form (no norm weight, no h
// or res outputs, s = bf16(1 + scale), batch-major tokens with rows_per_mod tokens per
// batch element) for rows of 256 NV elements held in registers.  Each CTA owns a
// contiguous block of rows and keeps the modulation of the batch element holding the
// block's middle row in shared memory (s as fp32, the shift as bf16); rows of another
// batch element (a block straddling a boundary) read theirs from global memory.
template <int NV, int QK>
__global__ void __launch_bounds__(512, 1) rms_mod_simple_kernel(const RmsArgs a, const WarpRingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NVEC = 32 * NV;
  const int lane = threadIdx.x & 31;
  const int W = blockDim.x >> 5;
  // cache: s of elements 8c..8c+3 at cache_lo[c], 8c+4..8c+7 at cache_hi[c] (lane-contiguous
  // 16-byte reads), then the bf16 shift
  float4* cache_lo = reinterpret_cast<float4*>(smem + kWarpRingHeader + static_cast<size_t>(W) * g.stages * g.slot_bytes);
  float4* cache_hi = cache_lo + NVEC;
  uint4* cache_b = reinterpret_cast<uint4*>(cache_hi + NVEC);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * g.cta_rows;
  const int64_t r1 = min(a.S, r0 + g.cta_rows);
  const int64_t cm = r0 < r1 ? ((r0 + r1 - 1) >> 1) / a.rows_per_mod : -1;
  if (cm >= 0) {
    for (int c = threadIdx.x; c < NVEC; c += blockDim.x) {
      const uint4 su = ld_v4(a.scale + cm * a.ld_mod + 8 * c);
      float2 sf[4];
      unpack_pairs(
          make_uint4(one_plus_bf16x2(su.x), one_plus_bf16x2(su.y), one_plus_bf16x2(su.z), one_plus_bf16x2(su.w)), sf);
      cache_lo[c] = make_float4(sf[0].x, sf[0].y, sf[1].x, sf[1].y);
      cache_hi[c] = make_float4(sf[2].x, sf[2].y, sf[3].x, sf[3].y);
      cache_b[c] = ld_v4(a.shift + cm * a.ld_mod + 8 * c);
    }
  }
  __syncthreads();
  int64_t cur_m = -1;
  int64_t seg_end = -1;
  auto src = [&](int64_t r) -> const void* { return a.x + r * a.ld_x; };
  warp_row_loop_reg(
      smem, g, a.S, src, [&](const uint8_t* slot, int64_t) { return load_row_regs<NV>(slot, lane); },
      [&](int64_t row, RowRegs<NV>& r) {
        const float inv = row_inv_reg<NV>(r, a.eps);
        int64_t m;
        if (row < seg_end) {
          m = cur_m;
        } else {
          m = row / a.rows_per_mod;
          seg_end = (m + 1) * a.rows_per_mod;
        }
        cur_m = m;
        float amax = 0.f;
        if (m == cm) {
          const float2 inv2 = make_float2(inv, inv);
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int c = 32 * k + lane;
            const float4 s0 = cache_lo[c];
            const float4 s1 = cache_hi[c];
            const float2 sf[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w), make_float2(s1.x, s1.y),
                                  make_float2(s1.z, s1.w)};
            r.v[k] = rms_h_simple8(r.v[k], inv2, sf, cache_b[c], amax);
          }
        } else {
          const __nv_bfloat16* srow = a.scale + m * a.ld_mod;
          const __nv_bfloat16* brow = a.shift + m * a.ld_mod;
#pragma unroll
          for (int k = 0; k < NV; ++k) r.v[k] = rms_h_simple_global8(srow, brow, 32 * k + lane, r.v[k], inv, &amax);
        }
        amax = warp_max_nonneg(amax);
        // max |bf16(h)| = bf16(max |h|): rounding is monotone and symmetric
        const QuantRow qr = quant_row<QK>(__bfloat162float(__float2bfloat16_rn(amax)));
        if (lane == 0) a.q_scale[row] = qr.scale;
        uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll
        for (int k = 0; k < NV; ++k) store_q<QK>(qrow, 32 * k + lane, r.v[k], qr);
      });
}

// ---------------------------------------------------------------- tensorwise (reference) norm
// The reference's fused_rms_mod_quant and its per-segment driver (src/ck_fused_mod_norm_quant.py:
// 23-55, src/ck_fused_patch.py:105-136) derive one scale for the whole tensor from the
// float32 max of |h|, so h must be the reference's to the last bit: these kernels sum the
// squares in the reference's own order.  Its kernel accumulates x^2 into a 2048-lane float32
// vector chunk by chunk (lane i += x[2048 c + i]^2; BLOCK_K = 2048 in both callers) and
// reduces the vector with tl.sum, which Triton evaluates (CPU interpreter: numpy's pairwise
// summation) as a balanced binary tree over 16 leaves of 128 lanes, each leaf summed by 8
// interleaved accumulators r_j (lanes 8 t + j, t = 0..15, in order) and combined as
// ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)).
//
// One warp computes it from a row in the padded layout: lane 2 b + e owns leaf b's
// accumulators 4 e .. 4 e + 3 and folds their chunks in order with a mixed-precision fma
// (x^2 of a bf16 value is exact, so fma(x, x, acc) = RN(acc + x^2)); the eight accumulators
// of a leaf combine as above (the two halves across the lane pair), and the leaves by a
// butterfly (xor 2, 4, 8, 16), which is the pairwise tree.  At a given (t, chunk) the 32
// lanes read 8 bytes at the same offset of 16 consecutive pieces: with the 272-byte piece
// pitch each half-warp covers all 32 banks once.
constexpr int kRefBlock = 2048;

// NCH > 0: the row's chunk count as a compile-time constant (loops unrolled); 0: D / 2048
// rounded up, at run time.
template <int NCH = 0>
__device__ __forceinline__ float ref_sumsq_warp(const uint8_t* row, int D, int lane) {
  const int b = lane >> 1;
  const int e = lane & 1;
  const int nch = NCH > 0 ? NCH : (D + kRefBlock - 1) / kRefBlock;
  float2 r01 = make_float2(0.f, 0.f), r23 = make_float2(0.f, 0.f);
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    float2 e01 = make_float2(0.f, 0.f), e23 = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < nch; ++c) {
      const int el = c * kRefBlock + b * 128 + t * 8 + e * 4;   // this lane's 4 elements (all in or all out)
      if (el < D) {
        const uint2 v = *reinterpret_cast<const uint2*>(row + (el >> 7) * kPiecePitch + (el & 127) * 2);
        e01 = sumsq_bf16x2(e01, v.x);
        e23 = sumsq_bf16x2(e23, v.y);
      }
    }
    if (t == 0) {
      r01 = e01;
      r23 = e23;
    } else {
      r01 = make_float2(__fadd_rn(r01.x, e01.x), __fadd_rn(r01.y, e01.y));
      r23 = make_float2(__fadd_rn(r23.x, e23.x), __fadd_rn(r23.y, e23.y));
    }
  }
  float v = __fadd_rn(__fadd_rn(r01.x, r01.y), __fadd_rn(r23.x, r23.y));
#pragma unroll
  for (int off = 1; off <= 16; off <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  return v;
}

__device__ __forceinline__ float rms_inv_of(float ss, float D, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, D), eps)));
}

// The modulation row of `row` (mod_index, or batch-major rows_per_mod with the division done
// only when a batch element ends; rows are visited in increasing order).
__device__ __forceinline__ int64_t mod_row_of(const RmsArgs& a, int64_t row, int64_t& cur_m, int64_t& seg_end) {
  if (a.mod_index) return static_cast<int64_t>(__ldg(a.mod_index + row));
  if (row >= seg_end || cur_m < 0) {
    cur_m = row / a.rows_per_mod;
    seg_end = (cur_m + 1) * a.rows_per_mod;
  }
  return cur_m;
}

// Phase A of the tensorwise norm, one row per warp (rows of at most kWarpRowMaxBytes, padded
// layout, NCH = the row's 2048-element chunks): h and res stored, each lane's running max of
// the float32 |h|, folded into the tensor's amax word at the end.
template <int NCH>
__global__ void __launch_bounds__(1024) rms_mod_tw_warp_kernel(const RmsArgs a, const WarpRingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int nvec = a.D >> 3;
  const float fD = static_cast<float>(a.D);
  int64_t cur_m = -1, seg_end = -1;
  float tw_max = 0.f;
  auto src = [&](int64_t r) -> const void* { return a.x + r * a.ld_x; };
  warp_row_loop(smem, g, a.S, src, [&](int64_t row, uint8_t* slot) {
    const float inv = rms_inv_of(ref_sumsq_warp<NCH>(slot, a.D, lane), fD, a.eps);
    const float2 inv2 = make_float2(inv, inv);
    const int64_t m = mod_row_of(a, row, cur_m, seg_end);
#pragma unroll 2
    for (int c = lane; c < nvec; c += 32) {
      float2 s[4], b[4], x[4], h[4];
      load_mod8(a, m, c, s, b);
      rms_h8(lds_v4(slot + padded_vec(c)), inv2, s, b, a.w, c, x, h);
      tw_max = absmax_f2x4(tw_max, h);
      rms_store8(a, row, c, x, h);
    }
  });
  flush_amax(a.amax, tw_max);
}

// A register-resident row and its sum of squares in the reference's order.
template <int NV>
struct RowRegsSS {
  uint4 v[NV];
  float ss;
};

// h and res of one vector from x, inv, the norm weight (HAS_W), the fp32 multiplier pairs s
// and the packed bf16 shift: h = RN(RN(RN(RN(x * inv) * w) * s) + b), the product with w left
// out without a weight (the order of rms_h8), res = bf16(h + x) when asked; folds the float32
// |h| into amax.
template <bool HAS_W>
__device__ __forceinline__ uint4 rms_h_res8(const uint4& xu, float2 inv2, const uint4& wu, const float2 (&s)[4],
                                            const uint4& bu, float& amax, bool want_res, uint4& res) {
  const uint32_t xw[4] = {xu.x, xu.y, xu.z, xu.w};
  const uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
  const uint32_t bw[4] = {bu.x, bu.y, bu.z, bu.w};
  uint32_t hw[4], rw[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 x = bf2_to_f2(xw[p]);
    float2 t = mul2_rn(x, inv2);
    if constexpr (HAS_W) t = mul2_rn(t, bf2_to_f2(ww[p]));
    const float2 h = add_f32_bf16x2(mul2_rn(t, s[p]), bw[p]);
    amax = max3_abs(amax, h.x, h.y);
    hw[p] = f2_to_bf2(h);
    if (want_res) rw[p] = f2_to_bf2(add2_rn(h, x));
  }
  if (want_res) res = make_uint4(rw[0], rw[1], rw[2], rw[3]);
  return make_uint4(hw[0], hw[1], hw[2], hw[3]);
}

// Shared memory after the warp rings of the cached norm kernels: the multiplier s of the cached
// modulation row as fp32 (elements 8c..8c+3 at [c], 8c+4..8c+7 at [NVEC + c], lane-contiguous
// 16-byte reads), its shift as bf16 ([2 NVEC + c]) and, with a weight, the norm weight as bf16
// ([3 NVEC + c]): 6 D bytes, 8 D with a weight.
template <int NV>
__device__ __forceinline__ float4* mod_cache_of(uint8_t* smem, const WarpRingGeom& g) {
  return reinterpret_cast<float4*>(smem + kWarpRingHeader +
                                   static_cast<size_t>(blockDim.x >> 5) * g.stages * g.slot_bytes);
}

// Fills the CTA's modulation cache (and norm weight) for the modulation row of its block's
// middle row; returns that row, -1 for an empty block.  The caller synchronises the CTA.
template <int NV, bool HAS_W>
__device__ __forceinline__ int64_t fill_mod_cache(const RmsArgs& a, const WarpRingGeom& g, float4* cache) {
  constexpr int NVEC = 32 * NV;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * g.cta_rows;
  const int64_t r1 = min(a.S, r0 + g.cta_rows);
  if (r0 >= r1) return -1;
  const int64_t mid = (r0 + r1 - 1) >> 1;
  const int64_t cm = a.mod_index ? static_cast<int64_t>(__ldg(a.mod_index + mid)) : mid / a.rows_per_mod;
  uint4* cache_b = reinterpret_cast<uint4*>(cache + 2 * NVEC);
  for (int c = threadIdx.x; c < NVEC; c += blockDim.x) {
    uint4 su = ld_v4(a.scale + cm * a.ld_mod + 8 * c);
    if (!a.scale_is_multiplier)
      su = make_uint4(one_plus_bf16x2(su.x), one_plus_bf16x2(su.y), one_plus_bf16x2(su.z), one_plus_bf16x2(su.w));
    float2 sf[4];
    unpack_pairs(su, sf);
    cache[c] = make_float4(sf[0].x, sf[0].y, sf[1].x, sf[1].y);
    cache[NVEC + c] = make_float4(sf[2].x, sf[2].y, sf[3].x, sf[3].y);
    cache_b[c] = ld_v4(a.shift + cm * a.ld_mod + 8 * c);
    if constexpr (HAS_W) cache_b[NVEC + c] = ld_v4(a.w + 8 * c);
  }
  return cm;
}

// s (fp32 pairs) and the packed shift of vector c of modulation row m: from the cache when m is
// the cached row, else from global memory.
template <int NV>
__device__ __forceinline__ void mod_of(const RmsArgs& a, const float4* cache, bool cached, int64_t m, int c,
                                       float2 (&sf)[4], uint4& bu) {
  constexpr int NVEC = 32 * NV;
  if (cached) {
    const float4 s0 = cache[c];
    const float4 s1 = cache[NVEC + c];
    sf[0] = make_float2(s0.x, s0.y);
    sf[1] = make_float2(s0.z, s0.w);
    sf[2] = make_float2(s1.x, s1.y);
    sf[3] = make_float2(s1.z, s1.w);
    bu = reinterpret_cast<const uint4*>(cache + 2 * NVEC)[c];
  } else {
    uint4 su = ld_v4(a.scale + m * a.ld_mod + 8 * c);
    if (!a.scale_is_multiplier)
      su = make_uint4(one_plus_bf16x2(su.x), one_plus_bf16x2(su.y), one_plus_bf16x2(su.z), one_plus_bf16x2(su.w));
    unpack_pairs(su, sf);
    bu = ld_v4(a.shift + m * a.ld_mod + 8 * c);
  }
}

// h (and res, when asked) of vector c of a row whose modulation row m is not the CTA's cached
// one: the modulation read from global memory.  Out of line (rare), with the row's vector passed
// by value, so that the caller's row stays in registers; stores h / res when their rows are
// given and folds |h| into *amax.
template <bool HAS_W>
__device__ __noinline__ uint4 rms_h_res_global8(const __nv_bfloat16* srow, const __nv_bfloat16* brow, int multiplier,
                                                int c, uint4 xu, float inv, uint4 wu, float* amax,
                                                __nv_bfloat16* rrow, __nv_bfloat16* hrow) {
  uint4 su = ld_v4(srow + 8 * c);
  if (!multiplier)
    su = make_uint4(one_plus_bf16x2(su.x), one_plus_bf16x2(su.y), one_plus_bf16x2(su.z), one_plus_bf16x2(su.w));
  float2 sf[4];
  unpack_pairs(su, sf);
  const uint4 bu = ld_v4(brow + 8 * c);
  float mx = *amax;
  uint4 ru;
  const uint4 hu = rms_h_res8<HAS_W>(xu, make_float2(inv, inv), wu, sf, bu, mx, rrow != nullptr, ru);
  *amax = mx;
  if (rrow) *reinterpret_cast<uint4*>(rrow + 8 * c) = ru;
  if (hrow) *reinterpret_cast<uint4*>(hrow + 8 * c) = hu;
  return hu;
}

// The cached norm weight's vector c.
template <int NV>
__device__ __forceinline__ uint4 weight_of(const float4* cache, int c) {
  return reinterpret_cast<const uint4*>(cache + 2 * 32 * NV)[32 * NV + c];
}

// Phase A of the tensorwise norm for rows of 256 NV elements (every option of the entry
// point: norm weight when HAS_W, mod_index or batch-major rows_per_mod, scale as multiplier or
// s = bf16(1 + scale), res when asked): the warp sums the squares in the reference's order from
// the padded slot, copies the row into registers (lane l holding vectors 32 k + l) and refills
// the slot at once, then computes h from the registers.  Each CTA owns a contiguous block of
// rows and keeps in shared memory the modulation of the block's middle row (s as fp32, the
// shift as bf16) and the norm weight; rows with another modulation row read theirs from
// global memory.
template <int NV, bool HAS_W>
__global__ void __launch_bounds__(512, 1) rms_mod_tw_cached_kernel(const RmsArgs a, const WarpRingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int D = 256 * NV;
  constexpr int NCH = (D + kRefBlock - 1) / kRefBlock;
  const int lane = threadIdx.x & 31;
  float4* cache = mod_cache_of<NV>(smem, g);
  const int64_t cm = fill_mod_cache<NV, HAS_W>(a, g, cache);
  __syncthreads();
  int64_t cur_m = -1, seg_end = -1;
  float tw_max = 0.f;
  auto src = [&](int64_t r) -> const void* { return a.x + r * a.ld_x; };
  warp_row_loop_reg(
      smem, g, a.S, src,
      [&](const uint8_t* slot, int64_t) {
        RowRegsSS<NV> r;
        r.ss = ref_sumsq_warp<NCH>(slot, D, lane);
#pragma unroll
        for (int k = 0; k < NV; ++k) r.v[k] = lds_v4(slot + padded_vec(32 * k + lane));
        return r;
      },
      [&](int64_t row, RowRegsSS<NV>& r) {
        const float inv = rms_inv_of(r.ss, static_cast<float>(D), a.eps);
        const float2 inv2 = make_float2(inv, inv);
        const int64_t m = mod_row_of(a, row, cur_m, seg_end);
        __nv_bfloat16* hrow = a.h + row * a.ld_h;
        __nv_bfloat16* rrow = a.res ? a.res + row * a.ld_res : nullptr;
        // (the per-vector cached / global choice measured faster here than one branch per row
        // with an out-of-line global path, which the per-token kernel below uses)
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int c = 32 * k + lane;
          float2 sf[4];
          uint4 bu;
          mod_of<NV>(a, cache, m == cm, m, c, sf, bu);
          uint4 wu = make_uint4(0, 0, 0, 0);
          if constexpr (HAS_W) wu = weight_of<NV>(cache, c);
          uint4 ru;
          const uint4 hu = rms_h_res8<HAS_W>(r.v[k], inv2, wu, sf, bu, tw_max, rrow != nullptr, ru);
          if (rrow) *reinterpret_cast<uint4*>(rrow + 8 * c) = ru;
          *reinterpret_cast<uint4*>(hrow + 8 * c) = hu;
        }
      });
  flush_amax(a.amax, tw_max);
}

// RMSNorm + modulation + per-token quantisation with every option of the entry point (norm
// weight when HAS_W, mod_index or batch-major rows_per_mod, scale as multiplier, h / res
// outputs) for rows of 256 NV elements held in registers: the canonical sum of squares
// (row_inv_reg), the CTA's cached modulation row and norm weight (fill_mod_cache), and the
// quantiser of rms_mod_simple_kernel.
template <int NV, int QK, bool HAS_W>
__global__ void __launch_bounds__(512, 1) rms_mod_cached_kernel(const RmsArgs a, const WarpRingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  float4* cache = mod_cache_of<NV>(smem, g);
  const int64_t cm = fill_mod_cache<NV, HAS_W>(a, g, cache);
  __syncthreads();
  int64_t cur_m = -1, seg_end = -1;
  auto src = [&](int64_t r) -> const void* { return a.x + r * a.ld_x; };
  warp_row_loop_reg(
      smem, g, a.S, src, [&](const uint8_t* slot, int64_t) { return load_row_regs<NV>(slot, lane); },
      [&](int64_t row, RowRegs<NV>& r) {
        const int64_t m = mod_row_of(a, row, cur_m, seg_end);   // issued before the sum, which hides its latency
        const float inv = row_inv_reg<NV>(r, a.eps);
        const float2 inv2 = make_float2(inv, inv);
        __nv_bfloat16* hrow = a.h ? a.h + row * a.ld_h : nullptr;
        __nv_bfloat16* rrow = a.res ? a.res + row * a.ld_res : nullptr;
        float amax = 0.f;
        if (m == cm) {
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int c = 32 * k + lane;
            float2 sf[4];
            uint4 bu;
            mod_of<NV>(a, cache, true, m, c, sf, bu);
            uint4 wu = make_uint4(0, 0, 0, 0);
            if constexpr (HAS_W) wu = weight_of<NV>(cache, c);
            uint4 ru;
            const uint4 hu = rms_h_res8<HAS_W>(r.v[k], inv2, wu, sf, bu, amax, rrow != nullptr, ru);
            if (rrow) *reinterpret_cast<uint4*>(rrow + 8 * c) = ru;
            if (hrow) *reinterpret_cast<uint4*>(hrow + 8 * c) = hu;
            r.v[k] = hu;
          }
        } else {
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int c = 32 * k + lane;
            uint4 wu = make_uint4(0, 0, 0, 0);
            if constexpr (HAS_W) wu = weight_of<NV>(cache, c);
            r.v[k] = rms_h_res_global8<HAS_W>(a.scale + m * a.ld_mod, a.shift + m * a.ld_mod, a.scale_is_multiplier,
                                              c, r.v[k], inv, wu, &amax, rrow, hrow);
          }
        }
        amax = warp_max_nonneg(amax);
        // max |bf16(h)| = bf16(max |h|): rounding is monotone and symmetric
        const QuantRow qr = quant_row<QK>(__bfloat162float(__float2bfloat16_rn(amax)));
        if (lane == 0) a.q_scale[row] = qr.scale;
        uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
#pragma unroll
        for (int k = 0; k < NV; ++k) store_q<QK>(qrow, 32 * k + lane, r.v[k], qr);
      });
}

// The same for longer rows, one CTA (row group of T threads) per row: its first warp sums
// the squares in the reference's order while the others wait, then every thread takes the
// vectors t, t + T, ... of the h pass.
__global__ void __launch_bounds__(512) rms_mod_tw_cta_kernel(const RmsArgs a, const RingGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int T = blockDim.x;
  const RowGroup grp = row_group(T);
  const int nvec = a.D >> 3;
  const float fD = static_cast<float>(a.D);
  int64_t cur_m = -1, seg_end = -1;
  float tw_max = 0.f;
  auto src = [&](int64_t r, int) -> const void* { return a.x + r * a.ld_x; };
  row_loop(smem, g, grp, a.S, src, [&](int64_t row, uint8_t* slot, const RingState& rs) {
    if (grp.t < 32) {
      const float ss = ref_sumsq_warp(slot, a.D, grp.t);
      if (grp.t == 0) rs.red_sum[0] = ss;
    }
    group_sync(grp);
    const float inv = rms_inv_of(rs.red_sum[0], fD, a.eps);
    const float2 inv2 = make_float2(inv, inv);
    const int64_t m = mod_row_of(a, row, cur_m, seg_end);
    for (int c = grp.t; c < nvec; c += T) {
      float2 s[4], b[4], x[4], h[4];
      load_mod8(a, m, c, s, b);
      rms_h8(lds_v4(slot + padded_vec(c)), inv2, s, b, a.w, c, x, h);
      tw_max = absmax_f2x4(tw_max, h);
      rms_store8(a, row, c, x, h);
    }
    // rs.red_sum[0] is rewritten only after the next row's group barrier in row_loop
  });
  flush_amax(a.amax, tw_max);
}

// ---------------------------------------------------------------- SwiGLU
// act for one vector from the gate and up rows in the slot (sigmoid table `sig` in shared
// memory, its shared-memory address); returns bf16(act) and folds the float32 |act| into
// amax32 when asked.
__device__ __forceinline__ uint4 swiglu8(const uint8_t* gate, const uint8_t* up, int c, uint32_t sig,
                                         float& amax32, bool tensorwise) {
  float2 uv[4], act[4];
  const uint4 gu = lds_v4(gate + 16 * c);
  const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
  unpack_pairs(lds_v4(up + 16 * c), uv);
#pragma unroll
  for (int p = 0; p < 4; ++p) act[p] = silu_mul2(gw[p], uv[p], sig);
  if (tensorwise) amax32 = absmax_f2x4(amax32, act);
  return make_uint4(f2_to_bf2(act[0]), f2_to_bf2(act[1]), f2_to_bf2(act[2]), f2_to_bf2(act[3]));
}

// Shared-memory bytes of one row group's ring.
__host__ __device__ inline size_t ring_bytes(const RingGeom& g) {
  return static_cast<size_t>(kRingHeader) + static_cast<size_t>(g.stages) * g.slot_bytes;
}

// SwiGLU + quantisation, CTA-per-row form: blockDim.x / T row groups of T threads, each with
// its own ring; the sigmoid table (32 KB) sits in front of the rings and is shared by the
// groups.  Thread t of a group owns the vectors t, t + T, ... of a row.
template <int V, int MODE>
__global__ void __launch_bounds__(1024) swiglu_kernel(const SwigluArgs a, const RingGeom g, const int T) {
  extern __shared__ __align__(1024) uint8_t smem[];
  load_sigmoid_table(reinterpret_cast<uint32_t*>(smem), threadIdx.x, blockDim.x);
  const uint32_t sig = smem_u32(smem);
  __syncthreads();
  const RowGroup grp = row_group(T);
  uint8_t* ring = smem + kSigmoidBytes + static_cast<size_t>(grp.index) * ring_bytes(g);
  const int nvec = a.F >> 3;
  auto src = [&](int64_t r, int part) -> const void* { return (part ? a.up : a.gate) + r * a.ld_in; };
  float tw_max = 0.f;   // tensorwise: running max of |act| over this thread's rows
  row_loop(ring, g, grp, a.M, src, [&](int64_t row, uint8_t* slot, const RingState& rs) {
    const uint8_t* up = slot + g.part_bytes;
    uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
    uint32_t m2 = 0;
    float amax32 = 0.f;
    constexpr bool kTw = MODE == kModeTensorwise;
    if constexpr (V > 0) {
      uint4 av[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = grp.t + T * i;
        av[i] = make_uint4(0, 0, 0, 0);
        if (c < nvec) {
          av[i] = swiglu8(slot, up, c, sig, amax32, kTw);
          m2 = absmax4(m2, av[i]);
          if (a.act) *reinterpret_cast<uint4*>(a.act + row * a.ld_act + 8 * c) = av[i];
        }
      }
      if constexpr (!kTw) {
        constexpr int QK = MODE;
        const QuantRow qr = quant_row<QK>(block_max(grp, pair_max(m2), rs.red_max));
        if (grp.t == 0) a.q_scale[row] = qr.scale;
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const int c = grp.t + T * i;
          if (c < nvec) store_q<QK>(qrow, c, av[i], qr);
        }
      }
    } else {
      for (int c = grp.t; c < nvec; c += T) {
        const uint4 au = swiglu8(slot, up, c, sig, amax32, kTw);
        m2 = absmax4(m2, au);
        if constexpr (!kTw) *reinterpret_cast<uint4*>(slot + 16 * c) = au;   // act replaces the gate row
        if (a.act) *reinterpret_cast<uint4*>(a.act + row * a.ld_act + 8 * c) = au;
      }
      if constexpr (!kTw) {
        constexpr int QK = MODE;
        slot_written();
        const QuantRow qr = quant_row<QK>(block_max(grp, pair_max(m2), rs.red_max));   // barrier: act complete
        if (grp.t == 0) a.q_scale[row] = qr.scale;
        for (int c = grp.t; c < nvec; c += T) store_q<QK>(qrow, c, lds_v4(slot + 16 * c), qr);
      }
    }
    if constexpr (kTw) tw_max = fmaxf(tw_max, amax32);
  });
  if constexpr (MODE == kModeTensorwise) flush_amax(a.amax, tw_max);
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
  const int64_t G = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (a.ld_h == a.D && a.ld_q == a.D) {
    // contiguous rows: one flat run of vectors, four loads in flight per thread
    const int64_t total = a.S * nvec;
    const uint4* hv = reinterpret_cast<const uint4*>(a.h);
    uint2* qv = reinterpret_cast<uint2*>(a.q);
    int64_t v = t0;
    for (; v + 3 * G < total; v += 4 * G) {
      uint4 u[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) u[i] = ld_v4(hv + v + i * G);
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[v + i * G] = quant8<QK>(u[i], qr);
    }
    for (; v < total; v += G) qv[v] = quant8<QK>(ld_v4(hv + v), qr);
  } else {
    // strided rows: warps over rows, lanes over a row's vectors
    const int lane = threadIdx.x & 31;
    for (int64_t row = t0 >> 5; row < a.S; row += G >> 5) {
      const __nv_bfloat16* hrow = a.h + row * a.ld_h;
      uint8_t* qrow = static_cast<uint8_t*>(a.q) + row * a.ld_q;
      for (int c = lane; c < nvec; c += 32) *reinterpret_cast<uint2*>(qrow + 8 * c) = quant8<QK>(ld_v4(hrow + 8 * c), qr);
    }
  }
}

// ---------------------------------------------------------------------------
// per-token quantisation with the row maxima given (the fc1 GEMM's SwiGLU epilogue reports
// max |act| per row): a pure stream, one row per warp, no reduction and no row kept whole.
// q_scale[m] = max(amax[m] / qmax, 1e-12), q = the same quantiser as t8g_quant_rows, so
// the result equals quant_rows(act) bit for bit.
// ---------------------------------------------------------------------------
struct QuantGivenRowsArgs {
  const __nv_bfloat16* x;
  int64_t ld_x;
  const float* row_amax;
  void* q;
  int64_t ld_q;
  float* q_scale;
  int64_t S;
  int D;
};

template <int QK>
__global__ void __launch_bounds__(256) quant_rows_given_amax_kernel(const QuantGivenRowsArgs a) {
  const int lane = threadIdx.x & 31;
  const int nvec = a.D >> 3;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < a.S;
       row += warps) {
    const QuantRow qr = quant_row<QK>(__ldg(a.row_amax + row));
    if (lane == 0) a.q_scale[row] = qr.scale;
    const uint4* xr = reinterpret_cast<const uint4*>(a.x + row * a.ld_x);
    uint2* qr_out = reinterpret_cast<uint2*>(static_cast<uint8_t*>(a.q) + row * a.ld_q);
    int c = lane;
    for (; c + 7 * 32 < nvec; c += 8 * 32) {
      uint4 u[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) u[i] = ld_v4(xr + c + 32 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) qr_out[c + 32 * i] = quant8<QK>(u[i], qr);
    }
    for (; c < nvec; c += 32) qr_out[c] = quant8<QK>(ld_v4(xr + c), qr);
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
