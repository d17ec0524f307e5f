// Persistent, warp-specialised 8-bit GEMM with a fused dequantisation epilogue
// for sm_100a (tcgen05 tensor cores, TMEM accumulators, TMA in and out).
//
//   out[m, n] = cast( ((f32(acc[m, n]) * xs[m]) * ws[n or 0]) + f32(bias[n]) )
//   acc[m, n] = sum_k A[m, k] * W[n, k]        (int8 -> int32, or e4m3 -> f32)
//
// Replaces the Triton `_kernel` of src/ck_int8_patch_thor.py:67-106 (epilogue
// :101-106) behind comfy-kitchen's `_C.cutlass_int8_dequant`; the float
// operations are the reference's, in its order, each rounded separately.
//
// CTA layout (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A and W tiles -> 4-stage shared-memory ring
//               (L2 priority: A normal, W evict-last, output stores evict-first)
//   warp 1      MMA issuer:   tcgen05.mma 128x256x32 into one of two TMEM
//               accumulators (2 x 256 columns), commit frees smem stages
//   warps 2..5  epilogue:     TMEM -> registers (tcgen05.ld), dequant, convert,
//               swizzled smem staging, TMA store; releases the accumulator so
//               the MMA of the next tile overlaps this tile's epilogue
// Tiles are visited n-fastest, so the whole weight matrix of a DiT projection
// (<= 75 MB) stays in L2 while activation row panels stream from HBM once.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "f32x2.cuh"
#include "ptx.cuh"
#include "sigmoid.cuh"

namespace t8g {
namespace gemm {

enum InKind : int { kInI8 = 0, kInE4M3 = 1 };
enum OutKind : int { kOutBF16 = 0, kOutF16 = 1, kOutF32 = 2, kOutSwiglu = 3, kOutGated = 4 };
// kOutSwiglu: the GEMM's bf16 output columns come in 128-column gate / up blocks (weights
// interleaved so that every 256-column tile holds 128 gate columns and the matching 128 up
// columns); the epilogue stores act = silu(gate) * up (bf16, half the columns) instead.
// kOutGated: bf16 output updated as a gated residual, out = res + gate[row's gate row] * y
// (the DiT block's `x + gate * proj(...)`), with y the bf16 GEMM output; out may be res.

constexpr int BM = 128;          // tile rows (tokens)
constexpr int BN = 256;          // tile columns (output channels)
constexpr int BK = 128;          // K bytes per stage = one 128-byte swizzle row
constexpr int MMA_K = 32;        // K of one tcgen05.mma for 8-bit operands
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int EPI_COLS = 32;               // columns per epilogue chunk
constexpr int EPI_BUF_BYTES = 32 * 128;    // 32 rows x (32 cols x <= 4 bytes)
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 2 * BN;     // double-buffered accumulator

struct Smem {
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  uint8_t epi[EPI_WARPS][2][EPI_BUF_BYTES];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
};
constexpr size_t SMEM_BYTES = sizeof(Smem) + 1024;   // + slack to align the base to 1024 B

struct Args {
  const float* xs;    // [M] per-token activation scale
  const float* ws;    // [N] per-channel weight scale, or [1]
  const void* bias;   // [N] in the output type, or nullptr
  int ws_stride;      // 1: per channel, 0: one scalar
  int vec_ok;         // ws and bias are 16-byte aligned
  int M, N, K;
  // kOutGated only: out = bf16(res + bf16(gate[grow] * bf16(y))), y the dequantised GEMM
  // output and grow = gate_index[m] (or m / rows_per_gate); res and gate are bf16
  const void* res;
  const void* gate;
  const int32_t* gate_index;
  int64_t ld_res, ld_gate, rows_per_gate;
  // kOutSwiglu only, optional: float32 [M], zeroed by the host; receives max |bf16(act)| of
  // every row (an atomic max per row and tile), so a per-token quantiser can stream act
  float* row_amax;
};

template <int OUT>
struct OutTraits;
template <>
struct OutTraits<kOutBF16> {
  static constexpr int kBytes = 2;
  __device__ static float to_f32(const void* p, int i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  }
  __device__ static uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct OutTraits<kOutSwiglu> : OutTraits<kOutBF16> {};
template <>
struct OutTraits<kOutGated> : OutTraits<kOutBF16> {};
template <>
struct OutTraits<kOutF16> {
  static constexpr int kBytes = 2;
  __device__ static float to_f32(const void* p, int i) {
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
  }
  __device__ static uint32_t pack2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct OutTraits<kOutF32> {
  static constexpr int kBytes = 4;
  __device__ static float to_f32(const void* p, int i) { return reinterpret_cast<const float*>(p)[i]; }
};

// Load 32 consecutive per-channel weight scales and biases for columns [n0, n0+32).
template <int OUT>
__device__ __forceinline__ void load_channel_params(const Args& a, int n0, float (&wsv)[32], float (&bv)[32]) {
  const bool full = n0 + 32 <= a.N;
  if (a.ws_stride == 0) {
    const float w0 = __ldg(a.ws);
#pragma unroll
    for (int j = 0; j < 32; ++j) wsv[j] = w0;
  } else if (full && a.vec_ok) {
    const float4* p = reinterpret_cast<const float4*>(a.ws + n0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 t = __ldg(p + q);
      wsv[4 * q + 0] = t.x;
      wsv[4 * q + 1] = t.y;
      wsv[4 * q + 2] = t.z;
      wsv[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) wsv[j] = (n0 + j < a.N) ? __ldg(a.ws + n0 + j) : 0.f;
  }
  if (a.bias == nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j) bv[j] = 0.f;
  } else if (full && a.vec_ok) {
    if constexpr (OutTraits<OUT>::kBytes == 2) {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.bias) + n0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 t = __ldg(p + q);
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint16_t lo = static_cast<uint16_t>(w[e] & 0xFFFFu), hi = static_cast<uint16_t>(w[e] >> 16);
          bv[8 * q + 2 * e + 0] = OutTraits<OUT>::to_f32(&lo, 0);
          bv[8 * q + 2 * e + 1] = OutTraits<OUT>::to_f32(&hi, 0);
        }
      }
    } else {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.bias) + n0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 t = __ldg(p + q);
        bv[4 * q + 0] = t.x;
        bv[4 * q + 1] = t.y;
        bv[4 * q + 2] = t.z;
        bv[4 * q + 3] = t.w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) bv[j] = (n0 + j < a.N) ? OutTraits<OUT>::to_f32(a.bias, n0 + j) : 0.f;
  }
}

// Epilogue of one 32-row slice of an output tile: TMEM columns [0, BN) of the lanes
// at `t_row` -> fp32 dequant in the reference order -> output type -> swizzled
// staging buffer (two per warp, alternating) -> TMA store at (n_tile0 + 32c, row0).
template <int IN, int OUT>
__device__ __forceinline__ void epilogue_tile(const Args& args, const CUtensorMap* tm_out,
                                              uint8_t (*bufs)[EPI_BUF_BYTES], int& ebuf, uint32_t t_row, int row0,
                                              int n_tile0, int lane, uint64_t pol_out) {
  const int row = row0 + lane;
  const float xs_r = row < args.M ? __ldg(args.xs + row) : 0.f;
  const int nchunks = min(BN / EPI_COLS, (args.N - n_tile0 + EPI_COLS - 1) / EPI_COLS);
  for (int c = 0; c < nchunks; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * EPI_COLS), r);
    tmem_ld_wait();
    const int n0 = n_tile0 + c * EPI_COLS;
    float wsv[32], bv[32];
    load_channel_params<OUT>(args, n0, wsv, bv);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float f = (IN == kInI8) ? __int2float_rn(static_cast<int>(r[j])) : __uint_as_float(r[j]);
      f = __fmul_rn(f, xs_r);
      f = __fmul_rn(f, wsv[j]);
      if (args.bias != nullptr) f = __fadd_rn(f, bv[j]);
      v[j] = f;
    }
    // the staging buffer used two chunks ago must have been read by its TMA store
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    uint8_t* buf = bufs[ebuf];
    if constexpr (OutTraits<OUT>::kBytes == 2) {
      // 32 rows x 64 B, 64-byte swizzle: 16-byte chunk q of row r lives at chunk q ^ ((r >> 1) & 3)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = OutTraits<OUT>::pack2(v[8 * q + 0], v[8 * q + 1]);
        w.y = OutTraits<OUT>::pack2(v[8 * q + 2], v[8 * q + 3]);
        w.z = OutTraits<OUT>::pack2(v[8 * q + 4], v[8 * q + 5]);
        w.w = OutTraits<OUT>::pack2(v[8 * q + 6], v[8 * q + 7]);
        const int pq = q ^ ((lane >> 1) & 3);
        *reinterpret_cast<uint4*>(buf + lane * 64 + pq * 16) = w;
      }
    } else {
      // 32 rows x 128 B, 128-byte swizzle: chunk q of row r lives at chunk q ^ (r & 7)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 w = make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        const int pq = q ^ (lane & 7);
        *reinterpret_cast<float4*>(buf + lane * 128 + pq * 16) = w;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tm_out, buf, n0, row0, pol_out);
      bulk_commit_group();
    }
    ebuf ^= 1;
  }
}

template <int IN, int OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_dequant_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_out, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_n = (args.N + BN - 1) / BN;
  const int tiles_m = (args.M + BM - 1) / BM;
  const int num_tiles = tiles_m * tiles_n;
  const int kblocks = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], EPI_WARPS);
    }
    mbar_init(&s.drain, 1);
    fence_mbarrier_init();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
    prefetch_tensormap(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // A row panels are re-read by every CTA of the panel (tiles run n-fastest): normal
      // priority; W is re-read by every panel: keep it.
      const uint64_t pol_a = policy_evict_normal();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int tm = tile / tiles_n;
        const int tn = tile - tm * tiles_n;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[stage], STAGE_BYTES);
          tma_load_2d(s.a[stage], &tm_a, &s.full[stage], kb * BK, tm * BM, pol_a);
          tma_load_2d(s.b[stage], &tm_b, &s.full[stage], kb * BK, tn * BN, pol_b);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every issued copy must land before the CTA may exit.
      for (int i = 0; i < STAGES && i < issued; ++i) {
        const int n = issued - 1 - i;
        if (!mbar_wait(&s.full[n % STAGES], static_cast<uint32_t>((n / STAGES) & 1), kStatusTimeoutDrain)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = (IN == kInI8) ? make_idesc(2, 1, 1, BM, BN)   // s32 <- s8 x s8
                                               : make_idesc(1, 0, 0, BM, BN);  // f32 <- e4m3 x e4m3
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true, any = false;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!mbar_wait(&s.tmem_empty[acc], acc_phase ^ 1u, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.a[stage]);
          const uint32_t b0 = smem_u32(s.b[stage]);
#pragma unroll
          for (int k = 0; k < BK / MMA_K; ++k) {
            const uint64_t ad = smem_desc_k_sw128(a0 + k * MMA_K);
            const uint64_t bd = smem_desc_k_sw128(b0 + k * MMA_K);
            const uint32_t accumulate = (kb | k) != 0 ? 1u : 0u;
            if constexpr (IN == kInI8)
              mma_i8(d_tmem, ad, bd, idesc, accumulate);
            else
              mma_f8(d_tmem, ad, bd, idesc, accumulate);
          }
          tc_commit(&s.empty[stage]);
          any = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&s.tmem_full[acc]);
      }
      if (any) {
        // All MMAs (and their shared-memory reads) complete before teardown.
        tc_commit(&s.drain);
        mbar_wait(&s.drain, 0, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;           // staging slot of this warp
    const int quarter = warp & 3;      // TMEM lanes [32*quarter, 32*quarter+32) are readable by this warp
    const uint64_t pol_out = policy_evict_first();   // the output is not re-read here
    int local = 0;
    int ebuf = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int tm = tile / tiles_n;
      const int tn = tile - tm * tiles_n;
      const int acc = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      if (!mbar_wait(&s.tmem_full[acc], acc_phase, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const int row0 = tm * BM + quarter * 32;
      if (row0 < args.M) {
        epilogue_tile<IN, OUT>(args, &tm_out, s.epi[ew], ebuf, tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                                                 static_cast<uint32_t>(acc * BN),
                               row0, tn * BN, lane, pol_out);
      }
      // hand the accumulator back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.tmem_empty[acc]);
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Per-tile channel parameters staged in shared memory by the epilogue warps:
// ws[n_tile0 + j] and f32(bias[n_tile0 + j]) for j < BN (0 past N).
struct TileParams {
  float ws[BN];
  float bias[BN];
  uint32_t bias2[BN / 2];   // 2-byte outputs: the bias as packed pairs of the output type
};

template <int OUT, int TBN = BN>
__device__ __forceinline__ void stage_tile_params(const Args& args, int n_tile0, int e, int ne, TileParams& tp) {
  for (int j = e; j < TBN; j += ne) {
    const int n = n_tile0 + j;
    const bool in = n < args.N;
    tp.ws[j] = in ? __ldg(args.ws + (args.ws_stride ? n : 0)) : 0.f;
    tp.bias[j] = (in && args.bias) ? OutTraits<OUT>::to_f32(args.bias, n) : 0.f;
  }
  if constexpr (OutTraits<OUT>::kBytes == 2) {
    const uint16_t* b16 = static_cast<const uint16_t*>(args.bias);
    for (int j = e; j < TBN / 2; j += ne) {
      const int n = n_tile0 + 2 * j;
      const uint32_t lo = (args.bias && n < args.N) ? b16[n] : 0u;
      const uint32_t hi = (args.bias && n + 1 < args.N) ? b16[n + 1] : 0u;
      tp.bias2[j] = lo | (hi << 16);
    }
  }
}

// Epilogue of one 32-row slice with the tile's parameters in shared memory and the
// TMEM loads software-pipelined (the load of chunk c+1 overlaps the math of chunk c).
template <int IN, int OUT, int EPB>
__device__ __forceinline__ void epilogue_tile_staged(const Args& args, const CUtensorMap* tm_out,
                                                     uint8_t (*bufs)[EPB], int& ebuf, uint32_t t_row,
                                                     int row0, int n_tile0, int lane, uint64_t pol_out, float xs_r,
                                                     const TileParams& tp) {
  const int nchunks = min(BN / EPI_COLS, (args.N - n_tile0 + EPI_COLS - 1) / EPI_COLS);
  const bool has_bias = args.bias != nullptr;
  uint32_t r[32];
  tmem_ld_32x32b_x32(t_row, r);
  for (int c = 0; c < nchunks; ++c) {
    tmem_ld_wait_regs(r);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (IN == kInI8) ? __int2float_rn(static_cast<int>(r[j])) : __uint_as_float(r[j]);
    if (c + 1 < nchunks) tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((c + 1) * EPI_COLS), r);
    const float4* wq = reinterpret_cast<const float4*>(tp.ws + c * EPI_COLS);
    if constexpr (OutTraits<OUT>::kBytes == 2) {
      // packed products, then the bias added from its 16-bit pair (mixed-precision add)
      const uint4* bq2 = reinterpret_cast<const uint4*>(tp.bias2 + c * EPI_COLS / 2);
      const float2 xs2 = make_float2(xs_r, xs_r);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 w0 = wq[2 * q], w1 = wq[2 * q + 1];
        const float2 wp[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                              make_float2(w1.z, w1.w)};
        const uint4 b4 = has_bias ? bq2[q] : make_uint4(0, 0, 0, 0);
        const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int j = 8 * q + 2 * p;
          float2 f = mul2_rn(mul2_rn(make_float2(v[j], v[j + 1]), xs2), wp[p]);
          if (has_bias) f = (OUT == kOutF16) ? add_f32_f16x2(f, bw[p]) : add_f32_bf16x2(f, bw[p]);
          v[j] = f.x;
          v[j + 1] = f.y;
        }
      }
    } else {
      const float4* bq = reinterpret_cast<const float4*>(tp.bias + c * EPI_COLS);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 w4 = wq[q];
        const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
        float bb[4] = {0.f, 0.f, 0.f, 0.f};
        if (has_bias) {
          const float4 b4 = bq[q];
          bb[0] = b4.x; bb[1] = b4.y; bb[2] = b4.z; bb[3] = b4.w;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float f = __fmul_rn(v[4 * q + e], xs_r);
          f = __fmul_rn(f, wv[e]);
          if (has_bias) f = __fadd_rn(f, bb[e]);
          v[4 * q + e] = f;
        }
      }
    }
    const int n0 = n_tile0 + c * EPI_COLS;
    // the staging buffer used two chunks ago must have been read by its TMA store
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    uint8_t* buf = bufs[ebuf];
    if constexpr (OutTraits<OUT>::kBytes == 2) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = OutTraits<OUT>::pack2(v[8 * q + 0], v[8 * q + 1]);
        w.y = OutTraits<OUT>::pack2(v[8 * q + 2], v[8 * q + 3]);
        w.z = OutTraits<OUT>::pack2(v[8 * q + 4], v[8 * q + 5]);
        w.w = OutTraits<OUT>::pack2(v[8 * q + 6], v[8 * q + 7]);
        const int pq = q ^ ((lane >> 1) & 3);
        *reinterpret_cast<uint4*>(buf + lane * 64 + pq * 16) = w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 w = make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        const int pq = q ^ (lane & 7);
        *reinterpret_cast<float4*>(buf + lane * 128 + pq * 16) = w;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tm_out, buf, n0, row0, pol_out);
      bulk_commit_group();
    }
    ebuf ^= 1;
  }
  if (nchunks == 0) tmem_ld_wait_regs(r);
}

__device__ __align__(16) uint8_t g_zero16[16];
__device__ __forceinline__ const void* rbuf_src_dummy() { return g_zero16; }

// acc -> float for 64 columns: int32 converted (RN), fp32 taken as is
template <int IN>
__device__ __forceinline__ void acc_to_f32_64(const uint32_t (&r0)[32], const uint32_t (&r1)[32], float (&v)[64]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    v[j] = (IN == kInI8) ? __int2float_rn(static_cast<int>(r0[j])) : __uint_as_float(r0[j]);
    v[32 + j] = (IN == kInI8) ? __int2float_rn(static_cast<int>(r1[j])) : __uint_as_float(r1[j]);
  }
}

// Dequantise 64 columns (chunk c of the tile) of one row and pack them to the 2-byte output
// type: ((acc * xs) * ws) + bias in f32, the bias added from its 16-bit pair.
template <int OUT>
__device__ __forceinline__ void dequant_pack64(const TileParams& tp, int c, const float (&v)[64], float2 xs2,
                                               bool has_bias, uint32_t (&packed)[32]) {
  const float4* wq = reinterpret_cast<const float4*>(tp.ws + c * 64);
  const uint4* bq2 = reinterpret_cast<const uint4*>(tp.bias2 + c * 32);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 w0 = wq[2 * q], w1 = wq[2 * q + 1];
    const float2 wp[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                          make_float2(w1.z, w1.w)};
    const uint4 b4 = has_bias ? bq2[q] : make_uint4(0, 0, 0, 0);
    const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int j = 8 * q + 2 * p;
      float2 f = mul2_rn(mul2_rn(make_float2(v[j], v[j + 1]), xs2), wp[p]);
      if (has_bias) f = (OUT == kOutF16) ? add_f32_f16x2(f, bw[p]) : add_f32_bf16x2(f, bw[p]);
      packed[4 * q + p] = OutTraits<OUT>::pack2(f.x, f.y);
    }
  }
}

// Stage one row's 64 packed 2-byte values in the warp's staging buffer (32 rows x 128 B,
// 128-byte swizzle: 16-byte piece q of row r at q ^ (r & 7)) and store the 32 x 64 box at
// (x, y) with TMA; the buffer used two stores ago must have been read first.
template <int EPB>
__device__ __forceinline__ void store_chunk64(const CUtensorMap* tm_out, uint8_t (*bufs)[EPB], int& ebuf, int lane,
                                              const uint32_t (&packed)[32], int x, int y, uint64_t pol_out) {
  if (lane == 0) bulk_wait_group_read<1>();
  __syncwarp();
  uint8_t* buf = bufs[ebuf];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint4 w = make_uint4(packed[4 * q + 0], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    *reinterpret_cast<uint4*>(buf + lane * 128 + ((q ^ (lane & 7)) * 16)) = w;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tm_out, buf, x, y, pol_out);
    bulk_commit_group();
  }
  ebuf ^= 1;
}

// ---------------------------------------------------------------- gated residual
// The residual rows of a warp's 32 x 256 slice of a tile are copied into shared memory
// (4 chunks of 32 rows x 128 B, the staging layout: 16-byte piece q of row r at q ^ (r & 7))
// with cp.async when the tile's epilogue begins, before the accumulator is ready, so the
// copies overlap the tile's MMA; each chunk's output then replaces its residual in place and
// is stored from there with TMA.  When the 32 rows share one gate row (one batch element),
// that row's 256 columns are copied next to them and read as broadcasts.
struct GatedSlice {
  const uint16_t* gate_row;   // this lane's gate row at the tile's first column (null: row >= M)
  bool shared_gate;           // every valid row of the warp uses lane 0's gate row
};

__device__ __forceinline__ GatedSlice gated_prefetch(const Args& args, uint8_t* rbuf, uint8_t* gbuf, int row0,
                                                     int n_tile0, int lane) {
  GatedSlice g;
  const int m = row0 + lane;
  const int tile_cols = min(BN, args.N - n_tile0);
  const uint16_t* res_row = nullptr;
  int64_t grow = -1;
  if (m < args.M) {
    res_row = static_cast<const uint16_t*>(args.res) + static_cast<int64_t>(m) * args.ld_res + n_tile0;
    grow = args.gate_index ? static_cast<int64_t>(__ldg(args.gate_index + m)) : m / args.rows_per_gate;
  }
  g.gate_row = m < args.M ? static_cast<const uint16_t*>(args.gate) + grow * args.ld_gate + n_tile0 : nullptr;
  const int64_t grow0 = __shfl_sync(0xffffffffu, grow, 0);
  g.shared_gate = __all_sync(0xffffffffu, m >= args.M || grow == grow0);
  // the previous tile's stores must have read the buffer before it is refilled
  if (lane == 0) bulk_wait_group_read<0>();
  __syncwarp();
#pragma unroll
  for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int col = c * 64 + 8 * q;
      const bool in = res_row != nullptr && col < tile_cols;
      cp_async_16(rbuf + c * 4096 + lane * 128 + ((q ^ (lane & 7)) * 16),
                  in ? static_cast<const void*>(res_row + col) : rbuf_src_dummy(), in ? 16u : 0u);
    }
  }
  if (g.shared_gate) {
    const uint16_t* g0 = static_cast<const uint16_t*>(args.gate) + grow0 * args.ld_gate + n_tile0;
    const bool in = 8 * lane < tile_cols;
    cp_async_16(gbuf + lane * 16, in ? static_cast<const void*>(g0 + 8 * lane) : rbuf_src_dummy(), in ? 16u : 0u);
  }
  cp_async_commit();
  return g;
}

// Epilogue of one 32-row slice with the gated residual (kOutGated, bf16): for each 64-column
// chunk, y = the plain epilogue's bf16 value, then out = bf16(res + bf16(gate * y)) in
// torch's order, written over the chunk's residual and stored from there.
template <int IN>
__device__ __forceinline__ void epilogue_tile_gated(const Args& args, const CUtensorMap* tm_out, uint8_t* rbuf,
                                                    const uint8_t* gbuf, const GatedSlice& gs, uint32_t t_row,
                                                    int row0, int n_tile0, int lane, uint64_t pol_out, float xs_r,
                                                    const TileParams& tp) {
  const int tile_cols = min(BN, args.N - n_tile0);
  const int nchunks = (tile_cols + 63) / 64;
  const bool has_bias = args.bias != nullptr;
  const float2 xs2 = make_float2(xs_r, xs_r);
  uint32_t r0[32], r1[32];
  tmem_ld_32x32b_x32(t_row, r0);
  tmem_ld_32x32b_x32(t_row + 32u, r1);
  cp_async_wait_all();   // issued when the tile began: long done
  __syncwarp();          // the shared gate row came from every lane's copy
  for (int c = 0; c < nchunks; ++c) {
    tmem_ld_wait_regs(r0);
    tmem_ld_wait_regs(r1);
    float v[64];
    acc_to_f32_64<IN>(r0, r1, v);
    if (c + 1 < nchunks) {
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((c + 1) * 64), r0);
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((c + 1) * 64 + 32), r1);
    }
    uint32_t packed[32];
    dequant_pack64<kOutGated>(tp, c, v, xs2, has_bias, packed);
    uint8_t* slot = rbuf + c * 4096;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int col = c * 64 + 8 * q;
      uint4* cell = reinterpret_cast<uint4*>(slot + lane * 128 + ((q ^ (lane & 7)) * 16));
      const uint4 r4 = *cell;
      uint4 g4;
      if (gs.shared_gate)
        g4 = *reinterpret_cast<const uint4*>(gbuf + (c * 8 + q) * 16);
      else
        g4 = (gs.gate_row != nullptr && col < tile_cols) ? __ldg(reinterpret_cast<const uint4*>(gs.gate_row + col))
                                                         : make_uint4(0, 0, 0, 0);
      const uint32_t rw[4] = {r4.x, r4.y, r4.z, r4.w};
      const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
      uint32_t o[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint32_t t = f2_to_bf2(mul_bf16x2_exact(gw[p], packed[4 * q + p]));   // bf16(gate * y)
        o[p] = f2_to_bf2(add_f32_bf16x2(bf2_to_f2(rw[p]), t));                      // bf16(res + t)
      }
      *cell = make_uint4(o[0], o[1], o[2], o[3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tm_out, slot, n_tile0 + c * 64, row0, pol_out);
      bulk_commit_group();
    }
  }
  if (nchunks == 0) {
    tmem_ld_wait_regs(r0);
    tmem_ld_wait_regs(r1);
  }
}

// Epilogue of one 32-row slice for 2-byte outputs, 64 columns per chunk: two 32-column
// TMEM loads per chunk (the next chunk's loads overlap this chunk's math), packed
// products, the bias added from its 16-bit pair, and a 32 x 64 TMA store of full
// 128-byte rows from a 128-byte-swizzled staging buffer.
template <int IN, int OUT, int EPB, int TBN = BN>
__device__ __forceinline__ void epilogue_tile_staged64(const Args& args, const CUtensorMap* tm_out,
                                                       uint8_t (*bufs)[EPB], int& ebuf, uint32_t t_row, int row0,
                                                       int n_tile0, int lane, uint64_t pol_out, float xs_r,
                                                       const TileParams& tp) {
  static_assert(EPB >= 32 * 128, "staging buffer holds 32 rows of 128 bytes");
  const int nchunks = min(TBN / 64, (args.N - n_tile0 + 63) / 64);
  const bool has_bias = args.bias != nullptr;
  const float2 xs2 = make_float2(xs_r, xs_r);
  uint32_t r0[32], r1[32];
  tmem_ld_32x32b_x32(t_row, r0);
  tmem_ld_32x32b_x32(t_row + 32u, r1);
  for (int c = 0; c < nchunks; ++c) {
    tmem_ld_wait_regs(r0);
    tmem_ld_wait_regs(r1);
    float v[64];
    acc_to_f32_64<IN>(r0, r1, v);
    if (c + 1 < nchunks) {
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((c + 1) * 64), r0);
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((c + 1) * 64 + 32), r1);
    }
    uint32_t packed[32];
    dequant_pack64<OUT>(tp, c, v, xs2, has_bias, packed);
    store_chunk64<EPB>(tm_out, bufs, ebuf, lane, packed, n_tile0 + c * 64, row0, pol_out);
  }
  if (nchunks == 0) {
    tmem_ld_wait_regs(r0);
    tmem_ld_wait_regs(r1);
  }
}

// SwiGLU epilogue of one 32-row slice: tile columns [0, 128) are gate and [128, 256) the
// matching up columns.  Each value is dequantised and rounded to bf16 exactly as the plain
// epilogue stores it, then act = (g * sigmoid(g)) * u with the row kernel's exact sigmoid
// (sigmoid.cuh, table `sig` in shared memory), rounded to bf16 and stored at act columns
// [n_tile0 / 2, n_tile0 / 2 + 128).
template <int IN, int EPB>
__device__ __forceinline__ void epilogue_tile_swiglu(const Args& args, const CUtensorMap* tm_out,
                                                     uint8_t (*bufs)[EPB], int& ebuf, uint32_t t_row, int row0,
                                                     int n_tile0, int lane, uint64_t pol_out, float xs_r,
                                                     const TileParams& tp, uint32_t sig) {
  const bool has_bias = args.bias != nullptr;
  const float2 xs2 = make_float2(xs_r, xs_r);
  constexpr int kChunks = BN / 2 / EPI_COLS;
  uint32_t m2 = 0;   // max |act| of this lane's row over the tile (packed bf16 pair)
  uint32_t rg[32], ru[32];
  tmem_ld_32x32b_x32(t_row, rg);
  tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(BN / 2), ru);
#pragma unroll 1
  for (int c = 0; c < kChunks; ++c) {
    tmem_ld_wait_regs(rg);
    tmem_ld_wait_regs(ru);
    float2 gf[16], uf[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      gf[p] = (IN == kInI8) ? make_float2(__int2float_rn(static_cast<int>(rg[2 * p])),
                                          __int2float_rn(static_cast<int>(rg[2 * p + 1])))
                            : make_float2(__uint_as_float(rg[2 * p]), __uint_as_float(rg[2 * p + 1]));
      uf[p] = (IN == kInI8) ? make_float2(__int2float_rn(static_cast<int>(ru[2 * p])),
                                          __int2float_rn(static_cast<int>(ru[2 * p + 1])))
                            : make_float2(__uint_as_float(ru[2 * p]), __uint_as_float(ru[2 * p + 1]));
    }
    // the next chunk's accumulator loads while this one computes
    if (c + 1 < kChunks) {
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((c + 1) * EPI_COLS), rg);
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(BN / 2 + (c + 1) * EPI_COLS), ru);
    }
    const float2* wg = reinterpret_cast<const float2*>(tp.ws + c * EPI_COLS);
    const float2* wu = reinterpret_cast<const float2*>(tp.ws + BN / 2 + c * EPI_COLS);
    const uint32_t* bg = tp.bias2 + c * EPI_COLS / 2;
    const uint32_t* bu = tp.bias2 + (BN / 2 + c * EPI_COLS) / 2;
    uint32_t act[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      // gate and up exactly as the plain epilogue stores them: ((acc * xs) * ws) + bias, bf16
      float2 g = mul2_rn(mul2_rn(gf[p], xs2), wg[p]);
      float2 u = mul2_rn(mul2_rn(uf[p], xs2), wu[p]);
      if (has_bias) {
        g = add_f32_bf16x2(g, bg[p]);
        u = add_f32_bf16x2(u, bu[p]);
      }
      act[p] = f2_to_bf2(silu_mul2(f2_to_bf2(g), bf2_to_f2(f2_to_bf2(u)), sig));
      m2 = absmax_bf16x2(m2, act[p]);
    }
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    uint8_t* buf = bufs[ebuf];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = make_uint4(act[4 * q + 0], act[4 * q + 1], act[4 * q + 2], act[4 * q + 3]);
      const int pq = q ^ ((lane >> 1) & 3);
      *reinterpret_cast<uint4*>(buf + lane * 64 + pq * 16) = w;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tm_out, buf, n_tile0 / 2 + c * EPI_COLS, row0, pol_out);
      bulk_commit_group();
    }
    ebuf ^= 1;
  }
  if (args.row_amax != nullptr && row0 + lane < args.M) {
    // rows of the 32-row slice past M hold garbage accumulators: only valid rows report
    const float m = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xFFFF0000u));
    if (m > 0.f) atomicMax(reinterpret_cast<int*>(args.row_amax + row0 + lane), __float_as_int(m));
  }
}

// ===========================================================================
// 2-SM variant: a cluster of two CTAs (one per SM of a TPC) computes a 256x256
// output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32).
//   CTA r loads its own A rows [tm*256 + 128r, +128) and its own half of W, rows
//   [tn*256 + 128r, +128), into its own shared memory; the loads of both CTAs
//   complete on the leader's (r = 0) `full` barrier; every CTA loads only its own
//   operands.
//   The leader's single MMA thread issues the pair MMA, which reads the operands
//   of both CTAs and accumulates rows 128r..128r+127 in CTA r's TMEM; its commits
//   free the stage in both CTAs and hand each CTA its accumulator.
//   Each CTA's epilogue warps store their own 128 rows and report the
//   accumulator free on the leader's `tmem_empty` barrier.
// Per SM this halves W's share of the shared-memory fill and of the tensor
// core's operand reads compared with the 1-SM kernel.  The epilogue stages each
// tile's channel parameters in shared memory before waiting for its accumulator
// and pipelines its TMEM loads.  With few 256-wide tiles (small M) the host picks
// 128- or 64-column tiles (template TBN), so that more pairs share the problem.
// ===========================================================================
constexpr int P_BM = 256;                   // tile rows per CTA pair
constexpr int P_ROWS = 128;                 // rows of A (and of W) per CTA
constexpr int P_A_BYTES = P_ROWS * BK;
constexpr int P_B_BYTES = P_ROWS * BK;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;   // per CTA

// Ring depth, tile width and epilogue staging per output type: five 32 KB stages (per CTA)
// and two staging buffers per epilogue warp (32 x 64 of a 2-byte output, 32 x 32 of fp32);
// the gated epilogue keeps four stages and stores from its residual buffers instead; narrow
// tiles (TBN = 128 / 64 columns, plain 2-byte outputs, for problems with few tiles) load
// TBN / 2 rows of W per CTA.
template <int OUT, int TBN = BN>
struct PairCfg {
  static_assert(TBN == BN || ((TBN == 128 || TBN == 64) && (OUT == kOutBF16 || OUT == kOutF16)),
                "narrow tiles serve the plain 2-byte outputs");
  static constexpr int kBRows = TBN / 2;             // rows of W per CTA
  static constexpr int kBBytes = kBRows * BK;
  // 2-byte outputs are stored in 32 x 64 boxes (full 128-byte rows, 128-byte swizzle),
  // fp32 and the SwiGLU epilogue in 32 x 32 boxes
  static constexpr int kEpiCols = (OutTraits<OUT>::kBytes == 2 && OUT != kOutSwiglu) ? 64 : EPI_COLS;
  static constexpr int kEpiBytes = OUT == kOutGated ? 16 : 32 * kEpiCols * OutTraits<OUT>::kBytes;
  // kOutGated stores from its residual buffers (a warp's 32 x 256 slice of the tile, 16 KB)
  // instead of the staging buffers, and keeps four stages to make room for them
  static constexpr int kStages = OUT == kOutGated ? 4 : 5;
  static constexpr int kResBytes = OUT == kOutGated ? 4 * 32 * 128 : 16;
  static constexpr int kSigEntries = OUT == kOutSwiglu ? kSigmoidEntries : 4;
};

template <int STAGES, int EPB, int RESB, int BBYTES = P_B_BYTES, int SIGN = 4>
struct SmemPair {
  uint8_t a[STAGES][P_A_BYTES];
  uint8_t b[STAGES][BBYTES];
  alignas(1024) uint8_t epi[EPI_WARPS][2][EPB];
  alignas(1024) uint8_t res[EPI_WARPS][RESB];        // kOutGated: residual / output chunks
  uint8_t gate[EPI_WARPS][RESB > 16 ? 512 : 16];     // kOutGated: a shared gate row
  alignas(16) uint32_t sig[SIGN];                    // kOutSwiglu: the sigmoid table
  TileParams params[2];   // channel parameters of the tile in each accumulator
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
};
template <int OUT, int TBN = BN>
using SmemPairOf = SmemPair<PairCfg<OUT, TBN>::kStages, PairCfg<OUT, TBN>::kEpiBytes, PairCfg<OUT, TBN>::kResBytes,
                            PairCfg<OUT, TBN>::kBBytes, PairCfg<OUT, TBN>::kSigEntries>;
template <int OUT, int TBN = BN>
constexpr size_t pair_smem_bytes() { return sizeof(SmemPairOf<OUT, TBN>) + 1024; }   // + slack to align to 1024 B
static_assert(pair_smem_bytes<kOutBF16>() <= 227 * 1024 && pair_smem_bytes<kOutF32>() <= 227 * 1024 &&
                  pair_smem_bytes<kOutGated>() <= 227 * 1024 && pair_smem_bytes<kOutSwiglu>() <= 227 * 1024,
              "pair kernel shared memory exceeds the per-CTA limit");

template <int IN, int OUT, int TBN = BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_dequant_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                             const __grid_constant__ CUtensorMap tm_out, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  using Cfg = PairCfg<OUT, TBN>;
  constexpr int P_STAGES = Cfg::kStages;
  constexpr uint32_t kTmemCols = 2 * TBN;   // double-buffered accumulator
  SmemPairOf<OUT, TBN>& s = *reinterpret_cast<SmemPairOf<OUT, TBN>*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int tiles_n = (args.N + TBN - 1) / TBN;
  const int tiles_m = (args.M + P_BM - 1) / P_BM;
  const int num_tiles = tiles_m * tiles_n;
  const int kblocks = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < P_STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], 2 * EPI_WARPS);
    }
    mbar_init(&s.drain, 1);
    fence_mbarrier_init();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
    prefetch_tensormap(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc_pair(&s.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // both CTAs' barriers initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_normal();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += npairs) {
        const int tm = tile / tiles_n;
        const int tn = tile - tm * tiles_n;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&s.full[stage], 2 * (P_A_BYTES + Cfg::kBBytes));
          const uint32_t bar = mapa_shared(smem_u32(&s.full[stage]), 0);
          tma_load_2d_pair(s.a[stage], &tm_a, bar, kb * BK, tm * P_BM + static_cast<int>(rank) * P_ROWS, pol_a);
          tma_load_2d_pair(s.b[stage], &tm_b, bar, kb * BK, tn * TBN + static_cast<int>(rank) * Cfg::kBRows, pol_b);
          ++issued;
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // the leader sees every copy of the pair land on its `full` barriers
      if (rank == 0) {
        for (int i = 0; i < P_STAGES && i < issued; ++i) {
          const int n = issued - 1 - i;
          if (!mbar_wait(&s.full[n % P_STAGES], static_cast<uint32_t>((n / P_STAGES) & 1), kStatusTimeoutDrain)) break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = (IN == kInI8) ? make_idesc(2, 1, 1, P_BM, TBN)   // s32 <- s8 x s8
                                               : make_idesc(1, 0, 0, P_BM, TBN);  // f32 <- e4m3 x e4m3
      // cluster addresses of the barrier arrays in both CTAs (8 bytes per barrier)
      const uint32_t empty0[2] = {mapa_shared(smem_u32(&s.empty[0]), 0), mapa_shared(smem_u32(&s.empty[0]), 1)};
      const uint32_t tfull0[2] = {mapa_shared(smem_u32(&s.tmem_full[0]), 0),
                                  mapa_shared(smem_u32(&s.tmem_full[0]), 1)};
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true, any = false;
      for (int tile = pair; ok && tile < num_tiles; tile += npairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!mbar_wait(&s.tmem_empty[acc], acc_phase ^ 1u, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TBN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.a[stage]);
          const uint32_t b0 = smem_u32(s.b[stage]);
#pragma unroll
          for (int k = 0; k < BK / MMA_K; ++k) {
            const uint64_t ad = smem_desc_k_sw128(a0 + k * MMA_K);
            const uint64_t bd = smem_desc_k_sw128(b0 + k * MMA_K);
            const uint32_t accumulate = (kb | k) != 0 ? 1u : 0u;
            if constexpr (IN == kInI8)
              mma_i8_pair(d_tmem, ad, bd, idesc, accumulate);
            else
              mma_f8_pair(d_tmem, ad, bd, idesc, accumulate);
          }
          tc_commit_pair(empty0[0] + 8u * static_cast<uint32_t>(stage));
          tc_commit_pair(empty0[1] + 8u * static_cast<uint32_t>(stage));
          any = true;
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(tfull0[0] + 8u * static_cast<uint32_t>(acc));
        tc_commit_pair(tfull0[1] + 8u * static_cast<uint32_t>(acc));
      }
      if (any) {
        tc_commit_pair(mapa_shared(smem_u32(&s.drain), 0));
        mbar_wait(&s.drain, 0, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int e = threadIdx.x - 64;   // 0..127 over the epilogue warps
    const uint64_t pol_out = policy_evict_first();
    uint32_t tempty_bar[2];
    tempty_bar[0] = mapa_shared(smem_u32(&s.tmem_empty[0]), 0);
    tempty_bar[1] = mapa_shared(smem_u32(&s.tmem_empty[1]), 0);
    int local = 0;
    int ebuf = 0;
    // the sigmoid table; the first tile's named barrier orders these writes before any read
    if constexpr (OUT == kOutSwiglu) load_sigmoid_table(s.sig, e, 128);
    for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
      const int tm = tile / tiles_n;
      const int tn = tile - tm * tiles_n;
      const int acc = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      const int row0 = tm * P_BM + static_cast<int>(rank) * P_ROWS + quarter * 32;
      // channel parameters and the row scale load while the MMA still runs
      stage_tile_params<OUT, TBN>(args, tn * TBN, e, 128, s.params[acc]);

      const float xs_r = row0 + lane < args.M ? __ldg(args.xs + row0 + lane) : 0.f;
      [[maybe_unused]] GatedSlice gs{};
      if constexpr (OUT == kOutGated) {
        if (row0 < args.M) gs = gated_prefetch(args, s.res[ew], s.gate[ew], row0, tn * TBN, lane);
      }
      const bool ok = mbar_wait(&s.tmem_full[acc], acc_phase, kStatusTimeoutEpilogue);
      // all four warps staged the parameters; they leave together if any wait ran out
      if (named_bar_any(1, 128, !ok)) break;
      tc_fence_after();
      if (row0 < args.M) {
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * TBN);
        if constexpr (OUT == kOutGated)
          epilogue_tile_gated<IN>(args, &tm_out, s.res[ew], s.gate[ew], gs, t_row, row0, tn * TBN, lane, pol_out, xs_r,
                                  s.params[acc]);
        else if constexpr (OUT == kOutSwiglu)
          epilogue_tile_swiglu<IN, Cfg::kEpiBytes>(args, &tm_out, s.epi[ew], ebuf, t_row, row0, tn * TBN, lane, pol_out,
                                                   xs_r, s.params[acc], smem_u32(s.sig));
        else if constexpr (Cfg::kEpiCols == 64)
          epilogue_tile_staged64<IN, OUT, Cfg::kEpiBytes, TBN>(args, &tm_out, s.epi[ew], ebuf, t_row, row0, tn * TBN,
                                                               lane, pol_out, xs_r, s.params[acc]);
        else
          epilogue_tile_staged<IN, OUT, Cfg::kEpiBytes>(args, &tm_out, s.epi[ew], ebuf, t_row, row0, tn * TBN, lane,
                                                        pol_out, xs_r, s.params[acc]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_bar[acc]);
    }
    if constexpr (OUT == kOutGated) cp_async_wait_all();   // a residual copy left by a wait that gave up
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // the pair's MMAs, copies and cross-CTA signals are all done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace gemm
}  // namespace t8g
