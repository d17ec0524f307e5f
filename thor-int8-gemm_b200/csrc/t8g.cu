// C ABI of the B200 quantized linear-layer path (declared in include/thor_int8_gemm_b200.h).
//
// Host side only: argument validation, TMA tensor-map encoding, launch shapes.
// Single translation unit: the kernels live in the included headers.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "../../include/thor_int8_gemm_b200.h"
#include "gemm.cuh"
#include "ptx.cuh"
#include "rows.cuh"

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(T8G_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define T8G_CHECK_CUDA(expr, what)           \
  do {                                       \
    cudaError_t e_ = (expr);                 \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// ----------------------------------------------------------------- devices
struct DeviceInfo {
  bool known = false;
  int sms = 0;
  int major = 0, minor = 0;
};
constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int current_device(int* dev, DeviceInfo* info) {
  T8G_CHECK_CUDA(cudaGetDevice(dev), "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(T8G_ERR_UNSUPPORTED, "device ordinal %d out of range", *dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[*dev];
  if (!d.known) {
    T8G_CHECK_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, *dev), "cudaDeviceGetAttribute");
    T8G_CHECK_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, *dev), "cudaDeviceGetAttribute");
    T8G_CHECK_CUDA(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, *dev), "cudaDeviceGetAttribute");
    d.known = true;
  }
  *info = d;
  if (d.major != 10 || d.minor != 0)
    return fail(T8G_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200) only", *dev,
                d.major, d.minor);
  return T8G_OK;
}

// Sets the dynamic shared-memory limit of `fn` once per device.
template <typename F>
int ensure_smem_attr(F fn, int dev, size_t bytes, std::atomic<bool>* done_per_device) {
  if (done_per_device[dev].load(std::memory_order_acquire)) return T8G_OK;
  // setting the attribute twice (two threads racing on the first call) is harmless
  T8G_CHECK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
                 "cudaFuncSetAttribute");
  done_per_device[dev].store(true, std::memory_order_release);
  return T8G_OK;
}

// ----------------------------------------------------------------- tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_2d_uncached(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t ld_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(T8G_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(T8G_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return T8G_OK;
}

// Recently encoded tensor maps of this thread: a layer calls the GEMM with the same weight,
// and often the same activation and output buffers, every step, so most maps repeat.
struct MapKey {
  const void* base;
  uint64_t inner, outer, ld_bytes;
  uint32_t box_inner, box_outer;
  int dt, sw;
  bool operator==(const MapKey& o) const {
    return base == o.base && inner == o.inner && outer == o.outer && ld_bytes == o.ld_bytes &&
           box_inner == o.box_inner && box_outer == o.box_outer && dt == o.dt && sw == o.sw;
  }
};
struct MapCache {
  static constexpr int kEntries = 16;
  MapKey key[kEntries] = {};
  CUtensorMap map[kEntries];
  bool used[kEntries] = {};
  int next = 0;
};

// 2-D row-major tensor [outer, inner] with row pitch `ld_bytes`, box [box_outer, box_inner].
int encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t ld_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  static thread_local MapCache cache;
  const MapKey key = {base, inner, outer, ld_bytes, box_inner, box_outer, static_cast<int>(dt), static_cast<int>(sw)};
  for (int i = 0; i < MapCache::kEntries; ++i) {
    if (cache.used[i] && cache.key[i] == key) {
      *m = cache.map[i];
      return T8G_OK;
    }
  }
  int rc = encode_2d_uncached(m, dt, base, inner, outer, ld_bytes, box_inner, box_outer, sw);
  if (rc) return rc;
  const int slot = cache.next;
  cache.next = (slot + 1) % MapCache::kEntries;
  cache.key[slot] = key;
  cache.map[slot] = *m;
  cache.used[slot] = true;
  return T8G_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// ----------------------------------------------------------------- GEMM
// 2-SM launch: clusters of two CTAs, grid = 2 x min(tiles, SMs / 2).
template <int IN, int OUT, int TBN = t8g::gemm::BN>
int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                     const t8g::gemm::Args& args, int dev, int sms, cudaStream_t stream) {
  using namespace t8g::gemm;
  static std::atomic<bool> attr_done[kMaxDevices] = {};
  auto kern = gemm_dequant_pair_kernel<IN, OUT, TBN>;
  int rc = ensure_smem_attr(kern, dev, pair_smem_bytes<OUT, TBN>(), attr_done);
  if (rc) return rc;
  const int64_t tiles = static_cast<int64_t>((args.M + P_BM - 1) / P_BM) * ((args.N + TBN - 1) / TBN);
  const int64_t pairs = tiles < sms / 2 ? tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = pair_smem_bytes<OUT, TBN>();
  cfg.stream = stream;
  cfg.attrs = nullptr;   // the kernel declares its cluster shape (2, 1, 1)
  cfg.numAttrs = 0;
  T8G_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, to, args), "gemm pair launch");
  return T8G_OK;
}

template <int IN, int OUT>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const t8g::gemm::Args& args,
                int dev, int sms, cudaStream_t stream) {
  using namespace t8g::gemm;
  static std::atomic<bool> attr_done[kMaxDevices] = {};
  auto kern = gemm_dequant_kernel<IN, OUT>;
  int rc = ensure_smem_attr(kern, dev, SMEM_BYTES, attr_done);
  if (rc) return rc;
  const int64_t tiles = static_cast<int64_t>((args.M + BM - 1) / BM) * ((args.N + BN - 1) / BN);
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  kern<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ta, tb, to, args);
  T8G_CHECK_CUDA(cudaGetLastError(), "gemm launch");
  return T8G_OK;
}

// K = 0: the sum over k is empty and the accumulator 0, so out = cast(((0 * xs[m]) * ws[n]) +
// bias[n]) in the epilogue's order (a NaN or infinite scale gives NaN, as it does there).
__global__ void gemm_k0_kernel(const float* xs, const float* ws, int64_t ws_numel, const void* bias, void* out,
                               int out_dtype, int64_t M, int64_t N, int64_t ld_out) {
  const int64_t total = M * N;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float v = __fmul_rn(__fmul_rn(0.0f, xs[m]), ws[ws_numel == 1 ? 0 : n]);
    if (out_dtype == T8G_OUT_BF16) {
      if (bias) v = __fadd_rn(v, __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]));
      static_cast<__nv_bfloat16*>(out)[m * ld_out + n] = __float2bfloat16_rn(v);
    } else if (out_dtype == T8G_OUT_F16) {
      if (bias) v = __fadd_rn(v, __half2float(static_cast<const __half*>(bias)[n]));
      static_cast<__half*>(out)[m * ld_out + n] = __float2half_rn(v);
    } else {
      if (bias) v = __fadd_rn(v, static_cast<const float*>(bias)[n]);
      static_cast<float*>(out)[m * ld_out + n] = v;
    }
  }
}

int gemm_entry(int in_kind, const void* x, const void* w, const float* x_scale, const float* w_scale,
               int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* out, int out_dtype, int64_t M,
               int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream_) {
  using namespace t8g::gemm;
  g_last_error[0] = '\0';
  if (M < 0 || N < 0 || K < 0) return fail(T8G_ERR_INVALID_ARGUMENT, "bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31))
    return fail(T8G_ERR_UNSUPPORTED, "M, N and K must each be below 2^31");
  if (out_dtype < T8G_OUT_BF16 || out_dtype > T8G_OUT_F32) return fail(T8G_ERR_INVALID_ARGUMENT, "unknown out_dtype %d", out_dtype);
  if (M == 0 || N == 0) return T8G_OK;
  if (K == 0) {
    // an empty sum: no operand is read, the epilogue alone runs
    if (!x_scale || !w_scale || !out) return fail(T8G_ERR_INVALID_ARGUMENT, "null operand pointer");
    if (w_scale_numel != 1 && w_scale_numel != N)
      return fail(T8G_ERR_INVALID_ARGUMENT, "w_scale numel %lld is neither 1 nor N=%lld", (long long)w_scale_numel, (long long)N);
    if (bias_numel != 0 && bias_numel != N)
      return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel %lld is neither 0 nor N=%lld", (long long)bias_numel, (long long)N);
    if (bias_numel == N && !bias) return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel is N but bias is null");
    if (ld_out < N) return fail(T8G_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
    const int64_t total = M * N;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 8));
    gemm_k0_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream_)>>>(
        x_scale, w_scale, w_scale_numel, bias_numel ? bias : nullptr, out, out_dtype, M, N, ld_out);
    T8G_CHECK_CUDA(cudaGetLastError(), "gemm (K = 0) launch");
    return T8G_OK;
  }
  if (!x || !w || !x_scale || !w_scale || !out) return fail(T8G_ERR_INVALID_ARGUMENT, "null operand pointer");
  if (w_scale_numel != 1 && w_scale_numel != N)
    return fail(T8G_ERR_INVALID_ARGUMENT, "w_scale numel %lld is neither 1 nor N=%lld", (long long)w_scale_numel, (long long)N);
  if (bias_numel != 0 && bias_numel != N)
    return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel %lld is neither 0 nor N=%lld", (long long)bias_numel, (long long)N);
  if (bias_numel == N && !bias) return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel is N but bias is null");
  const int esz = out_dtype == T8G_OUT_F32 ? 4 : 2;
  if (ld_x < K || ld_w < K || ld_out < N) return fail(T8G_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
  if (ld_x % 16 || ld_w % 16 || (ld_out * esz) % 16)
    return fail(T8G_ERR_INVALID_ARGUMENT, "row strides must be multiples of 16 bytes (ld_x=%lld ld_w=%lld ld_out=%lld)",
                (long long)ld_x, (long long)ld_w, (long long)ld_out);
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16))
    return fail(T8G_ERR_INVALID_ARGUMENT, "x, w and out must be 16-byte aligned");
  if (!aligned(x_scale, 4) || !aligned(w_scale, 4)) return fail(T8G_ERR_INVALID_ARGUMENT, "scales must be 4-byte aligned");

  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc) return rc;

  // The 2-SM kernel (CTA pairs, 256-row tiles) runs whenever there is more than one
  // 128-row block or narrow tiles apply; T8G_GEMM_SM=1 in the environment forces the 1-SM
  // kernel.
  const char* sm_env = getenv("T8G_GEMM_SM");
  const bool force_1sm = sm_env && sm_env[0] == '1';
  // Tile width of the 2-SM kernel (2-byte outputs): 256 columns, or 128 / 64 when 256-wide
  // tiles would leave more than half of the CTA pairs idle (small M): narrower tiles put more
  // SMs on the problem, each with a shorter tile.  Otherwise 256: a narrower tile streams its
  // activation panel for fewer output columns, and measured per tile at 0.81x (192 columns)
  // and 0.55x (128) the 256-column rate at M = 8192 and 32768 -- more than any fuller last
  // wave returns (M = 8192, N = 3072: 2678 TOPS at 256, 2446 at 192, 1685 at 128, L2-warm).
  // T8G_GEMM_TBN=256|128|64 forces a width (tuning).
  const int64_t pairs_avail = info.sms / 2;
  const int64_t tiles_m = (M + P_BM - 1) / P_BM;
  int tbn = BN;
  if (esz == 2) {
    while (tbn > 64 && tiles_m * ((N + tbn - 1) / tbn) * 2 < pairs_avail) tbn /= 2;
    if (const char* force = getenv("T8G_GEMM_TBN")) {
      const int f = atoi(force);
      if (f == 256 || f == 128 || f == 64) tbn = f;
    }
  }
  const bool pair = (M > BM || tbn < BN) && !force_1sm;
  const CUtensorMapDataType in_dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap ta, tb, to;
  rc = encode_2d(&ta, in_dt, x, K, M, ld_x, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&tb, in_dt, w, K, N, ld_w, BK, pair ? static_cast<uint32_t>(tbn / 2) : BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const CUtensorMapDataType out_dt = out_dtype == T8G_OUT_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : out_dtype == T8G_OUT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  // the 2-SM kernel stores 2-byte outputs in 32 x 64 boxes (128-byte rows), the 1-SM kernel
  // and fp32 outputs in 32 x 32 boxes
  const bool box64 = pair && esz == 2;
  rc = encode_2d(&to, out_dt, out, N, M, ld_out * esz, box64 ? 64 : EPI_COLS, 32,
                 esz == 2 && !box64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  Args args = {};
  args.xs = x_scale;
  args.ws = w_scale;
  args.bias = bias_numel ? bias : nullptr;
  args.ws_stride = w_scale_numel == 1 ? 0 : 1;
  args.vec_ok = aligned(w_scale, 16) && (bias_numel == 0 || aligned(bias, 16));
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  if (pair && tbn != BN) {
    // narrow tiles (2-byte outputs only)
    const bool f16 = out_dtype == T8G_OUT_F16;
    if (in_kind == kInI8) {
      if (tbn == 128)
        return f16 ? launch_gemm_pair<kInI8, kOutF16, 128>(ta, tb, to, args, dev, info.sms, st)
                   : launch_gemm_pair<kInI8, kOutBF16, 128>(ta, tb, to, args, dev, info.sms, st);
      return f16 ? launch_gemm_pair<kInI8, kOutF16, 64>(ta, tb, to, args, dev, info.sms, st)
                 : launch_gemm_pair<kInI8, kOutBF16, 64>(ta, tb, to, args, dev, info.sms, st);
    }
    if (tbn == 128)
      return f16 ? launch_gemm_pair<kInE4M3, kOutF16, 128>(ta, tb, to, args, dev, info.sms, st)
                 : launch_gemm_pair<kInE4M3, kOutBF16, 128>(ta, tb, to, args, dev, info.sms, st);
    return f16 ? launch_gemm_pair<kInE4M3, kOutF16, 64>(ta, tb, to, args, dev, info.sms, st)
               : launch_gemm_pair<kInE4M3, kOutBF16, 64>(ta, tb, to, args, dev, info.sms, st);
  }
  if (pair) {
    if (in_kind == kInI8) {
      switch (out_dtype) {
        case T8G_OUT_BF16: return launch_gemm_pair<kInI8, kOutBF16>(ta, tb, to, args, dev, info.sms, st);
        case T8G_OUT_F16: return launch_gemm_pair<kInI8, kOutF16>(ta, tb, to, args, dev, info.sms, st);
        default: return launch_gemm_pair<kInI8, kOutF32>(ta, tb, to, args, dev, info.sms, st);
      }
    }
    switch (out_dtype) {
      case T8G_OUT_BF16: return launch_gemm_pair<kInE4M3, kOutBF16>(ta, tb, to, args, dev, info.sms, st);
      case T8G_OUT_F16: return launch_gemm_pair<kInE4M3, kOutF16>(ta, tb, to, args, dev, info.sms, st);
      default: return launch_gemm_pair<kInE4M3, kOutF32>(ta, tb, to, args, dev, info.sms, st);
    }
  }
  if (in_kind == kInI8) {
    switch (out_dtype) {
      case T8G_OUT_BF16: return launch_gemm<kInI8, kOutBF16>(ta, tb, to, args, dev, info.sms, st);
      case T8G_OUT_F16: return launch_gemm<kInI8, kOutF16>(ta, tb, to, args, dev, info.sms, st);
      default: return launch_gemm<kInI8, kOutF32>(ta, tb, to, args, dev, info.sms, st);
    }
  }
  switch (out_dtype) {
    case T8G_OUT_BF16: return launch_gemm<kInE4M3, kOutBF16>(ta, tb, to, args, dev, info.sms, st);
    case T8G_OUT_F16: return launch_gemm<kInE4M3, kOutF16>(ta, tb, to, args, dev, info.sms, st);
    default: return launch_gemm<kInE4M3, kOutF32>(ta, tb, to, args, dev, info.sms, st);
  }
}

// GEMM with the SwiGLU epilogue: w holds the fc1 weight with gate and up rows interleaved in
// 128-row blocks (2F rows), act receives silu(gate) * up as bf16 [M, F].  Always the 2-SM
// kernel (its 256-column tiles pair 128 gate with 128 up columns).
int gemm_swiglu_entry(int in_kind, const void* x, const void* w, const float* x_scale, const float* w_scale,
                      int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t M, int64_t F,
                      int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_act, void* stream_,
                      float* row_amax = nullptr) {
  using namespace t8g::gemm;
  g_last_error[0] = '\0';
  if (M < 0 || F < 0 || K < 1) return fail(T8G_ERR_INVALID_ARGUMENT, "bad sizes M=%lld F=%lld K=%lld", (long long)M, (long long)F, (long long)K);
  if (F % 128) return fail(T8G_ERR_INVALID_ARGUMENT, "F=%lld must be a multiple of 128", (long long)F);
  const int64_t N = 2 * F;
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31))
    return fail(T8G_ERR_UNSUPPORTED, "M, 2F and K must each be below 2^31");
  if (M == 0 || F == 0) return T8G_OK;
  if (!x || !w || !x_scale || !w_scale || !act) return fail(T8G_ERR_INVALID_ARGUMENT, "null operand pointer");
  if (w_scale_numel != 1 && w_scale_numel != N)
    return fail(T8G_ERR_INVALID_ARGUMENT, "w_scale numel %lld is neither 1 nor 2F=%lld", (long long)w_scale_numel, (long long)N);
  if (bias_numel != 0 && bias_numel != N)
    return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel %lld is neither 0 nor 2F=%lld", (long long)bias_numel, (long long)N);
  if (bias_numel == N && !bias) return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel is 2F but bias is null");
  if (ld_x < K || ld_w < K || ld_act < F) return fail(T8G_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
  if (ld_x % 16 || ld_w % 16 || (ld_act * 2) % 16)
    return fail(T8G_ERR_INVALID_ARGUMENT, "row strides must be multiples of 16 bytes");
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(act, 16))
    return fail(T8G_ERR_INVALID_ARGUMENT, "x, w and act must be 16-byte aligned");
  if (!aligned(x_scale, 4) || !aligned(w_scale, 4)) return fail(T8G_ERR_INVALID_ARGUMENT, "scales must be 4-byte aligned");
  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc) return rc;
  CUtensorMap ta, tb, to;
  rc = encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x, K, M, ld_x, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K, N, ld_w, BK, P_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, act, F, M, ld_act * 2, EPI_COLS, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  Args args = {};
  args.xs = x_scale;
  args.ws = w_scale;
  args.bias = bias_numel ? bias : nullptr;
  args.ws_stride = w_scale_numel == 1 ? 0 : 1;
  args.vec_ok = aligned(w_scale, 16) && (bias_numel == 0 || aligned(bias, 16));
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.row_amax = row_amax;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  if (row_amax) T8G_CHECK_CUDA(cudaMemsetAsync(row_amax, 0, static_cast<size_t>(M) * sizeof(float), st),
                               "cudaMemsetAsync(row_amax)");
  if (in_kind == kInI8) return launch_gemm_pair<kInI8, kOutSwiglu>(ta, tb, to, args, dev, info.sms, st);
  return launch_gemm_pair<kInE4M3, kOutSwiglu>(ta, tb, to, args, dev, info.sms, st);
}

// GEMM whose epilogue applies the DiT block's gated residual: out = bf16(res + bf16(gate[g] *
// y)) with y the bf16 dequantised GEMM output and g = gate_index[m] (or m / rows_per_gate).
// bf16 output only; out may be res itself (each element is read before it is stored).
// Always the 2-SM kernel.
int gemm_gated_entry(int in_kind, const void* x, const void* w, const float* x_scale, const float* w_scale,
                     int64_t w_scale_numel, const void* bias, int64_t bias_numel, const void* res, int64_t ld_res,
                     const void* gate, int64_t ld_gate, const int32_t* gate_index, int64_t rows_per_gate, void* out,
                     int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream_) {
  using namespace t8g::gemm;
  g_last_error[0] = '\0';
  if (M < 0 || N < 0 || K < 1) return fail(T8G_ERR_INVALID_ARGUMENT, "bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31))
    return fail(T8G_ERR_UNSUPPORTED, "M, N and K must each be below 2^31");
  if (N % 8) return fail(T8G_ERR_INVALID_ARGUMENT, "N=%lld must be a multiple of 8", (long long)N);
  if (M == 0 || N == 0) return T8G_OK;
  if (!x || !w || !x_scale || !w_scale || !out || !res || !gate)
    return fail(T8G_ERR_INVALID_ARGUMENT, "null operand pointer");
  if (!gate_index && rows_per_gate < 1)
    return fail(T8G_ERR_INVALID_ARGUMENT, "rows_per_gate must be positive when gate_index is null");
  if (w_scale_numel != 1 && w_scale_numel != N)
    return fail(T8G_ERR_INVALID_ARGUMENT, "w_scale numel %lld is neither 1 nor N=%lld", (long long)w_scale_numel, (long long)N);
  if (bias_numel != 0 && bias_numel != N)
    return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel %lld is neither 0 nor N=%lld", (long long)bias_numel, (long long)N);
  if (bias_numel == N && !bias) return fail(T8G_ERR_INVALID_ARGUMENT, "bias numel is N but bias is null");
  if (ld_x < K || ld_w < K || ld_out < N || ld_res < N || ld_gate < N)
    return fail(T8G_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
  if (ld_x % 16 || ld_w % 16 || ld_out % 8 || ld_res % 8 || ld_gate % 8)
    return fail(T8G_ERR_INVALID_ARGUMENT, "row strides must be multiples of 16 bytes");
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16) || !aligned(res, 16) || !aligned(gate, 16))
    return fail(T8G_ERR_INVALID_ARGUMENT, "x, w, out, res and gate must be 16-byte aligned");
  if (!aligned(x_scale, 4) || !aligned(w_scale, 4) || !aligned(gate_index, 4))
    return fail(T8G_ERR_INVALID_ARGUMENT, "scales and gate_index must be 4-byte aligned");
  if (out != res) {
    // out and res are either the same matrix or disjoint
    const uintptr_t o0 = reinterpret_cast<uintptr_t>(out), r0 = reinterpret_cast<uintptr_t>(res);
    const uintptr_t o1 = o0 + static_cast<uintptr_t>(((M - 1) * ld_out + N) * 2);
    const uintptr_t r1 = r0 + static_cast<uintptr_t>(((M - 1) * ld_res + N) * 2);
    if (o0 < r1 && r0 < o1) return fail(T8G_ERR_INVALID_ARGUMENT, "out overlaps res without being res");
  } else if (ld_out != ld_res) {
    return fail(T8G_ERR_INVALID_ARGUMENT, "out is res but ld_out != ld_res");
  }
  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc) return rc;
  CUtensorMap ta, tb, to;
  rc = encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x, K, M, ld_x, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K, N, ld_w, BK, P_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, out, N, M, ld_out * 2, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Args args = {};
  args.xs = x_scale;
  args.ws = w_scale;
  args.bias = bias_numel ? bias : nullptr;
  args.ws_stride = w_scale_numel == 1 ? 0 : 1;
  args.vec_ok = aligned(w_scale, 16) && (bias_numel == 0 || aligned(bias, 16));
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.res = res;
  args.gate = gate;
  args.gate_index = gate_index;
  args.ld_res = ld_res;
  args.ld_gate = ld_gate;
  args.rows_per_gate = gate_index ? 1 : rows_per_gate;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  if (in_kind == kInI8) return launch_gemm_pair<kInI8, kOutGated>(ta, tb, to, args, dev, info.sms, st);
  return launch_gemm_pair<kInE4M3, kOutGated>(ta, tb, to, args, dev, info.sms, st);
}

// ----------------------------------------------------------------- row kernels
// Row-group shape: V = max(3, ceil(nvec / 512)) 16-byte vectors per thread and
// T = 32 * ceil(nvec / (32 V)) threads (nvec = D / 8); kernels are unrolled for V = 3
// and 4 and generic beyond (kernel parameter 0).  The oracle restates this rule.
struct RowShape {
  int T;
  int V;   // 3, 4, or 0 for the generic kernel
};

RowShape row_shape(int64_t D) {
  const int64_t nvec = (D + 7) / 8;
  int64_t v = (nvec + 511) / 512;
  if (v < 3) v = 3;
  int64_t t = 32 * ((nvec + 32 * v - 1) / (32 * v));
  if (t < 32) t = 32;
  RowShape r;
  r.T = static_cast<int>(t);
  r.V = v <= 4 ? static_cast<int>(v) : 0;
  return r;
}

// Row-group shape of the SwiGLU kernels, whose only reduction is a max (any order):
// V = max(kSwigluVecs, ceil(nvec / 1024)) vectors per thread and T = 32 * ceil(nvec /
// (32 V)) <= 1024 threads; V in {2, 3, 6} runs an unrolled kernel, longer rows the
// generic one.
constexpr int kSwigluVecs = 3;

RowShape swiglu_shape(int64_t F) {
  const int64_t nvec = (F + 7) / 8;
  int64_t v = (nvec + 1023) / 1024;
  if (v < kSwigluVecs) v = kSwigluVecs;
  int64_t t = 32 * ((nvec + 32 * v - 1) / (32 * v));
  if (t < 32) t = 32;
  RowShape r;
  r.T = static_cast<int>(t);
  r.V = (v == 2 || v == 3 || v == 6) ? static_cast<int>(v) : 0;
  return r;
}

// Ring geometry of a row kernel: `parts` operand rows of D bf16 per slot (the depth
// is set at launch).
t8g::rows::RingGeom ring_geom(int64_t D, int parts, bool padded = false) {
  t8g::rows::RingGeom g;
  g.parts = parts;
  g.part_bytes = static_cast<uint32_t>(D * 2);
  g.padded = padded ? 1 : 0;
  const uint32_t part_slot = padded ? t8g::rows::padded_row_bytes(g.part_bytes) : g.part_bytes;
  g.slot_bytes = (static_cast<uint32_t>(parts) * part_slot + 127u) & ~127u;
  g.stages = 2;
  return g;
}

size_t ring_smem(const t8g::rows::RingGeom& g) { return t8g::rows::ring_bytes(g); }

constexpr size_t kRowSmemLimit = 226 * 1024;

int check_row_shape(const char* what, int64_t S, int64_t D, int quant_kind, int parts) {
  if (S < 0 || D < 0) return fail(T8G_ERR_INVALID_ARGUMENT, "%s: negative size", what);
  if (D % 8) return fail(T8G_ERR_INVALID_ARGUMENT, "%s: row length %lld is not a multiple of 8", what, (long long)D);
  const int64_t dmax = parts == 1 ? 49152 : 24576;
  if (D > dmax) return fail(T8G_ERR_UNSUPPORTED, "%s: row length %lld exceeds %lld", what, (long long)D, (long long)dmax);
  if (quant_kind != T8G_QUANT_INT8 && quant_kind != T8G_QUANT_FP8_E4M3)
    return fail(T8G_ERR_INVALID_ARGUMENT, "%s: unknown quant_kind %d", what, quant_kind);
  if (S >= (int64_t(1) << 40)) return fail(T8G_ERR_UNSUPPORTED, "%s: too many rows", what);
  return T8G_OK;
}

int check_bf16_matrix(const char* what, const void* p, int64_t ld, int64_t D, bool required) {
  if (!p) return required ? fail(T8G_ERR_INVALID_ARGUMENT, "%s is null", what) : T8G_OK;
  if (!aligned(p, 16)) return fail(T8G_ERR_INVALID_ARGUMENT, "%s must be 16-byte aligned", what);
  if (ld < D || ld % 8) return fail(T8G_ERR_INVALID_ARGUMENT, "%s row stride %lld must be >= D and a multiple of 8", what, (long long)ld);
  return T8G_OK;
}

int check_q(const void* q, int64_t ld_q, int64_t D) {
  if (!q) return fail(T8G_ERR_INVALID_ARGUMENT, "q is null");
  if (!aligned(q, 8)) return fail(T8G_ERR_INVALID_ARGUMENT, "q must be 8-byte aligned");
  if (ld_q < D || ld_q % 8) return fail(T8G_ERR_INVALID_ARGUMENT, "q row stride must be >= D and a multiple of 8");
  return T8G_OK;
}

// Launch a persistent row kernel.  The ring depth is chosen from the occupancy the
// kernel gets: at most 16 CTAs per SM share ~216 KB of shared memory, each taking as
// many slots as fit (2..16), so 150-200 KB of rows are in flight per SM.  Grid =
// min(rows, SMs x resident CTAs).
// Raise a row kernel's dynamic shared-memory limit to kRowAttrBytes (the per-CTA maximum),
// once per kernel and device.
constexpr size_t kRowAttrBytes = 227 * 1024;

template <typename K>
int ensure_row_attr(K kern, int dev) {
  static std::mutex mu;
  static const void* attr_done[kMaxDevices][64] = {};
  std::lock_guard<std::mutex> lk(mu);
  int slot = 0;
  for (; slot < 64 && attr_done[dev][slot]; ++slot)
    if (attr_done[dev][slot] == reinterpret_cast<const void*>(kern)) return T8G_OK;
  T8G_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRowAttrBytes),
                 "cudaFuncSetAttribute(row kernel)");
  if (slot < 64) attr_done[dev][slot] = reinterpret_cast<const void*>(kern);
  return T8G_OK;
}

template <typename K, typename A>
int launch_rows(K kern, int T, const A& args, t8g::rows::RingGeom g, int64_t rows, int dev, int sms, cudaStream_t st,
                const char* what) {
  using t8g::rows::kMaxStages;
  using t8g::rows::kRingHeader;
  int rc = ensure_row_attr(kern, dev);
  if (rc) return rc;
  g.stages = 2;
  if (ring_smem(g) > kRowSmemLimit) return fail(T8G_ERR_UNSUPPORTED, "%s: row too long for the shared-memory ring", what);
  int occ = 0;
  T8G_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, T, ring_smem(g)), "occupancy query");
  const int n = occ < 1 ? 1 : occ > 16 ? 16 : occ;
  const size_t per_cta = (216 * 1024) / n;
  int stages = static_cast<int>((per_cta > kRingHeader ? per_cta - kRingHeader : 0) / g.slot_bytes);
  stages = stages < 2 ? 2 : stages > kMaxStages ? kMaxStages : stages;
  while (stages > 2 && ring_smem(t8g::rows::RingGeom{stages, g.slot_bytes, g.part_bytes, g.parts, g.padded}) > kRowSmemLimit)
    --stages;
  g.stages = stages;
  const size_t smem = ring_smem(g);
  T8G_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, T, smem), "occupancy query");
  if (occ < 1) occ = 1;
  const int64_t cap = static_cast<int64_t>(sms) * occ;
  const unsigned grid = static_cast<unsigned>(rows < cap ? rows : cap);
  kern<<<grid, T, smem, st>>>(args, g);
  T8G_CHECK_CUDA(cudaGetLastError(), what);
  return T8G_OK;
}

// Launch a warp-ring row kernel (one row per warp): kWarpStages slots per warp and as
// many warps per CTA as the shared-memory budget holds (216 KB by default; at most 32), one
// CTA per SM.
constexpr int kWarpStages = 2;

// `tail_bytes` of shared memory follow the rings (a kernel's own table); with
// `contiguous`, CTA b owns rows [b * cta_rows, (b + 1) * cta_rows) instead of a round-robin
// share.
struct WarpLaunch {
  int max_warps = t8g::rows::kWarpMaxWarps;
  size_t tail_bytes = 0;
  bool contiguous = false;
  bool padded = false;   // rows in 256-byte pieces at the padded pitch (reference-order reduction)
  size_t smem_budget = 216 * 1024;   // rings + tail
};

template <typename K, typename A, typename... Extra>
int launch_warp_rows(K kern, const A& args, uint32_t row_bytes, int64_t rows, int dev, int sms, cudaStream_t st,
                     const WarpLaunch& opt, const char* what, Extra... extra) {
  using namespace t8g::rows;
  int rc = ensure_row_attr(kern, dev);
  if (rc) return rc;
  WarpRingGeom g;
  g.row_bytes = row_bytes;
  g.padded = opt.padded ? 1 : 0;
  g.slot_bytes = ((opt.padded ? padded_row_bytes(row_bytes) : row_bytes) + 127u) & ~127u;
  g.stages = kWarpStages;
  const int64_t budget = static_cast<int64_t>(opt.smem_budget - kWarpRingHeader) - static_cast<int64_t>(opt.tail_bytes);
  int64_t warps = budget / (static_cast<int64_t>(g.stages) * g.slot_bytes);
  if (warps > opt.max_warps) warps = opt.max_warps;
  if (warps < 1) return fail(T8G_ERR_UNSUPPORTED, "%s: row too long for a warp ring", what);
  int64_t grid = (rows + warps - 1) / warps;
  if (grid > sms) grid = sms;
  g.cta_rows = opt.contiguous ? (rows + grid - 1) / grid : 0;
  const size_t smem = kWarpRingHeader + static_cast<size_t>(warps) * g.stages * g.slot_bytes + opt.tail_bytes;
  kern<<<static_cast<unsigned>(grid), static_cast<unsigned>(32 * warps), smem, st>>>(args, g, extra...);
  T8G_CHECK_CUDA(cudaGetLastError(), what);
  return T8G_OK;
}

// Launch the SwiGLU kernel: one CTA per SM holding the 32 KB sigmoid table and up to eight
// row groups of T threads (at most 1024 threads), each with a ring of as many slots (>= 2)
// as the rest of the CTA's shared memory holds.
template <typename K>
int launch_swiglu(K kern, int T, const t8g::rows::SwigluArgs& args, t8g::rows::RingGeom g, int64_t rows, int dev,
                  int sms, cudaStream_t st, const char* what) {
  using namespace t8g::rows;
  int rc = ensure_row_attr(kern, dev);
  if (rc) return rc;
  const size_t avail = kRowAttrBytes - t8g::kSigmoidBytes;
  int groups = 1024 / T;
  if (groups > 8) groups = 8;
  if (groups < 1) groups = 1;
  auto group_fits = [&](int n, int stages) {
    return static_cast<size_t>(n) * (kRingHeader + static_cast<size_t>(stages) * g.slot_bytes) <= avail;
  };
  while (groups > 1 && !group_fits(groups, 2)) --groups;
  if (!group_fits(groups, 2)) return fail(T8G_ERR_UNSUPPORTED, "%s: row too long for the shared-memory ring", what);
  int stages = 2;
  while (stages < kMaxStages && group_fits(groups, stages + 1)) ++stages;
  g.stages = stages;
  const size_t smem = t8g::kSigmoidBytes + static_cast<size_t>(groups) * ring_bytes(g);
  const int threads = groups * T;
  int occ = 0;
  T8G_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem), "occupancy query");
  if (occ < 1) occ = 1;
  const int64_t want = (rows + groups - 1) / groups;
  const int64_t cap = static_cast<int64_t>(sms) * occ;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  kern<<<grid, threads, smem, st>>>(args, g, T);
  T8G_CHECK_CUDA(cudaGetLastError(), what);
  return T8G_OK;
}

// Rows of D = 256 NV elements with these NV run the register-resident warp kernels
// (at most kRegWarps warps per CTA: their launch bound).
constexpr int kRegWarps = 16;

int reg_nv(int64_t D) {
  if (D % 256) return 0;
  const int64_t nv = D / 256;
  return (nv == 4 || nv == 6 || nv == 8 || nv == 12 || nv == 16) ? static_cast<int>(nv) : 0;
}

#define T8G_DISPATCH_NV(nv, CALL)                      \
  switch (nv) {                                        \
    case 4: { constexpr int NV = 4; CALL; break; }     \
    case 6: { constexpr int NV = 6; CALL; break; }     \
    case 8: { constexpr int NV = 8; CALL; break; }     \
    case 12: { constexpr int NV = 12; CALL; break; }   \
    default: { constexpr int NV = 16; CALL; break; }   \
  }

#define T8G_DISPATCH_SW(v, CALL)                       \
  switch (v) {                                         \
    case 2: { constexpr int V = 2; CALL; break; }      \
    case 3: { constexpr int V = 3; CALL; break; }      \
    case 6: { constexpr int V = 6; CALL; break; }      \
    default: { constexpr int V = 0; CALL; break; }     \
  }

#define T8G_DISPATCH_V(v, CALL)                        \
  switch (v) {                                         \
    case 3: { constexpr int V = 3; CALL; break; }      \
    case 4: { constexpr int V = 4; CALL; break; }      \
    default: { constexpr int V = 0; CALL; break; }     \
  }

int launch_checked(const char* what) {
  T8G_CHECK_CUDA(cudaGetLastError(), what);
  return T8G_OK;
}

int launch_quant_given(const t8g::rows::QuantGivenArgs& b, int quant_kind, int sms, cudaStream_t st) {
  using namespace t8g::rows;
  // 8 CTAs of 256 threads per SM; the kernel strides over vectors (contiguous rows) or rows
  const int64_t vecs = b.S * (b.D / 8);
  const int64_t want = (vecs + 255) / 256;
  const unsigned grid = static_cast<unsigned>(want < int64_t(sms) * 8 ? want : int64_t(sms) * 8);
  if (quant_kind == T8G_QUANT_FP8_E4M3)
    quant_given_amax_kernel<kQuantFp8><<<grid, 256, 0, st>>>(b);
  else
    quant_given_amax_kernel<kQuantInt8><<<grid, 256, 0, st>>>(b);
  return launch_checked("quant phase B launch");
}

// The tensorwise forms on an empty tensor: amax = 0, so the scale is the floor 1e-12, as the
// reference's amax and quant kernels give for no elements (src/ck_fused_mod_norm_quant.py:
// 92-111); phase B with no rows writes just the scale.
int empty_tensorwise(float* amax, float* scale_out, int quant_kind, void* stream_) {
  using namespace t8g::rows;
  if (!amax) return fail(T8G_ERR_INVALID_ARGUMENT, "amax scratch word is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  T8G_CHECK_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st), "cudaMemsetAsync(amax)");
  QuantGivenArgs b{};
  b.amax = amax;
  b.scale_out = scale_out;
  b.S = 0;
  b.D = 8;
  if (quant_kind == T8G_QUANT_FP8_E4M3)
    quant_given_amax_kernel<kQuantFp8><<<1, 32, 0, st>>>(b);
  else
    quant_given_amax_kernel<kQuantInt8><<<1, 32, 0, st>>>(b);
  return launch_checked("empty tensorwise scale");
}

int rms_common(bool tensorwise, const void* x, int64_t ld_x, const void* w, const void* shift, const void* scale,
               int64_t ld_mod, const int32_t* mod_index, int64_t rows_per_mod, int scale_is_multiplier, float eps,
               void* q, int64_t ld_q, float* q_scale, void* h, int64_t ld_h, void* res, int64_t ld_res,
               float* amax, float* scale_out, int64_t S, int64_t D, int quant_kind, void* stream_) {
  using namespace t8g::rows;
  g_last_error[0] = '\0';
  int rc = check_row_shape("rms_mod_quant", S, D, quant_kind, 1);
  if (rc) return rc;
  if (S == 0 || D == 0) return tensorwise ? empty_tensorwise(amax, scale_out, quant_kind, stream_) : T8G_OK;
  if ((rc = check_bf16_matrix("x", x, ld_x, D, true))) return rc;
  if ((rc = check_bf16_matrix("shift", shift, ld_mod, D, true))) return rc;
  if ((rc = check_bf16_matrix("scale", scale, ld_mod, D, true))) return rc;
  if (w && !aligned(w, 16)) return fail(T8G_ERR_INVALID_ARGUMENT, "w must be 16-byte aligned");
  if ((rc = check_bf16_matrix("h", h, ld_h, D, tensorwise))) return rc;
  if ((rc = check_bf16_matrix("res", res, ld_res, D, false))) return rc;
  if ((rc = check_q(q, ld_q, D))) return rc;
  if (!mod_index && rows_per_mod < 1) return fail(T8G_ERR_INVALID_ARGUMENT, "rows_per_mod must be >= 1 without mod_index");
  if (tensorwise && !amax) return fail(T8G_ERR_INVALID_ARGUMENT, "amax scratch word is null");
  if (!tensorwise && !q_scale) return fail(T8G_ERR_INVALID_ARGUMENT, "q_scale is null");
  int dev;
  DeviceInfo info;
  if ((rc = current_device(&dev, &info))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);

  RmsArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ld_x = ld_x;
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.shift = static_cast<const __nv_bfloat16*>(shift);
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.ld_mod = ld_mod;
  a.mod_index = mod_index;
  a.rows_per_mod = rows_per_mod < 1 ? 1 : rows_per_mod;
  a.scale_is_multiplier = scale_is_multiplier;
  a.eps = eps;
  a.q = q;
  a.ld_q = ld_q;
  a.q_scale = q_scale;
  a.h = static_cast<__nv_bfloat16*>(h);
  a.ld_h = ld_h;
  a.res = static_cast<__nv_bfloat16*>(res);
  a.ld_res = ld_res;
  a.amax = amax;
  a.S = S;
  a.D = static_cast<int>(D);
  const RowShape rsh = row_shape(D);
  const RingGeom g = ring_geom(D, 1);
  const uint32_t row_bytes = static_cast<uint32_t>(2 * D);
  const bool warp_rows = row_bytes <= kWarpRowMaxBytes;
  const int nv = reg_nv(D);
  const bool simple = !w && !h && !res && !mod_index && !scale_is_multiplier;
  WarpLaunch reg_launch;
  reg_launch.max_warps = kRegWarps;
  if (tensorwise) {
    // phase A sums the squares in the reference's order (rows in the padded layout)
    T8G_CHECK_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st), "cudaMemsetAsync(amax)");
    if (nv) {
      // the block's modulation row and the norm weight cached per CTA
      WarpLaunch o = reg_launch;
      o.padded = true;
      o.contiguous = true;
      o.tail_bytes = static_cast<size_t>((w ? 8 : 6) * D);   // fp32 multiplier + bf16 shift (+ bf16 weight)
      o.smem_budget = kRowSmemLimit;
      if (w) {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_tw_cached_kernel<NV, true>, a, row_bytes, S, dev, info.sms,
                                                  st, o, "rms_mod phase A"));
      } else {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_tw_cached_kernel<NV, false>, a, row_bytes, S, dev, info.sms,
                                                  st, o, "rms_mod phase A"));
      }
    } else if (warp_rows) {
      WarpLaunch o;
      o.padded = true;
      const int64_t nch = (D + kRefBlock - 1) / kRefBlock;   // 1..4 for rows of at most 16 KB
      switch (nch) {
        case 1: rc = launch_warp_rows(rms_mod_tw_warp_kernel<1>, a, row_bytes, S, dev, info.sms, st, o, "rms_mod phase A"); break;
        case 2: rc = launch_warp_rows(rms_mod_tw_warp_kernel<2>, a, row_bytes, S, dev, info.sms, st, o, "rms_mod phase A"); break;
        case 3: rc = launch_warp_rows(rms_mod_tw_warp_kernel<3>, a, row_bytes, S, dev, info.sms, st, o, "rms_mod phase A"); break;
        default: rc = launch_warp_rows(rms_mod_tw_warp_kernel<4>, a, row_bytes, S, dev, info.sms, st, o, "rms_mod phase A"); break;
      }
    } else {
      rc = launch_rows(rms_mod_tw_cta_kernel, rsh.T, a, ring_geom(D, 1, true), S, dev, info.sms, st,
                       "rms_mod phase A");
    }
    if (rc) return rc;
    QuantGivenArgs b;
    b.h = a.h;
    b.ld_h = ld_h;
    b.q = q;
    b.ld_q = ld_q;
    b.amax = amax;
    b.scale_out = scale_out;
    b.S = S;
    b.D = a.D;
    return launch_quant_given(b, quant_kind, info.sms, st);
  }
  if (nv) {
    const bool fp8 = quant_kind == T8G_QUANT_FP8_E4M3;
    if (simple) {
      WarpLaunch o = reg_launch;
      o.tail_bytes = static_cast<size_t>(6 * D);   // fp32 multiplier + bf16 shift of one batch element
      o.contiguous = true;
      if (fp8) {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_simple_kernel<NV, kQuantFp8>, a, row_bytes, S, dev,
                                                  info.sms, st, o, "rms_mod_quant"));
      } else {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_simple_kernel<NV, kQuantInt8>, a, row_bytes, S, dev,
                                                  info.sms, st, o, "rms_mod_quant"));
      }
    } else {
      // every other option: the block's modulation row and the norm weight cached per CTA
      WarpLaunch o = reg_launch;
      o.contiguous = true;
      o.tail_bytes = static_cast<size_t>((w ? 8 : 6) * D);   // fp32 multiplier + bf16 shift (+ bf16 weight)
      o.smem_budget = kRowSmemLimit;
      if (fp8 && w) {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_cached_kernel<NV, kQuantFp8, true>, a, row_bytes, S, dev,
                                                  info.sms, st, o, "rms_mod_quant"));
      } else if (fp8) {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_cached_kernel<NV, kQuantFp8, false>, a, row_bytes, S, dev,
                                                  info.sms, st, o, "rms_mod_quant"));
      } else if (w) {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_cached_kernel<NV, kQuantInt8, true>, a, row_bytes, S, dev,
                                                  info.sms, st, o, "rms_mod_quant"));
      } else {
        T8G_DISPATCH_NV(nv, rc = launch_warp_rows(rms_mod_cached_kernel<NV, kQuantInt8, false>, a, row_bytes, S, dev,
                                                  info.sms, st, o, "rms_mod_quant"));
      }
    }
    return rc;
  }
  if (warp_rows) {
    if (quant_kind == T8G_QUANT_FP8_E4M3)
      return launch_warp_rows(rms_mod_warp_kernel<kQuantFp8>, a, row_bytes, S, dev, info.sms, st, WarpLaunch{}, "rms_mod_quant", rsh.T);
    return launch_warp_rows(rms_mod_warp_kernel<kQuantInt8>, a, row_bytes, S, dev, info.sms, st, WarpLaunch{}, "rms_mod_quant", rsh.T);
  }
  if (quant_kind == T8G_QUANT_FP8_E4M3) {
    T8G_DISPATCH_V(rsh.V, rc = launch_rows(rms_mod_kernel<V, kQuantFp8>, rsh.T, a, g, S, dev, info.sms, st, "rms_mod_quant"));
  } else {
    T8G_DISPATCH_V(rsh.V, rc = launch_rows(rms_mod_kernel<V, kQuantInt8>, rsh.T, a, g, S, dev, info.sms, st, "rms_mod_quant"));
  }
  return rc;
}

int swiglu_common(bool tensorwise, const void* gate, const void* up, int64_t ld_in, void* q, int64_t ld_q,
                  float* q_scale, void* act, int64_t ld_act, float* amax, float* scale_out, int64_t M, int64_t F,
                  int quant_kind, void* stream_) {
  using namespace t8g::rows;
  g_last_error[0] = '\0';
  int rc = check_row_shape("swiglu_quant", M, F, quant_kind, 2);
  if (rc) return rc;
  if (M == 0 || F == 0) return tensorwise ? empty_tensorwise(amax, scale_out, quant_kind, stream_) : T8G_OK;
  if ((rc = check_bf16_matrix("gate", gate, ld_in, F, true))) return rc;
  if ((rc = check_bf16_matrix("up", up, ld_in, F, true))) return rc;
  if ((rc = check_bf16_matrix("act", act, ld_act, F, tensorwise))) return rc;
  if ((rc = check_q(q, ld_q, F))) return rc;
  if (tensorwise && !amax) return fail(T8G_ERR_INVALID_ARGUMENT, "amax scratch word is null");
  if (!tensorwise && !q_scale) return fail(T8G_ERR_INVALID_ARGUMENT, "q_scale is null");
  int dev;
  DeviceInfo info;
  if ((rc = current_device(&dev, &info))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  SwigluArgs a;
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.up = static_cast<const __nv_bfloat16*>(up);
  a.ld_in = ld_in;
  a.q = q;
  a.ld_q = ld_q;
  a.q_scale = q_scale;
  a.act = static_cast<__nv_bfloat16*>(act);
  a.ld_act = ld_act;
  a.amax = amax;
  a.M = M;
  a.F = static_cast<int>(F);
  const RowShape rsh = swiglu_shape(F);
  const RingGeom g = ring_geom(F, 2);
  if (tensorwise) {
    T8G_CHECK_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st), "cudaMemsetAsync(amax)");
    T8G_DISPATCH_SW(rsh.V, rc = launch_swiglu(swiglu_kernel<V, kModeTensorwise>, rsh.T, a, g, M, dev, info.sms, st, "swiglu phase A"));
    if (rc) return rc;
    QuantGivenArgs b;
    b.h = a.act;
    b.ld_h = ld_act;
    b.q = q;
    b.ld_q = ld_q;
    b.amax = amax;
    b.scale_out = scale_out;
    b.S = M;
    b.D = a.F;
    return launch_quant_given(b, quant_kind, info.sms, st);
  }
  if (quant_kind == T8G_QUANT_FP8_E4M3) {
    T8G_DISPATCH_SW(rsh.V, rc = launch_swiglu(swiglu_kernel<V, kModeFp8>, rsh.T, a, g, M, dev, info.sms, st, "swiglu_quant"));
  } else {
    T8G_DISPATCH_SW(rsh.V, rc = launch_swiglu(swiglu_kernel<V, kModeInt8>, rsh.T, a, g, M, dev, info.sms, st, "swiglu_quant"));
  }
  return rc;
}

// ----------------------------------------------------------------- allocation-free scratch
// Backing store of t8g_rms_mod_quant_tensorwise_noalloc: the amax word at offset 0, the bf16
// intermediate h from offset kNoAllocHOffset.  Loaded with the module on every device that
// uses the library; host code reaches it only through the address cudaGetSymbolAddress
// returns for the current device (the symbol itself is a host-side stand-in).
static __device__ __align__(256) unsigned char g_noalloc_scratch[T8G_NOALLOC_SCRATCH_BYTES];
constexpr uint64_t kNoAllocHOffset = 256;

void* g_noalloc_addr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// The host-visible status mirror (t8g_status_mirror): one mapped pinned int for the process,
// its device address stored once per device.
int* g_mirror_host = nullptr;
bool g_mirror_set[kMaxDevices] = {};
std::mutex g_mirror_mu;

// Device address of g_noalloc_scratch on device `dev` (which must be current); looked up
// on the first use per device and cached.
int noalloc_scratch(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_noalloc_addr[dev]);
  return T8G_OK;
}

int swiglu_quant_entry(int in_kind, const void* x, const void* w, const float* x_scale, const float* w_scale,
                       int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t ld_act,
                       float* act_amax, void* q, int64_t ld_q, float* q_scale, int64_t M, int64_t F, int64_t K,
                       int64_t ld_x, int64_t ld_w, int quant_kind, void* stream) {
  using namespace t8g::rows;
  g_last_error[0] = '\0';
  if (quant_kind != T8G_QUANT_INT8 && quant_kind != T8G_QUANT_FP8_E4M3)
    return fail(T8G_ERR_INVALID_ARGUMENT, "unknown quant_kind %d", quant_kind);
  if (M > 0 && F > 0) {
    if (!act_amax || !aligned(act_amax, 4)) return fail(T8G_ERR_INVALID_ARGUMENT, "act_amax must be a 4-byte aligned [M] buffer");
    if (!q_scale) return fail(T8G_ERR_INVALID_ARGUMENT, "q_scale is null");
    int rc = check_q(q, ld_q, F);
    if (rc) return rc;
  }
  int rc = gemm_swiglu_entry(in_kind, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, act, M, F, K, ld_x,
                             ld_w, ld_act, stream, act_amax);
  if (rc || M == 0 || F == 0) return rc;
  int dev;
  DeviceInfo info;
  if ((rc = current_device(&dev, &info))) return rc;
  QuantGivenRowsArgs a;
  a.x = static_cast<const __nv_bfloat16*>(act);
  a.ld_x = ld_act;
  a.row_amax = act_amax;
  a.q = q;
  a.ld_q = ld_q;
  a.q_scale = q_scale;
  a.S = M;
  a.D = static_cast<int>(F);
  const int64_t warps = static_cast<int64_t>(info.sms) * 64;   // 8 CTAs of 8 warps per SM
  const int64_t ctas = (std::min<int64_t>(M, warps) + 7) / 8;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (quant_kind == T8G_QUANT_FP8_E4M3)
    quant_rows_given_amax_kernel<kQuantFp8><<<static_cast<unsigned>(ctas), 256, 0, st>>>(a);
  else
    quant_rows_given_amax_kernel<kQuantInt8><<<static_cast<unsigned>(ctas), 256, 0, st>>>(a);
  return launch_checked("quant of act launch");
}

}  // namespace

extern "C" {

const char* t8g_version(void) { return "0.1.0"; }

const char* t8g_last_error(void) { return g_last_error; }

int t8g_get_device(int* device) {
  g_last_error[0] = '\0';
  if (!device) return fail(T8G_ERR_INVALID_ARGUMENT, "device is null");
  T8G_CHECK_CUDA(cudaGetDevice(device), "cudaGetDevice");
  return T8G_OK;
}

int t8g_set_device(int device) {
  g_last_error[0] = '\0';
  T8G_CHECK_CUDA(cudaSetDevice(device), "cudaSetDevice");
  return T8G_OK;
}

int t8g_device_status(void* stream, int* status) {
  g_last_error[0] = '\0';
  if (!status) return fail(T8G_ERR_INVALID_ARGUMENT, "status is null");
  T8G_CHECK_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
  int v = 0;
  T8G_CHECK_CUDA(cudaMemcpyFromSymbol(&v, t8g::g_device_status, sizeof(int)), "cudaMemcpyFromSymbol");
  if (v != 0) {
    const int zero = 0;
    T8G_CHECK_CUDA(cudaMemcpyToSymbol(t8g::g_device_status, &zero, sizeof(int)), "cudaMemcpyToSymbol");
  }
  *status = v;
  return T8G_OK;
}

int t8g_status_mirror(int** host_word) {
  g_last_error[0] = '\0';
  if (!host_word) return fail(T8G_ERR_INVALID_ARGUMENT, "host_word is null");
  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mirror_mu);
  if (!g_mirror_host) {
    void* p = nullptr;
    T8G_CHECK_CUDA(cudaHostAlloc(&p, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable),
                   "cudaHostAlloc(status mirror)");
    g_mirror_host = static_cast<int*>(p);
    *g_mirror_host = 0;
  }
  if (!g_mirror_set[dev]) {
    void* dptr = nullptr;
    T8G_CHECK_CUDA(cudaHostGetDevicePointer(&dptr, g_mirror_host, 0), "cudaHostGetDevicePointer(status mirror)");
    T8G_CHECK_CUDA(cudaMemcpyToSymbol(t8g::g_status_mirror, &dptr, sizeof(dptr)), "cudaMemcpyToSymbol(status mirror)");
    g_mirror_set[dev] = true;
  }
  *host_word = g_mirror_host;
  return T8G_OK;
}

int t8g_gemm_i8_dequant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                        int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* out, int out_dtype,
                        int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream) {
  return gemm_entry(t8g::gemm::kInI8, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, out, out_dtype, M, N,
                    K, ld_x, ld_w, ld_out, stream);
}

int t8g_gemm_fp8_dequant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                         int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* out, int out_dtype,
                         int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream) {
  return gemm_entry(t8g::gemm::kInE4M3, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, out, out_dtype, M,
                    N, K, ld_x, ld_w, ld_out, stream);
}

int t8g_gemm_i8_swiglu(const void* x, const void* w, const float* x_scale, const float* w_scale,
                       int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t M, int64_t F,
                       int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_act, void* stream) {
  return gemm_swiglu_entry(t8g::gemm::kInI8, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, act, M, F, K,
                           ld_x, ld_w, ld_act, stream);
}

int t8g_gemm_fp8_swiglu(const void* x, const void* w, const float* x_scale, const float* w_scale,
                        int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t M, int64_t F,
                        int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_act, void* stream) {
  return gemm_swiglu_entry(t8g::gemm::kInE4M3, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, act, M, F,
                           K, ld_x, ld_w, ld_act, stream);
}

int t8g_gemm_i8_swiglu_quant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                             int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t ld_act,
                             float* act_amax, void* q, int64_t ld_q, float* q_scale, int64_t M, int64_t F, int64_t K,
                             int64_t ld_x, int64_t ld_w, int quant_kind, void* stream) {
  return swiglu_quant_entry(t8g::gemm::kInI8, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, act, ld_act,
                            act_amax, q, ld_q, q_scale, M, F, K, ld_x, ld_w, quant_kind, stream);
}

int t8g_gemm_fp8_swiglu_quant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                              int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t ld_act,
                              float* act_amax, void* q, int64_t ld_q, float* q_scale, int64_t M, int64_t F, int64_t K,
                              int64_t ld_x, int64_t ld_w, int quant_kind, void* stream) {
  return swiglu_quant_entry(t8g::gemm::kInE4M3, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, act, ld_act,
                            act_amax, q, ld_q, q_scale, M, F, K, ld_x, ld_w, quant_kind, stream);
}

int t8g_gemm_i8_gated(const void* x, const void* w, const float* x_scale, const float* w_scale,
                      int64_t w_scale_numel, const void* bias, int64_t bias_numel, const void* res, int64_t ld_res,
                      const void* gate, int64_t ld_gate, const int32_t* gate_index, int64_t rows_per_gate, void* out,
                      int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream) {
  return gemm_gated_entry(t8g::gemm::kInI8, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, res, ld_res, gate,
                          ld_gate, gate_index, rows_per_gate, out, M, N, K, ld_x, ld_w, ld_out, stream);
}

int t8g_gemm_fp8_gated(const void* x, const void* w, const float* x_scale, const float* w_scale,
                       int64_t w_scale_numel, const void* bias, int64_t bias_numel, const void* res, int64_t ld_res,
                       const void* gate, int64_t ld_gate, const int32_t* gate_index, int64_t rows_per_gate, void* out,
                       int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream) {
  return gemm_gated_entry(t8g::gemm::kInE4M3, x, w, x_scale, w_scale, w_scale_numel, bias, bias_numel, res, ld_res,
                          gate, ld_gate, gate_index, rows_per_gate, out, M, N, K, ld_x, ld_w, ld_out, stream);
}

int t8g_quant_rows(const void* x, int64_t ld_x, void* q, int64_t ld_q, float* q_scale, int64_t S, int64_t D,
                   int quant_kind, void* stream) {
  using namespace t8g::rows;
  g_last_error[0] = '\0';
  int rc = check_row_shape("quant_rows", S, D, quant_kind, 1);
  if (rc) return rc;
  if (S == 0 || D == 0) return T8G_OK;
  if ((rc = check_bf16_matrix("x", x, ld_x, D, true))) return rc;
  if ((rc = check_q(q, ld_q, D))) return rc;
  if (!q_scale) return fail(T8G_ERR_INVALID_ARGUMENT, "q_scale is null");
  int dev;
  DeviceInfo info;
  if ((rc = current_device(&dev, &info))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  QuantRowsArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ld_x = ld_x;
  a.q = q;
  a.ld_q = ld_q;
  a.q_scale = q_scale;
  a.S = S;
  a.D = static_cast<int>(D);
  const uint32_t row_bytes = static_cast<uint32_t>(2 * D);
  if (const int nv = reg_nv(D)) {
    WarpLaunch o;
    o.max_warps = kRegWarps;
    if (quant_kind == T8G_QUANT_FP8_E4M3) {
      T8G_DISPATCH_NV(nv, rc = launch_warp_rows(quant_rows_warp_reg_kernel<NV, kQuantFp8>, a, row_bytes, S, dev,
                                                info.sms, st, o, "quant_rows"));
    } else {
      T8G_DISPATCH_NV(nv, rc = launch_warp_rows(quant_rows_warp_reg_kernel<NV, kQuantInt8>, a, row_bytes, S, dev,
                                                info.sms, st, o, "quant_rows"));
    }
    return rc;
  }
  if (row_bytes <= kWarpRowMaxBytes) {
    if (quant_kind == T8G_QUANT_FP8_E4M3)
      return launch_warp_rows(quant_rows_warp_kernel<kQuantFp8>, a, row_bytes, S, dev, info.sms, st, WarpLaunch{}, "quant_rows");
    return launch_warp_rows(quant_rows_warp_kernel<kQuantInt8>, a, row_bytes, S, dev, info.sms, st, WarpLaunch{}, "quant_rows");
  }
  const RowShape rsh = row_shape(D);
  const RingGeom g = ring_geom(D, 1);
  if (quant_kind == T8G_QUANT_FP8_E4M3) {
    T8G_DISPATCH_V(rsh.V, rc = launch_rows(quant_rows_kernel<V, kQuantFp8>, rsh.T, a, g, S, dev, info.sms, st, "quant_rows"));
  } else {
    T8G_DISPATCH_V(rsh.V, rc = launch_rows(quant_rows_kernel<V, kQuantInt8>, rsh.T, a, g, S, dev, info.sms, st, "quant_rows"));
  }
  return rc;
}

int t8g_rms_mod_quant(const void* x, int64_t ld_x, const void* w, const void* shift, const void* scale,
                      int64_t ld_mod, const int32_t* mod_index, int64_t rows_per_mod, int scale_is_multiplier,
                      float eps, void* q, int64_t ld_q, float* q_scale, void* h, int64_t ld_h, void* res,
                      int64_t ld_res, int64_t S, int64_t D, int quant_kind, void* stream) {
  return rms_common(false, x, ld_x, w, shift, scale, ld_mod, mod_index, rows_per_mod, scale_is_multiplier, eps, q,
                    ld_q, q_scale, h, ld_h, res, ld_res, nullptr, nullptr, S, D, quant_kind, stream);
}

int t8g_rms_mod_quant_tensorwise(const void* x, int64_t ld_x, const void* w, const void* shift,
                                 const void* scale, int64_t ld_mod, const int32_t* mod_index,
                                 int64_t rows_per_mod, int scale_is_multiplier, float eps, void* q,
                                 int64_t ld_q, void* h, int64_t ld_h, void* res, int64_t ld_res, float* amax,
                                 float* scale_out, int64_t S, int64_t D, int quant_kind, void* stream) {
  return rms_common(true, x, ld_x, w, shift, scale, ld_mod, mod_index, rows_per_mod, scale_is_multiplier, eps, q,
                    ld_q, nullptr, h, ld_h, res, ld_res, amax, scale_out, S, D, quant_kind, stream);
}

int t8g_swiglu_quant(const void* gate, const void* up, int64_t ld_in, void* q, int64_t ld_q, float* q_scale,
                     void* act, int64_t ld_act, int64_t M, int64_t F, int quant_kind, void* stream) {
  return swiglu_common(false, gate, up, ld_in, q, ld_q, q_scale, act, ld_act, nullptr, nullptr, M, F, quant_kind,
                       stream);
}

int t8g_swiglu_quant_tensorwise(const void* gate, const void* up, int64_t ld_in, void* q, int64_t ld_q,
                                void* act, int64_t ld_act, float* amax, float* scale_out, int64_t M, int64_t F,
                                int quant_kind, void* stream) {
  return swiglu_common(true, gate, up, ld_in, q, ld_q, nullptr, act, ld_act, amax, scale_out, M, F, quant_kind,
                       stream);
}

int t8g_rms_mod_quant_tensorwise_noalloc(const void* x, int64_t ld_x, const void* w, const void* shift,
                                         const void* scale, int64_t ld_mod, const int32_t* mod_index,
                                         int64_t rows_per_mod, int scale_is_multiplier, float eps, void* q,
                                         int64_t ld_q, void* res, int64_t ld_res, float* scale_out, int64_t S,
                                         int64_t D, int quant_kind, void* stream) {
  g_last_error[0] = '\0';
  if (S < 0 || D < 0) return fail(T8G_ERR_INVALID_ARGUMENT, "no-alloc tensorwise: negative size");
  const uint64_t cap = (T8G_NOALLOC_SCRATCH_BYTES - kNoAllocHOffset) / 2;
  if (S != 0 && D != 0 && static_cast<uint64_t>(S) > cap / static_cast<uint64_t>(D))
    return fail(T8G_ERR_UNSUPPORTED,
                "no-alloc tensorwise: S*D = %lld elements exceeds the built-in scratch (%llu elements, "
                "%u bytes); use t8g_rms_mod_quant_tensorwise with caller-provided buffers",
                (long long)(S * D), (unsigned long long)cap, (unsigned)T8G_NOALLOC_SCRATCH_BYTES);
  unsigned char* base = nullptr;
  if (S != 0 && D != 0) {
    int dev;
    DeviceInfo info;
    int rc = current_device(&dev, &info);
    if (rc) return rc;
    if ((rc = noalloc_scratch(dev, &base))) return rc;
  }
  float* amax = reinterpret_cast<float*>(base);
  void* h = base ? base + kNoAllocHOffset : nullptr;
  return rms_common(true, x, ld_x, w, shift, scale, ld_mod, mod_index, rows_per_mod, scale_is_multiplier, eps, q,
                    ld_q, nullptr, h, D, res, ld_res, amax, scale_out, S, D, quant_kind, stream);
}

int t8g_wait_selftest(uint64_t limit_ns, int* gave_up, void* stream) {
  g_last_error[0] = '\0';
  if (!gave_up) return fail(T8G_ERR_INVALID_ARGUMENT, "gave_up is null");
  if (limit_ns > 2000000000ull) return fail(T8G_ERR_INVALID_ARGUMENT, "limit above 2 s");
  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc) return rc;
  t8g::rows::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, gave_up);
  return launch_checked("wait_selftest launch");
}

}  // extern "C"
