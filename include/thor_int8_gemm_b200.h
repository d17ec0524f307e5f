/*
 * thor_int8_gemm_b200 -- C ABI of the B200 (sm_100a) quantized linear-layer path.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types.  Every entry
 * point validates its arguments on the host, launches asynchronously on
 * `stream` (a cudaStream_t; NULL is the legacy default stream) and returns
 * T8G_OK or a nonzero T8G_ERR_* code; t8g_last_error() then holds a message.
 * Device pointers must be CUDA device (or managed) memory of the current
 * device.  Row strides (ld_*) are in elements.  Matrices are row-major.
 *
 * Reference interfaces replaced (paths inside kylixs/thor-int8-gemm):
 *   comfy-kitchen _C.cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out,
 *       dtype_code, stream)                  src/ck_int8_patch_thor.py:143-168
 *       (kernel + launcher                   src/ck_int8_patch_thor.py:67-125)
 *   fused_rms_mod_quant(x, w, s, b, eps)     src/ck_fused_mod_norm_quant.py:121-145
 *   fused_swiglu_quant(gate, up)             src/ck_fused_mod_norm_quant.py:148-167
 *   per-segment norm_mod_quant driver        src/ck_fused_patch.py:105-136
 */
#ifndef THOR_INT8_GEMM_B200_H_
#define THOR_INT8_GEMM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* return codes */
#define T8G_OK 0
#define T8G_ERR_INVALID_ARGUMENT 1  /* shape, stride, alignment or null pointer */
#define T8G_ERR_UNSUPPORTED 2       /* device is not sm_100, or size beyond a limit */
#define T8G_ERR_CUDA 3              /* a CUDA runtime / driver call failed */

/* output element types of the GEMMs */
#define T8G_OUT_BF16 0
#define T8G_OUT_F16 1
#define T8G_OUT_F32 2

/* quantised element types */
#define T8G_QUANT_INT8 0            /* int8, scale = amax / 127, round half to even, clamp +-127 */
#define T8G_QUANT_FP8_E4M3 1        /* float8_e4m3fn, scale = amax / 448, RNE, clamp +-448 */

/* Library version string, e.g. "0.1.0". */
const char* t8g_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* t8g_last_error(void);

/* Reads and clears the device status word of the current device after
 * synchronising `stream`.  *status = 0 when no kernel recorded a problem;
 * otherwise the code of the first bounded wait that ran out (0x101..0x104),
 * in which case that kernel's output is incomplete. */
int t8g_device_status(void* stream, int* status);

/* A host-visible mirror of the status word: *host_word receives the address of a mapped,
 * pinned host int that every kernel of this library also writes (with a system-visible
 * store) when one of its bounded waits runs out, on every device this was called for.  A
 * caller can poll it without synchronising or calling CUDA -- the comfy-kitchen proxy checks
 * it on every call and stops using the library after a wait ran out -- and clears it by
 * writing 0.  Set-up (once per device, with that device current) copies the address to the
 * device, so make the first call before any stream capture. */
int t8g_status_mirror(int** host_word);

/* The calling thread's current CUDA device, and setting it (cudaGetDevice /
 * cudaSetDevice of the runtime this library uses), for callers without their own. */
int t8g_get_device(int* device);
int t8g_set_device(int device);

/*
 * out[m, n] = cast( ((float(acc[m, n]) * x_scale[m]) * w_scale[n or 0]) + float(bias[n]) )
 * acc[m, n] = sum_k x[m, k] * w[n, k]   (int8 x int8, exact int32)
 *
 * Replaces comfy-kitchen's _C.cutlass_int8_dequant, which the reference proxies
 * at src/ck_int8_patch_thor.py:143 (epilogue order :101-106, identical to
 * _gemm_intmm at src/ck_int8_patch_intmm.py:63-71).
 *   x        [M, K] int8, row stride ld_x          w   [N, K] int8, row stride ld_w
 *   x_scale  [M] float32                           w_scale [w_scale_numel] float32, numel 1 or N
 *   bias     [bias_numel] in the output type, numel 0 (then may be NULL) or N
 *   out      [M, N] of out_dtype (T8G_OUT_*), row stride ld_out
 * Requirements: x, w, out 16-byte aligned; ld_x, ld_w multiples of 16;
 * ld_out * element size a multiple of 16; 0 <= K; M, N, K < 2^31.
 * M == 0 or N == 0 is a no-op.  K == 0 (which the proxy's K % 16 rule lets through) is an
 * empty sum: out = cast(((0 * x_scale[m]) * w_scale[n]) + bias[n]), x and w are not read.
 */
int t8g_gemm_i8_dequant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                        int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* out, int out_dtype,
                        int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out,
                        void* stream);

/* float8_e4m3fn twin of t8g_gemm_i8_dequant (fp32 tensor-core accumulation).
 * The reference routes fp8 linears to comfy's _scaled_mm (src/ck_fused_patch.py:14-17,
 * :126-136); this is the same operator shape with per-token / per-channel scales. */
int t8g_gemm_fp8_dequant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                         int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* out, int out_dtype,
                         int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out,
                         void* stream);

/*
 * fc1 GEMM with the SwiGLU fused into its epilogue:
 *   y[m, n]   = bf16( ((float(acc[m, n]) * x_scale[m]) * w_scale[n or 0]) + float(bias[n]) )
 *   act[m, j] = bf16( silu(gate) * up )   with gate / up the bf16 y values of fc1 channels
 *               j and F + j (the SwiGLU of t8g_swiglu_quant, bit for bit)
 * The reference computes y with the GEMM, copies its halves and runs the SwiGLU kernel
 * (src/ck_fused_patch.py:139-149, src/ck_fused_mod_norm_quant.py:59-73); here y never
 * reaches memory.  w, w_scale and bias are the fc1 parameters with gate and up rows
 * interleaved in blocks of 128: row 256 t + i holds gate channel 128 t + i and row
 * 256 t + 128 + i up channel 128 t + i (i < 128).
 *   x [M, K] int8 (ld_x), w [2F, K] int8 (ld_w), x_scale [M], w_scale numel 1 or 2F,
 *   bias numel 0 or 2F (bf16), act [M, F] bf16 (ld_act).
 * Requirements: F a multiple of 128; alignment and strides as t8g_gemm_i8_dequant.
 * The per-token quantisation of act is t8g_quant_rows.
 */
int t8g_gemm_i8_swiglu(const void* x, const void* w, const float* x_scale, const float* w_scale,
                       int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t M, int64_t F,
                       int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_act, void* stream);

/* float8_e4m3fn twin of t8g_gemm_i8_swiglu. */
int t8g_gemm_fp8_swiglu(const void* x, const void* w, const float* x_scale, const float* w_scale,
                        int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t M, int64_t F,
                        int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_act, void* stream);

/*
 * fc1 + SwiGLU + per-token quantisation of act for the next linear (the reference's
 * swiglu_linear up to fc2's input, src/ck_fused_patch.py:139-149): t8g_gemm_i8_swiglu, whose
 * epilogue also reports act_amax[m] = max_j |act[m, j]| (bf16 values; an atomic max per row and
 * tile into the caller's float32 [M] buffer, zeroed by this call), then a streaming pass
 *   q_scale[m] = max(act_amax[m] / qmax, 1e-12),  q[m, j] = cvt(clamp(act[m, j] / q_scale[m]))
 * equal bit for bit to t8g_quant_rows(act).  A row's scale needs the whole row, which spans
 * many GEMM tiles, so q cannot be written by the epilogue itself; with the row maxima known the
 * quantiser reads act once as a plain stream (no row held in shared memory, no reduction).
 *   act [M, F] bf16 (ld_act, also returned), act_amax float32 [M] scratch, q [M, F] of
 *   quant_kind (ld_q), q_scale float32 [M]; the rest as t8g_gemm_i8_swiglu.
 */
int t8g_gemm_i8_swiglu_quant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                             int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t ld_act,
                             float* act_amax, void* q, int64_t ld_q, float* q_scale, int64_t M, int64_t F, int64_t K,
                             int64_t ld_x, int64_t ld_w, int quant_kind, void* stream);

/* float8_e4m3fn twin of t8g_gemm_i8_swiglu_quant (quant_kind selects act's codes). */
int t8g_gemm_fp8_swiglu_quant(const void* x, const void* w, const float* x_scale, const float* w_scale,
                              int64_t w_scale_numel, const void* bias, int64_t bias_numel, void* act, int64_t ld_act,
                              float* act_amax, void* q, int64_t ld_q, float* q_scale, int64_t M, int64_t F, int64_t K,
                              int64_t ld_x, int64_t ld_w, int quant_kind, void* stream);

/*
 * Fused-dequant GEMM whose epilogue applies the DiT block's gated residual, the stock
 * `x = _mod_gate(x, gate, proj(h), mod_segments)` after the attention and MLP projections
 * (the block's call order, src/ck_fused_patch.py:153-172), in torch's bf16 operation order:
 *   y   = bf16(f32(acc) * x_scale[m] * w_scale[n] + f32(bias[n]))      (as t8g_gemm_i8_dequant)
 *   t   = bf16(f32(gate[g, n]) * f32(y))
 *   out = bf16(f32(res[m, n]) + f32(t)),   g = gate_index[m] if non-NULL, else m / rows_per_gate.
 *   res, out bf16 [M, N] (ld_res, ld_out); gate bf16 [n_gate, N] (ld_gate); gate_index int32 [M]
 *   (trusted to hold rows of gate).  out may be res itself (in-place update); otherwise the
 *   two must not overlap.  The bf16 projection output y is never written to memory.
 * Requirements as t8g_gemm_i8_dequant with a bf16 output, plus N a multiple of 8, res/gate
 * 16-byte aligned and ld_res, ld_gate multiples of 8.
 */
int t8g_gemm_i8_gated(const void* x, const void* w, const float* x_scale, const float* w_scale,
                      int64_t w_scale_numel, const void* bias, int64_t bias_numel, const void* res, int64_t ld_res,
                      const void* gate, int64_t ld_gate, const int32_t* gate_index, int64_t rows_per_gate, void* out,
                      int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream);

/* float8_e4m3fn twin of t8g_gemm_i8_gated. */
int t8g_gemm_fp8_gated(const void* x, const void* w, const float* x_scale, const float* w_scale,
                       int64_t w_scale_numel, const void* bias, int64_t bias_numel, const void* res, int64_t ld_res,
                       const void* gate, int64_t ld_gate, const int32_t* gate_index, int64_t rows_per_gate, void* out,
                       int64_t M, int64_t N, int64_t K, int64_t ld_x, int64_t ld_w, int64_t ld_out, void* stream);

/*
 * Per-token quantisation of a bf16 matrix: q_scale[m] = max(amax_k |x[m,k]| / qmax, 1e-12),
 * q[m, k] = cvt(clamp(x[m, k] / q_scale[m])).  This is the activation quantiser that
 * comfy-kitchen's int8_linear runs in front of _C.cutlass_int8_dequant (its code is not
 * in the reference; the call chain is src/ck_int8_patch_thor.py:201-210 -> :143).
 *   x [S, D] bf16 (ld_x), q [S, D] (ld_q) of quant_kind, q_scale [S] float32.
 * Requirements: D a multiple of 8, D <= 49152; x 16-byte aligned, ld_x a multiple of 8;
 * q 8-byte aligned, ld_q a multiple of 8.
 */
int t8g_quant_rows(const void* x, int64_t ld_x, void* q, int64_t ld_q, float* q_scale, int64_t S, int64_t D,
                   int quant_kind, void* stream);

/*
 * One-pass RMSNorm + adaLN modulation + per-token quantisation.
 *   inv  = 1 / sqrt(sum_k x^2 / D + eps)
 *   s    = scale_is_multiplier ? scale[mrow] : bf16(1 + scale[mrow])   (src/ck_fused_patch.py:120)
 *   h    = (((x * inv) * w) * s) + shift[mrow]                          (src/ck_fused_mod_norm_quant.py:51)
 *   q, q_scale = per-token quantisation of bf16(h)
 *   res  = bf16(h + x)                                                   (:53)
 * mrow = mod_index[row] if mod_index != NULL, else row / rows_per_mod.
 *   x [S, D] bf16; w [D] bf16 or NULL (no affine weight); shift, scale [n_mod, D] bf16 with
 *   row stride ld_mod; h, res optional bf16 outputs (NULL to skip).
 * Requirements as t8g_quant_rows, plus 16-byte aligned shift/scale/w/h/res and strides
 * that are multiples of 8.
 */
int t8g_rms_mod_quant(const void* x, int64_t ld_x, const void* w, const void* shift, const void* scale,
                      int64_t ld_mod, const int32_t* mod_index, int64_t rows_per_mod, int scale_is_multiplier,
                      float eps, void* q, int64_t ld_q, float* q_scale, void* h, int64_t ld_h, void* res,
                      int64_t ld_res, int64_t S, int64_t D, int quant_kind, void* stream);

/*
 * The reference's fused_rms_mod_quant (src/ck_fused_mod_norm_quant.py:121-145) and its
 * per-segment driver (src/ck_fused_patch.py:105-136): writes h and res (bf16), takes
 * amax = max |h| over the whole tensor in float32, then q = cvt(clamp(bf16(h) / scale))
 * with scale = max(amax / qmax, 1e-12) written to *scale_out.  `amax` is a caller-provided
 * float32 device word that this call zeroes first.  h is required (it feeds the second
 * pass); res may be NULL.
 */
int t8g_rms_mod_quant_tensorwise(const void* x, int64_t ld_x, const void* w, const void* shift,
                                 const void* scale, int64_t ld_mod, const int32_t* mod_index,
                                 int64_t rows_per_mod, int scale_is_multiplier, float eps, void* q,
                                 int64_t ld_q, void* h, int64_t ld_h, void* res, int64_t ld_res, float* amax,
                                 float* scale_out, int64_t S, int64_t D, int quant_kind, void* stream);

/*
 * One-pass SwiGLU + per-token quantisation:
 *   act = bf16((gate * sigmoid(gate)) * up)       (src/ck_fused_mod_norm_quant.py:71)
 *   q, q_scale = per-token quantisation of act; act optionally stored.
 * gate and up are [M, F] bf16 with the common row stride ld_in, so the two halves of a
 * [M, 2F] fc1 output are read in place (gate = y, up = y + F, ld_in = 2F).
 * Requirements as t8g_quant_rows with D = F, except F <= 24576.
 */
int t8g_swiglu_quant(const void* gate, const void* up, int64_t ld_in, void* q, int64_t ld_q, float* q_scale,
                     void* act, int64_t ld_act, int64_t M, int64_t F, int quant_kind, void* stream);

/*
 * The reference's fused_swiglu_quant (src/ck_fused_mod_norm_quant.py:148-167): act bf16,
 * amax over float32 |act|, q from bf16 act with one scale (written to *scale_out).  `amax`
 * is a caller-provided float32 device word that this call zeroes first; act is required.
 */
int t8g_swiglu_quant_tensorwise(const void* gate, const void* up, int64_t ld_in, void* q, int64_t ld_q,
                                void* act, int64_t ld_act, float* amax, float* scale_out, int64_t M, int64_t F,
                                int quant_kind, void* stream);

/*
 * Allocation-free variant of t8g_rms_mod_quant_tensorwise.  No counterpart in the reference.
 *
 * Some callers cannot allocate device memory at the point where they quantise: plugins
 * hosted by a process whose allocator owns every byte of the GPU, C callers with no CUDA
 * allocator of their own, and code paths where cudaMalloc's implicit device-wide
 * synchronisation is not acceptable.  The tensorwise form needs two scratch buffers (the
 * float32 amax word and the bf16 intermediate h that the second pass quantises), which
 * t8g_rms_mod_quant_tensorwise takes from its caller.  This entry point takes neither: both
 * live in one file-scope device array of T8G_NOALLOC_SCRATCH_BYTES that every GPU which
 * loads the library holds until the process exits.  The caller passes only inputs and
 * outputs (q, optional res, scale_out).
 *
 * Limit: S * D * 2 + 256 <= T8G_NOALLOC_SCRATCH_BYTES (S * D <= 8388480 elements, e.g.
 * 2730 rows of 3072); larger problems are rejected with T8G_ERR_UNSUPPORTED.  The first
 * call on a device looks up the array's device address (once per device, with that device
 * current), so make that first call before any stream capture.  The call zeroes the amax
 * word itself.  All calls share the one array and it keeps the last call's contents, so
 * calls that overlap on the GPU (other streams, other host threads on the same device)
 * race; serialise them.  Arguments and results otherwise as t8g_rms_mod_quant_tensorwise.
 */
#define T8G_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int t8g_rms_mod_quant_tensorwise_noalloc(const void* x, int64_t ld_x, const void* w, const void* shift,
                                         const void* scale, int64_t ld_mod, const int32_t* mod_index,
                                         int64_t rows_per_mod, int scale_is_multiplier, float eps, void* q,
                                         int64_t ld_q, void* res, int64_t ld_res, float* scale_out, int64_t S,
                                         int64_t D, int quant_kind, void* stream);

/* Bounded-wait self-test: one kernel waits `limit_ns` on an mbarrier that nothing
 * completes, gives up, records status 0x1FF and writes 1 to the device int *gave_up.
 * Used by the tests to show that a wait which runs out ends the kernel with a status
 * the host can read, leaving the context usable. */
int t8g_wait_selftest(uint64_t limit_ns, int* gave_up, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* THOR_INT8_GEMM_B200_H_ */
