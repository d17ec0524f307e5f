"""CPU oracle for the quantized linear-layer path (TEST INFRASTRUCTURE ONLY).

This module restates, on the CPU with numpy (and torch CPU for the int8 matmul),
the arithmetic of the reference's hot path.  It is the checker the CUDA kernels
are compared against; nothing in the shipped package imports it.  Only `tests/`,
`__graft_entry__.smoke()` and the CPU legs of `bench.py` may use it.

Reference functions restated here (paths inside the reference project):

* `_gemm_intmm`                      src/ck_int8_patch_intmm.py:63-71
  (same epilogue order as the Triton `_kernel`, src/ck_int8_patch_thor.py:101-106)
* `_rms_mod_res_amax_kernel`         src/ck_fused_mod_norm_quant.py:23-55
* `_swiglu_amax_kernel`              src/ck_fused_mod_norm_quant.py:59-73
* `_quant_fp8_amax_kernel`           src/ck_fused_mod_norm_quant.py:92-111
* `_make_scale`                      src/ck_fused_mod_norm_quant.py:114-118
* `fused_rms_mod_quant`              src/ck_fused_mod_norm_quant.py:121-145
* `fused_swiglu_quant`               src/ck_fused_mod_norm_quant.py:148-167
* `1 + scale` rounded in bf16        src/ck_fused_patch.py:119-121
* the block's gated residual         src/ck_fused_patch.py:160-161, :172 (comfy `_mod_gate`)

Per-token quantisation (scale = amax/127 or amax/448 per row, round half to
even, clamp) has no code in the reference: it lives in comfy-kitchen's
`int8_linear`, which is not vendored.  Its definition here follows the
workload description (per-token scale = absmax/127, RNE, clamp +-127) plus the
reference's SCALE_MIN = 1e-12 floor (src/ck_fused_mod_norm_quant.py:141); that
part of the parity is unpinned against the stock library.

Pinning: `tests/golden/make_golden.py` runs the reference's own code (the
`_gemm_intmm` path natively, the Triton kernels through Triton's CPU
interpreter with an RNE-correct float converter) and stores the outputs under
`tests/golden/`; `tests/test_oracle_golden.py` checks this module against them.

Floating-point conventions (all IEEE-754 binary32, round-to-nearest-even,
every operation rounded separately, no fused multiply-add):
the GEMM epilogue is  out = cast(((f32(acc) * xs[m]) * ws[n]) + f32(bias[n]));
the RMS norm is       inv = 1 / sqrt(ss / D + eps),
                      h   = (((x * inv) * w) * s) + b;
where the sum of squares `ss` follows, in the tensorwise (reference-signature)
forms, the reference's own order (`rms_sum_squares_reference`), and in the
per-token forms, which have no reference counterpart, the library's canonical
tree (`rms_sum_squares`); the CUDA kernels implement each the same way.
The SwiGLU's exponential is correctly rounded (`exp_f32`).
"""
from __future__ import annotations

import numpy as np

try:  # torch is used only for the fast exact int8 x int8 -> int32 CPU matmul
    import torch
except Exception:  # pragma: no cover - torch is present in every supported setup
    torch = None

SCALE_MIN = np.float32(1e-12)      # src/ck_fused_mod_norm_quant.py:141
F8_E4M3_MAX = np.float32(448.0)    # src/ck_fused_mod_norm_quant.py:19
INT8_QMAX = np.float32(127.0)

QUANT_INT8 = "int8"
QUANT_FP8 = "fp8_e4m3"

# Canonical launch shape of the row kernels: one row is handled by T threads,
# V = max(3, ceil(nvec / 512)) 16-byte vectors (8 bf16 values) per thread and
# T = 32 * ceil(nvec / (32 * V)), nvec = D / 8 (rows up to ROW_MAX_D values).
ROW_MAX_D = 49152


# --------------------------------------------------------------------------
# scalar formats
# --------------------------------------------------------------------------
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def bf16_ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 ulps between two arrays of bf16 bit patterns (+0 == -0)."""
    a = np.asarray(a_bits, np.uint16).astype(np.int64)
    b = np.asarray(b_bits, np.uint16).astype(np.int64)
    oa = np.where(a & 0x8000, -(a & 0x7FFF), a & 0x7FFF)
    ob = np.where(b & 0x8000, -(b & 0x7FFF), b & 0x7FFF)
    return np.abs(oa - ob)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> float32 value of its bf16 rounding."""
    return bf16_to_f32(f32_to_bf16(x))


def f16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> IEEE binary16 bit patterns (numpy casts with RNE)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def _e4m3_table() -> np.ndarray:
    """Values of the 128 non-negative float8_e4m3fn codes (0x7F is NaN)."""
    vals = np.zeros(128, dtype=np.float64)
    for code in range(128):
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0:
            vals[code] = (m / 8.0) * 2.0 ** -6
        else:
            vals[code] = (1.0 + m / 8.0) * 2.0 ** (e - 7)
    vals[0x7F] = np.nan
    return vals


_E4M3_POS = _e4m3_table()
_E4M3_FINITE = _E4M3_POS[:0x7F]          # codes 0x00..0x7E, strictly increasing


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    """float8_e4m3fn codes (uint8) -> float32 values."""
    codes = np.asarray(codes, dtype=np.uint8)
    mag = _E4M3_POS[codes & 0x7F]
    out = np.where(codes & 0x80, -mag, mag)
    return out.astype(np.float32)


def f32_to_e4m3(v: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn codes, round to nearest even, saturating to +-448.

    Same result as the hardware conversion `cvt.rn.satfinite.e4m3x2.f32` for
    finite inputs; the quantisers always clamp to +-448 before converting
    (src/ck_fused_mod_norm_quant.py:110-111), so saturation never decides a
    value there.
    """
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v).astype(np.float64)
    a = np.minimum(a, 448.0)
    hi = np.searchsorted(_E4M3_FINITE, a, side="left")       # first value >= a
    hi = np.minimum(hi, len(_E4M3_FINITE) - 1)
    lo = np.maximum(hi - 1, 0)
    d_hi = _E4M3_FINITE[hi] - a
    d_lo = a - _E4M3_FINITE[lo]
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((hi & 1) == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(a == _E4M3_FINITE[hi], hi, code).astype(np.uint8)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    out = code | sign
    return np.where(np.isnan(v), np.uint8(0x7F), out).astype(np.uint8)


# --------------------------------------------------------------------------
# quantisers
# --------------------------------------------------------------------------
def _qmax(kind: str) -> np.float32:
    if kind == QUANT_INT8:
        return INT8_QMAX
    if kind == QUANT_FP8:
        return F8_E4M3_MAX
    raise ValueError(f"unknown quant kind {kind!r}")


def scale_from_amax(amax: np.ndarray, kind: str) -> np.ndarray:
    """scale = max(amax / qmax, 1e-12)  (src/ck_fused_mod_norm_quant.py:107,118)."""
    amax = np.asarray(amax, dtype=np.float32)
    return np.maximum(amax / _qmax(kind), SCALE_MIN).astype(np.float32)


def quantize_with_scale(v: np.ndarray, scale: np.ndarray, kind: str) -> np.ndarray:
    """q = clamp(v / scale) converted to the 8-bit code (IEEE divide).

    fp8: clamp to +-448 then RNE convert (src/ck_fused_mod_norm_quant.py:109-111).
    int8: round half to even then clamp to +-127.
    Returns uint8 codes for fp8 and int8 values for int8.
    """
    q = (np.asarray(v, dtype=np.float32) / np.asarray(scale, dtype=np.float32)).astype(np.float32)
    if kind == QUANT_FP8:
        q = np.minimum(np.maximum(q, -F8_E4M3_MAX), F8_E4M3_MAX)
        return f32_to_e4m3(q)
    q = np.clip(np.rint(q), -127.0, 127.0)
    return q.astype(np.int8)


def quant_rows(x: np.ndarray, kind: str):
    """Per-token (per-row) quantisation of float32 values of a bf16 matrix.

    scale[m] = max(amax_k |x[m,k]| / qmax, 1e-12); q = quantize(x / scale[m]).
    Returns (q, scale) with q int8 (int8 kind) or uint8 e4m3 codes (fp8 kind).
    """
    x = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x), axis=-1) if x.shape[-1] else np.zeros(x.shape[:-1], np.float32)
    scale = scale_from_amax(amax, kind)
    return quantize_with_scale(x, scale[..., None], kind), scale


# --------------------------------------------------------------------------
# GEMM with fused dequant epilogue
# --------------------------------------------------------------------------
def int_matmul_nt(a8: np.ndarray, w8: np.ndarray) -> np.ndarray:
    """acc[m, n] = sum_k a[m, k] * w[n, k], exact int32."""
    a8 = np.ascontiguousarray(a8, dtype=np.int8)
    w8 = np.ascontiguousarray(w8, dtype=np.int8)
    if torch is not None and a8.shape[0] > 0 and w8.shape[0] > 0 and a8.shape[1] > 0:
        acc = torch._int_mm(torch.from_numpy(a8), torch.from_numpy(w8).t())
        return acc.numpy().astype(np.int32)
    return (a8.astype(np.int64) @ w8.astype(np.int64).T).astype(np.int32)


def dequant_epilogue(acc_f32: np.ndarray, xs: np.ndarray, ws: np.ndarray,
                     bias_f32: np.ndarray | None) -> np.ndarray:
    """((acc * xs[m]) * ws[n or 0]) + bias[n], each op rounded in float32.

    src/ck_int8_patch_intmm.py:65-69 (and src/ck_int8_patch_thor.py:101-104).
    """
    o = np.asarray(acc_f32, dtype=np.float32)
    o = (o * np.asarray(xs, np.float32).reshape(-1, 1)).astype(np.float32)
    ws = np.asarray(ws, np.float32).reshape(-1)
    o = (o * (ws.reshape(1, -1) if ws.size > 1 else ws.reshape(1, 1))).astype(np.float32)
    if bias_f32 is not None and np.asarray(bias_f32).size:
        o = (o + np.asarray(bias_f32, np.float32).reshape(1, -1)).astype(np.float32)
    return o


def cast_out(o: np.ndarray, out_dtype: str) -> np.ndarray:
    """float32 result -> output bit patterns ('bf16' / 'f16' uint16, 'f32' float32)."""
    if out_dtype == "bf16":
        return f32_to_bf16(o)
    if out_dtype == "f16":
        return f16_bits(o)
    if out_dtype == "f32":
        return np.asarray(o, dtype=np.float32)
    raise ValueError(out_dtype)


def out_to_f32(bits: np.ndarray, out_dtype: str) -> np.ndarray:
    if out_dtype == "bf16":
        return bf16_to_f32(bits)
    if out_dtype == "f16":
        return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)
    return np.asarray(bits, np.float32)


def gemm_i8_dequant(x8, w8, xs, ws, bias_f32=None, out_dtype="bf16"):
    """out = cast(((f32(x8 @ w8^T) * xs) * ws) + bias) -- `_gemm_intmm`."""
    acc = int_matmul_nt(x8, w8)
    return cast_out(dequant_epilogue(acc.astype(np.float32), xs, ws, bias_f32), out_dtype)


def fp8_matmul_nt_f64(a_codes, w_codes) -> np.ndarray:
    """sum_k a[m,k] * w[n,k] over e4m3 codes, in float64 (products exact)."""
    a = e4m3_to_f32(a_codes).astype(np.float64)
    w = e4m3_to_f32(w_codes).astype(np.float64)
    return a @ w.T


def gemm_fp8_dequant(a_codes, w_codes, xs, ws, bias_f32=None, out_dtype="bf16"):
    """fp8 e4m3 variant of the same epilogue; the accumulator is formed in
    float64 and rounded once to float32 (the tensor core's fp32 accumulation
    order differs, so GPU results are compared with a stated tolerance)."""
    acc = fp8_matmul_nt_f64(a_codes, w_codes).astype(np.float32)
    return cast_out(dequant_epilogue(acc, xs, ws, bias_f32), out_dtype)


def fp8_gemm_tolerance(a_codes, w_codes, xs, ws, K: int) -> np.ndarray:
    """Per-element bound on |gpu - oracle| before the output cast for the fp8 GEMM:
    K * 2^-22 * sum_k |a||w| scaled by |xs||ws| (fp32 accumulation error)."""
    a = np.abs(e4m3_to_f32(a_codes).astype(np.float64))
    w = np.abs(e4m3_to_f32(w_codes).astype(np.float64))
    mag = a @ w.T
    ws = np.asarray(ws, np.float64).reshape(-1)
    sc = np.abs(np.asarray(xs, np.float64)).reshape(-1, 1) * np.abs(ws.reshape(1, -1) if ws.size > 1 else ws.reshape(1, 1))
    return mag * sc * (max(K, 1) * 2.0 ** -22)


def gated_residual(res_f32, gate_rows_f32, y_f32) -> np.ndarray:
    """The block's gated residual update after the attention and MLP projections,
    `x = _mod_gate(x, gate, y, mod_segments)` (call sites src/ck_fused_patch.py:160-161 and
    :172; comfy's `_mod_gate` itself is not vendored, so this is the plain x + gate * y
    form, unpinned against comfy) in torch's bf16 eager order: t = bf16(gate * y) computed
    in float32, then bf16(x + t).  All inputs are bf16 values held as float32, gate_rows
    already expanded to the rows of y.  Returns bf16 bits."""
    t = round_bf16((np.asarray(gate_rows_f32, np.float32) * np.asarray(y_f32, np.float32)).astype(np.float32))
    return f32_to_bf16((np.asarray(res_f32, np.float32) + t).astype(np.float32))


# --------------------------------------------------------------------------
# RMSNorm + adaLN modulation (+ quant)
# --------------------------------------------------------------------------
def row_threads(D: int) -> int:
    """Threads that cooperate on one row in the row kernels (canonical shape)."""
    if D > ROW_MAX_D:
        raise ValueError(f"row length {D} exceeds {ROW_MAX_D}")
    nvec = (D + 7) // 8
    v = max(3, (nvec + 511) // 512)
    return max(32, 32 * ((nvec + 32 * v - 1) // (32 * v)))


def rms_sum_squares(x: np.ndarray) -> np.ndarray:
    """Sum of squares of each row of float32 values (bf16-representable), in
    the canonical order of the CUDA row kernel:

    * the row is split in 16-byte vectors of 8 values, vector c = t + T*i goes
      to thread t (T = row_threads(D));
    * each thread keeps two float32 accumulators, one for the even and one for
      the odd element of every bf16 pair, and adds the squares of its vectors
      in order (i ascending, pairs in order) -- a packed FMA in the kernel;
    * the thread's value is even + odd;
    * each 32-thread warp combines its lanes by a butterfly: for offset in
      16, 8, 4, 2, 1: v = v + v[lane ^ offset];
    * warp results are added left to right: ((w0 + w1) + w2) + ...

    Squares of bf16 values are exact in float32, so the kernel's FMA and the
    separate multiply-add here round identically.
    """
    x = np.asarray(x, dtype=np.float32)
    S, D = x.shape
    T = row_threads(D)
    nvec = (D + 7) // 8
    V = (nvec + T - 1) // T
    padded = np.zeros((S, V * T * 8), dtype=np.float32)
    padded[:, :D] = x
    xv = padded.reshape(S, V, T, 8)
    acc_e = np.zeros((S, T), dtype=np.float32)
    acc_o = np.zeros((S, T), dtype=np.float32)
    for i in range(V):
        blk = xv[:, i]
        for p in range(4):
            e = blk[:, :, 2 * p]
            o = blk[:, :, 2 * p + 1]
            acc_e = (acc_e + e * e).astype(np.float32)
            acc_o = (acc_o + o * o).astype(np.float32)
    acc = (acc_e + acc_o).astype(np.float32)
    W = T // 32
    lanes = acc.reshape(S, W, 32)
    idx = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        lanes = (lanes + lanes[:, :, idx ^ off]).astype(np.float32)
    tot = lanes[:, 0, 0].copy()
    for w in range(1, W):
        tot = (tot + lanes[:, w, 0]).astype(np.float32)
    return tot


REF_BLOCK_K = 2048     # src/ck_fused_mod_norm_quant.py:124 and src/ck_fused_patch.py:115


def rms_sum_squares_reference(x: np.ndarray, block: int = REF_BLOCK_K) -> np.ndarray:
    """Sum of squares of each row in the order of the reference's norm kernel
    (src/ck_fused_mod_norm_quant.py:35-41), as its tl.sum evaluates:

    * a float32 vector of `block` lanes accumulates the squares chunk by chunk,
      lane i += x[block * c + i]^2 for c = 0, 1, ... (missing elements count 0);
    * tl.sum of that vector is numpy's pairwise summation (Triton's interpreter
      calls np.sum): for 2048 lanes a balanced binary tree over 16 leaves of 128
      lanes, each leaf summed by 8 interleaved accumulators r_j (lanes 8t + j,
      t = 0..15, in order) combined as ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)).

    The tensorwise CUDA kernels (`rms_mod_tw_*`) compute exactly this.
    """
    x = np.asarray(x, dtype=np.float32)
    S, D = x.shape
    if block % 128 or block & (block - 1):
        raise ValueError("block must be a power of two multiple of 128")
    nch = max(1, -(-D // block))
    padded = np.zeros((S, nch * block), dtype=np.float32)
    padded[:, :D] = x
    sq = (padded * padded).astype(np.float32)            # exact: squares of bf16 values
    lanes = sq[:, :block].copy()
    for c in range(1, nch):
        lanes = (lanes + sq[:, c * block:(c + 1) * block]).astype(np.float32)
    leaves = lanes.reshape(S, block // 128, 16, 8)        # [row, leaf, t, j]
    r = leaves[:, :, 0, :].copy()
    for t in range(1, 16):
        r = (r + leaves[:, :, t, :]).astype(np.float32)
    f = lambda a, b: (a + b).astype(np.float32)           # noqa: E731
    leaf = f(f(f(r[..., 0], r[..., 1]), f(r[..., 2], r[..., 3])),
             f(f(r[..., 4], r[..., 5]), f(r[..., 6], r[..., 7])))
    while leaf.shape[1] > 1:
        leaf = f(leaf[:, 0::2], leaf[:, 1::2])
    return leaf[:, 0]


def rms_inv(ss: np.ndarray, D: int, eps: float) -> np.ndarray:
    """inv = 1 / sqrt(ss / D + eps) in float32 (reference: rsqrt(sum/K + eps),
    src/ck_fused_mod_norm_quant.py:41)."""
    mean = (np.asarray(ss, np.float32) / np.float32(D)).astype(np.float32)
    v = (mean + np.float32(eps)).astype(np.float32)
    return (np.float32(1.0) / np.sqrt(v)).astype(np.float32)


def mod_multiplier(scale_f32: np.ndarray, scale_is_multiplier: bool) -> np.ndarray:
    """s = scale as given, or bf16(1 + scale) as src/ck_fused_patch.py:120 does
    (`1.0 + scale[row].to(bf16)` rounds the sum to bf16)."""
    if scale_is_multiplier:
        return np.asarray(scale_f32, np.float32)
    return round_bf16((np.float32(1.0) + np.asarray(scale_f32, np.float32)).astype(np.float32))


def rms_mod_h(x, inv, w, s, b):
    """h = (((x * inv) * w) * s) + b in float32 (src/ck_fused_mod_norm_quant.py:51)."""
    t = (x * inv.reshape(-1, 1)).astype(np.float32)
    if w is not None:
        t = (t * w).astype(np.float32)
    t = (t * s).astype(np.float32)
    return (t + b).astype(np.float32)


def rms_mod_quant_per_token(x, shift, scale, *, w=None, mod_index=None, rows_per_mod=None,
                            scale_is_multiplier=False, eps=1e-6, kind=QUANT_FP8):
    """One-pass RMSNorm + modulation + per-token quant (float32 inputs holding
    bf16 values).

    h    = rms-norm(x) * s + shift, with s = bf16(1 + scale) for the row's
           modulation vector (mod_index[r], or r // rows_per_mod);
    h16  = bf16(h), res = bf16(h + x);
    q, qs = quant_rows(h16)  -- the quantiser sees the bf16 h, exactly what a
           separate quantiser given the bf16 h tensor would produce.
    Returns (q, qscale, h16 bits, res bits).
    """
    x = np.asarray(x, np.float32)
    S, D = x.shape
    if mod_index is None:
        rpm = rows_per_mod if rows_per_mod else S
        mod_index = np.arange(S) // max(rpm, 1)
    mod_index = np.asarray(mod_index, np.int64)
    s = mod_multiplier(np.asarray(scale, np.float32), scale_is_multiplier)[mod_index]
    b = np.asarray(shift, np.float32)[mod_index]
    inv = rms_inv(rms_sum_squares(x), D, eps)
    h = rms_mod_h(x, inv, None if w is None else np.asarray(w, np.float32), s, b)
    h16 = round_bf16(h)
    res = f32_to_bf16((h + x).astype(np.float32))
    q, qs = quant_rows(h16, kind)
    return q, qs, f32_to_bf16(h16), res


def rms_mod_res_tensorwise(x, w, s, b, eps=1e-5):
    """The reference's `fused_rms_mod_quant` (src/ck_fused_mod_norm_quant.py:121-145):
    h = rms(x)*w*s + b (float32), h16 = bf16(h), res = bf16(h + x),
    amax = max |h| over the whole tensor in float32 (before the bf16 cast,
    :54-55), scale = max(amax/448, 1e-12), q = e4m3(clamp(h16/scale, +-448)).
    Returns (q codes, scale, h16 bits, res bits, amax).

    The sum of squares follows the reference's own order
    (`rms_sum_squares_reference`), so h, the float32 amax and the scale are the
    reference's bit for bit.
    """
    x = np.asarray(x, np.float32)
    S, D = x.shape
    inv = rms_inv(rms_sum_squares_reference(x), D, eps)
    h = rms_mod_h(x, inv, None if w is None else np.asarray(w, np.float32),
                  np.asarray(s, np.float32), np.asarray(b, np.float32))
    amax = np.float32(np.max(np.abs(h))) if h.size else np.float32(0)
    scale = scale_from_amax(amax, QUANT_FP8)
    h16 = round_bf16(h)
    q = quantize_with_scale(h16, scale, QUANT_FP8)
    return q, scale, f32_to_bf16(h16), f32_to_bf16((h + x).astype(np.float32)), amax


# --------------------------------------------------------------------------
# SwiGLU (+ quant)
# --------------------------------------------------------------------------
def exp_f32(x) -> np.ndarray:
    """exp of float32 values, correctly rounded to float32.

    Evaluated in float64 (numpy's exp is accurate to well under one float64 ulp) and
    rounded once to float32.  A double rounding can only differ from the correctly
    rounded result when exp(x) lies within about 2^-29 float32 ulps of a rounding
    boundary; tests/test_oracle_golden.py checks every bf16 input against a
    multi-precision evaluation, and bf16 inputs are all this oracle feeds it.

    numpy's own float32 exp (which Triton's CPU interpreter calls for tl.exp) is not
    correctly rounded: it is off by one or two ulps on ~5 % of bf16 inputs, and its
    SIMD kernels differ between CPUs.  The GPU's compiled Triton uses an approximate
    exp2 instead.  The correctly rounded value is the one definition of
    sigmoid(g) = 1 / (1 + exp(-g)) that no platform's shortcut decides; on every golden
    vector the reference produced it gives the same act bits as the interpreter did."""
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        return np.exp(np.asarray(x, np.float32).astype(np.float64)).astype(np.float32)


def sigmoid_f32(g) -> np.ndarray:
    """sigmoid(g) = RN(1 / RN(1 + exp_f32(-g))) in float32 (Triton's tl.sigmoid,
    `1 / (1 + exp(-x))`, with the exponential correctly rounded)."""
    e = exp_f32(-np.asarray(g, np.float32))
    with np.errstate(over="ignore"):
        return (np.float32(1.0) / (np.float32(1.0) + e)).astype(np.float32)


def silu_mul(gate, up) -> np.ndarray:
    """act = (g * sigmoid(g)) * u in float32 (src/ck_fused_mod_norm_quant.py:71),
    each product rounded separately."""
    g = np.asarray(gate, np.float32)
    u = np.asarray(up, np.float32)
    return ((g * sigmoid_f32(g)).astype(np.float32) * u).astype(np.float32)


def swiglu_quant_per_token(gate, up, kind=QUANT_INT8):
    """act16 = bf16(silu(g) * u); q, qs = quant_rows(act16).
    Returns (q, qscale, act16 bits)."""
    act16 = round_bf16(silu_mul(gate, up))
    q, qs = quant_rows(act16, kind)
    return q, qs, f32_to_bf16(act16)


def swiglu_tensorwise(gate, up):
    """The reference's `fused_swiglu_quant` (src/ck_fused_mod_norm_quant.py:148-167):
    amax over float32 |act| (before the bf16 store, :71-73), q from bf16 act."""
    a = silu_mul(gate, up)
    amax = np.float32(np.max(np.abs(a))) if a.size else np.float32(0)
    scale = scale_from_amax(amax, QUANT_FP8)
    a16 = round_bf16(a)
    return quantize_with_scale(a16, scale, QUANT_FP8), scale, f32_to_bf16(a16), amax


def quant_tensorwise_given(h16_f32, amax, kind=QUANT_FP8):
    """`_quant_fp8_amax_kernel` given h and the device amax (:103-111)."""
    scale = scale_from_amax(np.float32(amax), kind)
    return quantize_with_scale(h16_f32, scale, kind), scale
