"""torch-facing wrappers of the C ABI.

torch provides device memory and the current stream only; every computation
runs in the library's sm_100a kernels.  Tensors must be CUDA tensors with a
unit stride along their last dimension.  Calls are asynchronous on the given
stream (default: torch's current stream of the tensor's device).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

OUT_CODE = {torch.bfloat16: _lib.OUT_BF16, torch.float16: _lib.OUT_F16, torch.float32: _lib.OUT_F32}
QUANT_CODE = {"int8": _lib.QUANT_INT8, "fp8_e4m3": _lib.QUANT_FP8_E4M3}
QUANT_DTYPE = {"int8": torch.int8, "fp8_e4m3": torch.float8_e4m3fn}
F8_E4M3_MAX = 448.0


# torch's current raw cudaStream_t without building a Stream object (2 us -> 0.1 us a call)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(device, stream=None) -> int:
    if stream is None:
        idx = device.index if isinstance(device, torch.device) else device
        if idx is None:
            idx = torch.cuda.current_device()
        if _raw_stream is not None:
            return _raw_stream(idx)
        return torch.cuda.current_stream(idx).cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


class _on:
    """Makes `device` the current CUDA device inside the block (a no-op when it already is)."""
    __slots__ = ("idx", "prev")

    def __init__(self, device):
        self.idx = device.index if isinstance(device, torch.device) else device

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.idx is not None and self.idx != self.prev:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.idx is not None and self.idx != self.prev:
            torch.cuda.set_device(self.prev)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need_cuda(name, t, dtype=None, ndim=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
    if dtype is not None and t.dtype not in (dtype if isinstance(dtype, tuple) else (dtype,)):
        raise TypeError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    if t.dim() >= 1 and t.numel() and t.stride(-1) != 1:
        raise ValueError(f"{name} must have unit stride in its last dimension")


def gemm_dequant(x: torch.Tensor, w: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor,
                 bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 out_dtype: torch.dtype = torch.bfloat16, stream=None) -> torch.Tensor:
    """out = cast(((f32(x @ w^T) * x_scale[:, None]) * w_scale) + bias).

    x [M, K] and w [N, K] are both int8 (exact int32 accumulation) or both
    float8_e4m3fn (fp32 accumulation); x_scale [M] float32; w_scale [N] or [1]
    float32; bias [N] in the output dtype or None/empty; out [M, N] bf16/fp16/fp32.
    """
    if out is None and x.dim() == 2 and w.dim() == 2:
        out = torch.empty(x.shape[0], w.shape[0], dtype=out_dtype, device=x.device)
    if not _gemm_args_ok(x, w, x_scale, w_scale, bias, out):
        _gemm_args_explain(x, w, x_scale, w_scale, bias, out)
    M, K = x.shape
    N = w.shape[0]
    nb = 0 if bias is None else bias.numel()
    fn = _lib.load().t8g_gemm_i8_dequant if x.dtype is torch.int8 else _lib.load().t8g_gemm_fp8_dequant
    idx = x.get_device()
    with _on(idx):
        rc = fn(x.data_ptr(), w.data_ptr(), x_scale.data_ptr(), w_scale.data_ptr(), w_scale.numel(),
                bias.data_ptr() if nb else None, nb, out.data_ptr(), OUT_CODE[out.dtype], M, N, K, x.stride(0),
                w.stride(0), out.stride(0), _stream_handle(idx, stream))
    if rc:
        _lib.check(rc)
    return out


_GEMM_IN = (torch.int8, torch.float8_e4m3fn)


def _gemm_args_ok(x, w, xs, ws, bias, out) -> bool:
    """The common case of gemm_dequant's argument rules, checked cheaply; a False sends the
    call through _gemm_args_explain, which raises the precise error."""
    try:
        xd = x.dtype
        if xd not in _GEMM_IN or w.dtype is not xd or x.dim() != 2 or w.dim() != 2 or out is None or out.dim() != 2:
            return False
        M, K = x.shape
        N, Kw = w.shape
        if Kw != K or out.shape[0] != M or out.shape[1] != N or out.dtype not in OUT_CODE:
            return False
        if not (x.is_cuda and w.is_cuda and xs.is_cuda and ws.is_cuda and out.is_cuda):
            return False
        d = x.get_device()
        if w.get_device() != d or xs.get_device() != d or ws.get_device() != d or out.get_device() != d:
            return False
        if (M and K and x.stride(1) != 1) or (N and K and w.stride(1) != 1) or (M and N and out.stride(1) != 1):
            return False
        if xs.dtype is not torch.float32 or ws.dtype is not torch.float32:
            return False
        if xs.numel() != M or not xs.is_contiguous() or ws.numel() not in (1, N) or not ws.is_contiguous():
            return False
        if bias is not None and bias.numel():
            if (not bias.is_cuda or bias.get_device() != d or bias.dtype is not out.dtype or bias.numel() != N
                    or not bias.is_contiguous()):
                return False
        return True
    except (AttributeError, TypeError, ValueError):
        return False


def _gemm_args_explain(x, w, x_scale, w_scale, bias, out) -> None:
    _need_cuda("x", x, _GEMM_IN, 2)
    _need_cuda("w", w, x.dtype, 2)
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"w has K={w.shape[1]}, x has K={K}")
    _need_cuda("x_scale", x_scale, torch.float32)
    _need_cuda("w_scale", w_scale, torch.float32)
    if x_scale.numel() != M or not x_scale.is_contiguous():
        raise ValueError("x_scale must be a contiguous float32 tensor with M elements")
    if w_scale.numel() not in (1, N) or not w_scale.is_contiguous():
        raise ValueError("w_scale must be a contiguous float32 tensor with 1 or N elements")
    _need_cuda("out", out, tuple(OUT_CODE), 2)
    if tuple(out.shape) != (M, N):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(M, N)}")
    if bias is not None and bias.numel():
        _need_cuda("bias", bias, out.dtype)
        if bias.numel() != N or not bias.is_contiguous():
            raise ValueError("bias must be contiguous with N elements, in the output dtype")
    ts = [x, w, x_scale, w_scale, out] + ([bias] if bias is not None and bias.numel() else [])
    if len({t.get_device() for t in ts}) != 1:
        raise ValueError("x, w, the scales, bias and out must be on one CUDA device")
    raise ValueError("gemm_dequant: arguments rejected")   # the fast check and this one disagree


SWIGLU_BLOCK = 128


def interleave_gate_up(t: torch.Tensor, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    """Reorder an fc1 parameter whose first half (along dim 0) is gate and second half up
    into the layout of gemm_swiglu: blocks of `block` gate rows followed by the matching
    `block` up rows.  Works for the weight [2F, K], its per-channel scales [2F] and the
    bias [2F]; done once when the weights are loaded."""
    n = t.shape[0]
    if n % (2 * block):
        raise ValueError(f"dim 0 ({n}) must be a multiple of {2 * block}")
    F = n // 2
    g = t[:F].reshape(F // block, block, *t.shape[1:])
    u = t[F:].reshape(F // block, block, *t.shape[1:])
    return torch.stack([g, u], dim=1).reshape(t.shape).contiguous()


def gemm_swiglu(x: torch.Tensor, w_il: torch.Tensor, x_scale: torch.Tensor, w_scale_il: torch.Tensor,
                bias_il: torch.Tensor | None = None, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """act = bf16(silu(gate) * up) of the fc1 GEMM, fused: gate / up are the bf16 outputs
    the plain gemm_dequant would produce for fc1 channels j and F + j.  w_il, w_scale_il
    (numel 2F, or 1) and bias_il (bf16, 2F) come from interleave_gate_up; x int8 [M, K] or
    float8_e4m3fn; out [M, F] bf16."""
    _need_cuda("x", x, (torch.int8, torch.float8_e4m3fn), 2)
    _need_cuda("w", w_il, x.dtype, 2)
    M, K = x.shape
    N = w_il.shape[0]
    if w_il.shape[1] != K:
        raise ValueError(f"w has K={w_il.shape[1]}, x has K={K}")
    if N % (2 * SWIGLU_BLOCK):
        raise ValueError(f"w must have 2F rows with F a multiple of {SWIGLU_BLOCK}")
    F = N // 2
    _need_cuda("x_scale", x_scale, torch.float32)
    _need_cuda("w_scale", w_scale_il, torch.float32)
    if x_scale.numel() != M or not x_scale.is_contiguous():
        raise ValueError("x_scale must be a contiguous float32 tensor with M elements")
    if w_scale_il.numel() not in (1, N) or not w_scale_il.is_contiguous():
        raise ValueError("w_scale must be a contiguous float32 tensor with 1 or 2F elements")
    if out is None:
        out = torch.empty(M, F, dtype=torch.bfloat16, device=x.device)
    _need_cuda("out", out, torch.bfloat16, 2)
    if tuple(out.shape) != (M, F):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(M, F)}")
    nb = 0 if bias_il is None else bias_il.numel()
    if nb:
        _need_cuda("bias", bias_il, torch.bfloat16)
        if nb != N or not bias_il.is_contiguous():
            raise ValueError("bias must be contiguous bf16 with 2F elements")
    lib = _lib.load()
    fn = lib.t8g_gemm_i8_swiglu if x.dtype == torch.int8 else lib.t8g_gemm_fp8_swiglu
    with _on(x.device):
        rc = fn(_ptr(x), _ptr(w_il), _ptr(x_scale), _ptr(w_scale_il), w_scale_il.numel(),
                _ptr(bias_il) if nb else None, nb, _ptr(out), M, F, K, x.stride(0), w_il.stride(0), out.stride(0),
                _stream_handle(x.device, stream))
    _lib.check(rc)
    return out


def gemm_swiglu_quant(x: torch.Tensor, w_il: torch.Tensor, x_scale: torch.Tensor, w_scale_il: torch.Tensor,
                      bias_il: torch.Tensor | None = None, kind: str = "int8", act: torch.Tensor | None = None,
                      stream=None):
    """fc1 + SwiGLU + per-token quantisation of act in one call -> (q, q_scale, act): the SwiGLU
    epilogue also reports each row's max |act|, so the quantiser streams act once (equal bit
    for bit to quant_rows(gemm_swiglu(...)))."""
    _need_cuda("x", x, (torch.int8, torch.float8_e4m3fn), 2)
    _need_cuda("w", w_il, x.dtype, 2)
    M, K = x.shape
    N = w_il.shape[0]
    if w_il.shape[1] != K:
        raise ValueError(f"w has K={w_il.shape[1]}, x has K={K}")
    if N % (2 * SWIGLU_BLOCK):
        raise ValueError(f"w must have 2F rows with F a multiple of {SWIGLU_BLOCK}")
    F = N // 2
    _need_cuda("x_scale", x_scale, torch.float32)
    _need_cuda("w_scale", w_scale_il, torch.float32)
    if x_scale.numel() != M or not x_scale.is_contiguous():
        raise ValueError("x_scale must be a contiguous float32 tensor with M elements")
    if w_scale_il.numel() not in (1, N) or not w_scale_il.is_contiguous():
        raise ValueError("w_scale must be a contiguous float32 tensor with 1 or 2F elements")
    if act is None:
        act = torch.empty(M, F, dtype=torch.bfloat16, device=x.device)
    _need_cuda("act", act, torch.bfloat16, 2)
    if tuple(act.shape) != (M, F):
        raise ValueError(f"act has shape {tuple(act.shape)}, expected {(M, F)}")
    nb = 0 if bias_il is None else bias_il.numel()
    if nb:
        _need_cuda("bias", bias_il, torch.bfloat16)
        if nb != N or not bias_il.is_contiguous():
            raise ValueError("bias must be contiguous bf16 with 2F elements")
    amax = torch.empty(M, dtype=torch.float32, device=x.device)
    q = torch.empty(M, F, dtype=QUANT_DTYPE[kind], device=x.device)
    q_scale = torch.empty(M, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    fn = lib.t8g_gemm_i8_swiglu_quant if x.dtype == torch.int8 else lib.t8g_gemm_fp8_swiglu_quant
    with _on(x.device):
        rc = fn(_ptr(x), _ptr(w_il), _ptr(x_scale), _ptr(w_scale_il), w_scale_il.numel(),
                _ptr(bias_il) if nb else None, nb, _ptr(act), act.stride(0), _ptr(amax), _ptr(q), q.stride(0),
                _ptr(q_scale), M, F, K, x.stride(0), w_il.stride(0), QUANT_CODE[kind], _stream_handle(x.device, stream))
    _lib.check(rc)
    return q, q_scale, act


def gemm_gated(x: torch.Tensor, w: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor,
               bias: torch.Tensor | None, res: torch.Tensor, gate: torch.Tensor, *,
               rows_per_gate: int | None = None, gate_index: torch.Tensor | None = None,
               out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """The DiT block's gated residual with the projection GEMM fused in front of it:
    out = res + gate[g] * y in torch's bf16 order (t = bf16(gate * y), out = bf16(res + t)),
    y = gemm_dequant(x, w, x_scale, w_scale, bias) as bf16, never stored.  g is
    gate_index[m] (int32 [M]) or m // rows_per_gate (default: M // gate rows, which must
    divide M).  res [M, N] bf16; gate [n_gate, N] bf16; out [M, N] bf16, may be res itself
    (in-place update)."""
    _need_cuda("x", x, (torch.int8, torch.float8_e4m3fn), 2)
    _need_cuda("w", w, x.dtype, 2)
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"w has K={w.shape[1]}, x has K={K}")
    _need_cuda("x_scale", x_scale, torch.float32)
    _need_cuda("w_scale", w_scale, torch.float32)
    if x_scale.numel() != M or not x_scale.is_contiguous():
        raise ValueError("x_scale must be a contiguous float32 tensor with M elements")
    if w_scale.numel() not in (1, N) or not w_scale.is_contiguous():
        raise ValueError("w_scale must be a contiguous float32 tensor with 1 or N elements")
    _need_cuda("res", res, torch.bfloat16, 2)
    if tuple(res.shape) != (M, N):
        raise ValueError(f"res has shape {tuple(res.shape)}, expected {(M, N)}")
    if gate.dim() == 1:
        gate = gate.view(1, -1)
    _need_cuda("gate", gate, torch.bfloat16, 2)
    if gate.shape[1] != N or gate.shape[0] < 1:
        raise ValueError(f"gate must be [n_gate, {N}], got {tuple(gate.shape)}")
    if gate_index is not None:
        _need_cuda("gate_index", gate_index, torch.int32, 1)
        if gate_index.numel() != M or not gate_index.is_contiguous():
            raise ValueError("gate_index must be a contiguous int32 tensor with M elements")
        rpg = 0
    else:
        if rows_per_gate is None:
            if M % gate.shape[0]:
                raise ValueError(f"{M} rows do not split evenly over {gate.shape[0]} gate rows; pass gate_index")
            rows_per_gate = max(1, M // gate.shape[0])
        rpg = int(rows_per_gate)
        if rpg < 1 or (M and (M - 1) // rpg >= gate.shape[0]):
            raise ValueError(f"rows_per_gate={rpg} maps rows past the {gate.shape[0]} gate rows")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    _need_cuda("out", out, torch.bfloat16, 2)
    if tuple(out.shape) != (M, N):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(M, N)}")
    nb = 0 if bias is None else bias.numel()
    if nb:
        _need_cuda("bias", bias, torch.bfloat16)
        if nb != N or not bias.is_contiguous():
            raise ValueError("bias must be contiguous bf16 with N elements")
    lib = _lib.load()
    fn = lib.t8g_gemm_i8_gated if x.dtype == torch.int8 else lib.t8g_gemm_fp8_gated
    with _on(x.device):
        rc = fn(_ptr(x), _ptr(w), _ptr(x_scale), _ptr(w_scale), w_scale.numel(), _ptr(bias) if nb else None, nb,
                _ptr(res), res.stride(0), _ptr(gate), gate.stride(0), _ptr(gate_index), rpg, _ptr(out),
                M, N, K, x.stride(0), w.stride(0), out.stride(0), _stream_handle(x.device, stream))
    _lib.check(rc)
    return out


def quant_rows(x: torch.Tensor, kind: str = "int8", q: torch.Tensor | None = None,
               q_scale: torch.Tensor | None = None, stream=None):
    """Per-token quantisation of a bf16 [S, D] matrix -> (q [S, D], q_scale [S] float32)."""
    _need_cuda("x", x, torch.bfloat16, 2)
    S, D = x.shape
    if q is None:
        q = torch.empty(S, D, dtype=QUANT_DTYPE[kind], device=x.device)
    if q_scale is None:
        q_scale = torch.empty(S, dtype=torch.float32, device=x.device)
    _need_cuda("q", q, QUANT_DTYPE[kind], 2)
    with _on(x.device):
        rc = _lib.load().t8g_quant_rows(_ptr(x), x.stride(0), _ptr(q), q.stride(0), _ptr(q_scale), S, D,
                                        QUANT_CODE[kind], _stream_handle(x.device, stream))
    _lib.check(rc)
    return q, q_scale


def _mod_args(x, shift, scale, mod_index, rows_per_mod):
    S, D = x.shape
    for name, t in (("shift", shift), ("scale", scale)):
        _need_cuda(name, t, torch.bfloat16)
        if t.dim() == 1:
            if t.shape[0] != D:
                raise ValueError(f"{name} must have D={D} elements")
        elif t.dim() != 2 or t.shape[1] != D:
            raise ValueError(f"{name} must be [n_mod, D]")
    shift2 = shift.reshape(-1, D)
    scale2 = scale.reshape(-1, D)
    if shift2.stride(0) != scale2.stride(0):
        raise ValueError("shift and scale must share a row stride")
    if mod_index is not None:
        _need_cuda("mod_index", mod_index, torch.int32, 1)
        if mod_index.numel() != S or not mod_index.is_contiguous():
            raise ValueError("mod_index must be a contiguous int32 tensor with S elements")
        rows_per_mod = 1
    elif rows_per_mod is None:
        n_mod = shift2.shape[0]
        if S % n_mod:
            raise ValueError(f"{S} rows do not split evenly over {n_mod} modulation rows; pass mod_index")
        rows_per_mod = max(S // n_mod, 1)
    return shift2, scale2, rows_per_mod


def rms_mod_quant(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, *, w: torch.Tensor | None = None,
                  mod_index: torch.Tensor | None = None, rows_per_mod: int | None = None,
                  scale_is_multiplier: bool = False, eps: float = 1e-6, kind: str = "fp8_e4m3",
                  return_h: bool = False, return_res: bool = False, stream=None):
    """One-pass RMSNorm + adaLN modulation + per-token quantisation of x [S, D] bf16.

    h = rms_norm(x) * w * s + shift[row], s = bf16(1 + scale[row]) (or scale itself
    when scale_is_multiplier); the modulation row of token r is mod_index[r], or
    r // rows_per_mod (default: S split evenly over the rows of shift/scale).
    Returns (q, q_scale[, h][, res]).
    """
    _need_cuda("x", x, torch.bfloat16, 2)
    S, D = x.shape
    shift2, scale2, rpm = _mod_args(x, shift, scale, mod_index, rows_per_mod)
    if w is not None:
        _need_cuda("w", w, torch.bfloat16, 1)
        if w.numel() != D:
            raise ValueError("w must have D elements")
    q = torch.empty(S, D, dtype=QUANT_DTYPE[kind], device=x.device)
    q_scale = torch.empty(S, dtype=torch.float32, device=x.device)
    h = torch.empty_like(x) if return_h else None
    res = torch.empty_like(x) if return_res else None
    with _on(x.device):
        rc = _lib.load().t8g_rms_mod_quant(
            _ptr(x), x.stride(0), _ptr(w), _ptr(shift2), _ptr(scale2), shift2.stride(0), _ptr(mod_index), rpm,
            int(scale_is_multiplier), float(eps), _ptr(q), q.stride(0), _ptr(q_scale), _ptr(h), D, _ptr(res), D,
            S, D, QUANT_CODE[kind], _stream_handle(x.device, stream))
    _lib.check(rc)
    out = [q, q_scale]
    if return_h:
        out.append(h)
    if return_res:
        out.append(res)
    return tuple(out)


def rms_mod_quant_tensorwise(x, shift, scale, *, w=None, mod_index=None, rows_per_mod=None,
                             scale_is_multiplier=False, eps=1e-5, kind="fp8_e4m3", want_res=True, stream=None):
    """The reference's two-phase form: (q, scale 0-d tensor, h, res); one scale for the tensor."""
    _need_cuda("x", x, torch.bfloat16, 2)
    S, D = x.shape
    shift2, scale2, rpm = _mod_args(x, shift, scale, mod_index, rows_per_mod)
    if w is not None:
        _need_cuda("w", w, torch.bfloat16, 1)
    q = torch.empty(S, D, dtype=QUANT_DTYPE[kind], device=x.device)
    h = torch.empty_like(x)
    res = torch.empty_like(x) if want_res else None
    amax = torch.zeros((), dtype=torch.float32, device=x.device)
    qs = torch.empty((), dtype=torch.float32, device=x.device)
    with _on(x.device):
        rc = _lib.load().t8g_rms_mod_quant_tensorwise(
            _ptr(x), x.stride(0), _ptr(w), _ptr(shift2), _ptr(scale2), shift2.stride(0), _ptr(mod_index), rpm,
            int(scale_is_multiplier), float(eps), _ptr(q), q.stride(0), _ptr(h), D, _ptr(res), D, _ptr(amax),
            _ptr(qs), S, D, QUANT_CODE[kind], _stream_handle(x.device, stream))
    _lib.check(rc)
    return q, qs, h, res


def swiglu_quant(gate: torch.Tensor, up: torch.Tensor, kind: str = "int8", return_act: bool = False, stream=None):
    """act = bf16(silu(gate) * up), per-token quantised -> (q, q_scale[, act]).

    gate and up are [M, F] bf16 views with the same row stride (for example the
    two halves of a [M, 2F] fc1 output, read in place)."""
    _need_cuda("gate", gate, torch.bfloat16, 2)
    _need_cuda("up", up, torch.bfloat16, 2)
    if gate.shape != up.shape or gate.stride() != up.stride():
        raise ValueError("gate and up must have the same shape and strides")
    M, F = gate.shape
    q = torch.empty(M, F, dtype=QUANT_DTYPE[kind], device=gate.device)
    q_scale = torch.empty(M, dtype=torch.float32, device=gate.device)
    act = torch.empty(M, F, dtype=torch.bfloat16, device=gate.device) if return_act else None
    with _on(gate.device):
        rc = _lib.load().t8g_swiglu_quant(_ptr(gate), _ptr(up), gate.stride(0), _ptr(q), q.stride(0), _ptr(q_scale),
                                          _ptr(act), F, M, F, QUANT_CODE[kind], _stream_handle(gate.device, stream))
    _lib.check(rc)
    return (q, q_scale, act) if return_act else (q, q_scale)


def swiglu_quant_fc1(y: torch.Tensor, kind: str = "int8", return_act: bool = False, stream=None):
    """SwiGLU + quant of a [M, 2F] fc1 output whose first half is the gate."""
    F = y.shape[-1] // 2
    return swiglu_quant(y[:, :F], y[:, F:], kind=kind, return_act=return_act, stream=stream)


def swiglu_quant_tensorwise(gate, up, kind="fp8_e4m3", stream=None):
    """The reference's two-phase form: (q, scale 0-d tensor, act)."""
    _need_cuda("gate", gate, torch.bfloat16, 2)
    _need_cuda("up", up, torch.bfloat16, 2)
    if gate.shape != up.shape or gate.stride() != up.stride():
        raise ValueError("gate and up must have the same shape and strides")
    M, F = gate.shape
    q = torch.empty(M, F, dtype=QUANT_DTYPE[kind], device=gate.device)
    act = torch.empty(M, F, dtype=torch.bfloat16, device=gate.device)
    amax = torch.zeros((), dtype=torch.float32, device=gate.device)
    qs = torch.empty((), dtype=torch.float32, device=gate.device)
    with _on(gate.device):
        rc = _lib.load().t8g_swiglu_quant_tensorwise(_ptr(gate), _ptr(up), gate.stride(0), _ptr(q), q.stride(0),
                                                     _ptr(act), F, _ptr(amax), _ptr(qs), M, F, QUANT_CODE[kind],
                                                     _stream_handle(gate.device, stream))
    _lib.check(rc)
    return q, qs, act


def device_status(device=None, stream=None) -> int:
    """Synchronise and read/clear the device status word (0 = no wait ran out)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    st = ctypes.c_int(0)
    with _on(device):
        rc = _lib.load().t8g_device_status(_stream_handle(device, stream), ctypes.byref(st))
    _lib.check(rc)
    return st.value


_status_words = {}


def status_mirror(device=None):
    """The host-visible mirror of the device status word (a ctypes pointer to one int, shared by
    every device), set up for `device` on first use: nonzero once any kernel's bounded wait ran
    out.  Read it with `[0]`, clear it by assigning 0; no synchronisation or CUDA call involved."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    word = _status_words.get(device.index)
    if word is None:
        word = ctypes.POINTER(ctypes.c_int)()
        with _on(device):
            rc = _lib.load().t8g_status_mirror(ctypes.byref(word))
        _lib.check(rc)
        _status_words[device.index] = word
    return word


def wait_selftest(limit_ns: int = 20_000_000, device=None) -> int:
    """Run the bounded-wait self-test kernel; returns 1 if the wait gave up."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flag = torch.zeros(1, dtype=torch.int32, device=device)
    with _on(device):
        rc = _lib.load().t8g_wait_selftest(limit_ns, _ptr(flag), _stream_handle(device))
    _lib.check(rc)
    return int(flag.item())
