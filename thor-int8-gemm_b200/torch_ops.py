"""torch custom ops (namespace `t8g`) over the library's kernels, with fake (shape-only)
implementations, so that `torch.compile` can trace models that use them.

The reference keeps comfy-kitchen's `int8_linear` traceable by routing it, while
torch.compile traces, through comfy's own registered custom op instead of the eager
function that hands DLPack capsules to `_C` (src/ck_int8_patch_thor.py:191-216): a
FakeTensor has no storage to export.  These ops give the same property to this library's
entry points: under tracing only the fake implementation runs (output shapes and
dtypes), at run time the op calls the CUDA kernel on the current stream.

    t8g::gemm_dequant(x, w, x_scale, w_scale, bias?, out_dtype) -> out
    t8g::quant_rows(x, kind) -> (q, q_scale)
    t8g::int8_linear(x, w, w_scale, bias?, out_dtype) -> out      (per-token quant + GEMM)
    t8g::rms_mod_quant(x, shift, scale, w?, mod_index?, rows_per_mod, scale_is_multiplier,
                       eps, kind) -> (q, q_scale)
    t8g::swiglu_quant(y, kind) -> (q, q_scale)                     (y = [M, 2F] fc1 output)
    t8g::gemm_swiglu(x, w_il, x_scale, w_scale_il, bias_il?) -> act  (fc1 + SwiGLU epilogue)
    t8g::gemm_gated(x, w, x_scale, w_scale, bias?, res, gate, rows_per_gate) -> res + gate * y
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops

_QDTYPE = {"int8": torch.int8, "fp8_e4m3": torch.float8_e4m3fn}


def _qdtype(kind: str) -> torch.dtype:
    if kind not in _QDTYPE:
        raise ValueError(f"unknown quant kind {kind!r}")
    return _QDTYPE[kind]


@torch.library.custom_op("t8g::gemm_dequant", mutates_args=())
def gemm_dequant(x: torch.Tensor, w: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor,
                 bias: Optional[torch.Tensor], out_dtype: torch.dtype) -> torch.Tensor:
    return ops.gemm_dequant(x, w, x_scale, w_scale, bias, out_dtype=out_dtype)


@gemm_dequant.register_fake
def _(x, w, x_scale, w_scale, bias, out_dtype):
    torch._check(x.dim() == 2 and w.dim() == 2, lambda: "x and w must be 2-D")
    torch._check(x.shape[1] == w.shape[1], lambda: "x and w must share K")
    return x.new_empty((x.shape[0], w.shape[0]), dtype=out_dtype)


@torch.library.custom_op("t8g::quant_rows", mutates_args=())
def quant_rows(x: torch.Tensor, kind: str) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.quant_rows(x, kind)


@quant_rows.register_fake
def _(x, kind):
    torch._check(x.dim() == 2, lambda: "x must be 2-D")
    return x.new_empty(x.shape, dtype=_qdtype(kind)), x.new_empty((x.shape[0],), dtype=torch.float32)


@torch.library.custom_op("t8g::int8_linear", mutates_args=())
def int8_linear(x: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor, bias: Optional[torch.Tensor],
                out_dtype: torch.dtype) -> torch.Tensor:
    xq, xs = ops.quant_rows(x.reshape(-1, x.shape[-1]), "int8")
    out = ops.gemm_dequant(xq, w, xs, w_scale, bias, out_dtype=out_dtype)
    return out.reshape(*x.shape[:-1], w.shape[0])


@int8_linear.register_fake
def _(x, w, w_scale, bias, out_dtype):
    torch._check(x.shape[-1] == w.shape[1], lambda: "x and w must share K")
    return x.new_empty((*x.shape[:-1], w.shape[0]), dtype=out_dtype)


@torch.library.custom_op("t8g::rms_mod_quant", mutates_args=())
def rms_mod_quant(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, w: Optional[torch.Tensor],
                  mod_index: Optional[torch.Tensor], rows_per_mod: int, scale_is_multiplier: bool, eps: float,
                  kind: str) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.rms_mod_quant(x, shift, scale, w=w, mod_index=mod_index,
                             rows_per_mod=rows_per_mod if mod_index is None else None,
                             scale_is_multiplier=scale_is_multiplier, eps=eps, kind=kind)


@rms_mod_quant.register_fake
def _(x, shift, scale, w, mod_index, rows_per_mod, scale_is_multiplier, eps, kind):
    torch._check(x.dim() == 2, lambda: "x must be 2-D")
    return x.new_empty(x.shape, dtype=_qdtype(kind)), x.new_empty((x.shape[0],), dtype=torch.float32)


@torch.library.custom_op("t8g::swiglu_quant", mutates_args=())
def swiglu_quant(y: torch.Tensor, kind: str) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.swiglu_quant_fc1(y, kind=kind)


@swiglu_quant.register_fake
def _(y, kind):
    torch._check(y.dim() == 2 and y.shape[1] % 2 == 0, lambda: "y must be [M, 2F]")
    return y.new_empty((y.shape[0], y.shape[1] // 2), dtype=_qdtype(kind)), \
        y.new_empty((y.shape[0],), dtype=torch.float32)


@torch.library.custom_op("t8g::gemm_swiglu", mutates_args=())
def gemm_swiglu(x: torch.Tensor, w_il: torch.Tensor, x_scale: torch.Tensor, w_scale_il: torch.Tensor,
                bias_il: Optional[torch.Tensor]) -> torch.Tensor:
    return ops.gemm_swiglu(x, w_il, x_scale, w_scale_il, bias_il)


@gemm_swiglu.register_fake
def _(x, w_il, x_scale, w_scale_il, bias_il):
    torch._check(x.dim() == 2 and w_il.dim() == 2 and x.shape[1] == w_il.shape[1], lambda: "x [M, K], w [2F, K]")
    return x.new_empty((x.shape[0], w_il.shape[0] // 2), dtype=torch.bfloat16)


@torch.library.custom_op("t8g::gemm_swiglu_quant", mutates_args=())
def gemm_swiglu_quant(x: torch.Tensor, w_il: torch.Tensor, x_scale: torch.Tensor, w_scale_il: torch.Tensor,
                      bias_il: Optional[torch.Tensor], kind: str) -> tuple[torch.Tensor, torch.Tensor]:
    q, q_scale, _act = ops.gemm_swiglu_quant(x, w_il, x_scale, w_scale_il, bias_il, kind=kind)
    return q, q_scale


@gemm_swiglu_quant.register_fake
def _(x, w_il, x_scale, w_scale_il, bias_il, kind):
    torch._check(x.dim() == 2 and w_il.dim() == 2 and x.shape[1] == w_il.shape[1], lambda: "x [M, K], w [2F, K]")
    return x.new_empty((x.shape[0], w_il.shape[0] // 2), dtype=_qdtype(kind)), \
        x.new_empty((x.shape[0],), dtype=torch.float32)


@torch.library.custom_op("t8g::gemm_gated", mutates_args=())
def gemm_gated(x: torch.Tensor, w: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor,
               bias: Optional[torch.Tensor], res: torch.Tensor, gate: torch.Tensor, rows_per_gate: int) -> torch.Tensor:
    return ops.gemm_gated(x, w, x_scale, w_scale, bias, res, gate, rows_per_gate=rows_per_gate)


@gemm_gated.register_fake
def _(x, w, x_scale, w_scale, bias, res, gate, rows_per_gate):
    torch._check(x.dim() == 2 and w.dim() == 2 and x.shape[1] == w.shape[1], lambda: "x [M, K], w [N, K]")
    torch._check(res.shape[0] == x.shape[0] and res.shape[1] == w.shape[0], lambda: "res must be [M, N]")
    return res.new_empty(res.shape, dtype=torch.bfloat16)
